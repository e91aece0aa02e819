"""Expert parallelism over NVLink peer memory: the MoE layer with its experts sharded over the ranks,
the token rows crossing to their experts' ranks and back by stores into the peers' memory (the
ck_ep_peer_* kernels, include/ck_b200.h) instead of collective calls.

Each rank owns one device arena, which every peer maps through CUDA IPC:

    [flags: dispatch [32] u64 | return [32] u64 | step u64 | error i32]
    [receive rows  bf16 [world * cap, hidden]]      region s: the rows source rank s sent here
    [receive ids   int32 [world * cap, nsel]]       the slots' local experts, -1 where none
    [receive wts   fp32 [world * cap, nsel]]
    [receive token int32 [world * cap]]             the source's token number of each row
    [return rows   bf16 [cap * (nsel + n_shared), hidden]]   row t * nsel + k: the (token, slot)
                                                    output from its expert's rank; then the shared
                                                    expert's rows of the local tokens

A forward issues, on one stream and with no host wait: the route, the dispatch plan, the shared
expert (side stream), the dispatch stores, a barrier, the regroup of all world * cap received rows by
local expert (unused rows carry expert -1), the expert GEMMs, the return stores (from the down
projection's own epilogue when it runs on the grouped GEMM: every output row is stored straight into
its source's return buffer, so the return crosses NVLink while the GEMM runs), a barrier and the
combine.  It can therefore be captured in a CUDA graph and replayed.  The (token, slot) rows reach the
combine in the reference's order, computed by the same kernels as on one GPU, so the output equals
the single-GPU layer's bit for bit whenever both take the same expert-GEMM form (the few-token
matvec when world * cap <= 128 rows on the receiver and ntok <= 128 on one GPU, the GEMM above).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .moe import DECODE_TOKENS, FEW_TOKENS, MoeSpec, _align
from .ops import _dev, _ptr, _stream

MAX_RANKS = 32
WAIT_NS = 10_000_000_000  # a barrier gives up after 10 s and sets the error word


class EpPeers(ctypes.Structure):
    """ck_ep_peers (include/ck_b200.h)."""
    _fields_ = ([("world", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("cap", ctypes.c_uint32),
                 ("nsel", ctypes.c_uint32), ("hidden", ctypes.c_uint32), ("reserved", ctypes.c_uint32)] +
                [(n, ctypes.c_void_p * MAX_RANKS) for n in ("recv_x", "recv_ids", "recv_w", "recv_tok", "ret_y",
                                                             "dflag", "rflag")] +
                [(n, ctypes.c_void_p) for n in ("my_dflags", "my_rflags", "ctr", "err")])


def arena_layout(world, cap, nsel, hidden, n_shared):
    """Byte offsets of the arena's parts (every part 256-byte aligned) and its size."""
    off, out = 0, {}
    for name, nbytes in (("flags", 1024), ("recv_x", world * cap * hidden * 2), ("recv_ids", world * cap * nsel * 4),
                         ("recv_w", world * cap * nsel * 4), ("recv_tok", world * cap * 4),
                         ("ret_y", cap * (nsel + n_shared) * hidden * 2)):
        out[name] = off
        off += _align(nbytes)
    out["total"] = off
    return out


class PeerExpertParallelMoE:
    """The MoE layer, experts sharded over the ranks of a process group, exchange over peer memory.

    Rank r holds experts [r*E/W, (r+1)*E/W) and replicas of the router and the shared expert(s);
    it routes its own tokens (at most `max_tokens` per forward)."""

    def __init__(self, spec: MoeSpec, local_w_gate, local_w_up, local_w_down, s_gate, s_up, s_down, router_w, bias,
                 max_tokens: int, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        sp = self.spec = spec
        W = self.world
        if sp.n_experts % W or W > MAX_RANKS:
            raise ValueError("the experts must divide evenly over at most 32 ranks")
        self.el = sp.n_experts // W
        mb = sp.matrix_bytes
        self.w = [_dev(t, n, torch.uint8, self.el * mb) for t, n in
                  ((local_w_gate, "w_gate"), (local_w_up, "w_up"), (local_w_down, "w_down"))]
        self.s = [None, None, None] if sp.n_shared == 0 else [_dev(t, n, torch.uint8, sp.n_shared * mb) for t, n in
                                                               ((s_gate, "s_gate"), (s_up, "s_up"), (s_down, "s_down"))]
        self.router_w, self.bias = router_w, bias
        self.cap = T = max_tokens
        self._cfg = sp.cfg()
        dev = self.dev = router_w.device
        K, H, I, E = sp.nsel, sp.hidden, sp.inter, sp.n_experts
        L = _lib.load()
        # source side
        self.logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.route_ws = torch.empty(_align(L.ck_moe_route_workspace_bytes(ctypes.byref(self._cfg), T)),
                                    dtype=torch.uint8, device=dev)
        self.send_tok = torch.empty(T * min(W, K), dtype=torch.int32, device=dev)
        self.send_meta = torch.empty((T * min(W, K), 2 * K), dtype=torch.int32, device=dev)
        self.sizes = torch.empty((W, 2), dtype=torch.int64, device=dev)
        self.ret_pos = torch.empty(T * K, dtype=torch.int32, device=dev)
        self.counts = torch.empty(E, dtype=torch.int32, device=dev)
        self.iota = torch.arange(T * K, dtype=torch.int32, device=dev)
        self.h_sh = torch.empty((max(1, sp.n_shared) * T, I), dtype=torch.bfloat16, device=dev)
        self.sh_tiles = torch.empty((T // FEW_TOKENS + 2, 4), dtype=torch.int32, device=dev)
        self.sh_ntiles = torch.empty(1, dtype=torch.int32, device=dev)
        # receiver side: all world * cap rows, the unused ones carrying expert -1
        R = W * T
        P = R * K
        self.rows = R
        self.xp2 = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
        self.row_w2 = torch.empty(P, dtype=torch.float32, device=dev)
        self.pair_pos2 = torch.empty(P, dtype=torch.int32, device=dev)
        self.counts2 = torch.empty(self.el, dtype=torch.int32, device=dev)
        self.mt2 = L.ck_moe_max_tiles(R, K, self.el, 0)
        self.tiles2 = torch.empty((self.mt2, 4), dtype=torch.int32, device=dev)
        self.ntiles2 = torch.empty(1, dtype=torch.int32, device=dev)
        self.perm_ws2 = torch.empty(_align(L.ck_moe_permute_workspace_bytes(R, K, self.el)), dtype=torch.uint8,
                                    device=dev)
        self.h2 = torch.empty((P, I), dtype=torch.bfloat16, device=dev)
        self.bound = min(R, FEW_TOKENS) if R <= DECODE_TOKENS else 0
        if self.bound:
            # decode-sized receives: the few-token matvec writes y2, a return kernel sends its rows
            self.y2 = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
        else:
            # the grouped GEMM's epilogue stores each row in its source's return buffer itself
            self.row_dst = torch.empty(P, dtype=torch.int64, device=dev)
        self.side = torch.cuda.Stream(device=dev)
        # the arena, mapped by every peer
        self.lay = arena_layout(W, T, K, H, sp.n_shared)
        base = ctypes.c_void_p()
        _lib.check(L.ck_ep_arena_alloc(self.lay["total"], ctypes.byref(base)), "ck_ep_arena_alloc")
        self.base = base.value
        handle = ctypes.create_string_buffer(64)
        _lib.check(L.ck_ipc_get_handle(ctypes.c_void_p(self.base), handle), "ck_ipc_get_handle")
        handles = [None] * W
        dist.all_gather_object(handles, handle.raw, group=group)
        self.peer_base = []
        for d in range(W):
            if d == self.rank:
                self.peer_base.append(self.base)
                continue
            p = ctypes.c_void_p()
            _lib.check(L.ck_ipc_open_handle(ctypes.create_string_buffer(handles[d], 64), ctypes.byref(p)),
                       f"ck_ipc_open_handle (rank {d})")
            self.peer_base.append(p.value)
        lay, me = self.lay, self.rank
        pe = self.peers = EpPeers()
        pe.world, pe.rank, pe.cap, pe.nsel, pe.hidden = W, me, T, K, H
        for d in range(W):
            b = self.peer_base[d]
            pe.recv_x[d] = b + lay["recv_x"] + me * T * H * 2
            pe.recv_ids[d] = b + lay["recv_ids"] + me * T * K * 4
            pe.recv_w[d] = b + lay["recv_w"] + me * T * K * 4
            pe.recv_tok[d] = b + lay["recv_tok"] + me * T * 4
            pe.ret_y[d] = b + lay["ret_y"]
            pe.dflag[d] = b + lay["flags"] + 8 * me
            pe.rflag[d] = b + lay["flags"] + 256 + 8 * me
        pe.my_dflags = self.base + lay["flags"]
        pe.my_rflags = self.base + lay["flags"] + 256
        pe.ctr = self.base + lay["flags"] + 512
        pe.err = self.base + lay["flags"] + 520
        self.own = {k: ctypes.c_void_p(self.base + lay[k]) for k in ("recv_x", "recv_ids", "recv_w", "recv_tok",
                                                                      "ret_y")}
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)
        self.last_recv_pairs = 0

    def _shared_rows(self, T):
        """The shared expert's output rows of the local tokens, after the T * nsel routed rows."""
        return ctypes.c_void_p(self.base + self.lay["ret_y"] + T * self.spec.nsel * self.spec.hidden * 2)

    def forward(self, x, out=None, marks=None):
        """x bf16 [ntok, hidden] -> (out bf16 [ntok, hidden], ids int32 [ntok, nsel], wts fp32 [ntok, nsel],
        counts int32 [n_experts] of this rank's tokens).  `marks(name)` is called between phases."""
        sp, L = self.spec, _lib.load()
        mark = marks or (lambda name: None)
        T, H, I, K, E, W = x.shape[0], sp.hidden, sp.inter, sp.nsel, sp.n_experts, self.world
        if T > self.cap:
            raise ValueError("more tokens than the layer was sized for")
        dev, st = x.device, _stream()
        pe = ctypes.byref(self.peers)
        A = T * K
        ids = torch.empty((T, K), dtype=torch.int32, device=dev)
        wts = torch.empty((T, K), dtype=torch.float32, device=dev)
        out = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        mark("start")
        _lib.check(L.ck_ep_peer_begin(pe, st), "ck_ep_peer_begin")
        _lib.check(L.ck_moe_route(ctypes.byref(self._cfg), _ptr(x), T, _ptr(self.router_w), _ptr(self.bias),
                                  _ptr(self.logits), _ptr(ids), _ptr(wts), _ptr(self.route_ws),
                                  self.route_ws.numel(), st), "ck_moe_route")
        mark("route")
        _lib.check(L.ck_ep_dispatch_plan(_ptr(ids), _ptr(wts), T, K, E, W, _ptr(self.counts), _ptr(self.sizes),
                                         _ptr(self.send_tok), _ptr(self.send_meta), _ptr(self.ret_pos), st),
                   "ck_ep_dispatch_plan")
        mark("permute")
        main = torch.cuda.current_stream()
        side_done = None
        if sp.n_shared:
            self.side.wait_stream(main)
            sst = ctypes.c_void_p(self.side.cuda_stream)
            mb = sp.matrix_bytes
            sh_bound = min(T, FEW_TOKENS) if T <= DECODE_TOKENS else 0
            _lib.check(L.ck_token_tiles_n(_ptr(self.sh_tiles), _ptr(self.sh_ntiles), T,
                                          FEW_TOKENS if sh_bound else 192, sst), "ck_token_tiles_n")
            for s in range(sp.n_shared):
                hs = self.h_sh[s * T:(s + 1) * T]
                ys = ctypes.c_void_p(self._shared_rows(T).value + s * T * H * 2)
                _lib.check(L.ck_moe_expert_gemm_bounded(1, ctypes.c_void_p(self.s[0].data_ptr() + s * mb),
                                                         ctypes.c_void_p(self.s[1].data_ptr() + s * mb), None, None, 0,
                                                         1, 0, _ptr(x), T, _ptr(hs), T, None, _ptr(self.sh_tiles),
                                                         _ptr(self.sh_ntiles), self.sh_tiles.shape[0], I, H, 0,
                                                         sh_bound, ctypes.c_void_p(self.peers.err), sst),
                           "shared gate/up")
                _lib.check(L.ck_moe_expert_gemm_bounded(0, ctypes.c_void_p(self.s[2].data_ptr() + s * mb), None, None,
                                                         None, 0, 1, 0, _ptr(hs), T, ys, T, None,
                                                         _ptr(self.sh_tiles), _ptr(self.sh_ntiles),
                                                         self.sh_tiles.shape[0], H, I, 0, sh_bound,
                                                         ctypes.c_void_p(self.peers.err), sst), "shared down")
            side_done = torch.cuda.Event()
            side_done.record(self.side)
        mark("shared")
        _lib.check(L.ck_ep_peer_dispatch(pe, _ptr(x), _ptr(self.send_tok), _ptr(self.send_meta), _ptr(self.sizes), T,
                                         st), "ck_ep_peer_dispatch")
        _lib.check(L.ck_ep_peer_signal(pe, 0, st), "ck_ep_peer_signal")
        _lib.check(L.ck_ep_peer_wait(pe, 0, WAIT_NS, st), "ck_ep_peer_wait")
        mark("dispatch")
        R = self.rows
        _lib.check(L.ck_moe_permute(self.own["recv_ids"], self.own["recv_w"], self.own["recv_x"], R, K, self.el, 0,
                                    H, int(sp.mode == 4), _ptr(self.xp2), _ptr(self.row_w2), _ptr(self.pair_pos2),
                                    _ptr(self.counts2), _ptr(self.tiles2), _ptr(self.ntiles2), _ptr(self.perm_ws2),
                                    st), "regroup")
        if not self.bound:
            _lib.check(L.ck_ep_peer_return_rows(pe, _ptr(self.pair_pos2), self.own["recv_ids"], self.own["recv_tok"],
                                                _ptr(self.row_dst), st), "ck_ep_peer_return_rows")
        mark("regroup")
        err = ctypes.c_void_p(self.peers.err)
        _lib.check(L.ck_moe_expert_gemm_bounded(1, _ptr(self.w[0]), _ptr(self.w[1]), None, None, sp.matrix_bytes,
                                                 self.el, 0, _ptr(self.xp2), R * K, _ptr(self.h2), R * K,
                                                 _ptr(self.row_w2), _ptr(self.tiles2), _ptr(self.ntiles2), self.mt2, I,
                                                 H, 0, self.bound, err, st), "expert gate/up")
        mark("gate_up")
        if self.bound:
            _lib.check(L.ck_moe_expert_gemm_bounded(0, _ptr(self.w[2]), None, None, None, sp.matrix_bytes, self.el,
                                                     0, _ptr(self.h2), R * K, _ptr(self.y2), R * K, None,
                                                     _ptr(self.tiles2), _ptr(self.ntiles2), self.mt2, H, I, 1,
                                                     self.bound, err, st), "expert down")
            mark("down")
            mark("experts")
            _lib.check(L.ck_ep_peer_return(pe, _ptr(self.y2), _ptr(self.pair_pos2), self.own["recv_ids"],
                                           self.own["recv_tok"], st), "ck_ep_peer_return")
        else:
            # down projection and return in one kernel: each output row goes over NVLink to its source
            _lib.check(L.ck_moe_expert_gemm_rows(_ptr(self.w[2]), sp.matrix_bytes, self.el, _ptr(self.h2), R * K,
                                                  _ptr(self.row_dst), R * K, _ptr(self.tiles2), _ptr(self.ntiles2),
                                                  self.mt2, H, I, 1, err, st), "expert down + return")
            mark("down")
            mark("experts")
        _lib.check(L.ck_ep_peer_signal(pe, 1, st), "ck_ep_peer_signal")
        _lib.check(L.ck_ep_peer_wait(pe, 1, WAIT_NS, st), "ck_ep_peer_wait")
        mark("return")
        if side_done is not None:
            main.wait_event(side_done)
        _lib.check(L.ck_moe_combine(self.own["ret_y"], _ptr(ids), _ptr(wts), _ptr(self.iota), T, K, sp.n_shared, H,
                                    int(sp.mode == 3), _ptr(out), None, st), "combine")
        mark("combine")
        return out, ids, wts, self.counts

    __call__ = forward

    def check(self):
        """Synchronize and raise if a device-side wait of the last forward gave up."""
        _lib.check(_lib.load().ck_ep_peer_status(ctypes.byref(self.peers), _stream()), "ck_ep_peer_status")

    def recv_pairs(self) -> int:
        """(row, slot) pairs the last forward computed on this rank (synchronizes)."""
        return int(self.counts2.sum().item())

    def close(self):
        L = _lib.load()
        torch.cuda.synchronize(self.dev)
        for d, p in enumerate(getattr(self, "peer_base", [])):
            if d != self.rank and p:
                L.ck_ipc_close(ctypes.c_void_p(p))
        if getattr(self, "base", None):
            L.ck_ep_arena_free(ctypes.c_void_p(self.base))
            self.base = None

