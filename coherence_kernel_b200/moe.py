"""The batched MoE layer on B200: single GPU and expert-parallel over the GPUs of one box.

The reference runs an MoE FFN one token at a time (form/form-stdlib/dsv4-forward.fk:105-115,
moe-gate.fk:32-40, form/native/metal/moe-token.fk): route, bind the chosen experts' weights at
``t.off + e*nb02``, run three quantized matvecs per expert, combine.  Here a whole batch is routed
at once, the (token, slot) pairs are sorted by expert, each expert's rows run through one grouped
tensor-core GEMM, and the combine restores the reference's per-token summation order.

Two combine conventions, both the reference's:
  mode 3  softmax router, top-k, no renormalization; moe-mix order (ascending expert, acc + g*y)
  mode 4  sigmoid + bias, group-limited top-k, renormalized x wscale, weight inside the expert
          (dsv4-mid), dsv4-moe-acc order (selection list), then the shared expert.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .ops import _dev, _ptr, _stream, q4k_nbytes

# CK_MOE_FEW_TOKENS / CK_MOE_DECODE_TOKENS of ck_b200.h: batches up to DECODE_TOKENS tokens are
# permuted into tiles of at most FEW_TOKENS tokens and run the expert projections as the few-token
# grouped matvec
FEW_TOKENS = 5
DECODE_TOKENS = 128


@dataclass
class MoeSpec:
    hidden: int
    inter: int
    n_experts: int
    n_shared: int
    nsel: int
    mode: int            # 3 or 4
    ngroups: int = 1
    topk_groups: int = 1
    wscale: float = 1.0
    tau: float = 5e-5    # decision margin below which a token is re-routed in fp64

    def cfg(self) -> _lib.MoeConfig:
        return _lib.MoeConfig(self.hidden, self.inter, self.n_experts, self.n_shared, self.nsel, self.mode,
                              self.ngroups, self.topk_groups, self.wscale, self.tau)

    @property
    def matrix_bytes(self) -> int:
        return q4k_nbytes(self.inter * self.hidden)

    def flops_per_token(self) -> int:
        """Algorithmic FLOPs of one token: router + (nsel routed + n_shared) SwiGLU experts."""
        expert = 2 * 3 * self.hidden * self.inter
        return 2 * self.hidden * self.n_experts + (self.nsel + self.n_shared) * expert


class MoELayer:
    """One MoE layer with its weights resident in HBM (single GPU)."""

    def __init__(self, spec: MoeSpec, w_gate, w_up, w_down, s_gate, s_up, s_down, router_w, bias, max_tokens: int):
        self.spec = spec
        mb = spec.matrix_bytes
        E, S = spec.n_experts, spec.n_shared
        self.w = [_dev(w_gate, "w_gate", torch.uint8, E * mb), _dev(w_up, "w_up", torch.uint8, E * mb),
                  _dev(w_down, "w_down", torch.uint8, E * mb)]
        self.s = [None, None, None] if S == 0 else [_dev(s_gate, "s_gate", torch.uint8, S * mb),
                                                     _dev(s_up, "s_up", torch.uint8, S * mb),
                                                     _dev(s_down, "s_down", torch.uint8, S * mb)]
        self.router_w = _dev(router_w, "router_w", torch.float32, E * spec.hidden)
        self.bias = None if bias is None else _dev(bias, "bias", torch.float32, E)
        self.max_tokens = max_tokens
        self._cfg = spec.cfg()
        L = _lib.load()
        self.ws_bytes = L.ck_moe_workspace_bytes(ctypes.byref(self._cfg), max_tokens)
        if self.ws_bytes == 0:
            raise ValueError(f"unsupported MoE configuration {spec}")
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=w_gate.device)

    def forward(self, x, out=None, ids=None, wts=None, counts=None):
        """x bf16 [ntok, hidden] -> (out bf16 [ntok, hidden], ids int32 [ntok, nsel],
        wts fp32 [ntok, nsel], counts int32 [n_experts])."""
        sp = self.spec
        ntok = x.shape[0]
        if ntok > self.max_tokens:
            raise ValueError("more tokens than the layer's workspace was sized for")
        _dev(x, "x", (torch.bfloat16, torch.uint16, torch.int16), ntok * sp.hidden)
        dev = x.device
        out = out if out is not None else torch.empty((ntok, sp.hidden), dtype=torch.bfloat16, device=dev)
        ids = ids if ids is not None else torch.empty((ntok, sp.nsel), dtype=torch.int32, device=dev)
        wts = wts if wts is not None else torch.empty((ntok, sp.nsel), dtype=torch.float32, device=dev)
        counts = counts if counts is not None else torch.empty(sp.n_experts, dtype=torch.int32, device=dev)
        L = _lib.load()
        rc = L.ck_moe_layer_bf16(ctypes.byref(self._cfg), _ptr(x), ntok, _ptr(self.w[0]), _ptr(self.w[1]),
                                 _ptr(self.w[2]), _ptr(self.s[0]), _ptr(self.s[1]), _ptr(self.s[2]),
                                 _ptr(self.router_w), _ptr(self.bias), _ptr(ids), _ptr(wts), _ptr(counts), _ptr(out),
                                 _ptr(self.ws), self.ws_bytes, _stream())
        _lib.check(rc, "ck_moe_layer_bf16")
        return out, ids, wts, counts

    __call__ = forward

    def forward_steps(self, x, out, ids, wts, counts, marks=None):
        """The same layer as `forward`, issued step by step through the C ABI (route, permute,
        gate/up GEMM, down GEMM, combine) -- the sequence ck_moe_layer_bf16 runs internally.
        `marks(name)` is called between steps (the benchmark records CUDA events there)."""
        sp, L, st = self.spec, _lib.load(), _stream()
        T, H, I, K, E = x.shape[0], sp.hidden, sp.inter, sp.nsel, sp.n_experts
        A, R = T * K, T * K + sp.n_shared * T
        w = self._ws_views(T)
        mark = marks or (lambda name: None)
        cfg = ctypes.byref(self._cfg)
        w["err"].zero_()
        mark("start")
        _lib.check(L.ck_moe_route(cfg, _ptr(x), T, _ptr(self.router_w), _ptr(self.bias), _ptr(w["logits"]), _ptr(ids),
                                  _ptr(wts), _ptr(w["route"]), w["route"].numel(), st), "route")
        mark("route")
        _lib.check(L.ck_moe_permute(_ptr(ids), _ptr(wts), _ptr(x), T, K, E, sp.n_shared, H, int(sp.mode == 4),
                                    _ptr(w["xp"]), _ptr(w["row_w"]), _ptr(w["pair_pos"]), _ptr(counts), _ptr(w["tiles"]),
                                    _ptr(w["ntiles"]), _ptr(w["perm_ws"]), st), "permute")
        mark("permute")
        mb = sp.matrix_bytes
        bound = min(T, FEW_TOKENS) if T <= DECODE_TOKENS else 0  # the most tokens any tile holds
        _lib.check(L.ck_moe_expert_gemm_bounded(1, _ptr(self.w[0]), _ptr(self.w[1]), _ptr(self.s[0]), _ptr(self.s[1]),
                                                 mb, E, sp.n_shared, _ptr(w["xp"]), A + T, _ptr(w["h"]), R,
                                                 _ptr(w["row_w"]), _ptr(w["tiles"]), _ptr(w["ntiles"]), w["mt"], I, H, 0,
                                                 bound, _ptr(w["err"]), st), "gate/up")
        mark("gate_up")
        _lib.check(L.ck_moe_expert_gemm_bounded(0, _ptr(self.w[2]), None, _ptr(self.s[2]), None, mb, E, sp.n_shared,
                                                 _ptr(w["h"]), R, _ptr(w["y"]), R, None, _ptr(w["tiles"]),
                                                 _ptr(w["ntiles"]), w["mt"], H, I, 1, bound, _ptr(w["err"]), st), "down")
        mark("down")
        _lib.check(L.ck_moe_combine(_ptr(w["y"]), _ptr(ids), _ptr(wts), _ptr(w["pair_pos"]), T, K, sp.n_shared, H,
                                    int(sp.mode == 3), _ptr(out), None, st), "combine")
        mark("combine")
        return out, ids, wts, counts

    def _ws_views(self, T):
        """Views of the workspace laid out as ck_moe_layer_bf16 lays it out (api.cu moe_ws)."""
        sp, L = self.spec, _lib.load()
        K, H, I, E = sp.nsel, sp.hidden, sp.inter, sp.n_experts
        A, XR, R = T * K, T * K + T, T * K + sp.n_shared * T
        mt = L.ck_moe_max_tiles(T, K, E, sp.n_shared)
        off = 0
        views = {}

        def take(name, nbytes, dtype, shape):
            nonlocal off
            views[name] = self.ws[off:off + nbytes].view(dtype).view(shape)
            off += _align(nbytes)

        take("logits", T * E * 4, torch.float32, (T, E))
        rw = L.ck_moe_route_workspace_bytes(ctypes.byref(self._cfg), T)
        views["route"] = self.ws[off:off + rw]
        off += _align(rw)
        pw = L.ck_moe_permute_workspace_bytes(T, K, E)
        views["perm_ws"] = self.ws[off:off + pw]
        off += _align(pw)
        take("xp", XR * H * 2, torch.bfloat16, (XR, H))
        take("row_w", R * 4, torch.float32, (R,))
        take("pair_pos", A * 4, torch.int32, (A,))
        take("tiles", mt * 16, torch.int32, (mt, 4))
        take("ntiles", 4, torch.int32, (1,))
        take("h", R * I * 2, torch.bfloat16, (R, I))
        take("y", R * H * 2, torch.bfloat16, (R, H))
        take("err", 4, torch.int32, (1,))
        views["mt"] = mt
        return views

    def flagged(self, ntok) -> int:
        """Tokens the last layer re-routed in fp64 (synchronizes)."""
        w = self._ws_views(ntok)
        return _lib.load().ck_moe_route_flagged(ctypes.byref(self._cfg), ntok, _ptr(w["route"]), _stream())

    def status(self, ntok):
        """Synchronize and raise if a device-side wait of the last layer gave up."""
        _lib.check(_lib.load().ck_moe_layer_status(ctypes.byref(self._cfg), ntok, _ptr(self.ws), _stream()),
                   "ck_moe_layer_status")


def _align(n, a=256):
    return (n + a - 1) // a * a


def ep_dispatch_counts(ids, el, world):
    """The sizes of the deduplicated dispatch.  A token crosses to each rank that holds at least one
    of its experts once, however many of them live there.  Returns (destination rank of every slot
    [T, K], the token/rank incidence [T, W] bool, rows per destination rank [W], (token, slot)
    pairs per destination rank [W])."""
    er = torch.div(ids, el, rounding_mode="floor").long()
    mask = torch.zeros((ids.shape[0], world), dtype=torch.bool, device=ids.device)
    mask.scatter_(1, er, True)
    return er, mask, mask.sum(0), torch.bincount(er.reshape(-1), minlength=world)


def ep_dispatch_rows(ids, wts, er, mask, el, nrows):
    """The rows of the deduplicated dispatch, in (destination rank, token) order: the source token
    of every row [S] int32, the local expert of each of its slots [S, K] int32 (-1 where the slot's
    expert lives on another rank) and the slots' route weights [S, K] (0 there).  `nrows` is the
    row total, known on the host from the size exchange, so no step waits for the device."""
    dt = torch.nonzero_static(mask.t(), size=nrows)
    d, t = dt[:, 0], dt[:, 1]
    sel = er[t] == d.unsqueeze(1)
    me = torch.where(sel, ids[t].long() - (d * el).unsqueeze(1), torch.full_like(er[t], -1)).to(torch.int32)
    mw = torch.where(sel, wts[t], torch.zeros_like(wts[t]))
    return t.to(torch.int32), me, mw


def ep_return_positions(ids, el):
    """Where the return all-to-all leaves every (token, slot) pair's output row: the pairs sent to
    rank d come back as one block, in (token, slot) order, and the blocks arrive in rank order --
    the pairs' order after a stable sort by destination rank, so the position of a pair is its
    index in that sort."""
    er = torch.div(ids, el, rounding_mode="floor").reshape(-1)
    order = torch.argsort(er, stable=True)
    pos = torch.empty_like(order)
    pos[order] = torch.arange(order.numel(), device=ids.device)
    return pos.to(torch.int32)


class ExpertParallelMoE:
    """The MoE layer with experts sharded over the ranks of a process group (one GPU per rank).

    Rank r holds experts [r*E/W, (r+1)*E/W) and a replica of the router and the shared expert(s).
    Each rank routes its own tokens and sends every token once to each rank that holds at least
    one of its experts (with group-limited routing a token reaches at most topk_groups ranks),
    together with a small row naming the slots' local experts and weights; one all-to-all of the
    activation rows and one of the metadata (NCCL over NVLink).  The receiver regroups the
    (row, slot) pairs by local expert, runs the grouped GEMMs and returns every pair's output row,
    in (row, slot) order, with a second all-to-all; the source combines them in the reference's
    order, so the output equals the single-GPU layer's bit for bit.  The shared expert runs on
    the local tokens on a side stream, beside the exchange.
    """

    def __init__(self, spec: MoeSpec, local_w_gate, local_w_up, local_w_down, s_gate, s_up, s_down, router_w, bias,
                 max_tokens: int, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        sp = self.spec = spec
        if sp.n_experts % self.world:
            raise ValueError("the experts must divide evenly over the ranks")
        self.el = sp.n_experts // self.world
        mb = sp.matrix_bytes
        self.w = [_dev(t, n, torch.uint8, self.el * mb) for t, n in
                  ((local_w_gate, "w_gate"), (local_w_up, "w_up"), (local_w_down, "w_down"))]
        self.s = [None, None, None] if sp.n_shared == 0 else [_dev(t, n, torch.uint8, sp.n_shared * mb) for t, n in
                                                               ((s_gate, "s_gate"), (s_up, "s_up"), (s_down, "s_down"))]
        self.router_w = router_w
        self.bias = bias
        self.max_tokens = max_tokens
        self._cfg = sp.cfg()
        dev = router_w.device
        T, K, H, I, E, W = max_tokens, sp.nsel, sp.hidden, sp.inter, sp.n_experts, self.world
        A = T * K
        L = _lib.load()
        self.dev = dev
        # source side
        self.logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.route_ws = torch.empty(_align(L.ck_moe_route_workspace_bytes(ctypes.byref(self._cfg), T)),
                                    dtype=torch.uint8, device=dev)
        self.send_x = torch.empty((T * min(W, K), H), dtype=torch.bfloat16, device=dev)
        self.send_tok = torch.empty(T * min(W, K), dtype=torch.int32, device=dev)
        self.send_meta = torch.empty((T * min(W, K), 2 * K), dtype=torch.int32, device=dev)
        self.sizes = torch.empty((W, 2), dtype=torch.int64, device=dev)
        self.ret_pos = torch.empty(A, dtype=torch.int32, device=dev)
        self.y = torch.empty((A + sp.n_shared * T, H), dtype=torch.bfloat16, device=dev)
        self.h_sh = torch.empty((max(1, sp.n_shared) * T, I), dtype=torch.bfloat16, device=dev)
        self.sh_tiles = torch.empty((T // FEW_TOKENS + 2, 4), dtype=torch.int32, device=dev)
        self.sh_ntiles = torch.empty(1, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counts = torch.empty(E, dtype=torch.int32, device=dev)
        # receiver side: every rank may send each of its tokens here once
        R = T * W
        self.recv_x = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
        self.recv_meta = torch.empty((R, 2 * K), dtype=torch.int32, device=dev)
        P = R * K
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
        self.y2 = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
        self.y_recv = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
        self.side = torch.cuda.Stream(device=dev)  # the shared expert, beside the exchange
        self.last_recv_rows = 0
        self.last_recv_pairs = 0

    def forward(self, x, out=None, marks=None):
        """`marks(name)` is called between phases (a benchmark records CUDA events there)."""
        sp, L, dist = self.spec, _lib.load(), self.dist
        mark = marks or (lambda name: None)
        T, H, I, K, E, W = x.shape[0], sp.hidden, sp.inter, sp.nsel, sp.n_experts, self.world
        if T > self.max_tokens:
            raise ValueError("more tokens than the layer was sized for")
        A = T * K
        dev = x.device
        st = _stream()
        ids = torch.empty((T, K), dtype=torch.int32, device=dev)
        wts = torch.empty((T, K), dtype=torch.float32, device=dev)
        out = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        self.err.zero_()
        mark("start")
        _lib.check(L.ck_moe_route(ctypes.byref(self._cfg), _ptr(x), T, _ptr(self.router_w), _ptr(self.bias),
                                  _ptr(self.logits), _ptr(ids), _ptr(wts), _ptr(self.route_ws),
                                  self.route_ws.numel(), st), "ck_moe_route")
        mark("route")
        # the plan on the device: pairs per expert, (rows, pairs) per destination rank, the dispatch
        # rows with their metadata, and every pair's row in the return exchange
        _lib.check(L.ck_ep_dispatch_plan(_ptr(ids), _ptr(wts), T, K, E, W, _ptr(self.counts), _ptr(self.sizes),
                                         _ptr(self.send_tok), _ptr(self.send_meta), _ptr(self.ret_pos), st),
                   "ck_ep_dispatch_plan")
        mark("permute")
        # shared expert(s) on the local tokens, into y rows A + s*T .., on a side stream: launched
        # before the host waits for the split sizes, it overlaps the exchange and the expert GEMMs;
        # the combine waits for it
        main = torch.cuda.current_stream()
        side_done = None
        if sp.n_shared:
            self.side.wait_stream(main)
            sst = ctypes.c_void_p(self.side.cuda_stream)
            mb = sp.matrix_bytes
            # a decode-sized batch cuts the shared expert's tokens into tiles of at most FEW_TOKENS,
            # which stream the weights through the few-token grouped matvec
            sh_bound = min(T, FEW_TOKENS) if T <= DECODE_TOKENS else 0
            _lib.check(L.ck_token_tiles_n(_ptr(self.sh_tiles), _ptr(self.sh_ntiles), T,
                                          FEW_TOKENS if sh_bound else 192, sst), "ck_token_tiles_n")
            for s in range(sp.n_shared):
                hs = self.h_sh[s * T:(s + 1) * T]
                ys = self.y[A + s * T:A + (s + 1) * T]
                _lib.check(L.ck_moe_expert_gemm_bounded(1, ctypes.c_void_p(self.s[0].data_ptr() + s * mb),
                                                         ctypes.c_void_p(self.s[1].data_ptr() + s * mb), None, None, 0,
                                                         1, 0, _ptr(x), T, _ptr(hs), T, None, _ptr(self.sh_tiles),
                                                         _ptr(self.sh_ntiles), self.sh_tiles.shape[0], I, H, 0,
                                                         sh_bound, _ptr(self.err), sst), "shared gate/up")
                _lib.check(L.ck_moe_expert_gemm_bounded(0, ctypes.c_void_p(self.s[2].data_ptr() + s * mb), None, None,
                                                         None, 0, 1, 0, _ptr(hs), T, _ptr(ys), T, None,
                                                         _ptr(self.sh_tiles), _ptr(self.sh_ntiles),
                                                         self.sh_tiles.shape[0], H, I, 0, sh_bound, _ptr(self.err),
                                                         sst), "shared down")
            side_done = torch.cuda.Event()
            side_done.record(self.side)
        mark("shared")
        # the sizes: the one point where the host waits for the device
        rsizes = torch.empty_like(self.sizes)
        dist.all_to_all_single(rsizes, self.sizes, group=self.group)  # [src, (rows, pairs)]
        srow_l, spair_l, rrow_l, rpair_l = torch.cat([self.sizes.t(), rsizes.t()]).tolist()
        S, R, P = int(sum(srow_l)), int(sum(rrow_l)), int(sum(rpair_l))
        self.last_recv_rows, self.last_recv_pairs = R, P
        if S:
            _lib.check(L.ck_gather_rows(_ptr(x), _ptr(self.send_tok), _ptr(self.send_x), S, H * 2, st),
                       "dispatch rows")
        dist.all_to_all_single(self.recv_x[:R], self.send_x[:S], output_split_sizes=rrow_l, input_split_sizes=srow_l,
                               group=self.group)
        dist.all_to_all_single(self.recv_meta[:R], self.send_meta[:S], output_split_sizes=rrow_l,
                               input_split_sizes=srow_l, group=self.group)
        mark("dispatch")
        # regroup the received (row, slot) pairs by local expert (a stable counting sort that skips
        # the -1 slots), grouped GEMMs, then every pair's row back in (row, slot) order.  A
        # decode-sized receive (at most DECODE_TOKENS rows) is cut into tiles of at most FEW_TOKENS
        # by the permute, and the expert weights stream through the few-token grouped matvec.
        if P:
            bound = min(R, FEW_TOKENS) if R <= DECODE_TOKENS else 0
            rme = self.recv_meta[:R, :K].contiguous()
            rmw = self.recv_meta[:R, K:].contiguous().view(torch.float32)
            _lib.check(L.ck_moe_permute(_ptr(rme), _ptr(rmw), _ptr(self.recv_x), R, K, self.el, 0, H,
                                        int(sp.mode == 4), _ptr(self.xp2), _ptr(self.row_w2), _ptr(self.pair_pos2),
                                        _ptr(self.counts2), _ptr(self.tiles2), _ptr(self.ntiles2),
                                        _ptr(self.perm_ws2), st), "regroup")
            mark("regroup")
            _lib.check(L.ck_moe_expert_gemm_bounded(1, _ptr(self.w[0]), _ptr(self.w[1]), None, None, sp.matrix_bytes,
                                                     self.el, 0, _ptr(self.xp2), P, _ptr(self.h2), P,
                                                     _ptr(self.row_w2), _ptr(self.tiles2), _ptr(self.ntiles2),
                                                     self.mt2, I, H, 0, bound, _ptr(self.err), st), "expert gate/up")
            mark("gate_up")
            _lib.check(L.ck_moe_expert_gemm_bounded(0, _ptr(self.w[2]), None, None, None, sp.matrix_bytes, self.el,
                                                     0, _ptr(self.h2), P, _ptr(self.y2), P, None, _ptr(self.tiles2),
                                                     _ptr(self.ntiles2), self.mt2, H, I, 1, bound, _ptr(self.err), st),
                       "expert down")
            mark("down")
            pp = self.pair_pos2[:R * K]
            vidx = pp[torch.nonzero_static(pp >= 0, size=P).squeeze(1)]
            _lib.check(L.ck_gather_rows(_ptr(self.y2), _ptr(vidx), _ptr(self.y_recv), P, H * 2, st), "pair order")
        else:
            mark("regroup")
            mark("gate_up")
            mark("down")
        mark("experts")
        dist.all_to_all_single(self.y[:A], self.y_recv[:P], output_split_sizes=spair_l, input_split_sizes=rpair_l,
                               group=self.group)
        mark("return")
        if side_done is not None:
            main.wait_event(side_done)
        _lib.check(L.ck_moe_combine(_ptr(self.y), _ptr(ids), _ptr(wts), _ptr(self.ret_pos), T, K, sp.n_shared, H,
                                    int(sp.mode == 3), _ptr(out), None, st), "combine")
        mark("combine")
        return out, ids, wts, self.counts

    __call__ = forward

    def check(self):
        torch.cuda.current_stream().synchronize()
        if int(self.err.item()):
            raise _lib.CKError(f"a grouped-GEMM device wait timed out (role code {int(self.err.item())})")
