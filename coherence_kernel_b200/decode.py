"""A device-resident decode step: RMSNorm -> Q/K/V/O projections -> RMSNorm -> MoE layer, with the
residual adds, issued as one stream of kernels and replayable as one CUDA graph (the C ABI
ck_decode_step_* in include/ck_b200.h).

The reference's decode token spends most of its time in the joins between operations (about 400
host dispatches per forward, receipts/2026-07-22-ship-the-slot-map.md:135-145); here a captured
step is a single graph launch per token batch.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .moe import MoeSpec
from .ops import _dev, _ptr, _stream, q4k_nbytes


class DecodeStep:
    """One block's decode step with its weights resident in HBM.

    h fp32 [ntok, hidden] is updated in place; q, k, v fp32 [ntok, hidden] are written (the rows a
    KV cache keeps).  ``run`` issues every kernel; ``capture`` records one run over fixed buffers
    into a CUDA graph and ``replay`` relaunches it."""

    def __init__(self, spec: MoeSpec, wq, wk, wv, wo, g_attn, g_ffn, w_gate, w_up, w_down, s_gate, s_up, s_down,
                 router_w, bias, max_tokens: int, eps: float = 1e-6):
        H = spec.hidden
        self.spec, self.max_tokens = spec, max_tokens
        mb, E, S = spec.matrix_bytes, spec.n_experts, spec.n_shared
        self.dense = [_dev(w, n, torch.uint8, q4k_nbytes(H * H)) for w, n in ((wq, "wq"), (wk, "wk"), (wv, "wv"),
                                                                              (wo, "wo"))]
        self.g = [_dev(g_attn, "g_attn", torch.float32, H), _dev(g_ffn, "g_ffn", torch.float32, H)]
        self.moe = [_dev(w_gate, "w_gate", torch.uint8, E * mb), _dev(w_up, "w_up", torch.uint8, E * mb),
                    _dev(w_down, "w_down", torch.uint8, E * mb)]
        self.shared = [None] * 3 if S == 0 else [_dev(t, n, torch.uint8, S * mb) for t, n in
                                                 ((s_gate, "s_gate"), (s_up, "s_up"), (s_down, "s_down"))]
        self.router_w = _dev(router_w, "router_w", torch.float32, E * H)
        self.bias = None if bias is None else _dev(bias, "bias", torch.float32, E)
        self._cfg = _lib.DecodeConfig(H, max_tokens, eps, spec.cfg())
        L = _lib.load()
        self.ws_bytes = L.ck_decode_step_workspace_bytes(ctypes.byref(self._cfg))
        if self.ws_bytes == 0:
            raise ValueError(f"unsupported decode-step configuration (hidden {H}, {spec})")
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=w_gate.device)
        self._h = L.ck_decode_step_create(ctypes.byref(self._cfg), *[_ptr(t) for t in self.dense], _ptr(self.g[0]),
                                          _ptr(self.g[1]), *[_ptr(t) for t in self.moe],
                                          *[_ptr(t) for t in self.shared], _ptr(self.router_w), _ptr(self.bias),
                                          _ptr(self.ws), self.ws_bytes)
        if not self._h:
            raise ValueError("ck_decode_step_create refused the configuration or weights")

    def _check(self, h, q, k, v):
        ntok = h.shape[0]
        for t, n in ((h, "h"), (q, "q"), (k, "k"), (v, "v")):
            _dev(t, n, torch.float32, ntok * self.spec.hidden)
        if ntok > self.max_tokens:
            raise ValueError("more tokens than the step was sized for")
        return ntok

    def run(self, h, q, k, v):
        ntok = self._check(h, q, k, v)
        _lib.check(_lib.load().ck_decode_step_run(self._h, _ptr(h), _ptr(q), _ptr(k), _ptr(v), ntok, _stream()),
                   "ck_decode_step_run")

    def capture(self, h, q, k, v):
        """Record one run over these buffers into a CUDA graph on the current (non-default) stream."""
        ntok = self._check(h, q, k, v)
        _lib.check(_lib.load().ck_decode_step_capture(self._h, _ptr(h), _ptr(q), _ptr(k), _ptr(v), ntok, _stream()),
                   "ck_decode_step_capture")

    def replay(self):
        _lib.check(_lib.load().ck_decode_step_replay(self._h, _stream()), "ck_decode_step_replay")

    def status(self, ntok):
        _lib.check(_lib.load().ck_decode_step_status(self._h, ntok, _stream()), "ck_decode_step_status")

    def views(self, ntok):
        """The step's intermediates in its workspace: a (normed attention input, fp32), o (Wo v,
        fp32), b (normed MoE input, bf16), m (MoE output, bf16), ids / wts (the routing)."""
        H, K, T = self.spec.hidden, self.spec.nsel, self.max_tokens
        al = lambda n: (n + 255) // 256 * 256
        off, out = 0, {}
        for name, nb, dt, shape in (("a", T * H * 4, torch.float32, (T, H)), ("o", T * H * 4, torch.float32, (T, H)),
                                    ("b", T * H * 2, torch.bfloat16, (T, H)), ("m", T * H * 2, torch.bfloat16, (T, H)),
                                    ("ids", T * K * 4, torch.int32, (T, K)), ("wts", T * K * 4, torch.float32, (T, K))):
            out[name] = self.ws[off:off + nb].view(dt).view(shape)[:ntok]
            off += al(nb)
        return out

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.load().ck_decode_step_destroy(h)
            self._h = None
