"""ctypes face of the oracle (libckoracle.so, built from cpu_ref.c).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
it as the checker.  Nothing in the product imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_c_i64 = ctypes.c_int64
_p = ctypes.c_void_p


class MoeCfg(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int64), ("inter", ctypes.c_int64), ("n_experts", ctypes.c_int32),
                ("n_shared", ctypes.c_int32), ("nsel", ctypes.c_int32), ("mode", ctypes.c_int32),
                ("ngroups", ctypes.c_int32), ("topk_groups", ctypes.c_int32), ("wscale", ctypes.c_double)]


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE, "libckoracle.so"], check=True)
    return os.path.join(_HERE, "libckoracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libckoracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.ckr_f16.restype = ctypes.c_double
        L.ckr_f16.argtypes = [ctypes.c_uint32]
        L.ckr_bf16.restype = ctypes.c_double
        L.ckr_bf16.argtypes = [ctypes.c_uint32]
        for n in ("ckr_q80_at", "ckr_q4k_at", "ckr_q6k_at"):
            getattr(L, n).restype = ctypes.c_double
            getattr(L, n).argtypes = [_p, _c_i64, _c_i64]
        for n in ("ckr_q4k_codes", "ckr_q6k_codes"):
            getattr(L, n).restype = ctypes.c_uint32
            getattr(L, n).argtypes = [_p, _c_i64, _c_i64]
        for n in ("ckr_q80_dequant", "ckr_q4k_dequant", "ckr_q6k_dequant"):
            getattr(L, n).restype = None
            getattr(L, n).argtypes = [_p, _c_i64, _c_i64, _p]
        L.ckr_dot.restype = ctypes.c_double
        L.ckr_dot.argtypes = [_p, _p, _c_i64]
        for n in ("ckr_q80_matvec", "ckr_q4k_matvec", "ckr_q6k_matvec"):
            getattr(L, n).restype = None
            getattr(L, n).argtypes = [_p, _p, _p, _c_i64, _c_i64]
        L.ckr_q4k_matmul.restype = None
        L.ckr_q4k_matmul.argtypes = [_p, _p, _p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int]
        for n in ("ckr_exp", "ckr_sqrt", "ckr_ln", "ckr_sigmoid", "ckr_silu"):
            getattr(L, n).restype = ctypes.c_double
            getattr(L, n).argtypes = [ctypes.c_double]
        L.ckr_rmsnorm.restype = None
        L.ckr_rmsnorm.argtypes = [_p, _p, _c_i64, ctypes.c_double, _p]
        L.ckr_route_softmax.restype = None
        L.ckr_route_softmax.argtypes = [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p, _p]
        L.ckr_route_dsv4.restype = None
        L.ckr_route_dsv4.argtypes = [_p, _p, ctypes.c_int, ctypes.c_int, ctypes.c_double, _p, _p]
        L.ckr_route_sigmoid_group.restype = None
        L.ckr_route_sigmoid_group.argtypes = [_p, _p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_double, _p, _p, _p]
        L.ckr_moe_layer.restype = ctypes.c_int
        L.ckr_moe_layer.argtypes = [ctypes.POINTER(MoeCfg), _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                    _c_i64, _p, _p, _p, ctypes.c_int]
        L.ckr_moe_route.restype = ctypes.c_int
        L.ckr_moe_route.argtypes = [ctypes.POINTER(MoeCfg), _p, _p, _p, _c_i64, _p, _p, _p, ctypes.c_int]
        _LIB = L
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data


def q80_dequant(qb: np.ndarray, off: int, n: int) -> np.ndarray:
    w = np.empty(n, dtype=np.float64)
    lib().ckr_q80_dequant(_ptr(qb), off, n, _ptr(w))
    return w


def q4k_dequant(qb: np.ndarray, off: int, n: int) -> np.ndarray:
    w = np.empty(n, dtype=np.float64)
    lib().ckr_q4k_dequant(_ptr(qb), off, n, _ptr(w))
    return w


def q4k_at(qb: np.ndarray, idx: int) -> float:
    return lib().ckr_q4k_at(_ptr(qb), 0, idx)


def q4k_codes(qb: np.ndarray, idx: int):
    c = lib().ckr_q4k_codes(_ptr(qb), 0, idx)
    return c & 0xFF, (c >> 8) & 0xFF, c >> 16


def q6k_dequant(qb: np.ndarray, off: int, n: int) -> np.ndarray:
    w = np.empty(n, dtype=np.float64)
    lib().ckr_q6k_dequant(_ptr(qb), off, n, _ptr(w))
    return w


def q6k_codes(qb: np.ndarray, idx: int):
    """(q + 32, signed scale) of the weight at a flat index"""
    c = lib().ckr_q6k_codes(_ptr(qb), 0, idx)
    sc = (c >> 8) & 0xFF
    return c & 0xFF, sc - 256 if sc >= 128 else sc


def q6k_matvec(qb, x, rows, cols):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty(rows, dtype=np.float64)
    lib().ckr_q6k_matvec(_ptr(qb), _ptr(x), _ptr(y), rows, cols)
    return y


def rmsnorm(x, g, eps):
    x = np.ascontiguousarray(x, dtype=np.float64)
    g = np.ascontiguousarray(g, dtype=np.float64)
    out = np.empty_like(x)
    lib().ckr_rmsnorm(_ptr(x), _ptr(g), x.size, eps, _ptr(out))
    return out


def dot_rows(a, b):
    """out[i, k] = tb-dot's right fold of a[i] with b[k] (fp64 rows of equal length)."""
    a = np.ascontiguousarray(a, dtype=np.float64)
    b = np.ascontiguousarray(b, dtype=np.float64)
    out = np.empty((a.shape[0], b.shape[0]), dtype=np.float64)
    n, L = a.shape[1], lib()
    pa, pb = a.ctypes.data, b.ctypes.data
    for i in range(a.shape[0]):
        for k in range(b.shape[0]):
            out[i, k] = L.ckr_dot(ctypes.c_void_p(pa + 8 * n * i), ctypes.c_void_p(pb + 8 * n * k), n)
    return out


def q80_matvec(qb, x, rows, cols):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty(rows, dtype=np.float64)
    lib().ckr_q80_matvec(_ptr(qb), _ptr(x), _ptr(y), rows, cols)
    return y


def q4k_matvec(qb, x, rows, cols):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty(rows, dtype=np.float64)
    lib().ckr_q4k_matvec(_ptr(qb), _ptr(x), _ptr(y), rows, cols)
    return y


def q4k_matmul(qb, x, rows, cols, r0=0, r1=None, nthreads=None):
    """x [ntok, cols] (float64) -> y [ntok, rows]; only rows [r0, r1) are computed (others 0)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    ntok = x.shape[0]
    r1 = rows if r1 is None else r1
    y = np.zeros((ntok, rows), dtype=np.float64)
    lib().ckr_q4k_matmul(_ptr(qb), _ptr(x), _ptr(y), rows, cols, ntok, r0, r1,
                         nthreads or (os.cpu_count() or 1))
    return y


def route_softmax(logits, nsel, renorm):
    logits = np.ascontiguousarray(logits, dtype=np.float64)
    ids = np.empty(nsel, dtype=np.int32)
    wts = np.empty(nsel, dtype=np.float64)
    lib().ckr_route_softmax(_ptr(logits), logits.size, nsel, int(renorm), _ptr(ids), _ptr(wts), None)
    return ids, wts


def route_dsv4(logits, bias, nused, wscale):
    logits = np.ascontiguousarray(logits, dtype=np.float64)
    bias = np.ascontiguousarray(bias, dtype=np.float64)
    ids = np.empty(nused, dtype=np.int32)
    wts = np.empty(nused, dtype=np.float64)
    lib().ckr_route_dsv4(_ptr(logits), _ptr(bias), logits.size, nused, wscale, _ptr(ids), _ptr(wts))
    return ids, wts


def route_sigmoid_group(logits, bias, ngroups, topk_groups, nused, wscale):
    logits = np.ascontiguousarray(logits, dtype=np.float64)
    bias = np.ascontiguousarray(bias, dtype=np.float64)
    ids = np.empty(nused, dtype=np.int32)
    wts = np.empty(nused, dtype=np.float64)
    mg = np.zeros(1, dtype=np.float64)
    lib().ckr_route_sigmoid_group(_ptr(logits), _ptr(bias), logits.size, ngroups, topk_groups, nused,
                                  wscale, _ptr(ids), _ptr(wts), _ptr(mg))
    return ids, wts, float(mg[0])


def moe_cfg(hidden, inter, n_experts, n_shared, nsel, mode, ngroups=1, topk_groups=1, wscale=1.0):
    return MoeCfg(hidden, inter, n_experts, n_shared, nsel, mode, ngroups, topk_groups, wscale)


def moe_layer(cfg: MoeCfg, w, x_bf16, tokens, nthreads=None):
    """w: dict of uint8 arrays gate/up/down (experts concatenated) and s_gate/s_up/s_down (shared),
    float32 'router' [ne, hidden] and optional 'bias'. Returns (ids, wts, out) for the tokens."""
    tok = np.ascontiguousarray(tokens, dtype=np.int64)
    n = tok.size
    ids = np.empty((n, cfg.nsel), dtype=np.int32)
    wts = np.empty((n, cfg.nsel), dtype=np.float64)
    out = np.empty((n, cfg.hidden), dtype=np.float64)
    rc = lib().ckr_moe_layer(ctypes.byref(cfg), _ptr(w["gate"]), _ptr(w["up"]), _ptr(w["down"]),
                             _ptr(w.get("s_gate")), _ptr(w.get("s_up")), _ptr(w.get("s_down")),
                             _ptr(w["router"]), _ptr(w.get("bias")), _ptr(x_bf16), _ptr(tok), n,
                             _ptr(ids), _ptr(wts), _ptr(out), nthreads or (os.cpu_count() or 1))
    assert rc == 0, "oracle refused the MoE configuration"
    return ids, wts, out


def moe_route(cfg: MoeCfg, router, bias, x_bf16, nthreads=None):
    ntok = x_bf16.shape[0]
    ids = np.empty((ntok, cfg.nsel), dtype=np.int32)
    wts = np.empty((ntok, cfg.nsel), dtype=np.float64)
    mg = np.empty(ntok, dtype=np.float64)
    rc = lib().ckr_moe_route(ctypes.byref(cfg), _ptr(router), _ptr(bias), _ptr(x_bf16), ntok,
                             _ptr(ids), _ptr(wts), _ptr(mg), nthreads or (os.cpu_count() or 1))
    assert rc == 0, "oracle refused the router configuration"
    return ids, wts, mg
