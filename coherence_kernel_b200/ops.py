"""Torch-facing wrappers of the C ABI (include/ck_b200.h).

Tensors are device tensors; each wrapper checks dtype, device, contiguity and size, then calls
the library on torch's current CUDA stream.  Packed GGUF blocks travel as uint8 tensors, bf16
activations as torch.bfloat16 (or their uint16 bit patterns).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

Q8_0_BLOCK_BYTES, Q4K_BLOCK_BYTES = 34, 144


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dev(t, name, dtype=None, numel=None):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype not in (dtype if isinstance(dtype, tuple) else (dtype,)):
        raise ValueError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name} holds {t.numel()} elements, needs {numel}")
    return t


def q8_0_nbytes(n):
    return n // 32 * Q8_0_BLOCK_BYTES


def q4k_nbytes(n):
    return n // 256 * Q4K_BLOCK_BYTES


def q8_0_dequant(qb, off, n):
    _dev(qb, "qb", torch.uint8, q8_0_nbytes(((off + n + 31) // 32) * 32))
    w = torch.empty(n, dtype=torch.float32, device=qb.device)
    _lib.check(_lib.load().ck_q8_0_dequant_f32(_ptr(qb), _ptr(w), off, n, _stream()), "ck_q8_0_dequant_f32")
    return w


def q4k_dequant(qb, off, n, dtype=torch.float32):
    _dev(qb, "qb", torch.uint8, q4k_nbytes(((off + n + 255) // 256) * 256))
    w = torch.empty(n, dtype=dtype, device=qb.device)
    fn = _lib.load().ck_q4k_dequant_f32 if dtype == torch.float32 else _lib.load().ck_q4k_dequant_bf16
    _lib.check(fn(_ptr(qb), _ptr(w), off, n, _stream()), "ck_q4k_dequant")
    return w


def q8_0_matvec(qb, x, rows, cols, out=None):
    _dev(qb, "qb", torch.uint8, q8_0_nbytes(rows * cols))
    _dev(x, "x", torch.float32, cols)
    y = out if out is not None else torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().ck_q8_0_matvec_f32(_ptr(qb), _ptr(x), _ptr(y), rows, cols, _stream()), "ck_q8_0_matvec_f32")
    return y


def q4k_matvec(qb, x, rows, cols, out=None):
    _dev(qb, "qb", torch.uint8, q4k_nbytes(rows * cols))
    _dev(x, "x", torch.float32, cols)
    y = out if out is not None else torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().ck_q4k_matvec_f32(_ptr(qb), _ptr(x), _ptr(y), rows, cols, _stream()), "ck_q4k_matvec_f32")
    return y


def q4k_matvec_group(qbs, x, rows, cols, outs=None):
    """Up to four Q4_K matvecs of one shape on the same x, in one launch where the tensor-core
    kernel applies (ck_q4k_matvec_f32_group); returns the list of y."""
    if not 1 <= len(qbs) <= 4:
        raise ValueError("one to four matrices")
    for qb in qbs:
        _dev(qb, "qb", torch.uint8, q4k_nbytes(rows * cols))
    _dev(x, "x", torch.float32, cols)
    ys = list(outs) if outs is not None else [torch.empty(rows, dtype=torch.float32, device=x.device) for _ in qbs]
    n = len(qbs)
    qarr = (ctypes.c_void_p * n)(*[qb.data_ptr() for qb in qbs])
    yarr = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    _lib.check(_lib.load().ck_q4k_matvec_f32_group(n, qarr, _ptr(x), yarr, rows, cols, _stream()),
               "ck_q4k_matvec_f32_group")
    return ys


def q6k_nbytes(n_weights: int) -> int:
    return (n_weights + 255) // 256 * 210


def q6k_dequant(qb, off, n):
    _dev(qb, "qb", torch.uint8, q6k_nbytes(off + n))
    w = torch.empty(n, dtype=torch.float32, device=qb.device)
    _lib.check(_lib.load().ck_q6k_dequant_f32(_ptr(qb), _ptr(w), off, n, _stream()), "ck_q6k_dequant_f32")
    return w


def q6k_matvec(qb, x, rows, cols, out=None):
    _dev(qb, "qb", torch.uint8, q6k_nbytes(rows * cols))
    _dev(x, "x", torch.float32, cols)
    y = out if out is not None else torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().ck_q6k_matvec_f32(_ptr(qb), _ptr(x), _ptr(y), rows, cols, _stream()), "ck_q6k_matvec_f32")
    return y


def q6k_matmul_batch(qb, x, rows, cols):
    """fp32 x [ntok, cols] -> fp32 y [ntok, rows]."""
    ntok = x.shape[0]
    _dev(qb, "qb", torch.uint8, q6k_nbytes(rows * cols))
    _dev(x, "x", torch.float32, ntok * cols)
    y = torch.empty((ntok, rows), dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().ck_q6k_matmul_batch_f32(_ptr(qb), _ptr(x), _ptr(y), rows, cols, ntok, _stream()),
               "ck_q6k_matmul_batch_f32")
    return y


def matvec_ordered(ggml_type, qb, x, rows, cols):
    nb = {8: q8_0_nbytes, 12: q4k_nbytes, 14: q6k_nbytes}[ggml_type](rows * cols)
    _dev(qb, "qb", torch.uint8, nb)
    _dev(x, "x", torch.float32, cols)
    y = torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().ck_matvec_ordered_f32(ggml_type, _ptr(qb), _ptr(x), _ptr(y), rows, cols, _stream()),
               "ck_matvec_ordered_f32")
    return y


def q4k_matmul_batch(qb, x, rows, cols):
    """fp32 x [ntok, cols] -> fp32 y [ntok, rows]."""
    ntok = x.shape[0]
    _dev(qb, "qb", torch.uint8, q4k_nbytes(rows * cols))
    _dev(x, "x", torch.float32, ntok * cols)
    y = torch.empty((ntok, rows), dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().ck_q4k_matmul_batch_f32(_ptr(qb), _ptr(x), _ptr(y), rows, cols, ntok, _stream()),
               "ck_q4k_matmul_batch_f32")
    return y


class Q4KGemm:
    """Prefill GEMM on the tensor cores: Y[t, r] = X[t] . W[r], X bf16 [ntok, cols] -> Y bf16."""

    def __init__(self, qb, rows, cols, max_tokens):
        self.qb = _dev(qb, "qb", torch.uint8, q4k_nbytes(rows * cols))
        self.rows, self.cols = rows, cols
        L = _lib.load()
        self.ws_bytes = L.ck_q4k_gemm_workspace_bytes(max_tokens)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=qb.device)
        self.max_tokens = max_tokens

    def __call__(self, x, out=None):
        ntok = x.shape[0]
        if ntok > self.max_tokens:
            raise ValueError("more tokens than the workspace was sized for")
        _dev(x, "x", (torch.bfloat16, torch.uint16, torch.int16), ntok * self.cols)
        y = out if out is not None else torch.empty((ntok, self.rows), dtype=torch.bfloat16, device=x.device)
        _lib.check(_lib.load().ck_q4k_gemm_bf16(_ptr(self.qb), _ptr(x), _ptr(y), self.rows, self.cols, ntok,
                                                _ptr(self.ws), self.ws_bytes, _stream()), "ck_q4k_gemm_bf16")
        return y

    def status(self, ntok):
        """Synchronize and raise if a device-side wait of the last call (over ntok tokens) gave up."""
        _lib.check(_lib.load().ck_q4k_gemm_status(ntok, _ptr(self.ws), _stream()), "ck_q4k_gemm_status")


def route_softmax(logits, nsel, renorm=True):
    ntok, ne = logits.shape
    _dev(logits, "logits", torch.float32)
    ids = torch.empty((ntok, nsel), dtype=torch.int32, device=logits.device)
    wts = torch.empty((ntok, nsel), dtype=torch.float32, device=logits.device)
    _lib.check(_lib.load().ck_route_softmax_f32(_ptr(logits), _ptr(ids), _ptr(wts), ne, nsel, ntok, int(renorm),
                                                _stream()), "ck_route_softmax_f32")
    return ids, wts


def route_dsv4(logits, bias, nused, wscale):
    ntok, ne = logits.shape
    _dev(logits, "logits", torch.float32)
    _dev(bias, "bias", torch.float32, ne)
    ids = torch.empty((ntok, nused), dtype=torch.int32, device=logits.device)
    wts = torch.empty((ntok, nused), dtype=torch.float32, device=logits.device)
    _lib.check(_lib.load().ck_route_dsv4_f32(_ptr(logits), _ptr(bias), _ptr(ids), _ptr(wts), ne, nused, wscale, ntok,
                                             _stream()), "ck_route_dsv4_f32")
    return ids, wts
