"""Python face of the handle door (include/fk_cuda_carrier.h) -- what a Form cell does through
metal_pipeline / metal_buf_* / metal_enqueue / metal_sync, for tests and host tools.

``md_bind`` encodes the binding string exactly as the reference's Form encoder does
(form/form-stdlib/metal-door.fk:110-126): little-endian u32 n_buf, handles, n_const, constants,
optionally followed by the (threads_per_group, threadgroup_bytes[, dispatch_mode, barrier_before])
tail.  Float constants travel as their binary32 bit pattern (md-f32-bits, metal-door.fk:99-103).
"""
from __future__ import annotations

import ctypes
import struct

from . import _lib


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def md_bind(bufs, consts, tail=None) -> bytes:
    b = struct.pack("<I", len(bufs)) + b"".join(struct.pack("<I", h & 0xFFFFFFFF) for h in bufs)
    b += struct.pack("<I", len(consts)) + b"".join(struct.pack("<I", c & 0xFFFFFFFF) for c in consts)
    if tail is not None:
        b += b"".join(struct.pack("<I", v) for v in tail)
    return b


def _L():
    return _lib.load()


def pipeline(msl: str, name: str) -> int:
    m, n = msl.encode(), name.encode()
    return _L().fk_metal_pipeline_external(m, len(m), n, len(n))


def buf_alloc(nbytes: int) -> int:
    return _L().fk_metal_buf_alloc_external(nbytes)


def buf_from_file(path: str, off: int, length: int) -> int:
    p = path.encode()
    return _L().fk_metal_buf_from_file_external(p, len(p), off, length)


def buf_write(h: int, off: int, data: bytes) -> int:
    return _L().fk_metal_buf_write_external(h, off, data, len(data))


def enqueue(pipe: int, binding: bytes, threads: int) -> int:
    return _L().fk_metal_enqueue_external(pipe, binding, len(binding), threads)


def sync() -> int:
    return _L().fk_metal_sync_external()


def buf_read(h: int, off: int, length: int, cap: int | None = None):
    cap = length if cap is None else cap
    out = ctypes.create_string_buffer(max(cap, 1))
    n = _L().fk_metal_buf_read_external(h, off, length, out, cap)
    return None if n < 0 else out.raw[:n]


def status() -> str:
    out = ctypes.create_string_buffer(8192)
    n = _L().fk_metal_status_external(out, 8192)
    return out.raw[:max(n, 0)].decode(errors="replace")


def batch_concurrent() -> int:
    return _L().fk_metal_batch_concurrent_external()


def buf_free(h: int) -> int:
    return _L().fk_metal_buf_free_external(h)


def submit() -> int:
    return _L().fk_metal_submit_external()


def fence_wait(f: int) -> int:
    return _L().fk_metal_fence_wait_external(f)
