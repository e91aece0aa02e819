"""GGUF ingest: read a model file's tensor table on the host and put its quantized tensors in HBM.

The reference walks the same structures in Form over a byte source (form/form-stdlib/
equireach-gguf.fk:42-115 egg-*: header, key/value skip, tensor-info records, data base aligned
up), and its MoE decode cell emits the table with each tensor's absolute offset and byte length
(form/native/metal/moe-token.fk:121-160), then binds the tensors on the device with
metal_buf_from_file.  This module is the host side of that path for Python callers:

* ``read_table(path)`` parses the header (magic "GGUF", version, tensor count, key/value count),
  skips the key/value section value by value (arrays included), reads every tensor-info record
  (name, dims, ggml type, offset relative to the data base) and aligns the data base up to
  ``general.alignment`` (32 when the file does not set it);
* ``load(path, names, device)`` copies each tensor's bytes into HBM once (one host read and one
  host-to-device copy per tensor); the packed blocks are not repacked, so the kernels read them in
  the file's own GGUF layout.

Byte lengths by ggml type: F32 4 B / weight, F16 2 B / weight, Q8_0 34 B / 32, Q4_K 144 B / 256,
Q6_K 210 B / 256; any other type is refused rather than guessed.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
TYPE_BYTES = {0: (1, 4), 1: (1, 2), 8: (32, 34), 12: (256, 144), 14: (256, 210)}  # type: (weights, bytes)
# key/value value types: size of a fixed-size scalar, 8 = string, 9 = array
_SCALAR = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}


@dataclass
class TensorInfo:
    name: str
    dims: tuple
    ggml_type: int
    offset: int       # absolute byte offset in the file
    nbytes: int

    @property
    def n_weights(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n


class GGUFError(ValueError):
    pass


class _Reader:
    def __init__(self, data: bytes):
        self.b = data
        self.o = 0

    def take(self, fmt):
        n = struct.calcsize(fmt)
        if self.o + n > len(self.b):
            raise GGUFError("truncated GGUF header")
        v = struct.unpack_from(fmt, self.b, self.o)
        self.o += n
        return v[0] if len(v) == 1 else v

    def string(self) -> bytes:
        n = self.take("<Q")
        if self.o + n > len(self.b):
            raise GGUFError("truncated GGUF string")
        s = self.b[self.o:self.o + n]
        self.o += n
        return s

    def value(self, t):
        if t in _SCALAR:
            raw = self.b[self.o:self.o + _SCALAR[t]]
            self.o += _SCALAR[t]
            return raw
        if t == 8:
            return self.string()
        if t == 9:
            et, count = self.take("<I"), self.take("<Q")
            if et in _SCALAR:
                self.o += _SCALAR[et] * count
            else:
                for _ in range(count):
                    self.value(et)
            return None
        raise GGUFError(f"unknown key/value type {t}")


def read_table(path: str, header_bytes: int = 64 << 20):
    """(tensors by name in file order, data base, key/values that are scalars or strings)."""
    with open(path, "rb") as f:
        data = f.read(min(header_bytes, os.path.getsize(path)))
    r = _Reader(data)
    if r.take("<I") != GGUF_MAGIC:
        raise GGUFError(f"{path} is not a GGUF file")
    version = r.take("<I")
    if version not in (2, 3):
        raise GGUFError(f"GGUF version {version} is not supported")
    n_tensors, n_kv = r.take("<Q"), r.take("<Q")
    kv = {}
    for _ in range(n_kv):
        key = r.string().decode(errors="replace")
        t = r.take("<I")
        v = r.value(t)
        if t == 4 or t == 5:
            v = struct.unpack("<I" if t == 4 else "<i", v)[0]
        elif t == 8:
            v = v.decode(errors="replace")
        kv[key] = v
    infos = []
    for _ in range(n_tensors):
        name = r.string().decode(errors="replace")
        nd = r.take("<I")
        dims = tuple(r.take("<Q") for _ in range(nd))
        t, off = r.take("<I"), r.take("<Q")
        infos.append((name, dims, t, off))
    align = int(kv.get("general.alignment", 32))
    base = (r.o + align - 1) // align * align
    out = {}
    for name, dims, t, off in infos:
        if t not in TYPE_BYTES:
            raise GGUFError(f"tensor {name}: ggml type {t} has no known byte length")
        n = 1
        for d in dims:
            n *= d
        per, nb = TYPE_BYTES[t]
        if n % per:
            raise GGUFError(f"tensor {name}: {n} weights is not a whole number of blocks")
        out[name] = TensorInfo(name, dims, t, base + off, n // per * nb)
    return out, base, kv


def load(path: str, names=None, device="cuda"):
    """The named tensors (all by default) as uint8 device tensors of their packed bytes."""
    import torch
    table, _, _ = read_table(path)
    names = list(table) if names is None else names
    out = {}
    with open(path, "rb") as f:
        for name in names:
            ti = table[name]
            f.seek(ti.offset)
            raw = f.read(ti.nbytes)
            if len(raw) != ti.nbytes:
                raise GGUFError(f"tensor {name}: file ends inside its data")
            host = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
            out[name] = host.to(device)
    return out, table
