"""A small GGUF v3 writer for the ingest tests (test infrastructure): header, string and u32
key/values, tensor-info records, the data base aligned to `align`, every tensor's bytes at an
offset aligned to `align`."""
import struct


def write_gguf(path, tensors, kv=None, align=32):
    """tensors: list of (name, dims, ggml_type, raw bytes).  kv: {key: str | int}."""
    kv = dict(kv or {})
    if align != 32:
        kv["general.alignment"] = align

    def s(b):
        b = b.encode() if isinstance(b, str) else b
        return struct.pack("<Q", len(b)) + b

    out = bytearray(struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kv)))
    for k, v in kv.items():
        out += s(k)
        out += struct.pack("<I", 8) + s(v) if isinstance(v, str) else struct.pack("<II", 4, v)
    offs, cur = [], 0
    for _, _, _, raw in tensors:
        offs.append(cur)
        cur = (cur + len(raw) + align - 1) // align * align
    for (name, dims, t, _), off in zip(tensors, offs):
        out += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, off)
    base = (len(out) + align - 1) // align * align
    out += b"\x00" * (base - len(out))
    for (_, _, _, raw), off in zip(tensors, offs):
        out += b"\x00" * (base + off - len(out)) + raw
    with open(path, "wb") as f:
        f.write(bytes(out))
    return base
