"""The host-side GGUF tensor-table reader (coherence_kernel_b200/gguf.py), on CPU: the reference's
own mini-GGUF from weight-load-q4k-band.fk (one Q4_K tensor, tensor info at byte 41, data at 96,
and the band's weight pins decoded by the oracle from the located bytes), and a written file with
Q4_K, Q6_K, Q8_0, F16 and F32 tensors, a string key/value and a non-default alignment."""
import os

import numpy as np
import pytest

from coherence_kernel_b200 import gguf, synth
from gguf_file import write_gguf
from oracle import oracle as O

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_reference_mini_gguf(tmp_path):
    g = np.load(os.path.join(G, "gguf_golden.npz"))
    p = tmp_path / "band.gguf"
    g["band_gguf"].tofile(p)
    table, base, kv = gguf.read_table(str(p))
    assert len(table) == 1
    (ti,) = table.values()
    assert ti.ggml_type == 12 and ti.dims[0] == 256 and ti.nbytes == 144
    assert base == 96 and ti.offset == 96
    w = O.q4k_dequant(g["band_gguf"][ti.offset:ti.offset + 144], 0, 256)
    for i, v in g["band_pins"]:
        assert round(w[i] * 1e6) == v, i


@pytest.mark.parametrize("align", [32, 64])
def test_written_table(tmp_path, align):
    rng = np.random.default_rng(align)
    ts = [("blk.0.ffn_gate.weight", (512, 3), 12, synth.make_q4k(rng, 512 * 3).tobytes()),
          ("token_embd.weight", (256, 5), 14, synth.make_q6k(rng, 256 * 5).tobytes()),
          ("blk.0.attn_q.weight", (64, 7), 8, synth.make_q8_0(rng, 64 * 7).tobytes()),
          ("blk.0.ffn_gate_inp.weight", (96, 4), 1, rng.standard_normal(384).astype(np.float16).tobytes()),
          ("output_norm.weight", (100,), 0, rng.standard_normal(100).astype(np.float32).tobytes())]
    p = tmp_path / "m.gguf"
    base = write_gguf(str(p), ts, kv={"general.architecture": "llama", "llama.block_count": 1}, align=align)
    table, rbase, kv = gguf.read_table(str(p))
    assert rbase == base and kv["general.architecture"] == "llama" and kv["llama.block_count"] == 1
    data = p.read_bytes()
    for name, dims, t, raw in ts:
        ti = table[name]
        assert ti.dims == dims and ti.ggml_type == t and ti.offset % align == 0
        assert data[ti.offset:ti.offset + ti.nbytes] == raw


def test_unknown_type_is_refused(tmp_path):
    p = tmp_path / "bad.gguf"
    write_gguf(str(p), [("q2k.weight", (256,), 10, b"\x00" * 84)])
    with pytest.raises(gguf.GGUFError):
        gguf.read_table(str(p))
