"""GGUF ingest from Python: coherence_kernel_b200.gguf.load puts a file's packed tensors in HBM,
and the kernels decode them there -- Q4_K within one rounding of the oracle, Q6_K and Q8_0 bit for
bit -- with a Q6_K matvec on the loaded tensor within 1e-3 of sum |w x|."""
import numpy as np
import pytest
import torch

from coherence_kernel_b200 import gguf, ops, synth
from gguf_file import write_gguf
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_gguf_load_and_decode_on_device(tmp_path):
    rng = np.random.default_rng(41)
    q4, q6, q8 = synth.make_q4k(rng, 1024 * 3), synth.make_q6k(rng, 512 * 6), synth.make_q8_0(rng, 96 * 4)
    ts = [("a.weight", (1024, 3), 12, q4.tobytes()), ("b.weight", (512, 6), 14, q6.tobytes()),
          ("c.weight", (96, 4), 8, q8.tobytes())]
    p = tmp_path / "m.gguf"
    write_gguf(str(p), ts, align=64)
    dev, table = gguf.load(str(p), device="cuda")
    w4 = ops.q4k_dequant(dev["a.weight"], 0, 1024 * 3).cpu().numpy().astype(np.float64)
    r4 = O.q4k_dequant(q4, 0, 1024 * 3)
    assert np.all(np.abs(w4 - r4) <= 2.0 ** -24 * np.abs(r4))
    assert np.array_equal(ops.q6k_dequant(dev["b.weight"], 0, 512 * 6).cpu().numpy(),
                          O.q6k_dequant(q6, 0, 512 * 6).astype(np.float32))
    assert np.array_equal(ops.q8_0_dequant(dev["c.weight"], 0, 96 * 4).cpu().numpy(),
                          O.q80_dequant(q8, 0, 96 * 4).astype(np.float32))
    x = rng.standard_normal(512).astype(np.float32)
    y = ops.q6k_matvec(dev["b.weight"], torch.from_numpy(x).cuda(), 6, 512).cpu().numpy()
    w = O.q6k_dequant(q6, 0, 512 * 6).reshape(6, 512)
    assert np.all(np.abs(y - w @ x.astype(np.float64)) <= 1e-3 * (np.abs(w) @ np.abs(x.astype(np.float64))))
