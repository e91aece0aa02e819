"""Parity of the tensor-core Q4_K GEMM (tcgen05, bf16 MMA, fp32 accumulate) with the oracle.

Tolerance 2e-2 (bf16-MMA): per output |gpu - ref| <= 2e-2 * sum_j |w_j x_j|, and the normwise
max|gpu - ref| / max|ref| <= 2e-2.
"""
import numpy as np
import pytest
import torch

from coherence_kernel_b200 import ops, synth, workloads
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def run(rows, cols, ntok, seed, sample_rows=None):
    rng = np.random.default_rng(seed)
    q = synth.make_q4k(rng, rows * cols)
    xb = synth.make_bf16(rng, (ntok, cols))
    g = ops.Q4KGemm(torch.from_numpy(q).cuda(), rows, cols, max_tokens=ntok)
    y = g(torch.from_numpy(xb.view(np.int16)).cuda()).float().cpu().numpy()
    x64 = synth.bf16_bits_to_f32(xb).astype(np.float64)
    rs = np.arange(rows) if sample_rows is None else sample_rows
    w = np.stack([O.q4k_dequant(q, r * cols, cols) for r in rs])
    ref = x64 @ w.T            # fp64 reference for the sampled rows (tb-dot per (t, r) to 1e-15)
    bound = np.abs(x64) @ np.abs(w).T
    got = y[:, rs]
    assert np.all(np.abs(got - ref) <= 2e-2 * bound)
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()
    return got, ref


@pytest.mark.parametrize("rows,cols,ntok", [(128, 64, 16), (256, 512, 1), (256, 512, 17), (384, 1408, 300),
                                            (128, 256, 256), (512, 2048, 520), (256, 768, 4), (384, 1024, 8),
                                            (640, 2048, 3), (200, 512, 3), (256, 256, 2)])
def test_gemm_small(rows, cols, ntok):
    # up to 4 tokens, rows a multiple of 128 and cols of 256 take the few-token tensor-core matvec;
    # the rest (and 200 rows) the dequantizing GEMM
    run(rows, cols, ntok, seed=rows * 31 + ntok)


def test_gemm_matches_oracle_fold_exactly_enough():
    # the oracle's own right fold on a few (token, row) pairs, not numpy's matmul
    rows, cols, ntok = 256, 1024, 48
    got, _ = run(rows, cols, ntok, seed=5)
    rng = np.random.default_rng(5)
    q = synth.make_q4k(rng, rows * cols)
    xb = synth.make_bf16(rng, (ntok, cols))
    x64 = synth.bf16_bits_to_f32(xb).astype(np.float64)
    yo = O.q4k_matmul(q, x64, rows, cols)
    w = O.q4k_dequant(q, 0, rows * cols).reshape(rows, cols)
    assert np.all(np.abs(got - yo) <= 2e-2 * (np.abs(x64) @ np.abs(w).T))


@pytest.mark.parametrize("m", workloads.Q4K_PREFILL_M)
def test_prefill_shape_sampled(m):
    rows, cols = workloads.Q4K_PREFILL
    run(rows, cols, m, seed=m, sample_rows=np.unique(np.linspace(0, rows - 1, 48).astype(int)))
