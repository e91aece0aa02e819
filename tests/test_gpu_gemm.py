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


@pytest.mark.parametrize("rows,cols,ntok", [(1024, 2048, 300), (256, 512, 17), (512, 1408, 200), (200, 512, 33)])
def test_gemm_rows_scattered_equal_contiguous(rows, cols, ntok):
    """ck_moe_expert_gemm_rows (output row o stored at the address row_dst[o], the expert-parallel
    down projection that writes the return itself) gives, row for row, exactly the bits of the
    contiguous grouped GEMM, with the rows scattered in a shuffled order and nothing else written."""
    import ctypes

    from coherence_kernel_b200 import _lib
    from coherence_kernel_b200.ops import _ptr, _stream
    L = _lib.load()
    rng = np.random.default_rng(rows + ntok)
    q = torch.from_numpy(synth.make_q4k(rng, rows * cols)).cuda()
    x = torch.from_numpy(synth.make_bf16(rng, (ntok, cols)).view(np.int16)).cuda()
    mt = ntok // 16 + 2
    tiles = torch.empty((mt, 4), dtype=torch.int32, device="cuda")
    nt = torch.empty(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(L.ck_token_tiles(_ptr(tiles), _ptr(nt), ntok, _stream()), "ck_token_tiles")
    ref = torch.empty((ntok, rows), dtype=torch.int16, device="cuda")
    _lib.check(L.ck_moe_expert_gemm_bounded(0, _ptr(q), None, None, None, 0, 1, 0, _ptr(x), ntok, _ptr(ref), ntok,
                                            None, _ptr(tiles), _ptr(nt), mt, rows, cols, 0, 0, _ptr(err), _stream()),
               "ck_moe_expert_gemm_bounded")
    perm = torch.randperm(ntok, generator=torch.Generator().manual_seed(ntok)).cuda()
    dst = torch.full((ntok + 3, rows), 0x7ABC, dtype=torch.int16, device="cuda")
    row_dst = (dst.data_ptr() + perm.to(torch.int64) * rows * 2).contiguous()
    _lib.check(L.ck_moe_expert_gemm_rows(_ptr(q), 0, 1, _ptr(x), ntok, _ptr(row_dst), ntok, _ptr(tiles), _ptr(nt), mt,
                                         rows, cols, 0, _ptr(err), _stream()), "ck_moe_expert_gemm_rows")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(dst[perm], ref)
    assert bool((dst[ntok:] == 0x7ABC).all())
    # the entry refuses a missing row table
    assert L.ck_moe_expert_gemm_rows(_ptr(q), 0, 1, _ptr(x), ntok, None, ntok, _ptr(tiles), _ptr(nt), mt, rows,
                                     cols, 0, _ptr(err), _stream()) != 0
