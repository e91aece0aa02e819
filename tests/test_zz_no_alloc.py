"""ck_q4k_gemm_bf16_noalloc (fixed device scratch, no workspace argument) against ck_q4k_gemm_bf16.

Two calls in a row with different shapes -- the second reuses the scratch the first left behind --
each within the GEMM tolerance of the workspace entry point's result: normwise
max|noalloc - workspace| <= 2e-2 * max|workspace|.  Runs alone or after every other test.
"""
import numpy as np
import pytest
import torch

from coherence_kernel_b200 import _lib, ops, synth

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _inputs(rows, cols, ntok, seed):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(synth.make_q4k(rng, rows * cols)).cuda()
    x = torch.from_numpy(synth.make_bf16(rng, (ntok, cols)).view(np.int16)).cuda()
    return q, x


def _noalloc(q, x, rows, cols):
    ntok = x.shape[0]
    y = torch.empty((ntok, rows), dtype=torch.bfloat16, device=x.device)
    rc = _lib.load().ck_q4k_gemm_bf16_noalloc(ops._ptr(q), ops._ptr(x), ops._ptr(y), rows, cols, ntok,
                                              ops._stream())
    _lib.check(rc, "ck_q4k_gemm_bf16_noalloc")
    return y


def test_noalloc_matches_workspace_entry_two_calls():
    # call 1: K % 256 == 0 (TMA-staged packed weights); call 2: K = 1408 (rows straddle
    # superblocks) with more tokens, so the tile table it writes is longer than the first one's
    shapes = [(512, 2048, 300, 11), (384, 1408, 1000, 12)]
    cases = [(rows, cols) + _inputs(rows, cols, ntok, seed) for rows, cols, ntok, seed in shapes]
    got = [_noalloc(q, x, rows, cols) for rows, cols, q, x in cases]  # back to back, same stream
    for (rows, cols, q, x), y in zip(cases, got):
        ref = ops.Q4KGemm(q, rows, cols, max_tokens=x.shape[0])(x).float().cpu().numpy()
        y = y.float().cpu().numpy()
        assert np.isfinite(y).all()
        assert np.abs(y - ref).max() <= TOL * np.abs(ref).max()


def test_noalloc_rejects_more_tokens_than_its_scratch():
    limit = 65536
    rc = _lib.load().ck_q4k_gemm_bf16_noalloc(1, 1, 1, 128, 256, limit + 1, None)
    assert rc == -2  # CK_ESHAPE, refused on the host before any work is queued
    assert str(limit) in _lib.load().ck_last_error().decode()
