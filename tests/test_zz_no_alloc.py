"""ck_q4k_gemm_bf16_noalloc (fixed device scratch, no workspace argument) against ck_q4k_gemm_bf16.

Both entry points run the same kernels on the same inputs in the same order, so their outputs
must be equal bit for bit.  Three calls in a row -- the second reuses the scratch the first left
behind with a longer tile table, the third is a 3-token call (the few-token tensor-core path,
one tile of 3 tokens) right after the 1000-token one -- each compared with the workspace entry
point, and every call's error word read back through ck_q4k_gemm_bf16_noalloc_status.  Runs alone
or after every other test.
"""
import numpy as np
import pytest
import torch

from coherence_kernel_b200 import _lib, ops, synth

pytestmark = pytest.mark.gpu


def _inputs(rows, cols, ntok, seed):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(synth.make_q4k(rng, rows * cols)).cuda()
    x = torch.from_numpy(synth.make_bf16(rng, (ntok, cols)).view(np.int16)).cuda()
    return q, x


def _noalloc(q, x, rows, cols):
    ntok = x.shape[0]
    y = torch.empty((ntok, rows), dtype=torch.bfloat16, device=x.device)
    L = _lib.load()
    _lib.check(L.ck_q4k_gemm_bf16_noalloc(ops._ptr(q), ops._ptr(x), ops._ptr(y), rows, cols, ntok, ops._stream()),
               "ck_q4k_gemm_bf16_noalloc")
    _lib.check(L.ck_q4k_gemm_bf16_noalloc_status(ops._stream()), "ck_q4k_gemm_bf16_noalloc_status")
    return y


def test_noalloc_equals_workspace_entry_three_calls():
    # the set-up call: ntok 0, null pointers, before any real call
    assert _lib.load().ck_q4k_gemm_bf16_noalloc(None, None, None, 0, 0, 0, ops._stream()) == 0
    # call 1: K % 256 == 0 (TMA-staged packed weights); call 2: K = 1408 (rows straddle
    # superblocks) with more tokens, so the tile table it writes is longer than the first one's;
    # call 3: 3 tokens, n % 128 == 0 and k % 256 == 0 -- the few-token matvec over a one-tile table
    shapes = [(512, 2048, 300, 11), (384, 1408, 1000, 12), (640, 2048, 3, 13)]
    cases = [(rows, cols) + _inputs(rows, cols, ntok, seed) for rows, cols, ntok, seed in shapes]
    got = [_noalloc(q, x, rows, cols) for rows, cols, q, x in cases]  # back to back, same stream
    for (rows, cols, q, x), y in zip(cases, got):
        g = ops.Q4KGemm(q, rows, cols, max_tokens=x.shape[0])
        ref = g(x)
        g.status(x.shape[0])
        y, ref = y.view(torch.int16).cpu().numpy(), ref.view(torch.int16).cpu().numpy()
        assert np.isfinite(synth.bf16_bits_to_f32(y.view(np.uint16))).all()
        assert np.array_equal(y, ref), f"{rows}x{cols}, {x.shape[0]} tokens: not bit-equal"


def test_noalloc_rejects_more_tokens_than_its_scratch():
    limit = 65536
    rc = _lib.load().ck_q4k_gemm_bf16_noalloc(1, 1, 1, 128, 256, limit + 1, None)
    assert rc == -2  # CK_ESHAPE, refused on the host before any work is queued
    assert str(limit) in _lib.load().ck_last_error().decode()
