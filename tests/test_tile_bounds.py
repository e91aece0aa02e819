"""Host-side checks of the token-tile table bound (no GPU): ck_moe_max_tiles must hold every table
the permute can write -- decode-sized batches cut into tiles of CK_MOE_FEW_TOKENS, larger ones into
the grouped GEMM's tiles -- and must not shrink as the batch grows, since a caller sizes the table
once for its largest batch and then runs smaller ones through it."""
import os
import re

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GEMM_TILE_TOKENS = 192  # ck::GEMM_TILE_TOKENS


def header_define(name):
    src = open(os.path.join(REPO, "include", "ck_b200.h")).read()
    return int(re.search(r"#define\s+" + name + r"\s+(\d+)", src).group(1))


FEW = header_define("CK_MOE_FEW_TOKENS")
DECODE = header_define("CK_MOE_DECODE_TOKENS")


def tiles_of(count, bn):
    """Tiles of one segment of `count` rows (the permute's seg_tiles): ceil(count / bn)."""
    return 0 if count <= 0 else -(-count // bn)


def table_tiles(counts, ntok, n_shared):
    bn = FEW if ntok <= DECODE else GEMM_TILE_TOKENS
    return sum(tiles_of(int(c), bn) for c in counts) + n_shared * tiles_of(ntok, bn)


def worst_counts(ntok, nsel, n_experts, rng):
    """Expert counts of a batch: each token picks nsel distinct experts.  Besides random picks, the
    spread that maximises tiles (as many experts as possible just past a tile boundary)."""
    yield np.bincount(np.concatenate([rng.choice(n_experts, nsel, replace=False) for _ in range(ntok)]),
                      minlength=n_experts)
    for bn in (FEW, GEMM_TILE_TOKENS):
        c = np.zeros(n_experts, dtype=np.int64)
        left = ntok * nsel
        for e in range(n_experts):
            take = min(left, bn + 1, ntok)
            c[e] = take
            left -= take
        i = 0
        while left > 0:  # the rest one at a time, never above ntok per expert
            if c[i % n_experts] < ntok:
                c[i % n_experts] += 1
                left -= 1
            i += 1
        yield c


@pytest.mark.parametrize("nsel,n_experts,n_shared", [(8, 256, 1), (6, 64, 2), (4, 16, 1), (8, 32, 0)])
def test_max_tiles_holds_every_table_and_is_monotone(cuda_lib, nsel, n_experts, n_shared):
    rng = np.random.default_rng(nsel * 1000 + n_experts)
    sizes = list(range(1, 300)) + [DECODE - 1, DECODE, DECODE + 1, 511, 1024, 4096, 8192]
    bound = {n: cuda_lib.ck_moe_max_tiles(n, nsel, n_experts, n_shared) for n in sorted(set(sizes))}
    ns = sorted(bound)
    for a, b in zip(ns, ns[1:]):
        assert bound[b] >= bound[a], (a, b, bound[a], bound[b])
    for n in ns:
        for counts in worst_counts(n, min(nsel, n_experts), n_experts, rng):
            assert counts.sum() == n * min(nsel, n_experts)
            assert table_tiles(counts, n, n_shared) <= bound[n], (n, table_tiles(counts, n, n_shared), bound[n])


def test_decode_tiles_fit_two_accumulator_stages():
    # 3 digit rows per token in N = 16 accumulator columns per K step
    assert 3 * FEW <= 16
    assert DECODE >= FEW
