"""Parity of the Q6_K kernels with the oracle (GPU), directly and through the handle door.

Tolerances: Q6_K dequant is exact in fp32 ((d*sc)*q needs at most 25 significant bits and is
rounded once, q6k-msl.fk's own bit-exactness argument), so equality; the decode / batched matvecs
within 1e-3 * sum_j |w_j x_j| per row AND normwise max|y - ref| / max|ref| <= 1e-3; the
attestant-order kernel within the reference's derived bound (cols + ceil(cols/p) + p) * 2^-24 *
sum_j |w_j x_j| at p = 1 (qk-matvec-split.fk:41-54), and its split form at p parts equal to it bit
for bit at p = 1.
"""
import os

import numpy as np
import pytest
import torch

from coherence_kernel_b200 import carrier, ops, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
U = 2.0 ** -24


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_q6k_dequant_exact_on_reference_vectors():
    g = np.load(os.path.join(G, "q6k_golden.npz"))
    # the reference's two-superblock fixture, the band's real superblock, and a seeded tensor
    assert np.array_equal(ops.q6k_dequant(dev(g["fix"]), 0, 512).cpu().numpy(), g["fix_w"].astype(np.float32))
    w = ops.q6k_dequant(dev(g["band_sb"]), 0, 256).cpu().numpy()
    assert np.array_equal(w, g["band_w"].astype(np.float32))
    for i, v in g["band_pins"]:
        assert round(float(w[i]) * 1e6) == v
    r6, c6 = (int(v) for v in g["dims"])
    assert np.array_equal(ops.q6k_dequant(dev(g["q6"]), 0, r6 * c6).cpu().numpy(), g["w6"].astype(np.float32))


@pytest.mark.parametrize("n,off", [(1 << 20, 0), (1000, 37), (70000, 256 * 3 + 5)])
def test_q6k_dequant_large(n, off):
    rng = np.random.default_rng(n + off)
    q = synth.make_q6k(rng, ((off + n + 255) // 256) * 256)
    w = ops.q6k_dequant(dev(q), off, n).cpu().numpy()
    assert np.array_equal(w, O.q6k_dequant(q, off, n).astype(np.float32))


def test_q6k_matvec_golden():
    # fkwu's tb-matvec over q6m-flat-at rows that straddle superblocks (cols = 384)
    g = np.load(os.path.join(G, "q6k_golden.npz"))
    r6, c6 = (int(v) for v in g["dims"])
    w = g["w6"].reshape(r6, c6)
    bound = np.abs(w) @ np.abs(g["x6"].astype(np.float64))
    y = ops.q6k_matvec(dev(g["q6"]), dev(g["x6"]), r6, c6).cpu().numpy()
    assert np.all(np.abs(y - g["y6"]) <= 1e-3 * bound)
    yo = ops.matvec_ordered(14, dev(g["q6"]), dev(g["x6"]), r6, c6).cpu().numpy()
    assert np.all(np.abs(yo - g["y6"]) <= (2 * c6 + 1) * U * bound)


def check_rows(q, x, y, rows, cols, nsample=64):
    sample = np.unique(np.linspace(0, rows - 1, nsample).astype(int))
    x64 = x.astype(np.float64)
    refs = []
    for r in sample:
        w = O.q6k_dequant(q, r * cols, cols)
        ref = O.lib().ckr_dot(w.ctypes.data, x64.ctypes.data, cols)
        assert abs(y[r] - ref) <= 1e-3 * np.abs(w * x64).sum(), (r, y[r], ref)
        refs.append(ref)
    err = np.abs(y[sample] - np.array(refs)).max() / np.abs(np.array(refs)).max()
    print(f"normwise error q6k matvec {rows}x{cols}: {err:.3e}")
    assert err <= 1e-3


# shared-memory streaming kernel: one unit per thread (<= 4096 cols), two (<= 8192), four (<= 16384),
# several row slots per CTA (2048, 256 cols), ragged stage tails (odd rows, 7168 cols: 5880-byte
# rows); 11008 (an odd superblock count per row) and 384 (rows straddle superblocks) take the
# one-warp-per-row kernel
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (7168, 7168), (333, 7168), (129, 16384), (1000, 2048),
                                       (777, 256), (3072, 8192), (300, 11008), (10, 384), (5, 512)])
def test_q6k_matvec_sizes(rows, cols):
    rng = np.random.default_rng(rows * 5 + cols)
    q = synth.make_q6k(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = ops.q6k_matvec(dev(q), dev(x), rows, cols).cpu().numpy()
    assert np.all(np.isfinite(y))
    check_rows(q, x, y, rows, cols)


@pytest.mark.parametrize("ntok", [1, 3, 8])
def test_q6k_matmul_batch(ntok):
    rows, cols = 512, 2048
    rng = np.random.default_rng(ntok + 100)
    q = synth.make_q6k(rng, rows * cols)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    y = ops.q6k_matmul_batch(dev(q), dev(x), rows, cols).cpu().numpy()
    w = O.q6k_dequant(q, 0, rows * cols).reshape(rows, cols)
    ref = x.astype(np.float64) @ w.T
    assert np.all(np.abs(y - ref) <= 1e-3 * (np.abs(x.astype(np.float64)) @ np.abs(w).T))
    for t in range(ntok):
        assert np.abs(y[t] - ref[t]).max() <= 1e-3 * np.abs(ref[t]).max()


def test_q6k_door_names():
    """form_q6k_* through the handle door, with the reference's argument layouts: dequant equals the
    oracle bit for bit; the attestant within the derived bound; the split at one part equals the
    attestant bit for bit and at 5 parts + form_part_combine_f32 stays within its bound; the lane /
    slot forms and the batched form within 1e-3 of sum |w x|."""
    rows, cols, parts, ntok = 96, 1024, 5, 3
    rng = np.random.default_rng(21)
    q = synth.make_q6k(rng, rows * cols)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    w = O.q6k_dequant(q, 0, rows * cols).reshape(rows, cols)
    ref = x.astype(np.float64) @ w.T
    absb = np.abs(x.astype(np.float64)) @ np.abs(w).T
    hq = carrier.buf_alloc(q.nbytes)
    hx = carrier.buf_alloc(x.nbytes)
    hy = carrier.buf_alloc(ntok * rows * 4)
    hw = carrier.buf_alloc(rows * cols * 4)
    hp = carrier.buf_alloc(rows * parts * 4)
    carrier.buf_write(hq, 0, q.tobytes())
    carrier.buf_write(hx, 0, x.tobytes())

    def run(name, bufs, consts, threads, nbytes, h):
        p = carrier.pipeline("", name)
        assert p > 0, carrier.status()
        assert carrier.enqueue(p, carrier.md_bind(bufs, consts), threads) == 1, carrier.status()
        assert carrier.sync() == 1
        return np.frombuffer(carrier.buf_read(h, 0, nbytes), dtype=np.float32)

    wd = run("form_q6k_dequant_f32", [hq, hw], [0, rows * cols], rows * cols, rows * cols * 4, hw)
    assert np.array_equal(wd, w.reshape(-1).astype(np.float32))
    ya = run("form_q6k_matvec_f32", [hq, hx, hy], [rows, cols], rows, rows * 4, hy)
    assert np.all(np.abs(ya - ref[0]) <= (2 * cols + 1) * U * absb[0])
    p1 = run("form_q6k_matvec_part_f32", [hq, hx, hp], [rows, cols, 1], rows, rows * 4, hp)
    assert np.array_equal(p1, ya)
    h1 = run("form_q6k_matvec_hoist_f32", [hq, hx, hp], [rows, cols, 1], rows, rows * 4, hp)
    assert np.array_equal(h1, ya)
    run("form_q6k_matvec_part_f32", [hq, hx, hp], [rows, cols, parts], rows * parts, rows * parts * 4, hp)
    yc = run("form_part_combine_f32", [hp, hy], [rows, parts], rows, rows * 4, hy)
    chunk = -(-cols // parts)
    assert np.all(np.abs(yc - ref[0]) <= (cols + chunk + parts) * U * absb[0])
    for name in ("form_q6k_matvec_lane_f32", "form_q6k_matvec_slot_f32"):
        yl = run(name, [hq, hx, hy], [rows, cols], rows, rows * 4, hy)
        assert np.all(np.abs(yl - ref[0]) <= 1e-3 * absb[0])
    yb = run("form_q6k_matmul_batch_f32", [hq, hx, hy], [rows, cols, ntok], rows, ntok * rows * 4, hy)
    assert np.all(np.abs(yb.reshape(ntok, rows) - ref) <= 1e-3 * absb)
    for h in (hq, hx, hy, hw, hp):
        assert carrier.buf_free(h) == 1
