"""Parity of the dequant / decode-matvec kernels with the oracle (GPU).

Tolerances: Q8_0 dequant is exact in fp32 (d*q needs <= 19 significand bits, q8-0-msl.fk:17-21),
so equality; Q4_K dequant within one rounding |gpu - w| <= 2^-24 |w| (q4k-msl.fk:20-28); fp32
matvecs within 1e-3 * sum_j |w_j x_j| per row AND within the stated max relative error
max|y - ref| / max|ref| <= 1e-3 (normwise, fp32 accumulate), and the attestant-order kernel within
the reference's derived bound (cols + ceil(cols/p) + p) * 2^-24 * sum_j |w_j x_j| at p = 1
(qk-matvec-split.fk:41-54).  The achieved normwise error is printed (pytest -s shows it).
"""
import os

import numpy as np
import pytest
import torch

from coherence_kernel_b200 import ops, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
U = 2.0 ** -24


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


NORMWISE = 1e-3


def normwise(y, ref, what, tol=NORMWISE):
    """max|y - ref| / max|ref| <= tol; prints the achieved error."""
    y, ref = np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    print(f"normwise error {what}: {err:.3e}")
    assert err <= tol, (what, err)
    return err


def absdot(wq_deq, x, rows, cols):
    return np.abs(wq_deq.reshape(rows, cols)) @ np.abs(x.astype(np.float64))


def test_q8_0_dequant_exact_on_reference_fixture():
    f = np.load(os.path.join(G, "ref_fixtures.npz"))
    w = ops.q8_0_dequant(dev(f["q80"]), 0, 96).cpu().numpy()
    assert np.array_equal(w, f["w8"].astype(np.float32))


def test_q4k_dequant_one_rounding_on_reference_fixture():
    f = np.load(os.path.join(G, "ref_fixtures.npz"))
    w = ops.q4k_dequant(dev(f["q4k"]), 0, 512).cpu().numpy().astype(np.float64)
    assert np.all(np.abs(w - f["w4"]) <= U * np.abs(f["w4"]))


@pytest.mark.parametrize("n,off", [(4096 * 32, 0), (1000, 37), (1 << 20, 256)])
def test_dequant_large(n, off):
    rng = np.random.default_rng(n)
    q8 = synth.make_q8_0(rng, ((off + n + 31) // 32) * 32)
    q4 = synth.make_q4k(rng, ((off + n + 255) // 256) * 256)
    w8 = ops.q8_0_dequant(dev(q8), off, n).cpu().numpy()
    assert np.array_equal(w8, O.q80_dequant(q8, off, n).astype(np.float32))
    w4 = ops.q4k_dequant(dev(q4), off, n).cpu().numpy().astype(np.float64)
    ref = O.q4k_dequant(q4, off, n)
    assert np.all(np.abs(w4 - ref) <= U * np.abs(ref))


def test_matvec_golden():
    g = np.load(os.path.join(G, "quant_golden.npz"))
    r8, c8, r4, c4 = (int(v) for v in g["dims"])
    y8 = ops.q8_0_matvec(dev(g["q8"]), dev(g["x8"]), r8, c8).cpu().numpy()
    b8 = absdot(g["w8"], g["x8"], r8, c8)
    assert np.all(np.abs(y8 - g["y8"]) <= 1e-3 * b8)
    normwise(y8, g["y8"], "q8_0 golden")
    y4 = ops.q4k_matvec(dev(g["q4"]), dev(g["x4"]), r4, c4).cpu().numpy()   # rows straddle superblocks
    b4 = absdot(g["w4"], g["x4"], r4, c4)
    assert np.all(np.abs(y4 - g["y4"]) <= 1e-3 * b4)
    normwise(y4, g["y4"], "q4k golden")
    for kind, q, x, y, b, r, c in ((8, g["q8"], g["x8"], g["y8"], b8, r8, c8), (12, g["q4"], g["x4"], g["y4"], b4, r4, c4)):
        yo = ops.matvec_ordered(kind, dev(q), dev(x), r, c).cpu().numpy()
        assert np.all(np.abs(yo - y) <= (2 * c + 1) * U * b)


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (512, 1408), (7168, 7168), (300, 2048), (1000, 256), (777, 768),
                                       (130, 8192), (5, 512)])
def test_q4k_matvec_sizes(rows, cols):
    rng = np.random.default_rng(rows + cols)
    q = synth.make_q4k(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = ops.q4k_matvec(dev(q), dev(x), rows, cols).cpu().numpy()
    q4k_rows_check(q, x, y, rows, cols, nsample=64, what=f"q4k matvec {rows}x{cols}")


def q4k_rows_check(q, x, y, rows, cols, nsample=64, tol=1e-3, what="q4k matvec"):
    sample = np.unique(np.linspace(0, rows - 1, nsample).astype(int))
    x64 = x.astype(np.float64)
    refs = []
    for r in sample:
        w = O.q4k_dequant(q, r * cols, cols)
        ref = O.lib().ckr_dot(w.ctypes.data, x64.ctypes.data, cols)
        assert abs(y[r] - ref) <= tol * np.abs(w * x64).sum(), (r, y[r], ref)
        refs.append(ref)
    normwise(y[sample], refs, f"{what} ({len(sample)} rows)")


@pytest.mark.parametrize("rows,cols", [(4096, 11008), (19000, 4096), (1000, 8448), (777, 9216), (5, 8448),
                                       (300, 16384), (129, 12288)])
def test_q4k_matvec_tensor_core_shapes(rows, cols):
    """One token through the tensor-core matvec (from about 12 MB of weights, or cols beyond the
    streaming kernel's limit): ragged last tiles, K splits of 1, 2 and 4 CTAs, a 149-tile grid."""
    rng = np.random.default_rng(rows * 3 + cols)
    q = synth.make_q4k(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = ops.q4k_matvec(dev(q), dev(x), rows, cols).cpu().numpy()
    assert np.all(np.isfinite(y))
    q4k_rows_check(q, x, y, rows, cols, nsample=48, what=f"q4k tensor-core matvec {rows}x{cols}")


def test_q4k_matvec_tensor_core_dynamic_range():
    """x scaled per 32-value sub-block over 1e-40 .. 1e25, with all-zero sub-blocks: the matvec holds
    each sub-block of x as a fixed-point integer relative to its own power-of-two bound."""
    rows, cols = 777, 9216
    rng = np.random.default_rng(11)
    q = synth.make_q4k(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    x[0:256] = 0
    x[256:512] *= np.float32(1e-30)
    x[512:768] *= np.float32(1e25)
    x[768:800] = 0
    x[1024:1056] = np.float32(1e-40)
    x[2048:2080] *= np.float32(3e-12)
    y = ops.q4k_matvec(dev(q), dev(x), rows, cols).cpu().numpy()
    assert np.all(np.isfinite(y))
    q4k_rows_check(q, x, y, rows, cols, nsample=32, what="q4k tensor-core matvec, x over 1e-40..1e25")


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (64, 96), (1000, 2048), (999, 256), (513, 7168), (64, 8192),
                                       (3, 1280)])
def test_q8_0_matvec_sizes(rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    q = synth.make_q8_0(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = ops.q8_0_matvec(dev(q), dev(x), rows, cols).cpu().numpy()
    ref = O.q80_matvec(q, x.astype(np.float64), rows, cols)
    w = O.q80_dequant(q, 0, rows * cols)
    assert np.all(np.abs(y - ref) <= 1e-3 * absdot(w, x, rows, cols))
    normwise(y, ref, f"q8_0 matvec {rows}x{cols}")


@pytest.mark.parametrize("ntok", [1, 3, 8, 13])
def test_q4k_matmul_batch_fp32(ntok):
    rows, cols = 384, 1408
    rng = np.random.default_rng(ntok)
    q = synth.make_q4k(rng, rows * cols)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    y = ops.q4k_matmul_batch(dev(q), dev(x), rows, cols).cpu().numpy()
    ref = O.q4k_matmul(q, x.astype(np.float64), rows, cols)
    w = O.q4k_dequant(q, 0, rows * cols).reshape(rows, cols)
    bound = np.abs(x.astype(np.float64)) @ np.abs(w).T
    assert np.all(np.abs(y - ref) <= 1e-3 * bound)
    for t in range(ntok):
        normwise(y[t], ref[t], f"q4k batch fp32 token {t}/{ntok}")


def test_small_routers_golden():
    g = np.load(os.path.join(G, "route_golden.npz"))
    for t in ("e64", "e256"):
        ne, nsel, ng, tg = (int(v) for v in g[t + "_dims"])
        L = dev(g[t + "_logits"])
        ids, w = ops.route_softmax(L, nsel, renorm=True)
        assert np.array_equal(ids.cpu().numpy(), g[t + "_mm_ids"])
        assert np.allclose(w.cpu().numpy(), g[t + "_mm_wn"], rtol=1e-5, atol=1e-7)
        ids, w = ops.route_dsv4(L, dev(g[t + "_bias"]), nsel, 2.5)
        ok = np.array_equal(ids.cpu().numpy(), g[t + "_dr_ids"])
        assert ok
        assert np.allclose(w.cpu().numpy(), g[t + "_dr_w"], rtol=1e-5, atol=1e-6)


def test_bounded_wait_gives_up_and_reports():
    """A device wait that can never complete (an mbarrier nothing arrives on) gives up after its
    limit, records its code in the error word the host reads, and returns; the context stays usable."""
    from coherence_kernel_b200 import _lib
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    limit = 2_000_000  # 2 ms
    _lib.check(_lib.load().ck_wait_selftest(limit, err.data_ptr(), waited.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream), "ck_wait_selftest")
    torch.cuda.synchronize()
    assert int(err.item()) == 77
    assert limit <= int(waited.item()) < 200 * limit
    # the next launch on the same context runs normally
    f = np.load(os.path.join(G, "ref_fixtures.npz"))
    w = ops.q8_0_dequant(dev(f["q80"]), 0, 96).cpu().numpy()
    assert np.array_equal(w, f["w8"].astype(np.float32))


@pytest.mark.parametrize("rows,cols,n", [(7168, 7168, 3), (7168, 7168, 4), (4096, 11008, 2), (1024, 2048, 3)])
def test_q4k_matvec_group_equals_single_calls(rows, cols, n):
    """ck_q4k_matvec_f32_group: several matrices against one x in one launch (tensor-core shapes) or
    one after another (small ones); every y bit-identical to its own ck_q4k_matvec_f32."""
    rng = np.random.default_rng(rows + cols + n)
    qs = [torch.from_numpy(synth.make_q4k(rng, rows * cols)).cuda() for _ in range(n)]
    x = torch.from_numpy(rng.standard_normal(cols).astype(np.float32)).cuda()
    ys = ops.q4k_matvec_group(qs, x, rows, cols)
    torch.cuda.synchronize()
    for q, y in zip(qs, ys):
        assert torch.equal(y, ops.q4k_matvec(q, x, rows, cols))
