"""Every kernel name the handle door registers, dispatched the way a Form cell dispatches it
(metal_pipeline / md-bind / metal_enqueue / metal_sync / metal_buf_read), against the oracle.

Argument layouts are the reference's MSL signatures (buffers in [[buffer(i)]] order, then the
constants).  Bars, per name:
  dequant            Q8_0 bit-exact; Q4_K within one rounding u*|w| (q4k-msl.fk:20-28)
  attestant          the reference's derived bound (cols + ceil(cols/p) + p) * u * sum|w x| at p = 1
  part / hoist       bit-equal to the attestant at one part; at p parts + form_part_combine_f32
                     within the bound at p (qk-matvec-split.fk:41-54)
  lane/slot/wide/batch  1e-3 * sum|w x| per row (fp32 accumulation)
  f16 matvec         (cols + 2) * u * sum|w x| (any fp32 summation order)
  routers            ids bit-exact with the fkwu-pinned goldens, weights within 1e-5 relative
  swiglu forms       1e-6 relative to the fp64 restatement of ln-silu (llama-numerics.fk:29-34)
  scale / axpy / f32 matvec / moe_reduce   bit-exact against the same fp32 operations in order
(u = 2^-24.)
"""
import os

import numpy as np
import pytest

from coherence_kernel_b200 import carrier, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
U = 2.0 ** -24


class Door:
    def __init__(self):
        self.handles = []

    def buf(self, arr=None, nbytes=None):
        nbytes = arr.nbytes if arr is not None else nbytes
        h = carrier.buf_alloc(nbytes)
        assert h > 0, carrier.status()
        if arr is not None:
            assert carrier.buf_write(h, 0, np.ascontiguousarray(arr).tobytes()) == nbytes
        self.handles.append(h)
        return h

    def run(self, name, bufs, consts, threads):
        p = carrier.pipeline("", name)
        assert p > 0, carrier.status()
        assert carrier.enqueue(p, carrier.md_bind(bufs, consts), threads) == 1, carrier.status()
        assert carrier.sync() == 1

    def read(self, h, n, dtype=np.float32):
        return np.frombuffer(carrier.buf_read(h, 0, n * np.dtype(dtype).itemsize), dtype=dtype).copy()

    def close(self):
        for h in self.handles:
            assert carrier.buf_free(h) == 1


@pytest.fixture
def door(cuda_lib):
    d = Door()
    yield d
    d.close()


@pytest.mark.parametrize("kind", ["q8_0", "q4k"])
def test_quant_matvec_names(door, kind):
    rows, cols, ntok, parts = 96, 1024, 3, 6
    rng = np.random.default_rng(5 if kind == "q8_0" else 6)
    if kind == "q8_0":
        q = synth.make_q8_0(rng, rows * cols)
        w = O.q80_dequant(q, 0, rows * cols).reshape(rows, cols)
    else:
        q = synth.make_q4k(rng, rows * cols)
        w = O.q4k_dequant(q, 0, rows * cols).reshape(rows, cols)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    ref = x.astype(np.float64) @ w.T
    absb = np.abs(x.astype(np.float64)) @ np.abs(w).T
    hq, hx = door.buf(q), door.buf(x)
    hw = door.buf(nbytes=rows * cols * 4)
    hy = door.buf(nbytes=ntok * rows * 4)
    hp = door.buf(nbytes=rows * parts * 4)
    # dequant of a range that starts inside a block
    off, n = 37, rows * cols - 100
    door.run(f"form_{kind}_dequant_f32", [hq, hw], [off, n], n)
    wd = door.read(hw, n).astype(np.float64)
    wr = w.reshape(-1)[off:off + n]
    if kind == "q8_0":
        assert np.array_equal(wd, wr.astype(np.float32).astype(np.float64))
    else:
        assert np.all(np.abs(wd - wr) <= U * np.abs(wr))
    # the attestant
    door.run(f"form_{kind}_matvec_f32", [hq, hx, hy], [rows, cols], rows)
    ya = door.read(hy, rows)
    assert np.all(np.abs(ya - ref[0]) <= (2 * cols + 1) * U * absb[0])
    # the lane / slot / wide forms
    fast = (["form_q8_0_matvec_lane_f32", "form_q8_0_matvec_wide_f32"] if kind == "q8_0" else
            ["form_q4k_matvec_lane_f32", "form_q4k_matvec_slot_f32", "form_q4k_matvec_slot4_f32"])
    for name in fast:
        door.run(name, [hq, hx, hy], [rows, cols], rows)
        assert np.all(np.abs(door.read(hy, rows) - ref[0]) <= 1e-3 * absb[0]), name
    if kind == "q4k":
        for name in ("form_q4k_matvec_part_f32", "form_q4k_matvec_hoist_f32"):
            door.run(name, [hq, hx, hp], [rows, cols, 1], rows)
            assert np.array_equal(door.read(hp, rows), ya), name
        door.run("form_q4k_matvec_part_f32", [hq, hx, hp], [rows, cols, parts], rows * parts)
        door.run("form_part_combine_f32", [hp, hy], [rows, parts], rows)
        chunk = -(-cols // parts)
        assert np.all(np.abs(door.read(hy, rows) - ref[0]) <= (cols + chunk + parts) * U * absb[0])
        door.run("form_q4k_matmul_batch_f32", [hq, hx, hy], [rows, cols, ntok], rows)
        yb = door.read(hy, ntok * rows).reshape(ntok, rows)
        assert np.all(np.abs(yb - ref) <= 1e-3 * absb)


def test_f16_matvec_name(door):
    rows, cols = 64, 640
    rng = np.random.default_rng(8)
    wh = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float16)
    x = rng.standard_normal(cols).astype(np.float32)
    w = np.array([[O.lib().ckr_f16(int(b)) for b in row] for row in wh.view(np.uint16)])
    x64 = x.astype(np.float64)  # named: the C call reads through its pointer
    ref = np.array([O.lib().ckr_dot(w[r].ctypes.data, x64.ctypes.data, cols) for r in range(rows)])
    hw, hx, hy = door.buf(wh), door.buf(x), door.buf(nbytes=rows * 4)
    door.run("form_f16_matvec_f32", [hw, hx, hy], [rows, cols], rows)
    y = door.read(hy, rows)
    assert np.all(np.abs(y - ref) <= (cols + 2) * U * (np.abs(w) @ np.abs(x.astype(np.float64))))


def test_router_names(door):
    g = np.load(os.path.join(G, "route_golden.npz"))
    for t in ("e64", "e256"):
        ne, nsel, _, _ = (int(v) for v in g[t + "_dims"])
        hb = door.buf(g[t + "_bias"].astype(np.float32))
        hi, hw = door.buf(nbytes=nsel * 4), door.buf(nbytes=nsel * 4)
        names = ["form_moe_route_wide_f32"] + (["form_moe_route_f32"] if ne <= 64 else [])
        for i in range(g[t + "_logits"].shape[0]):
            hl = door.buf(g[t + "_logits"][i].astype(np.float32))
            for name in names:
                door.run(name, [hl, hi, hw], [ne, nsel], 1)
                assert np.array_equal(door.read(hi, nsel, np.uint32), g[t + "_mm_ids"][i]), (name, i)
                assert np.allclose(door.read(hw, nsel), g[t + "_mm_wn"][i], rtol=1e-5, atol=1e-7)
            door.run("form_dsv4_router_f32", [hl, hb, hi, hw], [ne, nsel, carrier.f32_bits(2.5)], 1)
            assert np.array_equal(door.read(hi, nsel, np.uint32), g[t + "_dr_ids"][i]), i
            assert np.allclose(door.read(hw, nsel), g[t + "_dr_w"][i], rtol=1e-5, atol=1e-6)


def _silu64(v):
    return np.array([O.lib().ckr_silu(float(a)) for a in v])


def test_swiglu_names(door):
    n, nexp = 1000, 4
    rng = np.random.default_rng(9)
    gte = (rng.standard_normal(n * nexp) * 3).astype(np.float32)
    up = (rng.standard_normal(n * nexp) * 3).astype(np.float32)
    wts = rng.random(nexp).astype(np.float32)
    hg, hu = door.buf(gte), door.buf(up)
    ho, hwt = door.buf(nbytes=n * nexp * 4), door.buf(wts)
    g64, u64 = gte.astype(np.float64), up.astype(np.float64)
    # form_swiglu_f32: silu(g) * u
    door.run("form_swiglu_f32", [hg, hu, ho], [n], n)
    ref = _silu64(g64[:n]) * u64[:n]
    assert np.allclose(door.read(ho, n), ref, rtol=1e-6, atol=1e-30)
    # form_dsv4_swiglu_f32: (silu(min(g, lim)) * clamp(u, -lim, lim)) * w, and with the clamp off
    for lim in (0.0, 2.0):
        door.run("form_dsv4_swiglu_f32", [hg, hu, ho], [n, carrier.f32_bits(0.75), carrier.f32_bits(lim)], n)
        gg, uu = (np.minimum(g64[:n], lim), np.clip(u64[:n], -lim, lim)) if lim else (g64[:n], u64[:n])
        assert np.allclose(door.read(ho, n), _silu64(gg) * uu * 0.75, rtol=1e-6, atol=1e-30), lim
    # form_dsv4_swiglu_experts: expert slot e of [nexp, n], weighted by wts[e]
    door.run("form_dsv4_swiglu_experts", [hg, hu, ho, hwt], [n, nexp, carrier.f32_bits(0.0)], n * nexp)
    ref = (_silu64(g64) * u64).reshape(nexp, n) * wts.astype(np.float64)[:, None]
    assert np.allclose(door.read(ho, n * nexp).reshape(nexp, n), ref, rtol=1e-6, atol=1e-30)


def test_elementwise_and_reduce_names(door):
    n, nexp, rows, cols = 777, 5, 40, 300
    rng = np.random.default_rng(10)
    x = rng.standard_normal(n).astype(np.float32)
    y0 = rng.standard_normal(n).astype(np.float32)
    a = np.float32(0.3)
    hx, hy = door.buf(x), door.buf(y0)
    for name in ("form_scale_f32", "form_dsv4_scale_f32"):
        door.run(name, [hx, hy], [carrier.f32_bits(float(a)), n], n)
        assert np.array_equal(door.read(hy, n), a * x)
    for name in ("form_axpy_f32", "form_dsv4_axpy_f32"):
        carrier.buf_write(hy, 0, y0.tobytes())
        door.run(name, [hx, hy], [carrier.f32_bits(float(a)), n], n)
        assert np.array_equal(door.read(hy, n), y0 + a * x)
    # form_dsv4_moe_reduce: out[d] = parts[0][d] + parts[1][d] + ... in ascending slot order, fp32
    parts = rng.standard_normal((nexp, n)).astype(np.float32)
    hp, ho = door.buf(parts), door.buf(nbytes=n * 4)
    door.run("form_dsv4_moe_reduce", [hp, ho], [n, nexp], n)
    acc = np.zeros(n, dtype=np.float32)
    for e in range(nexp):
        acc = acc + parts[e]
    assert np.array_equal(door.read(ho, n), acc)
    # form_dsv4_matvec_f32: one thread per row, j counting down, acc = w*x + acc in fp32
    W = rng.standard_normal((rows, cols)).astype(np.float32)
    xv = rng.standard_normal(cols).astype(np.float32)
    hW, hxv, hyv = door.buf(W), door.buf(xv), door.buf(nbytes=rows * 4)
    door.run("form_dsv4_matvec_f32", [hW, hxv, hyv], [rows, cols], rows)
    acc = np.zeros(rows, dtype=np.float32)
    for j in range(cols - 1, -1, -1):
        acc = (W[:, j] * xv[j]) + acc
    assert np.array_equal(door.read(hyv, rows), acc)
