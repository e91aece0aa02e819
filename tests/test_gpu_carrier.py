"""The handle door (fk_metal_*_external) through the C ABI, as a Form cell drives it (GPU).

Mirrors the reference's carrier contract (form/native/metal/fk-metal-carrier.m): handles with
generations, the three legal binding lengths, enqueue without waiting, sync counts, reads that
are all-or-nothing, refusals that speak through metal_status.
"""
import ctypes
import struct

import numpy as np
import pytest

from coherence_kernel_b200 import carrier, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_status_canary(cuda_lib):
    st = carrier.status()
    assert "metal_linked=true" in st and "metal_door=handle" in st


def test_q4k_matvec_through_the_door(cuda_lib, tmp_path):
    rows, cols = 96, 1408
    rng = np.random.default_rng(11)
    q = synth.make_q4k(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    path = tmp_path / "w.bin"
    pad = b"\x00" * 100
    path.write_bytes(pad + q.tobytes())
    hq = carrier.buf_from_file(str(path), 100, q.nbytes)
    hx = carrier.buf_alloc(cols * 4)
    hy = carrier.buf_alloc(rows * 4)
    assert hq and hx and hy
    assert carrier.buf_write(hx, 0, x.tobytes()) == cols * 4
    for name in ("form_q4k_matvec_f32", "form_q4k_matvec_lane_f32"):
        p = carrier.pipeline("// msl text kept for identity", name)
        assert p > 0, carrier.status()
        assert carrier.pipeline("// msl text kept for identity", name) == p   # same text + name = same handle
        assert carrier.enqueue(p, carrier.md_bind([hq, hx, hy], [rows, cols]), rows) == 1
        assert carrier.sync() == 1
        y = np.frombuffer(carrier.buf_read(hy, 0, rows * 4), dtype=np.float32)
        ref = O.q4k_matvec(q, x.astype(np.float64), rows, cols)
        w = O.q4k_dequant(q, 0, rows * cols).reshape(rows, cols)
        assert np.all(np.abs(y - ref) <= 1e-3 * (np.abs(w) @ np.abs(x)))
    # stale handles are refused after free
    assert carrier.buf_free(hy) == 1
    assert carrier.enqueue(p, carrier.md_bind([hq, hx, hy], [rows, cols]), rows) == -1
    assert "bad buffer handle" in carrier.status()
    for h in (hq, hx):
        assert carrier.buf_free(h) == 1


def test_binding_refusals(cuda_lib):
    hq = carrier.buf_alloc(144 * 4)
    hx = carrier.buf_alloc(256 * 4)
    hy = carrier.buf_alloc(4 * 4)
    p = carrier.pipeline("", "form_q4k_matvec_lane_f32")
    good = carrier.md_bind([hq, hx, hy], [4, 256])
    assert carrier.enqueue(p, good + b"\x00\x00\x00\x00", 4) == -1          # a length between the legal three
    assert "binding is" in carrier.status()
    assert carrier.enqueue(p, good[:-4], 4) == -1                           # truncated
    assert carrier.enqueue(p, carrier.md_bind([hq, hx, hy], [4, 256], tail=(0, 0, 0, 1)), 4) == -1
    assert "barrier_before is only legal in a concurrent batch" in carrier.status()
    assert carrier.enqueue(p, carrier.md_bind([hq, hx, hy], [8, 256]), 8) == -1   # y too small for 8 rows
    assert "needs" in carrier.status()
    assert carrier.enqueue(p, good, 0) == -1                                # threads must be positive
    assert carrier.pipeline("", "no_such_kernel") == 0
    # a concurrent batch accepts barrier_before; submit / fence_wait answer the dispatch count
    assert carrier.batch_concurrent() == 1
    assert carrier.enqueue(p, carrier.md_bind([hq, hx, hy], [4, 256], tail=(0, 0, 0, 1)), 4) == 1
    assert carrier.enqueue(p, good, 4) == 1
    f = carrier.submit()
    assert f > 0
    assert carrier.fence_wait(f) == 2
    assert carrier.fence_wait(f) == 0                                        # already drained
    assert carrier.buf_read(hy, 0, 8, cap=4) is None                        # len > cap: refused, no short read
    for h in (hq, hx, hy):
        assert carrier.buf_free(h) == 1


def test_routers_through_the_door(cuda_lib):
    logits = np.array([[0.1, 2.0, -1.0, 2.0, 0.5, 0.0, 1.5, -0.2]], dtype=np.float32)
    hl = carrier.buf_alloc(32)
    hi = carrier.buf_alloc(8)
    hw = carrier.buf_alloc(8)
    carrier.buf_write(hl, 0, logits.tobytes())
    p = carrier.pipeline("", "form_moe_route_f32")
    assert carrier.enqueue(p, carrier.md_bind([hl, hi, hw], [8, 2]), 1) == 1
    ids = np.frombuffer(carrier.buf_read(hi, 0, 8), dtype=np.uint32)
    ref_ids, ref_w = O.route_softmax(logits[0].astype(np.float64), 2, True)
    assert list(ids) == list(ref_ids) == [1, 3]                            # tie: the lower index first
    w = np.frombuffer(carrier.buf_read(hw, 0, 8), dtype=np.float32)
    assert np.allclose(w, ref_w, rtol=1e-6)
    for h in (hl, hi, hw):
        carrier.buf_free(h)
