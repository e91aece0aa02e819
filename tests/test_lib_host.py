"""Host-side checks that need no GPU: the library loads, exports every declared symbol, and the
handle door answers honestly when no device is present."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from coherence_kernel_b200 import _lib, synth

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("ck_b200.h", "fk_cuda_carrier.h"):
        src = open(os.path.join(REPO, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b((?:ck|fk)_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(cuda_lib):
    names = declared_symbols()
    assert len(names) >= 40
    for n in names:
        assert hasattr(cuda_lib, n), n
    assert names <= set(_lib.SIGNATURES), names - set(_lib.SIGNATURES)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answers")
def test_door_without_device_answers_unlinked(cuda_lib):
    buf = ctypes.create_string_buffer(4096)
    n = cuda_lib.fk_metal_status_external(buf, 4096)
    text = buf.raw[:n].decode()
    assert "metal_linked=false" in text and "metal_door=handle" in text
    assert cuda_lib.fk_metal_buf_alloc_external(64) == 0   # never a live handle
    assert cuda_lib.ck_device_ok() == 0


def test_workspace_sizing_is_host_only(cuda_lib):
    cfg = _lib.MoeConfig(7168, 2048, 256, 1, 8, 4, 8, 4, 2.5, 1e-4)
    ws = cuda_lib.ck_moe_workspace_bytes(ctypes.byref(cfg), 8192)
    A, R = 8192 * 8, 8192 * 9
    assert ws > (A + 8192) * 7168 * 2 + R * 7168 * 2 + R * 2048 * 2
    bad = _lib.MoeConfig(7168, 2048, 300, 1, 8, 4, 8, 4, 2.5, 1e-4)   # more than 256 experts
    assert cuda_lib.ck_moe_workspace_bytes(ctypes.byref(bad), 8192) == 0


def test_synth_q4k_scale_packing_roundtrip():
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    sc = rng.integers(0, 64, size=(64, 8))
    mn = rng.integers(0, 64, size=(64, 8))
    packed = synth.pack_q4k_scales(sc, mn)
    blk = np.zeros((64, 144), dtype=np.uint8)
    blk[:, 4:16] = packed
    flat = blk.reshape(-1)
    for b in range(64):
        for j in range(8):
            s, m, _ = O.q4k_codes(flat, b * 256 + j * 32)
            assert (s, m) == (sc[b, j], mn[b, j])


def test_synth_bf16_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-3], dtype=np.float32)
    b = synth.f32_to_bf16_bits(x)
    back = synth.bf16_bits_to_f32(b)
    ref = torch.tensor(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(back, ref)


def test_decode_step_create_and_destroy_on_the_host(cuda_lib):
    """ck_decode_step_create only records pointers and carves the workspace (no device work), so its
    argument list, its refusals and ck_decode_step_destroy are checked here without a GPU."""
    import ctypes

    from coherence_kernel_b200 import _lib, workloads
    L = _lib.load()
    cfg = _lib.DecodeConfig(7168, 16, 1e-6, workloads.MOE_DSV3.cfg())
    need = L.ck_decode_step_workspace_bytes(ctypes.byref(cfg))
    assert need > 0
    fake = [ctypes.c_void_p(0x10000 * (i + 1)) for i in range(15)]
    h = L.ck_decode_step_create(ctypes.byref(cfg), *fake[:14], fake[14], need)
    assert h
    L.ck_decode_step_destroy(h)
    assert not L.ck_decode_step_create(ctypes.byref(cfg), *fake[:14], fake[14], need - 1)   # short workspace
    assert not L.ck_decode_step_create(ctypes.byref(cfg), None, *fake[1:14], fake[14], need)  # missing weight
    bad = _lib.DecodeConfig(7000, 16, 1e-6, workloads.MOE_DSV3.cfg())
    assert L.ck_decode_step_workspace_bytes(ctypes.byref(bad)) == 0                          # hidden mismatch
    assert L.ck_decode_step_replay(None, None) == -3


def test_workspaces_grow_with_the_batch():
    """A workspace sized for a batch must hold every smaller batch (callers size it once for their
    largest): the route's and the layer's byte counts never fall as ntok grows, across the decode
    sizes, the split-K router sizes and beyond."""
    import ctypes
    from coherence_kernel_b200 import _lib, workloads
    L = _lib.load()
    for spec in (workloads.MOE_DSV3, workloads.MOE_SMALL):
        cfg = spec.cfg()
        for fn in (L.ck_moe_route_workspace_bytes, L.ck_moe_workspace_bytes):
            prev = 0
            for n in list(range(1, 5200, 13)) + [8192, 16384]:
                b = fn(ctypes.byref(cfg), n)
                assert b >= prev, (spec, n)
                prev = b
