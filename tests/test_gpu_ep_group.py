"""The expert-parallel layer driven by one process over two GPUs (ck_ep_group_*), directly through
the C ABI and through the handle door as the pipeline `ck_moe_layer_ep_bf16`: outputs, ids, weights
and per-expert counts equal the single-GPU layer's bit for bit (each (token, slot) row is computed
by the same kernels, and the combine reads the rows in the reference's order), at a decode-sized
batch (the few-token expert matvec on both sides) and a prefill-sized one (the grouped GEMM).

Needs two GPUs; skipped otherwise."""
import ctypes

import numpy as np
import pytest
import torch

from coherence_kernel_b200 import _lib, carrier, workloads
from coherence_kernel_b200.moe import MoELayer, MoeSpec
from coherence_kernel_b200.ops import _ptr

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

SPECS = {"dsv4": MoeSpec(1024, 512, 16, 1, 4, 4, 4, 2, 2.5), "softmax": MoeSpec(1024, 768, 8, 2, 3, 3)}


def weights(spec, ntok, seed):
    w = workloads.make_moe(spec, ntok, seed=seed)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    return w, {k: t(w[k]) for k in ("gate", "up", "down", "s_gate", "s_up", "s_down", "router", "bias")}, \
        t(w["x"].view(np.int16))


def single(spec, d, x):
    lay = MoELayer(spec, d["gate"], d["up"], d["down"], d["s_gate"], d["s_up"], d["s_down"], d["router"], d["bias"],
                   max_tokens=x.shape[0])
    out, ids, wts, counts = lay(x)
    lay.status(x.shape[0])
    return out, ids, wts, counts


@pytest.mark.parametrize("name", sorted(SPECS))
@pytest.mark.parametrize("ntok", [16, 512])
def test_ep_group_equals_single_gpu(name, ntok):
    spec = SPECS[name]
    torch.cuda.set_device(0)
    _, d, x = weights(spec, ntok, seed=21)
    ref = single(spec, d, x)
    L = _lib.load()
    cfg = spec.cfg()
    devs = (ctypes.c_int * 2)(0, 1)
    g = L.ck_ep_group_create(ctypes.byref(cfg), 2, devs, (ntok + 1) // 2)
    assert g
    try:
        _lib.check(L.ck_ep_group_load(g, *[_ptr(d[k]) for k in ("gate", "up", "down", "s_gate", "s_up", "s_down",
                                                                 "router", "bias")]), "ck_ep_group_load")
        for _ in range(2):  # a second forward: the barriers' step counters move on
            out = torch.empty_like(ref[0])
            ids, wts, counts = torch.empty_like(ref[1]), torch.empty_like(ref[2]), torch.empty_like(ref[3])
            _lib.check(L.ck_ep_group_forward(g, _ptr(x), ntok, _ptr(ids), _ptr(wts), _ptr(counts), _ptr(out),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                       "ck_ep_group_forward")
            _lib.check(L.ck_ep_group_status(g), "ck_ep_group_status")
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int16), ref[0].view(torch.int16))
            assert torch.equal(ids, ref[1]) and torch.equal(wts, ref[2]) and torch.equal(counts, ref[3])
    finally:
        L.ck_ep_group_destroy(g)


def test_ep_layer_through_the_door():
    """ck_moe_layer_ep_bf16 (14 buffers, 12 constants: ck_moe_layer_bf16's plus world) against
    ck_moe_layer_bf16 through the same door, bit for bit."""
    spec, ntok = SPECS["dsv4"], 64
    torch.cuda.set_device(0)
    w, _, _ = weights(spec, ntok, seed=22)
    cfg = spec.cfg()
    ws = _lib.load().ck_moe_workspace_bytes(ctypes.byref(cfg), ntok)
    bufs = [carrier.buf_alloc(int(np.ascontiguousarray(w[k]).nbytes)) for k in
            ("x", "gate", "up", "down", "s_gate", "s_up", "s_down", "router", "bias")]
    for h, k in zip(bufs, ("x", "gate", "up", "down", "s_gate", "s_up", "s_down", "router", "bias")):
        assert carrier.buf_write(h, 0, np.ascontiguousarray(w[k]).tobytes()) > 0
    K, H, E = spec.nsel, spec.hidden, spec.n_experts
    consts = [spec.hidden, spec.inter, E, spec.n_shared, K, spec.mode, spec.ngroups, spec.topk_groups,
              carrier.f32_bits(spec.wscale), carrier.f32_bits(spec.tau), ntok]
    results = {}
    for name, extra in (("ck_moe_layer_bf16", []), ("ck_moe_layer_ep_bf16", [2])):
        outs = [carrier.buf_alloc(n) for n in (ntok * K * 4, ntok * K * 4, E * 4, ntok * H * 2, ws)]
        p = carrier.pipeline("", name)
        assert p > 0, carrier.status()
        assert carrier.enqueue(p, carrier.md_bind(bufs + outs, consts + extra), ntok) == 1, carrier.status()
        assert carrier.sync() == 1
        results[name] = [carrier.buf_read(h, 0, n) for h, n in zip(outs[:4], (ntok * K * 4, ntok * K * 4, E * 4,
                                                                               ntok * H * 2))]
        for h in outs:
            carrier.buf_free(h)
    assert results["ck_moe_layer_bf16"] == results["ck_moe_layer_ep_bf16"]
    for h in bufs:
        carrier.buf_free(h)
