"""The drop-in: the reference's own runtime (fkwu, compiled from runtime/fkwu-uni.c) linked with the
CUDA carrier, running a Form cell that drives the handle door the way the reference's Metal cells
do (tests/fk/ck_door_q4k.fk), on a B200.

The runtime binary and the cell's program image are built where the reference tree is present
(__graft_entry__.build -> oracle/Makefile ref-cuda, oracle/build_images.py) and travel with the
repository as untracked build outputs.
"""
import ast
import os
import subprocess

import numpy as np
import pytest

from coherence_kernel_b200 import synth

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FKWU_CUDA = os.path.join(REPO, "oracle", "_ref", "fkwu-cuda")
IMAGE = os.path.join(REPO, "oracle", "_ref", "fk-cuda", "ck_door_q4k.fkb")


@pytest.mark.skipif(not (os.path.exists(FKWU_CUDA) and os.path.exists(IMAGE)),
                    reason="the reference runtime linked with the carrier was not built (no reference tree)")
@pytest.mark.parametrize("rows,cols", [(8, 256), (6, 384)])
def test_form_cell_drives_the_cuda_door(tmp_path, rows, cols):
    rng = np.random.default_rng(rows * cols)
    inp = tmp_path / "ck_in"
    inp.mkdir()
    np.array([rows, cols], dtype=np.uint32).tofile(inp / "meta.bin")
    q = synth.make_q4k(rng, rows * cols)
    q.tofile(inp / "q4.bin")
    x = rng.standard_normal(cols).astype(np.float32)
    x.tofile(inp / "x4.bin")
    p = subprocess.run([FKWU_CUDA, IMAGE], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("[")][-1]
    live, hq, hx, hy, pipe, enq, synced, gpu, form = ast.literal_eval(
        line.replace("true", "True").replace("false", "False"))
    assert live in (1, True), p.stdout
    assert hq > 0 and hx > 0 and hy > 0 and pipe > 0
    assert enq == 1 and synced == 1
    gpu, form = np.array(gpu), np.array(form)
    # form_q4k_matvec_f32 is the attestant order: within the reference's derived bound
    # (cols + ceil(cols/p) + p) * 2^-24 * sum|w x| at p = 1 (qk-matvec-split.fk:41-54)
    from oracle import oracle as O
    w = O.q4k_dequant(q, 0, rows * cols).reshape(rows, cols)
    bound = (2 * cols + 1) * 2.0 ** -24 * (np.abs(w) @ np.abs(x.astype(np.float64)))
    assert np.all(np.abs(gpu - form) <= bound)


def _run_cell(stem, cwd):
    image = os.path.join(REPO, "oracle", "_ref", "fk-cuda", stem + ".fkb")
    if not (os.path.exists(FKWU_CUDA) and os.path.exists(image)):
        pytest.skip("the reference runtime linked with the carrier was not built (no reference tree)")
    p = subprocess.run([FKWU_CUDA, image], cwd=cwd, capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stderr[-2000:]
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("[")][-1]
    return ast.literal_eval(line.replace("true", "True").replace("false", "False"))


@pytest.mark.parametrize("mode", [3, 4])
def test_form_cell_runs_the_moe_layer_through_the_door(tmp_path, mode):
    """The batched MoE layer as one enqueue of ck_moe_layer_bf16 from a Form cell on the reference
    runtime (14 buffers, 11 constants): ids and counts bit-exact with the oracle's routing, outputs
    within 2e-2 per token against the oracle's layer."""
    from coherence_kernel_b200 import _lib, carrier, workloads
    from coherence_kernel_b200.moe import MoeSpec
    spec = (MoeSpec(512, 256, 16, 1, 4, 4, 4, 2, 2.5) if mode == 4 else MoeSpec(512, 384, 8, 2, 3, 3))
    ntok = 12
    w = workloads.make_moe(spec, ntok, seed=31 + mode)
    inp = tmp_path / "ck_in"
    inp.mkdir()
    for k, f in (("x", "x.bin"), ("gate", "wg.bin"), ("up", "wu.bin"), ("down", "wd.bin"), ("s_gate", "sg.bin"),
                 ("s_up", "su.bin"), ("s_down", "sd.bin"), ("router", "router.bin"), ("bias", "bias.bin")):
        np.ascontiguousarray(w[k]).tofile(inp / f)
    cfg = spec.cfg()
    import ctypes
    ws = _lib.load().ck_moe_workspace_bytes(ctypes.byref(cfg), ntok)
    consts = [spec.hidden, spec.inter, spec.n_experts, spec.n_shared, spec.nsel, spec.mode, spec.ngroups,
              spec.topk_groups, carrier.f32_bits(spec.wscale), carrier.f32_bits(spec.tau), ntok]
    sizes = [w["x"].nbytes, w["gate"].nbytes, w["s_gate"].nbytes, w["router"].nbytes, w["bias"].nbytes, ws]
    np.array(consts + sizes + [0, 0, 0], dtype=np.uint32).tofile(inp / "moe_meta.bin")
    live, pipe, enq, synced, ids, counts, out = _run_cell("ck_door_moe", tmp_path)
    assert live in (1, True) and pipe > 0 and enq == 1 and synced == 1
    from oracle import oracle as O
    ocfg = O.moe_cfg(spec.hidden, spec.inter, spec.n_experts, spec.n_shared, spec.nsel, spec.mode, spec.ngroups,
                     spec.topk_groups, spec.wscale)
    rids, _, rout = O.moe_layer(ocfg, w, w["x"], np.arange(ntok))
    assert np.array_equal(np.array(ids).reshape(ntok, spec.nsel), rids)
    assert np.array_equal(np.array(counts), np.bincount(rids.reshape(-1), minlength=spec.n_experts))
    out = np.array(out).reshape(ntok, spec.hidden)
    for t in range(ntok):
        assert np.abs(out[t] - rout[t]).max() <= 2e-2 * np.abs(rout[t]).max(), t


@pytest.mark.parametrize("rows,cols,ntok", [(256, 512, 20), (256, 512, 3)])
def test_form_cell_runs_the_prefill_gemm_through_the_door(tmp_path, rows, cols, ntok):
    """The tensor-core Q4_K GEMM as one enqueue of ck_q4k_gemm_bf16 from a Form cell (the dequantizing
    GEMM at 20 tokens, the few-token tensor-core matvec at 3): within 2e-2 of sum |w x| per output."""
    from coherence_kernel_b200 import _lib
    rng = np.random.default_rng(rows + ntok)
    q = synth.make_q4k(rng, rows * cols)
    xb = synth.make_bf16(rng, (ntok, cols))
    inp = tmp_path / "ck_in"
    inp.mkdir()
    q.tofile(inp / "q4.bin")
    xb.tofile(inp / "xb.bin")
    ws = _lib.load().ck_q4k_gemm_workspace_bytes(ntok)
    np.array([rows, cols, ntok, ws], dtype=np.uint32).tofile(inp / "gemm_meta.bin")
    live, pipe, enq, synced, y = _run_cell("ck_door_gemm", tmp_path)
    assert live in (1, True) and pipe > 0 and enq == 1 and synced == 1
    from oracle import oracle as O
    w = O.q4k_dequant(q, 0, rows * cols).reshape(rows, cols)
    x64 = synth.bf16_bits_to_f32(xb).astype(np.float64)
    ref = x64 @ w.T
    y = np.array(y).reshape(ntok, rows)
    assert np.all(np.abs(y - ref) <= 2e-2 * (np.abs(x64) @ np.abs(w).T))
