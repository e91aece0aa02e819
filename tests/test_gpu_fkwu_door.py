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


def _gguf_case(tmp_path, raw_file: bytes, align=32):
    inp = tmp_path / "ck_in"
    inp.mkdir(exist_ok=True)
    (inp / "model.gguf").write_bytes(raw_file)
    np.array([len(raw_file), align], dtype=np.uint32).tofile(inp / "gguf_meta.bin")
    return _run_cell("ck_door_gguf", tmp_path)


def test_gguf_ingest_through_the_door(tmp_path):
    """GGUF ingest: a Form cell walks a model file's tensor table with the reference's egg-* recipes,
    binds every tensor's bytes in HBM with metal_buf_from_file at its absolute offset, and dequantizes
    it on the device through the door (Q4_K, Q6_K, Q8_0; F32 read back); the device weights equal the
    Form recipes' decode of the same file bytes (Q6_K, Q8_0 and F32 bit for bit, Q4_K within one
    rounding), and the table agrees with the host reader coherence_kernel_b200.gguf."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from gguf_file import write_gguf
    from coherence_kernel_b200 import gguf
    rng = np.random.default_rng(40)
    g6 = np.load(os.path.join(REPO, "tests", "golden", "q6k_golden.npz"))
    ts = [("blk.0.ffn_gate.weight", (256, 2), 12, synth.make_q4k(rng, 512).tobytes()),
          ("token_embd.weight", (256, 2), 14, np.concatenate([g6["band_sb"], synth.make_q6k(rng, 256)]).tobytes()),
          ("blk.0.attn_q.weight", (64, 2), 8, synth.make_q8_0(rng, 128).tobytes()),
          ("blk.0.ffn_gate_inp.weight", (8, 3), 0, rng.standard_normal(24).astype(np.float32).tobytes())]
    path = tmp_path / "written.gguf"
    write_gguf(str(path), ts, kv={"general.architecture": "llama"})
    table, base, _ = gguf.read_table(str(path))
    live, ok, ntens, start, dbase, tensors = _gguf_case(tmp_path, path.read_bytes())
    assert live in (1, True) and ok == 1 and ntens == len(ts) and dbase == base
    for (name, dims, t, raw), row in zip(ts, tensors):
        nlen, rt, nd, d0, d1, off, nbytes, h, gpu, form = row
        assert (nlen, rt, nd, d0, d1) == (len(name), t, 2, dims[0], dims[1])
        assert off == table[name].offset and nbytes == table[name].nbytes == len(raw) and h > 0
        gpu, form = np.array(gpu, dtype=np.float64), np.array(form, dtype=np.float64)
        if t == 12:
            assert np.all(np.abs(gpu - form) <= 2.0 ** -24 * np.abs(form)), name
        else:
            assert np.array_equal(gpu, form.astype(np.float32).astype(np.float64)), name


def test_reference_mini_gguf_through_the_door(tmp_path):
    """The reference's own mini-GGUF (weight-load-q4k-band.fk): tensor info at byte 41, data base 96,
    one Q4_K superblock bound in HBM through the door and dequantized there; the band's weight pins
    hold on the device values."""
    g = np.load(os.path.join(REPO, "tests", "golden", "gguf_golden.npz"))
    live, ok, ntens, start, dbase, tensors = _gguf_case(tmp_path, g["band_gguf"].tobytes())
    assert ok == 1 and ntens == 1 and start == int(g["band_tinfo_start"]) and dbase == 96
    (nlen, t, nd, d0, d1, off, nbytes, h, gpu, form), = tensors
    assert t == 12 and d0 == 256 and off == 96 and nbytes == 144
    gpu = np.array(gpu, dtype=np.float64)
    for i, v in g["band_pins"]:
        assert round(gpu[i] * 1e6) == v, (i, gpu[i])
