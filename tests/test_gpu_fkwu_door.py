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
