"""Compile the Form driver cells into self-contained fkwu program images (.fkb + .sym) over a
temporary writable copy of the reference's Form stdlib.  An image only loads in the binary that
wrote it, so the oracle's cells (oracle/fk/*.fk) are compiled by the reference runtime
(oracle/_ref/fkwu) into oracle/_ref/fk/, and the door cells (tests/fk/*.fk) by the same runtime
linked with the CUDA carrier (oracle/_ref/fkwu-cuda) into oracle/_ref/fk-cuda/.  The images run
without the reference tree, so they travel with the repository to a machine that has none.  Test
infrastructure only.

    python oracle/build_images.py --ref <the reference tree>   (or CK_REFERENCE=<tree>)
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


PRELUDES = ("ck_io.fk", "ck_group_route.fk")  # prelude cells, not programs


def _compile(binary: str, cells: list, out_dir: str, ref: str) -> list:
    os.makedirs(out_dir, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="ck_images_")
    built = []
    try:
        form = os.path.join(tmp, "form")
        shutil.copytree(os.path.join(ref, "form", "form-stdlib"), os.path.join(form, "form-stdlib"))
        os.makedirs(os.path.join(form, "ck"))
        os.makedirs(os.path.join(form, "ck_in"))
        for f in PRELUDES:
            shutil.copy(os.path.join(HERE, "fk", f), os.path.join(form, "ck", f))
        for path in cells:
            shutil.copy(path, os.path.join(form, "ck", os.path.basename(path)))
        for path in cells:
            f = os.path.basename(path)
            p = subprocess.run([binary, f"ck/{f}"], cwd=form, capture_output=True, text=True, timeout=600)
            if " error(s)" in p.stderr and "0 error(s)" not in p.stderr:
                raise RuntimeError(f"{f} does not compile cleanly:\n{p.stderr[-3000:]}")
            stem = f[:-3]
            for ext in (".fkb", ".sym"):
                shutil.copy(os.path.join(form, "ck", stem + ext), os.path.join(out_dir, stem + ext))
            built.append(stem)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return built


def build(ref: str) -> list:
    fkwu = os.path.join(HERE, "_ref", "fkwu")
    if not os.path.exists(fkwu):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)
    oracle_cells = [os.path.join(HERE, "fk", f) for f in sorted(os.listdir(os.path.join(HERE, "fk")))
                    if f.endswith(".fk") and f not in PRELUDES]
    built = _compile(fkwu, oracle_cells, os.path.join(HERE, "_ref", "fk"), ref)
    fkwu_cuda = os.path.join(HERE, "_ref", "fkwu-cuda")
    if os.path.exists(fkwu_cuda):
        door = os.path.join(REPO, "tests", "fk")
        door_cells = [os.path.join(door, f) for f in sorted(os.listdir(door)) if f.endswith(".fk")]
        built += [c + " (cuda)" for c in _compile(fkwu_cuda, door_cells, os.path.join(HERE, "_ref", "fk-cuda"), ref)]
    return built


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CK_REFERENCE"))
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref <the reference tree> (or CK_REFERENCE) is required")
    print("images:", build(a.ref))
