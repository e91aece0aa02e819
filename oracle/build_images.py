"""Compile the Form driver cells (oracle/fk/*.fk, tests/fk/*.fk) into self-contained fkwu program
images (.fkb + .sym) under oracle/_ref/fk/, using the reference runtime (oracle/_ref/fkwu) over a
temporary writable copy of the reference's Form stdlib.  The images run without the reference tree,
so they travel with the repository to a machine that has none.  Test infrastructure only.

    python oracle/build_images.py [--ref /root/reference]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def build(ref: str) -> list:
    fkwu = os.path.join(HERE, "_ref", "fkwu")
    if not os.path.exists(fkwu):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)
    out_dir = os.path.join(HERE, "_ref", "fk")
    os.makedirs(out_dir, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="ck_images_")
    built = []
    try:
        form = os.path.join(tmp, "form")
        shutil.copytree(os.path.join(ref, "form", "form-stdlib"), os.path.join(form, "form-stdlib"))
        os.makedirs(os.path.join(form, "ck"))
        os.makedirs(os.path.join(form, "ck_in"))
        cells = []
        for d in (os.path.join(HERE, "fk"), os.path.join(REPO, "tests", "fk")):
            for f in sorted(os.listdir(d)):
                if f.endswith(".fk"):
                    shutil.copy(os.path.join(d, f), os.path.join(form, "ck", f))
                    cells.append(f)
        for f in cells:
            if f in ("ck_io.fk", "ck_group_route.fk"):
                continue  # preludes, not programs
            p = subprocess.run([fkwu, f"ck/{f}"], cwd=form, capture_output=True, text=True, timeout=600)
            if " error(s)" in p.stderr and "0 error(s)" not in p.stderr:
                raise RuntimeError(f"{f} does not compile cleanly:\n{p.stderr[-3000:]}")
            stem = f[:-3]
            for ext in (".fkb", ".sym"):
                shutil.copy(os.path.join(form, "ck", stem + ext), os.path.join(out_dir, stem + ext))
            built.append(stem)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return built


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    print("images:", build(ap.parse_args().ref))
