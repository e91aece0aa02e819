"""Build the sm_100a shared library (libck_b200.so) and the carrier archive, in-tree.

    python -m coherence_kernel_b200.build [--force]

Every .cu under csrc/ is compiled with nvcc for sm_100a only; the objects are linked into
coherence_kernel_b200/libck_b200.so (the C ABI of include/ck_b200.h and include/fk_cuda_carrier.h)
and archived into coherence_kernel_b200/libck_carrier.a for linking into a C host such as the
reference runtime.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libck_b200.so")
ARCHIVE = os.path.join(PKG, "libck_carrier.a")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libck_b200.so")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers += [os.path.join(PKG, "..", "include", f) for f in os.listdir(os.path.join(PKG, "..", "include"))]
    jobs = []
    for f in sources():
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ, f[:-3] + ".o")
        if force or _stale(obj, [src] + headers):
            jobs.append((src, obj))
    cc = nvcc()

    def run(job):
        src, obj = job
        cmd = [cc, *ARCH, *NVFLAGS, "-c", src, "-o", obj]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{p.stderr[-6000:]}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    objs = [os.path.join(OBJ, f[:-3] + ".o") for f in sources()]
    if force or jobs or _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stderr[-4000:]}")
        if os.path.exists(ARCHIVE):
            os.remove(ARCHIVE)
        subprocess.run(["ar", "rcs", ARCHIVE, *objs], check=True)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(force=a.force, verbose=True)
    sys.exit(0)
