"""The tag-232 / tag-233 CUDA matvec doors (runtime/fkwu-uni.c:4753-5050: Windows-only in the
reference) served on Linux by this library's C ABI (include/fk_cuda_carrier.h).

A C host -- compiled here against libck_b200.so the way the reference runtime would link it --
does what the tag-233 op does with its Form lists: y = W.x through fk_cuda_go_external, then the
CPU's downward right fold of two roundings per term, counting the rows that agree bit for bit.
Every row must agree (the device kernel folds in the same order with the same roundings), at the
door's shapes up to its 4194304-weight limit, and the fixture witness (tag 232) answers 3 of 3."""
import os
import subprocess

import numpy as np
import pytest

from coherence_kernel_b200 import _lib

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "coherence_kernel_b200")

HOST = r"""
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "fk_cuda_carrier.h"
/* rows x cols from a fixed linear-congruential stream, values in [-1, 1) */
static unsigned st = 12345u;
static float rnd(void) { st = st * 1664525u + 1013904223u; return (float)((int)(st >> 8) - (1 << 23)) / (float)(1 << 23); }
int main(int argc, char **argv) {
    unsigned rows = (unsigned)atoi(argv[1]), cols = (unsigned)atoi(argv[2]);
    float *W = malloc((size_t)rows * cols * 4), *x = malloc((size_t)cols * 4), *y = malloc((size_t)rows * 4);
    for (size_t i = 0; i < (size_t)rows * cols; i++) W[i] = rnd();
    for (unsigned j = 0; j < cols; j++) x[j] = rnd();
    char name[256];
    long long rc = fk_cuda_go_external(W, x, y, rows, cols, name, sizeof name);
    if (rc < 0) { printf("REFUSED %lld\n", rc); return 1; }
    long long agree = 0;
    for (unsigned i = 0; i < rows; i++) {
        volatile float acc = 0.0f;
        for (long long j = (long long)cols - 1; j >= 0; j--) { volatile float p = W[(size_t)i * cols + j] * x[j]; acc = p + acc; }
        float c = acc;
        agree += memcmp(&c, &y[i], 4) == 0;
    }
    long long door = fk_cuda_matvec_f32_external(W, x, y, rows, cols);
    long long fixture = fk_cuda_matvec_fixture_external();
    printf("RESULT %s|%lld|%lld|%lld\n", name, agree, door, fixture);
    return 0;
}
"""


@pytest.fixture(scope="module")
def host_binary(tmp_path_factory, cuda_lib):
    d = tmp_path_factory.mktemp("cuda_door")
    (d / "host.c").write_text(HOST)
    exe = d / "host"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-I", os.path.join(REPO, "include"), str(d / "host.c"),
                    "-o", str(exe), f"-L{PKG}", "-l:libck_b200.so", f"-Wl,-rpath,{PKG}"], check=True)
    return str(exe)


@pytest.mark.parametrize("rows,cols", [(3, 4), (1000, 7), (4096, 1024), (1, 4194304)])
def test_cuda_matvec_door_bit_exact(host_binary, rows, cols):
    p = subprocess.run([host_binary, str(rows), str(cols)], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    name, agree, door, fixture = line[len("RESULT "):].split("|")
    assert "B200" in name
    assert int(agree) == rows and int(door) == rows and int(fixture) == 3


def test_cuda_matvec_door_refusals(cuda_lib):
    L = _lib.load()
    w = np.zeros(8, dtype=np.float32)
    assert L.fk_cuda_matvec_f32_external(w.ctypes.data, w.ctypes.data, w.ctypes.data, 2, 0) == -1
    assert L.fk_cuda_matvec_f32_external(w.ctypes.data, w.ctypes.data, w.ctypes.data, 4194305, 1) == -1
