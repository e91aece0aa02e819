"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference's own Form recipes on the reference's own runtime (fkwu, compiled from
runtime/fkwu-uni.c by oracle/Makefile) over seeded synthetic inputs, through the driver cells in
oracle/fk/, and writes inputs + fp64 outputs as small .npz fixtures beside this script.  It also
copies the reference's two real-weight fixtures (q4k-two-superblocks.bin, q8-0-three-blocks.bin)
and records every weight the reference decodes from them.

Needs the reference tree, named by --ref or CK_REFERENCE, and runs only where it is present; the
fixtures it writes are committed and are all that the tests read.

    python tests/golden/make_golden.py --ref <the reference tree> [--only quant,fixtures,route,moe]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from coherence_kernel_b200 import synth  # noqa: E402

FKWU = os.path.join(REPO, "oracle", "_ref", "fkwu")


def parse_form(text: str):
    """fkwu prints lists as [a, b, ...] with shortest round-trip floats; Python's literal parser
    reads the same digits back to the same doubles."""
    import ast
    line = [ln for ln in text.strip().splitlines() if ln.startswith("[")][-1]
    return ast.literal_eval(line.replace("nothing", "None"))


class FormRunner:
    def __init__(self, ref: str):
        self.tmp = tempfile.mkdtemp(prefix="ck_golden_")
        self.form = os.path.join(self.tmp, "form")
        shutil.copytree(os.path.join(ref, "form", "form-stdlib"), os.path.join(self.form, "form-stdlib"))
        os.makedirs(os.path.join(self.form, "ck"))
        for f in os.listdir(os.path.join(REPO, "oracle", "fk")):
            if f.endswith(".fk"):
                shutil.copy(os.path.join(REPO, "oracle", "fk", f), os.path.join(self.form, "ck", f))
        self.inp = os.path.join(self.form, "ck_in")
        os.makedirs(self.inp)

    def put(self, name: str, arr: np.ndarray):
        np.ascontiguousarray(arr).tofile(os.path.join(self.inp, name))

    def run(self, cell: str, timeout=3600):
        p = subprocess.run([FKWU, f"ck/{cell}"], cwd=self.form, capture_output=True, text=True,
                           timeout=timeout)
        if p.returncode != 0 or "error" in p.stderr.lower().replace("0 error(s)", ""):
            raise RuntimeError(f"fkwu {cell} failed rc={p.returncode}\n{p.stderr[-4000:]}\n{p.stdout[-2000:]}")
        return parse_form(p.stdout)

    def close(self):
        shutil.rmtree(self.tmp, ignore_errors=True)


def golden_quant(fr: FormRunner):
    rng = np.random.default_rng(0)
    r8, c8, r4, c4 = 16, 256, 12, 384   # Q4_K rows of 384 straddle superblocks at 128-weight halves
    q8 = synth.make_q8_0(rng, r8 * c8)
    q4 = synth.make_q4k(rng, r4 * c4)
    x8 = rng.standard_normal(c8).astype(np.float32)
    x4 = rng.standard_normal(c4).astype(np.float32)
    fr.put("meta.bin", np.array([r8, c8, r4, c4], dtype=np.uint32))
    fr.put("q8.bin", q8)
    fr.put("q4.bin", q4)
    fr.put("x8.bin", x8)
    fr.put("x4.bin", x4)
    rows8, y8, rows4, y4 = fr.run("ck_quant.fk")
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), q8=q8, q4=q4, x8=x8, x4=x4,
                        dims=np.array([r8, c8, r4, c4]), w8=np.array(rows8, dtype=np.float64).reshape(-1),
                        y8=np.array(y8, dtype=np.float64), w4=np.array(rows4, dtype=np.float64).reshape(-1),
                        y4=np.array(y4, dtype=np.float64))
    print("quant golden: q8", len(y8), "rows, q4", len(y4), "rows")


def golden_ref_fixtures(fr: FormRunner, ref: str):
    fx = os.path.join(ref, "form", "form-stdlib", "tests", "fixtures")
    out = {}
    for name, size in (("q4k-two-superblocks.bin", 288), ("q8-0-three-blocks.bin", 102)):
        data = open(os.path.join(fx, name), "rb").read()
        assert len(data) == size
        out[name] = np.frombuffer(data, dtype=np.uint8)
        print(name, hashlib.sha256(data).hexdigest())
    # the reference decodes every weight of both fixtures (q4m-flat-at / q80-flat-at)
    fr.put("meta.bin", np.array([3, 32, 2, 256], dtype=np.uint32))
    fr.put("q8.bin", out["q8-0-three-blocks.bin"])
    fr.put("q4.bin", out["q4k-two-superblocks.bin"])
    fr.put("x8.bin", np.ones(32, dtype=np.float32))
    fr.put("x4.bin", np.ones(256, dtype=np.float32))
    rows8, _, rows4, _ = fr.run("ck_quant.fk")
    np.savez_compressed(os.path.join(HERE, "ref_fixtures.npz"), q4k=out["q4k-two-superblocks.bin"],
                        q80=out["q8-0-three-blocks.bin"], w4=np.array(rows4).reshape(-1),
                        w8=np.array(rows8).reshape(-1))
    print("reference fixtures decoded:", len(np.array(rows4).reshape(-1)), "+", len(np.array(rows8).reshape(-1)))


def q6k_band_vectors(ref: str):
    """The real llama3.2:3b Q6_K superblock of the reference's q6k-dequant-band.fk (d, QL, QH,
    SCALES given inline there) as 210 raw bytes, and the band's twelve (index, round(w * 1e6)) pins."""
    import re
    text = open(os.path.join(ref, "form", "form-stdlib", "tests", "q6k-dequant-band.fk")).read()
    d = float(re.search(r"\(let d ([0-9.e-]+)\)", text).group(1))
    lists = {}
    for name in ("SCALES", "QL", "QH"):
        body = re.search(r"\(let " + name + r" \(list([^)]*)\)\)", text).group(1)
        lists[name] = [int(v) for v in body.split()]
    assert [len(lists[k]) for k in ("QL", "QH", "SCALES")] == [128, 64, 16]
    dh = np.array([d], dtype=np.float16)
    assert float(dh[0]) == d, "d is an f16 value"
    sb = np.concatenate([np.array(lists["QL"], dtype=np.uint8), np.array(lists["QH"], dtype=np.uint8),
                         np.array(lists["SCALES"], dtype=np.uint8), dh.view(np.uint8)])
    pins = [(int(i), int(v)) for i, v in
            re.findall(r"\(q6k-at (\d+) +d QL QH SCALES\) 1000000\.0\)\) (-?\d+)\)", text)]
    last = re.search(r"\(nth full 255\) 1000000\.0\)\) (-?\d+)\)", text)
    pins.append((255, int(last.group(1))))
    assert len(pins) == 12
    return sb, pins


def golden_q6k(fr: FormRunner, ref: str):
    """Q6_K through the reference's own q6m-flat-at and tb-matvec: a seeded tensor whose rows
    straddle superblocks (384 columns), the reference's two-superblock fixture, and the band's real
    superblock, whose twelve pins are kept beside the fp64 values fkwu decodes from it."""
    out = {}

    def run(q, rows, cols, x):
        fr.put("meta6.bin", np.array([rows, cols], dtype=np.uint32))
        fr.put("q6.bin", q)
        fr.put("x6.bin", x)
        w, y = fr.run("ck_q6k.fk")
        return np.array(w, dtype=np.float64).reshape(-1), np.array(y, dtype=np.float64)

    rng = np.random.default_rng(6)
    r6, c6 = 10, 384
    q6 = synth.make_q6k(rng, r6 * c6)
    x6 = rng.standard_normal(c6).astype(np.float32)
    out["q6"], out["x6"], out["dims"] = q6, x6, np.array([r6, c6])
    out["w6"], out["y6"] = run(q6, r6, c6, x6)
    fx = os.path.join(ref, "form", "form-stdlib", "tests", "fixtures", "q6k-two-superblocks.bin")
    data = open(fx, "rb").read()
    assert len(data) == 420
    print("q6k-two-superblocks.bin", hashlib.sha256(data).hexdigest())
    out["fix"] = np.frombuffer(data, dtype=np.uint8)
    out["fix_w"], _ = run(out["fix"], 2, 256, np.ones(256, dtype=np.float32))
    sb, pins = q6k_band_vectors(ref)
    out["band_sb"] = sb
    out["band_pins"] = np.array(pins, dtype=np.int64)
    out["band_w"], _ = run(sb, 1, 256, np.ones(256, dtype=np.float32))
    np.savez_compressed(os.path.join(HERE, "q6k_golden.npz"), **out)
    print("q6k golden:", len(out["y6"]), "rows,", len(out["fix_w"]), "fixture weights, 12 band pins")


def golden_gguf(ref: str):
    """The reference's mini-GGUF (header, one key/value, one Q4_K tensor-info record, the pad, one real
    superblock) from weight-load-q4k-band.fk, as bytes, with that band's pins: tensor-info start, type,
    dim0, data offset, and round(w * 1e6) at eight indices."""
    import re
    text = open(os.path.join(ref, "form", "form-stdlib", "tests", "weight-load-q4k-band.fk")).read()
    body = re.search(r"\(let g \(list(.*?)\)\)", text, re.S).group(1)
    g = np.array([int(v) for v in body.split()], dtype=np.uint8)
    pins = [(int(i), int(v)) for i, v in re.findall(r"\(wl-q4k-at g off (\d+) *\) +1000000\.0\)\) (-?\d+)\)", text)]
    last = re.search(r"\(nth full 255\) 1000000\.0\)\) (-?\d+)\)", text)
    pins.append((255, int(last.group(1))))
    ti = int(re.search(r"\(eq ti (\d+)\)", text).group(1))
    assert len(pins) == 8, pins
    np.savez_compressed(os.path.join(HERE, "gguf_golden.npz"), band_gguf=g, band_pins=np.array(pins, dtype=np.int64),
                        band_tinfo_start=np.array(ti))
    print("gguf golden:", g.size, "bytes, tensor info at", ti, ",", len(pins), "pins")


def golden_norm(fr: FormRunner):
    """ln-rmsnorm (llama-numerics.fk:40-50) on the reference runtime: a hidden-size vector and a
    short one with a large eps."""
    out = {}
    rng = np.random.default_rng(12)
    for tag, n, eps in (("h", 7168, 1e-6), ("s", 37, 0.25)):
        x = (rng.standard_normal(n) * 3).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        meta = np.zeros(2, dtype=np.uint32)
        meta[0] = n
        meta[1] = np.array([eps], dtype=np.float32).view(np.uint32)[0]
        fr.put("norm_meta.bin", meta)
        fr.put("xn.bin", x)
        fr.put("gn.bin", g)
        out[tag + "_x"], out[tag + "_g"], out[tag + "_eps"] = x, g, np.float32(eps)
        out[tag + "_out"] = np.array(fr.run("ck_norm.fk"), dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "norm_golden.npz"), **out)
    print("norm golden:", len(out["h_out"]), "+", len(out["s_out"]))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CK_REFERENCE"))
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref <the reference tree> (or CK_REFERENCE) is required")
    if not os.path.exists(FKWU):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "ref", f"REF={a.ref}"], check=True)
    fr = FormRunner(a.ref)
    try:
        todo = a.only.split(",") if a.only else ["quant", "fixtures", "route", "moe", "q6k", "gguf", "norm"]
        if "quant" in todo:
            golden_quant(fr)
        if "fixtures" in todo:
            golden_ref_fixtures(fr, a.ref)
        if "route" in todo:
            golden_route(fr)
        if "moe" in todo:
            golden_moe(fr)
        if "q6k" in todo:
            golden_q6k(fr, a.ref)
        if "gguf" in todo:
            golden_gguf(a.ref)
        if "norm" in todo:
            golden_norm(fr)
    finally:
        fr.close()


def golden_route(fr):
    rng = np.random.default_rng(1)
    cases = {}
    for tag, ne, nsel, ngroups, topkg, sigma in (("e64", 64, 6, 8, 4, 0.9), ("e256", 256, 8, 8, 4, 1.7)):
        ntok = 12
        logits = (rng.standard_normal((ntok, ne)) * sigma).astype(np.float32)
        bias = (rng.standard_normal(ne) * 0.01).astype(np.float32)
        # exact ties at the selection boundary: the lower index must win
        logits[0, :] = 0.0
        logits[1, 3] = logits[1, 40]
        logits[1, 3] = logits[1].max()
        logits[1, 40] = logits[1, 3]
        logits[2, : ne // 2] = logits[2, ne // 2:]
        fr.put("meta.bin", np.array([ne, nsel, ngroups, topkg, ntok], dtype=np.uint32))
        fr.put("logits.bin", logits)
        fr.put("bias.bin", bias)
        res = fr.run("ck_route.fk")
        cases[tag] = dict(
            logits=logits, bias=bias, dims=np.array([ne, nsel, ngroups, topkg]),
            mm_ids=np.array([r[0] for r in res], dtype=np.int32),
            mm_w=np.array([r[1] for r in res], dtype=np.float64),
            mm_wn=np.array([r[2] for r in res], dtype=np.float64),
            dr_ids=np.array([r[3] for r in res], dtype=np.int32),
            dr_w=np.array([r[4] for r in res], dtype=np.float64),
            sg_ids=np.array([r[5][0] for r in res], dtype=np.int32),
            sg_w=np.array([r[5][1] for r in res], dtype=np.float64))
    flat = {f"{t}_{k}": v for t, c in cases.items() for k, v in c.items()}
    np.savez_compressed(os.path.join(HERE, "route_golden.npz"), **flat)
    print("route golden:", {t: len(c["mm_ids"]) for t, c in cases.items()})


def golden_moe(fr):
    out = {}
    for mode, hidden, inter, ne, ns, nsel, ngroups, topkg, ntok in ((3, 256, 128, 16, 2, 4, 1, 1, 3),
                                                                     (4, 256, 64, 16, 1, 4, 4, 2, 3)):
        rng = np.random.default_rng(10 + mode)
        nw = inter * hidden
        W = {k: synth.make_q4k(rng, nw * n) for k, n in (("wg", ne), ("wu", ne), ("wd", ne),
                                                          ("sg", ns), ("su", ns), ("sd", ns))}
        router = synth.make_router(rng, ne, hidden)
        bias = synth.make_bias(rng, ne)
        x = synth.make_bf16(rng, (ntok, hidden))
        fr.put("meta.bin", np.array([mode, hidden, inter, ne, ns, nsel, ngroups, topkg, ntok], dtype=np.uint32))
        for k, v in W.items():
            fr.put(f"{k}.bin", v)
        fr.put("router.bin", router)
        fr.put("bias.bin", bias)
        fr.put("x.bin", x)
        res = fr.run("ck_moe.fk")
        p = f"m{mode}_"
        out.update({p + k: v for k, v in W.items()})
        out.update({p + "router": router, p + "bias": bias, p + "x": x,
                    p + "dims": np.array([mode, hidden, inter, ne, ns, nsel, ngroups, topkg, ntok]),
                    p + "ids": np.array([r[0] for r in res], dtype=np.int32),
                    p + "wts": np.array([r[1] for r in res], dtype=np.float64),
                    p + "out": np.array([r[2] for r in res], dtype=np.float64)})
        print("moe golden mode", mode, "tokens", len(res))
    np.savez_compressed(os.path.join(HERE, "moe_golden.npz"), **out)


if __name__ == "__main__":
    main()
