"""The oracle against the reference: fkwu-generated golden vectors and the reference's own pins."""
import os

import numpy as np
import pytest

from oracle import oracle as O

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_quant_golden_bit_exact():
    g = np.load(os.path.join(G, "quant_golden.npz"))
    r8, c8, r4, c4 = (int(v) for v in g["dims"])
    assert np.array_equal(O.q80_dequant(g["q8"], 0, r8 * c8), g["w8"])
    assert np.array_equal(O.q4k_dequant(g["q4"], 0, r4 * c4), g["w4"])
    assert np.array_equal(O.q80_matvec(g["q8"], g["x8"].astype(np.float64), r8, c8), g["y8"])
    assert np.array_equal(O.q4k_matvec(g["q4"], g["x4"].astype(np.float64), r4, c4), g["y4"])


def test_reference_fixtures_bit_exact():
    f = np.load(os.path.join(G, "ref_fixtures.npz"))
    assert np.array_equal(O.q4k_dequant(f["q4k"], 0, 512), f["w4"])
    assert np.array_equal(O.q80_dequant(f["q80"], 0, 96), f["w8"])
    # q8-0-msl-band.fk pins the stride crossings: w32*1e6 in (4634.857, 4634.858), w65 in (133.633, 133.634)
    w = O.q80_dequant(f["q80"], 0, 96) * 1e6
    assert 4634.857 < w[32] < 4634.858
    assert 133.633 < w[65] < 133.634


def test_q4k_dequant_band_pins():
    # form-stdlib/tests/q4k-dequant-band.fk:11-43: one superblock, 12 pinned round(w*1e6)
    d, dmin = 0.00010609626770019531, 0.0009484291076660156
    scales = [229, 178, 240, 255, 160, 107, 239, 191, 26, 174, 22, 179]
    qs = [135, 151, 157, 85, 141, 119, 132, 25, 148, 67, 236, 75, 75, 167, 115, 128, 174, 96, 117, 181, 88, 109, 101,
          142, 159, 152, 85, 156, 10, 167, 235, 213, 146, 203, 140, 191, 96, 14, 137, 172, 203, 135, 167, 205, 186, 152,
          140, 104, 105, 206, 186, 155, 173, 116, 185, 249, 234, 213, 153, 236, 74, 153, 105, 231, 185, 130, 215, 82,
          135, 196, 38, 164, 99, 99, 85, 43, 227, 52, 4, 143, 40, 178, 50, 41, 40, 68, 35, 182, 104, 119, 144, 218, 54,
          134, 1, 70, 58, 118, 95, 195, 183, 37, 121, 198, 151, 151, 119, 118, 105, 149, 136, 0, 246, 133, 186, 151,
          162, 154, 150, 168, 180, 87, 25, 135, 119, 107, 201, 187]
    blk = np.zeros(144, dtype=np.uint8)
    blk[0:2] = np.frombuffer(np.float16(d).tobytes(), dtype=np.uint8)
    blk[2:4] = np.frombuffer(np.float16(dmin).tobytes(), dtype=np.uint8)
    assert float(np.float16(d)) == d and float(np.float16(dmin)) == dmin
    blk[4:16] = scales
    blk[16:] = qs
    w = O.q4k_dequant(blk, 0, 256)
    pins = {0: -2871, 31: -10722, 32: 1656, 63: 28180, 64: -34391, 127: 33826, 128: 24084, 159: 5623,
            160: 29026, 191: -5137, 200: -6369, 255: 18738}
    for i, v in pins.items():
        assert round(w[i] * 1e6) == v, (i, w[i])


def test_q6k_golden_bit_exact():
    # fkwu's q6m-flat-at / tb-matvec (form-stdlib/q6k-msl.fk:62-81, transformer-block.fk:25-28) on a
    # seeded tensor whose rows straddle superblocks, and on the reference's two-superblock fixture
    g = np.load(os.path.join(G, "q6k_golden.npz"))
    r6, c6 = (int(v) for v in g["dims"])
    assert np.array_equal(O.q6k_dequant(g["q6"], 0, r6 * c6), g["w6"])
    assert np.array_equal(O.q6k_matvec(g["q6"], g["x6"].astype(np.float64), r6, c6), g["y6"])
    assert np.array_equal(O.q6k_dequant(g["fix"], 0, 512), g["fix_w"])


def test_q6k_dequant_band_pins():
    # form-stdlib/tests/q6k-dequant-band.fk: a real llama3.2:3b superblock (signed scales, both halves,
    # all four sub-groups, both nibbles), 12 pinned round(w*1e6) from gguf's dequantize
    g = np.load(os.path.join(G, "q6k_golden.npz"))
    w = O.q6k_dequant(g["band_sb"], 0, 256)
    assert np.array_equal(w, g["band_w"])  # fkwu's own decode of the same bytes
    for i, v in g["band_pins"]:
        assert round(w[i] * 1e6) == v, (i, w[i])


def test_rmsnorm_golden_bit_exact():
    # fkwu's ln-rmsnorm (llama-numerics.fk:40-50) with its tn-sqrt Newton iteration
    g = np.load(os.path.join(G, "norm_golden.npz"))
    for t in ("h", "s"):
        out = O.rmsnorm(g[t + "_x"].astype(np.float64), g[t + "_g"].astype(np.float64), float(g[t + "_eps"]))
        assert np.array_equal(out, g[t + "_out"]), t


def test_route_golden_bit_exact():
    g = np.load(os.path.join(G, "route_golden.npz"))
    for t in ("e64", "e256"):
        ne, nsel, ng, tg = (int(v) for v in g[t + "_dims"])
        L = g[t + "_logits"].astype(np.float64)
        B = g[t + "_bias"].astype(np.float64)
        for i in range(L.shape[0]):
            ids, w = O.route_softmax(L[i], nsel, False)
            assert np.array_equal(ids, g[t + "_mm_ids"][i]) and np.array_equal(w, g[t + "_mm_w"][i])
            _, w = O.route_softmax(L[i], nsel, True)
            assert np.array_equal(w, g[t + "_mm_wn"][i])
            ids, w = O.route_dsv4(L[i], B, nsel, 2.5)
            assert np.array_equal(ids, g[t + "_dr_ids"][i]) and np.array_equal(w, g[t + "_dr_w"][i])
            ids, w, _ = O.route_sigmoid_group(L[i], B, ng, tg, nsel, 2.5)
            assert np.array_equal(ids, g[t + "_sg_ids"][i]) and np.array_equal(w, g[t + "_sg_w"][i])
    # ties go to the lower index (row 1 ties experts 3 and 40 at the maximum)
    assert list(g["e64_mm_ids"][1][:2]) == [3, 40]


@pytest.mark.parametrize("mode", [3, 4])
def test_moe_layer_golden_bit_exact(mode):
    g = np.load(os.path.join(G, "moe_golden.npz"))
    p = f"m{mode}_"
    _, H, I, ne, ns, nsel, ng, tg, nt = (int(v) for v in g[p + "dims"])
    cfg = O.moe_cfg(H, I, ne, ns, nsel, mode, ng, tg, 2.5)
    w = dict(gate=g[p + "wg"], up=g[p + "wu"], down=g[p + "wd"], s_gate=g[p + "sg"], s_up=g[p + "su"],
             s_down=g[p + "sd"], router=g[p + "router"], bias=g[p + "bias"])
    ids, wts, out = O.moe_layer(cfg, w, g[p + "x"], np.arange(nt))
    assert np.array_equal(ids, g[p + "ids"])
    assert np.array_equal(wts, g[p + "wts"])
    assert np.array_equal(out, g[p + "out"])


def test_oracle_numerics_match_reference_recipes():
    # tn-exp / ln-sigmoid agree with libm to ~1e-15 relative (they are Taylor restatements)
    for x in (-7.5, -1.0, -0.3, 0.0, 0.25, 2.0, 9.0):
        assert abs(O.lib().ckr_exp(x) - np.exp(x)) <= 1e-13 * np.exp(x)
        assert abs(O.lib().ckr_sigmoid(x) - 1 / (1 + np.exp(-x))) <= 1e-14
    assert abs(O.lib().ckr_ln(3.7) - np.log(3.7)) < 1e-14
    assert abs(O.lib().ckr_sqrt(2.0) - np.sqrt(2.0)) < 1e-15
