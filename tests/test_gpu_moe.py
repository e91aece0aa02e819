"""Parity of the batched MoE layer with the oracle (GPU).

Expert ids and per-expert counts bit-exact (ids in the reference's list order: mm-topk best-first
for the softmax layer, dsv4-topk last-first for the DeepSeek-style layer); routing weights within
1e-5 relative (fp32); outputs normwise max|gpu - ref| / max|ref| <= 2e-2 per token (bf16 MMA).
At full size every token's routing is compared, and the outputs of at least 256 tokens that
together touch every expert.
"""
import os

import numpy as np
import pytest
import torch

from coherence_kernel_b200 import synth, workloads
from coherence_kernel_b200.moe import MoELayer, MoeSpec
from oracle import oracle as O

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def layer_for(spec, w, ntok):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return MoELayer(spec, t(w["gate"]), t(w["up"]), t(w["down"]),
                    t(w["s_gate"]) if spec.n_shared else None, t(w["s_up"]) if spec.n_shared else None,
                    t(w["s_down"]) if spec.n_shared else None, t(w["router"]), t(w["bias"]), max_tokens=ntok)


def run_layer(spec, w, x, keep=None):
    lay = layer_for(spec, w, x.shape[0])
    out, ids, wts, counts = lay(torch.from_numpy(x.view(np.int16)).cuda())
    lay.status(x.shape[0])
    if keep is not None:
        keep["logits"] = lay._ws_views(x.shape[0])["logits"].cpu().numpy()
        keep["flagged"] = lay.flagged(x.shape[0])
    return (out.float().cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy(), counts.cpu().numpy())


def check_outputs(out, ref, tol=2e-2):
    for i in range(ref.shape[0]):
        err = np.abs(out[i] - ref[i]).max()
        assert err <= tol * np.abs(ref[i]).max(), (i, err, np.abs(ref[i]).max())


@pytest.mark.parametrize("mode", [3, 4])
def test_moe_golden(mode):
    g = np.load(os.path.join(G, "moe_golden.npz"))
    p = f"m{mode}_"
    _, H, I, ne, ns, nsel, ng, tg, nt = (int(v) for v in g[p + "dims"])
    spec = MoeSpec(H, I, ne, ns, nsel, mode, ng, tg, 2.5 if mode == 4 else 1.0)
    w = dict(gate=g[p + "wg"], up=g[p + "wu"], down=g[p + "wd"], s_gate=g[p + "sg"], s_up=g[p + "su"],
             s_down=g[p + "sd"], router=g[p + "router"], bias=g[p + "bias"])
    out, ids, wts, counts = run_layer(spec, w, g[p + "x"])
    assert np.array_equal(ids, g[p + "ids"])
    assert np.allclose(wts, g[p + "wts"], rtol=1e-5, atol=1e-7)
    assert np.array_equal(counts, np.bincount(g[p + "ids"].reshape(-1), minlength=ne))
    check_outputs(out, g[p + "out"])


def test_moe_golden_after_gemm():
    # a grouped GEMM first leaves its accumulators in tensor memory; the router logits of a layer
    # whose K loop is shorter than the logit kernel's accumulator count must not pick them up
    from coherence_kernel_b200 import ops
    rng = np.random.default_rng(5)
    q = synth.make_q4k(rng, 512 * 2048)
    xb = synth.make_bf16(rng, (256, 2048))
    ops.Q4KGemm(torch.from_numpy(q).cuda(), 512, 2048, max_tokens=256)(torch.from_numpy(xb.view(np.int16)).cuda())
    torch.cuda.synchronize()
    for mode in (3, 4):
        test_moe_golden(mode)


@pytest.mark.parametrize("spec,ntok", [(MoeSpec(2048, 1408, 32, 2, 6, 3), 2048),
                                       (MoeSpec(7168, 2048, 16, 1, 8, 4, 8, 4, 2.5), 1024)])
def test_moe_layer_deterministic(spec, ntok):
    # the same inputs give the same bits: every shared-memory ring stage is handed back to its
    # producer only after its readers are done (a race shows up as differing output tiles)
    w = workloads.make_moe(spec, ntok, seed=3)
    lay = layer_for(spec, w, ntok)
    x = torch.from_numpy(w["x"].view(np.int16)).cuda()
    first = None
    for _ in range(4):
        out, ids, wts, counts = lay(x)
        lay.status(ntok)
        got = (out.view(torch.int16).clone(), ids.clone(), wts.clone(), counts.clone())
        if first is None:
            first = got
        else:
            for a, b in zip(first, got):
                assert torch.equal(a, b)


def full_size(spec, ntok, sample):
    w = workloads.make_moe(spec, ntok, seed=0)
    keep = {}
    out, ids, wts, counts = run_layer(spec, w, w["x"], keep)
    # the tensor-core logits (three-term bf16 split of the fp32 router) against fp64: their error
    # must sit far below the margin tau under which a token is re-routed exactly
    ref_logits = synth.bf16_bits_to_f32(w["x"]).astype(np.float64) @ w["router"].astype(np.float64).T
    lerr = np.abs(keep["logits"] - ref_logits).max()
    print(f"router logits max abs error {lerr:.3e}, tokens re-routed exactly {keep['flagged']}")
    # the margin is in score units: sigmoid(l) + b moves by at most |dl|/4, softmax order by |dl|
    score_err = lerr / 4 if spec.mode == 4 else lerr
    assert score_err <= spec.tau / 4
    cfg = O.moe_cfg(spec.hidden, spec.inter, spec.n_experts, spec.n_shared, spec.nsel, spec.mode, spec.ngroups,
                    spec.topk_groups, spec.wscale)
    rids, rwts, margin = O.moe_route(cfg, w["router"], w["bias"], w["x"])
    assert np.array_equal(ids, rids), np.argwhere((ids != rids).any(axis=1))[:10]
    assert np.array_equal(counts, np.bincount(rids.reshape(-1), minlength=spec.n_experts))
    assert np.allclose(wts, rwts, rtol=1e-5, atol=1e-7)
    toks = sample_tokens(ids, margin, spec.n_experts, sample)
    sids, swts, sout = O.moe_layer(cfg, w, w["x"], toks)
    assert np.array_equal(sids, ids[toks])
    check_outputs(out[toks], sout)
    err = max(np.abs(out[t] - sout[i]).max() / np.abs(sout[i]).max() for i, t in enumerate(toks))
    print(f"{len(toks)} tokens compared, every expert covered; worst per-token normwise error {err:.3e}")
    return margin


def sample_tokens(ids, margin, n_experts, sample):
    """Tokens whose outputs are compared with the oracle: a greedy cover of every routed expert (so
    every expert's token tiles and the shared-expert tiles they sit beside are exercised), the two
    lowest-margin tokens, the first and last token, then evenly spaced tokens up to `sample`."""
    ntok = ids.shape[0]
    order = np.random.default_rng(0).permutation(ntok)
    covered = np.zeros(n_experts, dtype=bool)
    pick = [0, ntok - 1] + list(np.argsort(margin)[:2])
    for t in pick:
        covered[ids[t]] = True
    for t in order:
        if covered.all():
            break
        if not covered[ids[t]].all():
            covered[ids[t]] = True
            pick.append(int(t))
    rest = sample - len(set(pick))
    if rest > 0:
        pick += list(np.linspace(0, ntok - 1, rest + 2).astype(int)[1:-1])
    have = set(int(t) for t in pick)
    for t in order:
        if len(have) >= sample:
            break
        have.add(int(t))
    assert covered[np.unique(ids)].all()
    return np.array(sorted(have), dtype=np.int64)


def test_moe_small_full_size():
    full_size(workloads.MOE_SMALL, workloads.MOE_SMALL_TOKENS, sample=256)


def test_moe_dsv3_full_size():
    margin = full_size(workloads.MOE_DSV3, workloads.MOE_DSV3_TOKENS, sample=256)
    assert margin.min() >= 0.0


def test_moe_exact_reroute_covers_ties():
    # token 0 has every logit 0 and the bias is 0: every score ties in fp32 and in fp64, the fast
    # path's margin is 0, and the exact re-route must pick the lower indices as the reference does
    spec = MoeSpec(256, 128, 16, 1, 4, 4, 4, 2, 2.5)
    w = workloads.make_moe(spec, 32, seed=7)
    w["x"][0, :] = 0
    w["bias"][:] = 0
    out, ids, wts, counts = run_layer(spec, w, w["x"])
    cfg = O.moe_cfg(256, 128, 16, 1, 4, 4, 4, 2, 2.5)
    rids, rwts, _ = O.moe_route(cfg, w["router"], w["bias"], w["x"])
    assert np.array_equal(ids, rids)


def test_moe_dsv3_decode_sizes():
    """At most 128 tokens (a decode-sized batch) the router logits run as a matvec with compensated
    float-pair sums (accurate to the logits' fp32 rounding), few flagged tokens take one exact fold
    chain per lane, and up to 128 tokens the expert projections run the few-token grouped matvec on
    tiles of at most 5 tokens: ids, counts and weights against the oracle's routing at 1, 3, 8, 16,
    64 and 128 tokens, outputs against the oracle's layer (all tokens up to 8, a sample beyond)."""
    spec = workloads.MOE_DSV3
    w = workloads.make_moe(spec, 128, seed=5)
    lay = layer_for(spec, w, 128)
    cfg = O.moe_cfg(spec.hidden, spec.inter, spec.n_experts, spec.n_shared, spec.nsel, spec.mode, spec.ngroups,
                    spec.topk_groups, spec.wscale)
    for n in (1, 3, 8, 16, 64, 128):
        x = np.ascontiguousarray(w["x"][:n])
        out, ids, wts, counts = lay(torch.from_numpy(x.view(np.int16)).cuda())
        lay.status(n)
        logits = lay._ws_views(n)["logits"].cpu().numpy()
        ref_logits = synth.bf16_bits_to_f32(x).astype(np.float64) @ w["router"].astype(np.float64).T
        assert np.abs(logits - ref_logits).max() <= 2e-6
        rids, rwts, _ = O.moe_route(cfg, w["router"], w["bias"], x)
        ids, wts, counts = ids.cpu().numpy(), wts.cpu().numpy(), counts.cpu().numpy()
        assert np.array_equal(ids, rids)
        assert np.array_equal(counts, np.bincount(rids.reshape(-1), minlength=spec.n_experts))
        assert np.allclose(wts, rwts, rtol=1e-5, atol=1e-7)
        toks = (np.arange(n) if n <= 8 else np.array([0, 9, 15]) if n == 16 else np.array([0, 9, 23, 40, 63]) if n == 64
                else np.array([0, 41, 64, 99, 127]))
        sids, _, sout = O.moe_layer(cfg, w, x, toks)
        assert np.array_equal(sids, ids[toks])
        check_outputs(out.float().cpu().numpy()[toks], sout)


def test_moe_decode_tie_reroute():
    # four tokens: the logits take the fp64 matvec, and token 0 (all-zero activations, zero bias)
    # ties everywhere, so the exact re-route's few-token form must pick the reference's experts
    spec = MoeSpec(256, 128, 16, 1, 4, 4, 4, 2, 2.5)
    w = workloads.make_moe(spec, 4, seed=9)
    w["x"][0, :] = 0
    w["bias"][:] = 0
    keep = {}
    out, ids, wts, counts = run_layer(spec, w, w["x"], keep)
    assert keep["flagged"] >= 1
    cfg = O.moe_cfg(256, 128, 16, 1, 4, 4, 4, 2, 2.5)
    rids, rwts, _ = O.moe_route(cfg, w["router"], w["bias"], w["x"])
    assert np.array_equal(ids, rids)
    assert np.allclose(wts, rwts, rtol=1e-5, atol=1e-7)
