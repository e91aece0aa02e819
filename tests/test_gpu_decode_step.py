"""The device-resident decode step (coherence_kernel_b200.decode.DecodeStep / ck_decode_step_*)
against the oracle, and its CUDA-graph replay against its eager run.

Per stage: the normed attention input within 1e-5 relative of the oracle's ln-rmsnorm of the same
h; q, k, v and the attention residual within 1e-3 of sum |w x| of the oracle's matvec of the step's
own normed input (fp32 accumulation); expert ids bit-exact with the oracle's routing of the step's
own bf16 MoE input, and the MoE output within 2e-2 per token normwise (bf16 MMA).  The replayed
graph equals the eager run bit for bit.
"""
import numpy as np
import pytest
import torch

from coherence_kernel_b200 import synth, workloads
from coherence_kernel_b200.decode import DecodeStep
from coherence_kernel_b200.moe import MoeSpec
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def make(spec, T, seed):
    rng = np.random.default_rng(seed)
    H = spec.hidden
    w = workloads.make_moe(spec, T, seed=seed)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dense = [synth.make_q4k(np.random.default_rng([seed, i]), H * H) for i in range(4)]
    g = [(1 + 0.1 * rng.standard_normal(H)).astype(np.float32) for _ in range(2)]
    step = DecodeStep(spec, *[t(d) for d in dense], t(g[0]), t(g[1]), t(w["gate"]), t(w["up"]), t(w["down"]),
                      t(w["s_gate"]), t(w["s_up"]), t(w["s_down"]), t(w["router"]), t(w["bias"]), max_tokens=T)
    h0 = (rng.standard_normal((T, H)) * 2).astype(np.float32)
    return step, w, dense, g, h0


def matvec_rows(q, x, H):
    x64 = x.astype(np.float64)
    w = O.q4k_dequant(q, 0, H * H).reshape(H, H)
    return w @ x64.T, np.abs(w) @ np.abs(x64).T


@pytest.mark.parametrize("spec,T", [(MoeSpec(1024, 512, 16, 1, 4, 4, 4, 2, 2.5), 3),
                                    (MoeSpec(2048, 1408, 64, 2, 6, 3), 5)])
def test_decode_step_matches_oracle(spec, T):
    step, w, dense, g, h0 = make(spec, T, seed=T)
    H = spec.hidden
    h = torch.from_numpy(h0).cuda()
    q, k, v = (torch.empty((T, H), device="cuda") for _ in range(3))
    step.run(h, q, k, v)
    step.status(T)
    vw = step.views(T)
    a = vw["a"].cpu().numpy()
    for i in range(T):
        ra = O.rmsnorm(h0[i].astype(np.float64), g[0].astype(np.float64), 1e-6)
        assert np.abs(a[i] - ra).max() <= 1e-5 * np.abs(ra).max()
    for out, qd in ((q, dense[0]), (k, dense[1]), (v, dense[2])):
        ref, bound = matvec_rows(qd, a, H)
        assert np.all(np.abs(out.cpu().numpy().T - ref) <= 1e-3 * bound)
    vv = v.cpu().numpy()
    ref, bound = matvec_rows(dense[3], vv, H)
    assert np.all(np.abs(vw["o"].cpu().numpy().T - ref) <= 1e-3 * bound)
    h1 = h0 + vw["o"].cpu().numpy()
    b = vw["b"].view(torch.int16).cpu().numpy().view(np.uint16)
    for i in range(T):
        rb = O.rmsnorm(h1[i].astype(np.float64), g[1].astype(np.float64), 1e-6)
        bf = synth.bf16_bits_to_f32(b[i]).astype(np.float64)
        assert np.abs(bf - rb).max() <= 2.0 ** -7 * np.abs(rb).max()
    cfg = O.moe_cfg(spec.hidden, spec.inter, spec.n_experts, spec.n_shared, spec.nsel, spec.mode, spec.ngroups,
                    spec.topk_groups, spec.wscale)
    rids, _, rout = O.moe_layer(cfg, w, np.ascontiguousarray(b), np.arange(T))
    assert np.array_equal(vw["ids"].cpu().numpy(), rids)
    m = vw["m"].float().cpu().numpy()
    for i in range(T):
        assert np.abs(m[i] - rout[i]).max() <= 2e-2 * np.abs(rout[i]).max(), i
    # h = h0 + Wo v + m, exactly as the two residual adds in fp32
    assert np.array_equal(h.cpu().numpy(), (h0 + vw["o"].cpu().numpy()) + m)


def test_decode_step_graph_replay_equals_eager():
    spec = workloads.MOE_DSV3
    T = 4
    step, w, dense, g, h0 = make(spec, T, seed=77)
    H = spec.hidden
    eager = torch.from_numpy(h0).cuda()
    q, k, v = (torch.empty((T, H), device="cuda") for _ in range(3))
    step.run(eager, q, k, v)  # also loads every kernel before the capture
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        hg = torch.from_numpy(h0).cuda()
        qg, kg, vg = (torch.empty((T, H), device="cuda") for _ in range(3))
        step.capture(hg, qg, kg, vg)
        hg.copy_(torch.from_numpy(h0).cuda())  # the capture recorded, it did not run
        step.replay()
        step.status(T)
    torch.cuda.synchronize()
    for a, b in ((eager, hg), (q, qg), (k, kg), (v, vg)):
        assert torch.equal(a, b)
    # a second replay continues from the updated state, like the next layer's step would
    with torch.cuda.stream(s):
        step.replay()
    torch.cuda.synchronize()
    step.run(eager, q, k, v)
    assert torch.equal(eager, hg)
