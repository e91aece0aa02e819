"""The benchmark workloads of the quantized path, as seeded synthetic inputs.

* ``Q8_MATVEC``     Q8_0 dequant-matvec, W 4096 x 4096, x fp32 [4096]
* ``Q4K_PREFILL``   Q4_K dequant-matmul, W 11008 x 4096, X bf16 [M, 4096], M in {1,16,128,512,2048}
* ``MOE_SMALL``     64 routed + 2 shared SwiGLU experts, hidden 2048, intermediate 1408, softmax
                    top-6 without renormalization, 4096 tokens
* ``MOE_DSV3``      256 routed + 1 shared SwiGLU experts, hidden 7168, intermediate 2048, sigmoid +
                    bias, group-limited top-4 of 8 groups (group score = sum of its top 2), top-8,
                    renormalized x 2.5, 8192 tokens
* ``DECODE``        MOE_DSV3 plus four dense 7168 x 7168 Q4_K matvecs at batch 1, 4, 16, 64

Weights and activations follow the stated distributions (see synth.py), all from
``numpy.random.default_rng(seed)``.
"""
from __future__ import annotations

import os

import numpy as np

from . import synth
from .moe import MoeSpec

MOE_SMALL = MoeSpec(hidden=2048, inter=1408, n_experts=64, n_shared=2, nsel=6, mode=3)
MOE_SMALL_TOKENS = 4096
MOE_DSV3 = MoeSpec(hidden=7168, inter=2048, n_experts=256, n_shared=1, nsel=8, mode=4, ngroups=8, topk_groups=4,
                   wscale=2.5)
MOE_DSV3_TOKENS = 8192
Q8_MATVEC = (4096, 4096)
Q4K_PREFILL = (11008, 4096)
Q4K_PREFILL_M = (1, 16, 128, 512, 2048)


def make_moe(spec: MoeSpec, ntok: int, seed: int = 0, experts=None):
    """Weights of every expert (or of the expert ids in `experts`), router, bias and tokens.

    Returns a dict of numpy arrays: gate / up / down (the experts' Q4_K tensors concatenated),
    s_gate / s_up / s_down (shared), router fp32 [ne, hidden], bias fp32 [ne], x bf16 bits
    [ntok, hidden].  Expert e's tensors are drawn from their own stream (seed, 1 + e) so any
    subset of experts can be regenerated identically.
    """
    from concurrent.futures import ThreadPoolExecutor
    nw = spec.inter * spec.hidden
    nb = synth.q4k_bytes(nw)
    ids = list(range(spec.n_experts) if experts is None else experts)
    out = {}
    for k, m in (("gate", 0), ("up", 1), ("down", 2)):
        for key, streams in ((k, [1 + e for e in ids]), ("s_" + k, [100000 + s for s in range(spec.n_shared)])):
            arr = np.empty(nb * len(streams), dtype=np.uint8)

            def fill(i, st=streams, a=arr, mm=m):
                a[i * nb:(i + 1) * nb] = synth.make_q4k(np.random.default_rng([seed, st[i], mm]), nw)

            with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
                list(ex.map(fill, range(len(streams))))
            out[key] = arr
    rng = np.random.default_rng([seed, 0])
    out["router"] = synth.make_router(rng, spec.n_experts, spec.hidden)
    out["bias"] = synth.make_bias(rng, spec.n_experts)
    out["x"] = synth.make_bf16(np.random.default_rng([seed, 200000]), (ntok, spec.hidden))
    return out
