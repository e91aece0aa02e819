"""The exact re-route's router logits (ck_router_exact_logits) against the oracle's right fold
(tb-dot, transformer-block.fk:25-26), bit for bit: the per-lane form (at most 128 listed tokens)
and the tiled form (more), at the DeepSeek-V3 router shape (256 experts, hidden 7168) and at a
small shape whose expert count is below one work item's 64 and whose row is shorter than the
copy ring."""
import ctypes

import numpy as np
import pytest
import torch

from coherence_kernel_b200 import _lib, synth
from coherence_kernel_b200.ops import _ptr
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def exact_logits(router, x_bf16, tokens):
    dev = "cuda"
    rw = torch.from_numpy(router).to(dev)
    x = torch.from_numpy(x_bf16.view(np.int16)).to(dev)
    lst = torch.from_numpy(np.asarray(tokens, dtype=np.uint32).view(np.int32)).to(dev)
    cnt = torch.tensor([len(tokens)], dtype=torch.int32, device=dev)
    ne, hidden = router.shape
    out = torch.full((max(len(tokens), 1), ne), float("nan"), dtype=torch.float64, device=dev)
    w64 = torch.empty((ne, hidden), dtype=torch.float64, device=dev)
    _lib.check(_lib.load().ck_router_exact_logits(_ptr(x), _ptr(rw), _ptr(lst), _ptr(cnt), ne, hidden, _ptr(out),
                                                  _ptr(w64), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "ck_router_exact_logits")
    torch.cuda.synchronize()
    return out.cpu().numpy()[:len(tokens)]


@pytest.mark.parametrize("ne,hidden,ntok", [(256, 7168, 300), (16, 96, 300)])
def test_exact_logits_match_the_reference_fold(ne, hidden, ntok):
    rng = np.random.default_rng([ne, hidden])
    router = synth.make_router(rng, ne, hidden)
    x = synth.make_bf16(rng, (ntok, hidden))
    xf = synth.bf16_bits_to_f32(x).astype(np.float64)
    for n in (1, 3, 40, 128, 129, 300):
        tokens = rng.choice(ntok, size=n, replace=False)
        got = exact_logits(router, x, tokens)
        ref = O.dot_rows(xf[tokens], router.astype(np.float64))
        assert np.array_equal(got, ref), (n, np.abs(got - ref).max())
