"""Expert parallelism on two and four GPUs, over NCCL collectives and over NVLink peer memory: the expert-parallel layer's output, ids and
weights equal the single-GPU layer's bit for bit (each token row is computed by the same kernels in
the same K order whichever tile it lands in, and the combine keeps the reference's order).  The
decode-sized cases (64 tokens in all) take the few-token grouped matvec on both sides.  Bit equality
needs both sides on the same side of the decode threshold (CK_MOE_DECODE_TOKENS): a rank whose share
is decode-sized routes with the compensated router and runs its shared expert on the few-token
matvec, so every prefill case gives each rank more than 128 tokens.

Runs as spawned ranks when the box has enough GPUs; skipped otherwise.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SPECS = {
    "dsv4": dict(hidden=1024, inter=512, n_experts=16, n_shared=1, nsel=4, mode=4, ngroups=4, topk_groups=2,
                 wscale=2.5),
    "softmax": dict(hidden=1024, inter=768, n_experts=8, n_shared=2, nsel=3, mode=3),
}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, name, NTOK, transport, q):
    import datetime

    import torch.distributed as dist

    from coherence_kernel_b200 import workloads
    from coherence_kernel_b200.ep_peer import PeerExpertParallelMoE
    from coherence_kernel_b200.moe import ExpertParallelMoE, MoELayer, MoeSpec
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        spec = MoeSpec(**SPECS[name])
        el = spec.n_experts // world
        w = workloads.make_moe(spec, NTOK, seed=11, experts=list(range(rank * el, (rank + 1) * el)))
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        T = NTOK // world
        x = t(w["x"][rank * T:(rank + 1) * T].view(np.int16))
        cls = PeerExpertParallelMoE if transport == "peer" else ExpertParallelMoE
        lay = cls(spec, t(w["gate"]), t(w["up"]), t(w["down"]), t(w["s_gate"]), t(w["s_up"]),
                                t(w["s_down"]), t(w["router"]), t(w["bias"]), max_tokens=T)
        out, ids, wts, _ = lay(x)
        lay.check()
        outs = [torch.empty_like(out) for _ in range(world)]
        idss = [torch.empty_like(ids) for _ in range(world)]
        wtss = [torch.empty_like(wts) for _ in range(world)]
        dist.all_gather(outs, out)
        dist.all_gather(idss, ids)
        dist.all_gather(wtss, wts)
        torch.cuda.synchronize()
        if rank == 0:
            wf = workloads.make_moe(spec, NTOK, seed=11)
            ref = MoELayer(spec, t(wf["gate"]), t(wf["up"]), t(wf["down"]), t(wf["s_gate"]), t(wf["s_up"]),
                           t(wf["s_down"]), t(wf["router"]), t(wf["bias"]), max_tokens=NTOK)
            rout, rids, rwts, _ = ref(t(wf["x"].view(np.int16)))
            ref.status(NTOK)
            same = (torch.equal(torch.cat(outs).view(torch.int16), rout.view(torch.int16)) and
                    torch.equal(torch.cat(idss), rids) and torch.equal(torch.cat(wtss), rwts))
            q.put(("ok" if same else "differs", transport))
        if transport == "peer":
            # a second forward over the same buffers (the barriers' step counters move on)
            dist.barrier()
            out2, ids2, _, _ = lay(x)
            lay.check()
            assert torch.equal(out2.view(torch.int16), out.view(torch.int16)) and torch.equal(ids2, ids)
            lay.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put(("error", repr(e)))
        raise


@pytest.mark.parametrize("transport", ["nccl", "peer"])
@pytest.mark.parametrize("name,world,ntok", [("dsv4", 2, 512), ("softmax", 2, 512), ("dsv4", 4, 1024),
                                             ("softmax", 4, 768), ("dsv4", 2, 64), ("dsv4", 4, 64)])
def test_expert_parallel_matches_single_gpu(name, world, ntok, transport):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, name, ntok, transport, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    verdict, info = q.get(timeout=5)
    assert verdict == "ok", info


@pytest.mark.parametrize("world,E,K,T", [(2, 16, 4, 300), (8, 256, 8, 1500), (4, 64, 8, 2048), (3, 48, 6, 1025),
                                         (2, 256, 8, 4096), (4, 256, 8, 2048), (8, 256, 8, 1024), (8, 256, 8, 16),
                                         (8, 256, 8, 1)])
def test_ep_dispatch_plan_matches_host_rules(world, E, K, T):
    """The device plan (one CTA) equals the host rules the gloo test exercises: pairs per expert,
    rows and pairs per rank, the dispatch rows in (rank, token) order with their metadata, and the
    return position of every (token, slot) pair."""
    import ctypes

    from coherence_kernel_b200 import _lib
    from coherence_kernel_b200.moe import ep_dispatch_counts, ep_dispatch_rows, ep_return_positions
    g = torch.Generator().manual_seed(T)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32).cuda()
    wts = torch.rand(T, K, generator=g).cuda()
    el = E // world
    rows_max = T * min(world, K)
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    sizes = torch.empty((world, 2), dtype=torch.int64, device="cuda")
    send_tok = torch.full((rows_max,), -7, dtype=torch.int32, device="cuda")
    meta = torch.full((rows_max, 2 * K), -7, dtype=torch.int32, device="cuda")
    ret_pos = torch.full((T * K,), -7, dtype=torch.int32, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    _lib.check(_lib.load().ck_ep_dispatch_plan(p(ids), p(wts), T, K, E, world, p(counts), p(sizes), p(send_tok),
                                               p(meta), p(ret_pos), None), "ck_ep_dispatch_plan")
    er, mask, srow, spair = ep_dispatch_counts(ids, el, world)
    S = int(srow.sum())
    tok, me, mw = ep_dispatch_rows(ids, wts, er, mask, el, S)
    assert torch.equal(counts.long(), torch.bincount(ids.reshape(-1).long(), minlength=E))
    assert torch.equal(sizes[:, 0], srow) and torch.equal(sizes[:, 1], spair)
    assert torch.equal(send_tok[:S], tok)
    assert torch.equal(meta[:S], torch.cat([me, mw.view(torch.int32)], dim=1))
    assert torch.equal(ret_pos, ep_return_positions(ids, el))


@pytest.mark.parametrize("cap,K,H,I", [(96, 4, 1024, 512), (40, 8, 7168, 2048)])
def test_fused_return_equals_return_kernel(cap, K, H, I):
    """On one GPU, with both 'ranks' of a two-rank peer table in local memory: the down projection
    that stores its rows through ck_ep_peer_return_rows' table (ck_moe_expert_gemm_rows) fills the
    return buffers with exactly the bits of the contiguous down projection followed by
    ck_ep_peer_return -- the same rows at the same (token, slot) places, nothing else written."""
    import ctypes

    from coherence_kernel_b200 import _lib, synth
    from coherence_kernel_b200.ep_peer import EpPeers
    from coherence_kernel_b200.ops import _ptr, _stream
    L, W = _lib.load(), 2
    g = torch.Generator().manual_seed(cap * K)
    rows = W * cap
    # received rows: each source's rows carry distinct tokens; about half the slots have a local expert
    ids_own = torch.where(torch.rand(rows, K, generator=g) < 0.5, 0, -1).to(torch.int32)
    tok_own = torch.cat([torch.randperm(cap, generator=g) for _ in range(W)]).to(torch.int32)
    valid = (ids_own.reshape(-1) >= 0).nonzero().reshape(-1)
    npairs = int(valid.numel())
    pair_pos2 = torch.full((rows * K,), -1, dtype=torch.int32)
    pair_pos2[valid] = torch.randperm(npairs, generator=g).to(torch.int32)
    ids_own, tok_own, pair_pos2 = ids_own.cuda(), tok_own.cuda(), pair_pos2.cuda()
    rng = np.random.default_rng(cap + K)
    w = torch.from_numpy(synth.make_q4k(rng, H * I)).cuda()
    h2 = torch.from_numpy(synth.make_bf16(rng, (npairs, I)).view(np.int16)).cuda()
    mt = npairs // 16 + 2
    tiles = torch.empty((mt, 4), dtype=torch.int32, device="cuda")
    nt = torch.empty(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _stream()
    _lib.check(L.ck_token_tiles(_ptr(tiles), _ptr(nt), npairs, st), "ck_token_tiles")
    keep = []  # buffers the peer table points at

    def table(ret):
        pe = EpPeers()
        pe.world, pe.rank, pe.cap, pe.nsel, pe.hidden = W, 0, cap, K, H
        for d in range(W):
            for name, n, dt in (("recv_x", cap * H, torch.int16), ("recv_ids", cap * K, torch.int32),
                                ("recv_w", cap * K, torch.float32), ("recv_tok", cap, torch.int32),
                                ("dflag", 1, torch.int64), ("rflag", 1, torch.int64)):
                b = torch.zeros(n, dtype=dt, device="cuda")
                keep.append(b)
                getattr(pe, name)[d] = b.data_ptr()
            pe.ret_y[d] = ret[d].data_ptr()
        for name in ("my_dflags", "my_rflags", "ctr", "err"):
            b = torch.zeros(W, dtype=torch.int64, device="cuda")
            keep.append(b)
            setattr(pe, name, b.data_ptr())
        return pe

    # the return kernel after the contiguous down projection
    ret_a = [torch.zeros((cap * K, H), dtype=torch.int16, device="cuda") for _ in range(W)]
    y2 = torch.empty((npairs, H), dtype=torch.int16, device="cuda")
    _lib.check(L.ck_moe_expert_gemm_bounded(0, _ptr(w), None, None, None, 0, 1, 0, _ptr(h2), npairs, _ptr(y2), npairs,
                                            None, _ptr(tiles), _ptr(nt), mt, H, I, 0, 0, _ptr(err), st), "down")
    pa = table(ret_a)
    _lib.check(L.ck_ep_peer_return(ctypes.byref(pa), _ptr(y2), _ptr(pair_pos2), _ptr(ids_own), _ptr(tok_own), st),
               "ck_ep_peer_return")
    # the down projection storing its rows itself
    ret_b = [torch.zeros((cap * K, H), dtype=torch.int16, device="cuda") for _ in range(W)]
    pb = table(ret_b)
    row_dst = torch.zeros(rows * K, dtype=torch.int64, device="cuda")
    _lib.check(L.ck_ep_peer_return_rows(ctypes.byref(pb), _ptr(pair_pos2), _ptr(ids_own), _ptr(tok_own),
                                        _ptr(row_dst), st), "ck_ep_peer_return_rows")
    _lib.check(L.ck_moe_expert_gemm_rows(_ptr(w), 0, 1, _ptr(h2), npairs, _ptr(row_dst), npairs, _ptr(tiles), _ptr(nt),
                                         mt, H, I, 0, _ptr(err), st), "ck_moe_expert_gemm_rows")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for d in range(W):
        assert torch.equal(ret_a[d], ret_b[d])
    assert int(sum((r != 0).any(dim=1).sum() for r in ret_a)) == npairs  # every pair row landed once
