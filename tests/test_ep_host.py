"""Expert-parallel dispatch/return bookkeeping on CPU ranks (gloo, world size 2 and 4).

The expert-parallel layer's host logic -- the deduplicated dispatch plan (one row per
(destination rank, token) with the slots' local experts and weights), the split sizes of the
all-to-alls and the position of every returned (token, slot) row -- exercised with the same
helpers ExpertParallelMoE uses, around a CPU stand-in for the GPU steps (the "expert" multiplies a
row by its global expert id + 1 and by the slot's route weight).  The result must equal the direct
computation, and every token must cross to each rank at most once.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from coherence_kernel_b200.moe import ep_dispatch_counts, ep_dispatch_rows, ep_return_positions


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, E, K, T, H, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        el = E // world
        g = torch.Generator().manual_seed(0)
        ids_all = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T * world)]).to(torch.int32)
        wts_all = torch.rand(T * world, K, generator=g)
        x_all = torch.randn(T * world, H, generator=g)
        sl = slice(rank * T, (rank + 1) * T)
        ids, wts, x = ids_all[sl], wts_all[sl], x_all[sl]
        er, mask, srow, spair = ep_dispatch_counts(ids, el, world)
        sizes = torch.stack([srow, spair], dim=1).to(torch.int64)
        rsizes = torch.empty_like(sizes)
        dist.all_to_all_single(rsizes, sizes)
        srow_l, spair_l, rrow_l, rpair_l = torch.cat([sizes.t(), rsizes.t()]).tolist()
        S, R, P = sum(srow_l), sum(rrow_l), sum(rpair_l)
        send_tok, me, mw = ep_dispatch_rows(ids, wts, er, mask, el, S)
        distinct = sum(len(set((ids[t] // el).tolist())) for t in range(T))
        ok = S == distinct and int(spair.sum()) == T * K
        meta = torch.cat([me, mw.view(torch.int32)], dim=1)
        recv_x = torch.empty(R, H)
        recv_meta = torch.empty(R, 2 * K, dtype=torch.int32)
        dist.all_to_all_single(recv_x, x[send_tok.long()], output_split_sizes=rrow_l, input_split_sizes=srow_l)
        dist.all_to_all_single(recv_meta, meta, output_split_sizes=rrow_l, input_split_sizes=srow_l)
        rme, rmw = recv_meta[:, :K], recv_meta[:, K:].contiguous().view(torch.float32)
        # the receiver: every valid (row, slot) pair in (row, slot) order
        rows, slots = torch.nonzero(rme >= 0, as_tuple=True)
        ok = ok and rows.numel() == P
        gexp = rme[rows, slots].float() + rank * el + 1
        y_recv = recv_x[rows] * (gexp * rmw[rows, slots]).unsqueeze(1)
        y_back = torch.empty(T * K, H)
        dist.all_to_all_single(y_back, y_recv, output_split_sizes=spair_l, input_split_sizes=rpair_l)
        pos = ep_return_positions(ids, el).long()
        out = y_back[pos].view(T, K, H).sum(1)
        ref = (x.unsqueeze(1) * ((ids.float() + 1) * wts).unsqueeze(2)).sum(1)
        ret[rank] = bool(ok and torch.allclose(out, ref, rtol=1e-5, atol=1e-5))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,E,K,T,H", [(2, 8, 2, 16, 4), (2, 32, 8, 64, 8), (4, 64, 8, 48, 4)])
def test_ep_exchange_round_trip_gloo(world, E, K, T, H):
    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), E, K, T, H, ret), nprocs=world, join=True,
                       start_method="spawn")
    assert dict(ret) == {r: True for r in range(world)}


def _worker_drop(rank, world, port, ret):
    """Rank 1 leaves between steps (before the sizes exchange); rank 0's exchange must end with an
    error within the process group's short timeout rather than wait for good."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    ids = torch.tensor([[0, 1]], dtype=torch.int32)
    er, mask, srow, spair = ep_dispatch_counts(ids, 1, world)
    sizes = torch.stack([srow, spair], dim=1).to(torch.int64)
    if rank == 1:
        ret[rank] = "left"
        os._exit(0)  # no collective in flight: the rank leaves between steps
    t0 = time.monotonic()
    try:
        dist.all_to_all_single(torch.empty_like(sizes), sizes)
        ret[rank] = "completed"
    except Exception:
        ret[rank] = "raised" if time.monotonic() - t0 < 60 else "late"
    os._exit(0)


def test_ep_exchange_detects_a_missing_rank():
    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    ctx = mp.start_processes(_worker_drop, args=(2, _free_port(), ret), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(120)
    assert dict(ret) == {0: "raised", 1: "left"}
