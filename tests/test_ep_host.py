"""Expert-parallel dispatch/return bookkeeping on CPU ranks (gloo, world size 2).

The expert-parallel layer's host logic -- the split sizes of the two all-to-alls and the local
expert of every received row -- exercised with the same helpers ExpertParallelMoE uses, around a
CPU stand-in for the GPU steps (stable counting sort by expert = a stable argsort; the "expert"
multiplies a row by its global expert id + 1).  The result must equal the direct computation.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from coherence_kernel_b200.moe import ep_recv_local_experts, ep_split_sizes


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
        g = torch.Generator().manual_seed(0)
        ids_all = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T * world)]).to(torch.int32)
        x_all = torch.randn(T * world, H, generator=g)
        ids, x = ids_all[rank * T:(rank + 1) * T], x_all[rank * T:(rank + 1) * T]
        flat = ids.reshape(-1)
        order = torch.argsort(flat, stable=True)          # ck_moe_permute's stable counting sort
        xp = x[order // K]
        counts = torch.bincount(flat, minlength=E).to(torch.int32)
        recv_counts_e = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts_e, counts)
        sc, rc = ep_split_sizes(counts, recv_counts_e, world)
        nrecv = int(sum(rc))
        recv = torch.empty(nrecv, H)
        dist.all_to_all_single(recv, xp, output_split_sizes=rc, input_split_sizes=sc)
        le = ep_recv_local_experts(recv_counts_e, world, nrecv)
        o2 = torch.argsort(le, stable=True)               # the receiver's regroup
        y2 = recv[o2] * (le[o2].float() + 1 + rank * (E // world)).unsqueeze(1)
        y_recv = torch.empty_like(y2)
        y_recv[o2] = y2                                   # restore arrival order
        y_back = torch.empty(T * K, H)
        dist.all_to_all_single(y_back, y_recv, output_split_sizes=sc, input_split_sizes=rc)
        y_pair = torch.empty_like(y_back)
        y_pair[order] = y_back
        out = y_pair.view(T, K, H).sum(1)
        ref = (x.unsqueeze(1) * (ids.float() + 1).unsqueeze(2)).sum(1)
        ret[rank] = bool(torch.allclose(out, ref)) and nrecv == int(recv_counts_e.sum())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("E,K,T,H", [(8, 2, 16, 4), (32, 8, 64, 8)])
def test_ep_exchange_round_trip_gloo(E, K, T, H):
    world = 2
    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), E, K, T, H, ret), nprocs=world, join=True,
                       start_method="spawn")
    assert dict(ret) == {0: True, 1: True}
