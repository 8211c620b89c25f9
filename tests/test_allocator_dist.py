"""Per-wave allgather of allocator scores across data-parallel ranks (gloo,
world size 2, CPU): every rank sees every rank's scores, the global terms
span all ranks, and each rank's allocation equals the single-process
allocation of its own requests with the union's global terms."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from specgrove_b200.allocator import (RequestScores, ScoreExchange, allocate_rank, allocate_tree_budgets,
                                      critical_path_weights)

OPTIONS = [15, 31, 63]


def _scores(rank):
    g = torch.Generator().manual_seed(100 + rank)
    n = 3 + rank
    return RequestScores(progress=[int(x) for x in torch.randint(0, 200, (n,), generator=g)],
                         ages=[int(x) for x in torch.randint(0, 40, (n,), generator=g)],
                         service_weights=[float(x) for x in torch.tensor([1.0, 2.0, 4.0])[torch.randint(0, 3, (n,),
                                                                                                     generator=g)]],
                         utilities=[[1.0 + float(torch.rand(1, generator=g)) * (k + 1) * 2 for k in range(3)]
                                    for _ in range(n)])


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ex = ScoreExchange(max_requests=8, num_tiers=3, device="cpu")
        mine = _scores(rank)
        ex.pack(mine)
        gathered = ex.exchange()
        alloc = allocate_rank(mine, gathered, OPTIONS, row_budget=400, criticality_weight=1.0, max_new_tokens=256,
                              fixed_row_equivalent=24.0)
        out[rank] = (gathered.clone(), list(alloc))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_score_exchange_and_allocation():
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    union = [_scores(r) for r in range(world)]
    lead = max(p for s in union for p in s.progress)
    oldest = max(a for s in union for a in s.ages)
    for rank in range(world):
        gathered, alloc = out[rank]
        assert torch.equal(gathered, out[0][0])                      # identical view on every rank
        assert ScoreExchange.global_terms(gathered) == (lead, oldest)
        s = union[rank]
        w = critical_path_weights(s.progress, s.ages, 1.0, 256, lead, oldest)
        w = [a * b for a, b in zip(w, s.service_weights)]
        expected = allocate_tree_budgets(w, OPTIONS, s.utilities, row_budget=400, fixed_row_equivalent=24.0)
        assert alloc == list(expected)
