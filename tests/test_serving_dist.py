"""The open-loop serving loop (specgrove_b200/serving.py) on two gloo ranks
(CPU) with a stand-in verify step: every arrival is assigned to exactly one
rank and every rank agrees on the assignment, the ranks take the same number
of exchanges, every request leaves with max_new_tokens tokens, the wave row
budget holds, and a rank's slots never exceed its arena."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from specgrove_b200.allocator import ScoreExchange
from specgrove_b200.serving import OpenLoopServer, ServeRequest

TIERS = [16, 32, 64]
MAX_NEW = 12


def _requests():
    rng = np.random.default_rng(3)
    arrivals = np.cumsum(rng.exponential(0.002, size=30))
    out = []
    for i, t in enumerate(arrivals):
        parents = [-1] + [int(rng.integers(0, j)) for j in range(1, 64)]
        tokens = [int(v) for v in rng.integers(0, 1000, size=64)]
        out.append(ServeRequest(i, float(t), int(rng.integers(16, 64)), float(rng.choice([1, 2, 4])), parents,
                                tokens, [1.0, 1.5 + i % 3, 2.0 + i % 5]))
    return out


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(rank)
        seen = {"rows": [], "slots": set(), "rids": set()}

        def step(trees, slots, lengths, rids, seed):
            seen["rows"].append(sum(len(t[0]) for t in trees))
            seen["slots"].update(slots)
            seen["rids"].update(rids)
            assert len(set(slots)) == len(slots)
            for (par, _), L in zip(trees, lengths):
                assert L + len(par) <= 200
            return [int(rng.integers(0, 3)) for _ in trees]

        ex = ScoreExchange(max_requests=4, num_tiers=len(TIERS), device="cpu")
        server = OpenLoopServer(_requests(), step, rank=rank, world=world, exchange=ex, num_slots=4, capacity=200,
                                tier_rows=TIERS, row_budget=160, max_new_tokens=MAX_NEW,
                                row_cost_curve=[(16, 2.0), (64, 3.0), (160, 6.0)], idle_sleep_s=1e-4)
        stats = server.run(seed=7)
        out[rank] = dict(tokens=stats.tokens, requests=stats.requests, exchanges=stats.exchanges,
                         rows=max(seen["rows"] or [0]), slots=sorted(seen["slots"]), rids=sorted(seen["rids"]),
                         assignment=[r.rank for r in server.requests])
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_open_loop_serving():
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    n = len(_requests())
    a0, a1 = out[0], out[1]
    assert a0["assignment"] == a1["assignment"]                    # one decision, taken on every rank
    assert sorted(a0["rids"] + a1["rids"]) == list(range(n))       # each request served by exactly one rank
    assert set(a0["rids"]).isdisjoint(a1["rids"])
    assert all(0 <= r < world for r in a0["assignment"])
    assert a0["exchanges"] == a1["exchanges"]                      # lockstep collectives
    assert a0["requests"] + a1["requests"] == n
    assert a0["tokens"] + a1["tokens"] == n * MAX_NEW
    assert max(a0["rows"], a1["rows"]) <= 160
    assert set(a0["slots"]) <= set(range(4)) and set(a1["slots"]) <= set(range(4))
    assert abs(a0["requests"] - a1["requests"]) <= n // 2          # least-loaded admission spreads the work


class _FakeDecoder:
    """Host stand-in for speculative.SpecDecoder: the same slot bookkeeping,
    admission (first token) and per-step token counts (1-3 per request)."""

    def __init__(self, num_slots, seed):
        from types import SimpleNamespace
        self.free_slots = list(range(num_slots))
        self.running = []
        self.rows_verified = 0
        self.target = SimpleNamespace(arena=SimpleNamespace(lengths=[0] * num_slots))
        self.rng = np.random.default_rng(seed)
        self.weights_seen = []

    def admit(self, reqs):
        for r in reqs:
            r.slot = self.free_slots.pop(0)
            self.target.arena.lengths[r.slot] = len(r.prompt)
            r.generated = [1]
        self.running.extend(reqs)

    def step(self):
        produced = 0
        self.weights_seen.append([r.weight for r in self.running])
        for r in self.running:
            n = int(self.rng.integers(1, 4))
            room = r.max_new_tokens - len(r.generated)
            r.generated.extend([2] * min(n, room))
            produced += min(n, room)
            self.target.arena.lengths[r.slot] += n
            self.rows_verified += 8
            if len(r.generated) >= r.max_new_tokens:
                r.done = True
                self.free_slots.append(r.slot)
        self.running = [r for r in self.running if not r.done]
        return produced


def _spec_worker(rank, world, port, out):
    from specgrove_b200.serving import SpecServer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dec = _FakeDecoder(4, seed=rank)
        reqs = _requests()
        prompts = {r.rid: [7] * r.prompt_len for r in reqs}
        ex = ScoreExchange(max_requests=4, num_tiers=len(TIERS), device="cpu")
        server = SpecServer(reqs, dec, prompts, rank=rank, world=world, exchange=ex, num_tiers=len(TIERS),
                            max_new_tokens=MAX_NEW, idle_sleep_s=1e-4, max_admit_per_wave=2)
        stats = server.run()
        out[rank] = dict(tokens=stats.tokens, requests=stats.requests, exchanges=stats.exchanges,
                         assignment=[r.rank for r in server.requests], free=sorted(dec.free_slots),
                         weights_ok=all(w > 0 for ws in dec.weights_seen for w in ws),
                         rids=sorted(r.rid for r in server.requests if r.rank == rank and r.finish is not None))
    finally:
        dist.destroy_process_group()


def test_two_rank_spec_server():
    """SpecServer (the serving loop over the speculative step) on two gloo
    ranks with a host stand-in for the decoder: one assignment on every rank,
    lockstep exchanges, every request served to max_new_tokens by one rank,
    every slot released."""
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_spec_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    n = len(_requests())
    a0, a1 = out[0], out[1]
    assert a0["assignment"] == a1["assignment"]
    assert a0["exchanges"] == a1["exchanges"]
    assert sorted(a0["rids"] + a1["rids"]) == list(range(n))
    assert a0["requests"] + a1["requests"] == n
    assert a0["tokens"] + a1["tokens"] == n * MAX_NEW
    assert a0["free"] == [0, 1, 2, 3] and a1["free"] == [0, 1, 2, 3]
    assert a0["weights_ok"] and a1["weights_ok"]
