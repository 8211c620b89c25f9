"""Open-loop serving of tree-verification waves over data-parallel ranks.

The request flow of the reference's open-loop serving experiments (serving
``scripts/run_openloop_scheduler_supplement.py:91-96`` Poisson arrivals,
``:250-298`` driver; admission at wave boundaries, serving
``continuous_tree_block_decode.py:1677-1717``; the exact-row tier allocator
of ``continuous_tree_block_decode.py:706-795``) with requests partitioned
across one process per GPU:

* arrivals follow a seeded Poisson process; at each wave boundary every rank
  sees the same arrivals (the global clock is the largest rank clock of the
  per-wave exchange) and assigns them, in arrival order, to the least-loaded
  rank (active plus queued requests, ties to the lower rank), so every rank
  makes the same decision without another message;
* a queued request takes a free arena slot; its prompt KV is synthetic (the
  prefill pass is not part of this step) and its slot length is the prompt
  length;
* every wave, each rank packs its requests' allocator scores (progress, age,
  service weight, per-tier draft utilities) plus its clock, load and done
  flag into the fixed-size allgather (``allocator.ScoreExchange``), solves
  its own exact-row knapsack with the global leading progress and oldest age
  (weights multiplied by the request's service weight), builds the wave from
  each request's canonical tree cut to its tier, runs one verify pass with
  commit, and reads the decisions back;
* a request leaves after ``max_new_tokens`` committed tokens (accepted nodes
  plus the bonus token each wave); the loop ends when every rank is done and
  every arrival has been assigned.  All ranks take the same number of
  exchanges.

``SpecServer`` runs the same loop on the full speculative step
(``speculative.SpecDecoder``): an admitted request's prompt is prefilled into
the target's arena and the draft cache (real prefill, not synthetic KV), and
every wave is one drafter pass, the on-device wave plan (trees, tier
knapsack with the critical-path weights of the global terms) and one verify
pass.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np
import torch

from .allocator import RequestScores, ScoreExchange, allocate_tree_budgets, critical_path_weights


@dataclass
class ServeRequest:
    rid: int
    arrival: float                 # seconds after the start
    prompt_len: int
    service_weight: float
    parents: list                  # canonical tree, root parent -1
    tokens: list                   # root input token first
    utilities: list                # draft expected tokens per tier option
    rank: int = -1
    slot: int = -1
    generated: int = 0
    admitted_wave: int = -1
    finish: float | None = None


def make_requests(num_requests: int, rate_per_s: float, prompt_range: tuple, tier_rows: Sequence[int], vocab: int,
                  seed: int = 0, block: int = 16, top_k: int = 4, draft_scale: float = 4.0,
                  device="cuda") -> list[ServeRequest]:
    """Seeded Poisson arrivals, log-uniform prompt lengths, service weights
    uniform over {1, 2, 4}, and one canonical best-first draft tree per
    request (block draft positions, top-k children per depth) with the draft
    utilities of every tier (rows including the root)."""
    from .workloads import best_first_tree
    rng = np.random.default_rng(seed)
    arrivals = np.cumsum(rng.exponential(1.0 / rate_per_s, size=num_requests))
    lo, hi = math.log(prompt_range[0]), math.log(prompt_range[1])
    prompts = np.exp(rng.uniform(lo, hi, size=num_requests)).astype(np.int64)
    weights = rng.choice([1.0, 2.0, 4.0], size=num_requests)
    gen = torch.Generator(device=device).manual_seed(seed)
    budget = max(tier_rows) - 1
    out = []
    for i in range(num_requests):
        draft = torch.randn((block, vocab), generator=gen, device=device) * draft_scale
        vals, idx = torch.topk(torch.log_softmax(draft, -1), top_k, dim=-1)
        parents, tokens, _, masses = best_first_tree(vals.tolist(), idx.tolist(), budget, [top_k] * block)
        tokens[0] = int(rng.integers(0, vocab))
        utilities = [1.0 + float(np.exp(np.asarray(masses[1:t])).sum()) for t in tier_rows]
        out.append(ServeRequest(i, float(arrivals[i]), int(prompts[i]), float(weights[i]), parents, tokens,
                                utilities))
    return out


@dataclass
class ServeStats:
    tokens: int = 0
    waves: int = 0
    rows: int = 0
    requests: int = 0
    exchanges: int = 0
    host_ms: float = 0.0
    admit_ms: float = 0.0          # SpecServer: prefill of admitted prompts (host clock; the call synchronizes)
    step_ms: float = 0.0           # SpecServer: speculative steps (host clock; the call synchronizes)
    rows_verified: int = 0         # SpecServer: rows of the verify waves
    finish_times: list = field(default_factory=list)


class OpenLoopServer:
    """One rank's serving loop.  ``step(trees, slots, lengths, request_ids,
    seed)`` runs one verify pass with commit and returns each request's
    accepted-node count (the host copy of accept_out[:, max_depth])."""

    def __init__(self, requests: Sequence[ServeRequest], step: Callable, *, rank: int, world: int,
                 exchange: ScoreExchange, num_slots: int, capacity: int, tier_rows: Sequence[int],
                 row_budget: int, max_new_tokens: int, criticality_weight: float = 1.0,
                 row_cost_curve: Sequence[tuple[int, float]] | None = None, clock: Callable = time.perf_counter,
                 idle_sleep_s: float = 5e-4):
        self.requests = sorted(requests, key=lambda r: r.arrival)
        self.step = step
        self.rank, self.world = rank, world
        self.exchange = exchange
        self.num_slots, self.capacity = num_slots, capacity
        self.tier_rows = list(tier_rows)
        self.options = [t - 1 for t in self.tier_rows]      # draft nodes of each tier
        self.row_budget = row_budget
        self.max_new = max_new_tokens
        self.criticality = criticality_weight
        self.curve = row_cost_curve
        self.clock = clock
        self.idle_sleep_s = idle_sleep_s
        self.lengths = [0] * num_slots

    def run(self, seed: int = 0) -> ServeStats:
        stats = ServeStats()
        t0 = self.clock()
        free = list(range(self.num_slots - 1, -1, -1))
        active: list[ServeRequest] = []
        queue: list[ServeRequest] = []
        assigned = 0
        wave = 0
        while True:
            h0 = self.clock()
            now = h0 - t0
            scores = RequestScores(progress=[r.generated for r in active],
                                   ages=[wave - r.admitted_wave for r in active],
                                   service_weights=[r.service_weight for r in active],
                                   utilities=[r.utilities for r in active])
            done = not active and not queue
            self.exchange.pack(scores, header=[now, len(active) + len(queue), 1.0 if done else 0.0])
            g = self.exchange.exchange().cpu()
            stats.exchanges += 1
            if bool((g[:, 0, 3] > 0).all()) and assigned == len(self.requests):
                break
            gclock = float(g[:, 0, 1].max())
            loads = g[:, 0, 2].tolist()
            while assigned < len(self.requests) and self.requests[assigned].arrival <= gclock:
                r = self.requests[assigned]
                r.rank = min(range(self.world), key=lambda k: (loads[k], k))
                loads[r.rank] += 1
                if r.rank == self.rank:
                    queue.append(r)
                assigned += 1
            while queue and free:
                r = queue.pop(0)
                r.slot = free.pop()
                r.admitted_wave = wave
                self.lengths[r.slot] = r.prompt_len
                active.append(r)
            if not active:
                stats.host_ms += (self.clock() - h0) * 1000
                time.sleep(self.idle_sleep_s)
                continue
            # global terms over every rank's requests (this rank's included;
            # requests admitted just now have progress 0 and age 0)
            lead, oldest = ScoreExchange.global_terms(g)
            weights = critical_path_weights([r.generated for r in active], [wave - r.admitted_wave for r in active],
                                            self.criticality, self.max_new, max(lead, 0), max(oldest, 1))
            weights = [w * r.service_weight for w, r in zip(weights, active)]
            alloc = allocate_tree_budgets(weights, self.options, [r.utilities for r in active],
                                          row_budget=self.row_budget, row_cost_curve=self.curve,
                                          fixed_row_equivalent=None if self.curve else 32.0)
            trees = [(r.parents[:b + 1], r.tokens[:b + 1]) for r, b in zip(active, alloc)]
            slots = [r.slot for r in active]
            lengths = [self.lengths[s] for s in slots]
            stats.host_ms += (self.clock() - h0) * 1000
            counts = self.step(trees, slots, lengths, [r.rid for r in active], seed + wave)
            h1 = self.clock()
            stats.waves += 1
            stats.rows += sum(len(t[0]) for t in trees)
            still = []
            for r, c in zip(active, counts):
                kept = int(c) + 1
                self.lengths[r.slot] += kept
                gained = min(kept, self.max_new - r.generated)
                r.generated += gained
                stats.tokens += gained
                if r.generated >= self.max_new:
                    r.finish = self.clock() - t0
                    stats.finish_times.append(r.finish - r.arrival)
                    stats.requests += 1
                    free.append(r.slot)
                else:
                    still.append(r)
            active = still
            wave += 1
            stats.host_ms += (self.clock() - h1) * 1000
        return stats


def make_prompts(requests: Sequence[ServeRequest], vocab: int, seed: int = 0) -> dict[int, list[int]]:
    """Seeded random prompt tokens of each request's prompt length."""
    g = torch.Generator().manual_seed(seed)
    return {r.rid: torch.randint(0, vocab, (r.prompt_len,), generator=g).tolist() for r in requests}


class SpecServer:
    """One rank's open-loop serving loop over a ``SpecDecoder`` (the decoder
    owns the arena slots; a queued request is admitted when one is free)."""

    def __init__(self, requests: Sequence[ServeRequest], decoder, prompts: dict, *, rank: int, world: int,
                 exchange: ScoreExchange, num_tiers: int, max_new_tokens: int, criticality_weight: float = 1.0,
                 clock: Callable = time.perf_counter, idle_sleep_s: float = 5e-4, max_admit_per_wave: int = 8):
        self.requests = sorted(requests, key=lambda r: r.arrival)
        self.decoder = decoder
        self.prompts = prompts
        self.rank, self.world = rank, world
        self.exchange = exchange
        self.num_tiers = num_tiers
        self.max_new = max_new_tokens
        self.criticality = criticality_weight
        self.clock = clock
        self.idle_sleep_s = idle_sleep_s
        self.max_admit = max_admit_per_wave

    def run(self) -> ServeStats:
        from .speculative import SpecRequest
        stats = ServeStats()
        t0 = self.clock()
        active: list[tuple[ServeRequest, SpecRequest]] = []
        queue: list[ServeRequest] = []
        assigned = 0
        wave = 0
        while True:
            h0 = self.clock()
            now = h0 - t0
            scores = RequestScores(progress=[len(s.generated) for _, s in active],
                                   ages=[wave - r.admitted_wave for r, _ in active],
                                   service_weights=[r.service_weight for r, _ in active],
                                   utilities=[[1.0] * self.num_tiers for _ in active])
            done = not active and not queue
            self.exchange.pack(scores, header=[now, len(active) + len(queue), 1.0 if done else 0.0])
            g = self.exchange.exchange().cpu()
            stats.exchanges += 1
            if bool((g[:, 0, 3] > 0).all()) and assigned == len(self.requests):
                break
            gclock = float(g[:, 0, 1].max())
            loads = g[:, 0, 2].tolist()
            while assigned < len(self.requests) and self.requests[assigned].arrival <= gclock:
                r = self.requests[assigned]
                r.rank = min(range(self.world), key=lambda k: (loads[k], k))
                loads[r.rank] += 1
                if r.rank == self.rank:
                    queue.append(r)
                assigned += 1
            admit = []
            while queue and len(self.decoder.free_slots) > len(admit) and len(admit) < self.max_admit:
                r = queue.pop(0)
                r.admitted_wave = wave
                admit.append((r, SpecRequest(r.rid, self.prompts[r.rid], self.max_new,
                                             weight=r.service_weight)))
            stats.host_ms += (self.clock() - h0) * 1000
            if admit:
                a0 = self.clock()
                self.decoder.admit([s for _, s in admit])
                stats.admit_ms += (self.clock() - a0) * 1000
                for r, s in admit:
                    r.slot = s.slot
                    r.generated = len(s.generated)
                    stats.tokens += len(s.generated)
                active.extend(admit)
            if not active:
                time.sleep(self.idle_sleep_s)
                continue
            h1 = self.clock()
            lead, oldest = ScoreExchange.global_terms(g)
            weights = critical_path_weights([len(s.generated) for _, s in active],
                                            [wave - r.admitted_wave for r, _ in active], self.criticality,
                                            self.max_new, max(lead, 0), max(oldest, 1))
            for (r, s), w in zip(active, weights):
                s.weight = w * r.service_weight
            stats.host_ms += (self.clock() - h1) * 1000
            rows_before = sum(self.decoder.target.arena.lengths[s.slot] for _, s in active)
            verified = self.decoder.rows_verified
            s0 = self.clock()
            stats.tokens += self.decoder.step()
            stats.step_ms += (self.clock() - s0) * 1000
            stats.rows_verified += self.decoder.rows_verified - verified
            stats.rows += sum(self.decoder.target.arena.lengths[s.slot] for _, s in active) - rows_before
            stats.waves += 1
            still = []
            for r, s in active:
                r.generated = len(s.generated)
                if s.done:
                    r.finish = self.clock() - t0
                    stats.finish_times.append(r.finish - r.arrival)
                    stats.requests += 1
                else:
                    still.append((r, s))
            active = still
            wave += 1
        return stats
