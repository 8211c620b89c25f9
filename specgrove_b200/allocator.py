"""Shared-budget tier allocation across data-parallel ranks.

Host-side planning that chooses each request's tree tier for the next wave.
It restates the reference's exact-row allocator
(continuous_tree_block_decode.py:560-568 ``_draft_tree_expected_tokens``,
:619-641 ``_global_wave_cost``, :706-795 ``_allocate_global_tree_budgets``):
a multiple-choice knapsack solved by dynamic programming over exact row
counts, maximising weighted draft-side expected tokens divided by the wave
cost, with causal critical-path weights
``1 + c * ((leading_progress - generated) / max_new_tokens + age / max_age)``.

With requests sharded over GPUs, the weights' global terms (the leading
request's progress, the oldest request's age) span every rank.
``ScoreExchange`` carries each rank's per-request scores in one fixed-size
fp64 tensor through ``torch.distributed.all_gather_into_tensor`` (NCCL over
NVLink on GPUs) once per wave; every rank then solves its own knapsack for its
own row budget with the global terms.  No KV, weights or activations are
exchanged.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import torch


def draft_tree_expected_tokens(prefix_log_masses: Sequence[float]) -> float:
    """1 + sum of draft prefix masses of the non-root nodes (:560-568)."""
    value = 1.0 + sum(math.exp(m) for m in prefix_log_masses[1:])
    if not math.isfinite(value) or value < 1.0:
        raise FloatingPointError("Invalid draft-tree expected-token utility")
    return value


def wave_cost(rows: int, fixed_row_equivalent: float | None,
              row_cost_curve: Sequence[tuple[int, float]] | None) -> float:
    """Piecewise-linear measured wave cost, or fixed + rows (:619-641)."""
    if rows < 1:
        raise ValueError("A Target wave must contain at least one row")
    if row_cost_curve is None:
        if fixed_row_equivalent is None or not math.isfinite(fixed_row_equivalent) or fixed_row_equivalent <= 0:
            raise ValueError("Missing global Target cost model")
        return fixed_row_equivalent + rows
    curve = tuple(row_cost_curve)
    if rows <= curve[0][0]:
        return curve[0][1]
    for (lr, lc), (rr, rc) in zip(curve, curve[1:]):
        if rows <= rr:
            return lc + (rows - lr) / (rr - lr) * (rc - lc)
    return curve[-1][1]


def critical_path_weights(progress: Sequence[int], ages: Sequence[int], criticality_weight: float,
                          max_new_tokens: int, leading_progress: int | None = None,
                          maximum_age: int | None = None) -> list[float]:
    """Per-request weights; global terms default to this request set's."""
    lead = max(progress) if leading_progress is None else leading_progress
    oldest = max(ages) if maximum_age is None else maximum_age
    return [1.0 + criticality_weight * ((lead - g) / max_new_tokens + a / max(1, oldest))
            for g, a in zip(progress, ages)]


def allocate_tree_budgets(weights: Sequence[float], budget_options: Sequence[int],
                          utilities: Sequence[Sequence[float]], *, row_budget: int,
                          fixed_row_equivalent: float | None = None,
                          row_cost_curve: Sequence[tuple[int, float]] | None = None) -> tuple[int, ...]:
    """Exact-row DP (:765-795): for every reachable row count keep the best
    weighted reward (ties -> lexicographically smaller allocation); pick the
    row count maximising reward / wave cost (ties -> fewer rows, larger trees)."""
    options = tuple(int(v) for v in budget_options)
    if (not weights or tuple(sorted(set(options))) != options or options[0] < 1
            or row_budget < len(weights) * (options[0] + 1)
            or (fixed_row_equivalent is None) == (row_cost_curve is None)
            or len(utilities) != len(weights) or any(len(u) != len(options) for u in utilities)):
        raise ValueError("Invalid global tree-budget allocation problem")
    frontier: dict[int, tuple[float, tuple[int, ...]]] = {0: (0.0, ())}
    for weight, values in zip(weights, utilities):
        updated: dict[int, tuple[float, tuple[int, ...]]] = {}
        for used, (reward, alloc) in frontier.items():
            for budget, utility in zip(options, values):
                rows = used + budget + 1
                if rows > row_budget:
                    continue
                cand = (reward + weight * utility, alloc + (budget,))
                prev = updated.get(rows)
                if (prev is None or cand[0] > prev[0] + 1e-12
                        or (abs(cand[0] - prev[0]) <= 1e-12 and cand[1] < prev[1])):
                    updated[rows] = cand
        frontier = updated
    if not frontier:
        raise RuntimeError("Global tree-budget allocator found no feasible wave")
    _, (_, allocation) = max(
        frontier.items(),
        key=lambda item: (item[1][0] / wave_cost(item[0], fixed_row_equivalent, row_cost_curve), -item[0],
                          tuple(-v for v in item[1][1])))
    return allocation


@dataclass
class RequestScores:
    """One rank's allocator inputs for its requests."""
    progress: list[int]           # tokens generated so far
    ages: list[int]               # waves since admission
    service_weights: list[float]  # per-request service weight (1 = plain)
    utilities: list[list[float]]  # expected tokens per tier


class ScoreExchange:
    """Fixed-size per-wave allgather of allocator scores.

    Layout per rank: row 0 = [request count, 0...]; rows 1..max_requests =
    [valid, progress, age, service weight, utility_0 .. utility_{T-1}] (fp64).
    """

    def __init__(self, max_requests: int, num_tiers: int, device, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.max_requests = max_requests
        self.num_tiers = num_tiers
        self.width = 4 + num_tiers
        self.local = torch.zeros((max_requests + 1, self.width), dtype=torch.float64, device=device)
        self.gathered = torch.zeros((self.world, max_requests + 1, self.width), dtype=torch.float64, device=device)

    def pack(self, scores: RequestScores) -> None:
        n = len(scores.progress)
        if n > self.max_requests:
            raise ValueError("more requests than the exchange was sized for")
        host = torch.zeros((self.max_requests + 1, self.width), dtype=torch.float64)
        host[0, 0] = n
        for i in range(n):
            host[1 + i, :4] = torch.tensor([1.0, scores.progress[i], scores.ages[i], scores.service_weights[i]],
                                           dtype=torch.float64)
            host[1 + i, 4:4 + len(scores.utilities[i])] = torch.tensor(scores.utilities[i], dtype=torch.float64)
        self.local.copy_(host, non_blocking=True)

    def exchange(self) -> torch.Tensor:
        """All ranks' score tables, [world, max_requests + 1, width]."""
        if self.world == 1:
            self.gathered[0].copy_(self.local)
        else:
            self.dist.all_gather_into_tensor(self.gathered.view(-1, self.width), self.local, group=self.group)
        return self.gathered

    @staticmethod
    def global_terms(gathered: torch.Tensor) -> tuple[int, int]:
        """(leading progress, maximum age) over every rank's valid requests."""
        g = gathered.cpu()
        valid = g[:, 1:, 0] > 0
        progress = g[:, 1:, 1][valid]
        ages = g[:, 1:, 2][valid]
        return int(progress.max().item()), int(ages.max().item())


def allocate_rank(scores: RequestScores, gathered: torch.Tensor, budget_options: Sequence[int], *,
                  row_budget: int, criticality_weight: float, max_new_tokens: int,
                  fixed_row_equivalent: float | None = None,
                  row_cost_curve: Sequence[tuple[int, float]] | None = None) -> tuple[int, ...]:
    """This rank's tiers, weighted with the global terms of all ranks and the
    per-request service weight (an extension: the reference has lag/age
    weights only)."""
    lead, oldest = ScoreExchange.global_terms(gathered)
    weights = critical_path_weights(scores.progress, scores.ages, criticality_weight, max_new_tokens, lead, oldest)
    weights = [w * sw for w, sw in zip(weights, scores.service_weights)]
    return allocate_tree_budgets(weights, budget_options, scores.utilities, row_budget=row_budget,
                                 fixed_row_equivalent=fixed_row_equivalent, row_cost_curve=row_cost_curve)
