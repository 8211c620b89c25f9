"""Shared-budget tier allocation across data-parallel ranks.

Host-side planning that chooses each request's tree tier for the next wave,
the role of the reference's exact-row allocator
(continuous_tree_block_decode.py:706-795, with the draft utility of :560-568
and the wave-cost model of :619-641).  The knapsack itself is native code in
the library (``sg_allocate_tiers``, include/specgrove_b200.h): one tier per
request, maximising weighted draft expected tokens divided by the measured
wave cost, with the critical-path weights
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

import ctypes
import math
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from . import _lib


def draft_tree_expected_tokens(prefix_log_masses: Sequence[float]) -> float:
    """Expected accepted tokens of a draft tree plus its bonus: one plus the
    draft probability mass of every non-root node's prefix."""
    masses = [math.exp(float(v)) for v in list(prefix_log_masses)[1:]]
    total = 1.0 + math.fsum(masses)
    if not (math.isfinite(total) and total >= 1.0):
        raise FloatingPointError("draft expected-token utility is not a finite value >= 1")
    return total


def critical_path_weights(progress: Sequence[int], ages: Sequence[int], criticality_weight: float,
                          max_new_tokens: int, leading_progress: int | None = None,
                          maximum_age: int | None = None) -> list[float]:
    """Per-request weights; the global terms default to this request set's
    own leading progress and oldest age."""
    lead = max(progress) if leading_progress is None else leading_progress
    oldest = max(1, max(ages) if maximum_age is None else maximum_age)
    weights = []
    for generated, age in zip(progress, ages):
        lag = (lead - generated) / max_new_tokens
        weights.append(1.0 + criticality_weight * (lag + age / oldest))
    return weights


def allocate_tree_budgets(weights: Sequence[float], budget_options: Sequence[int],
                          utilities: Sequence[Sequence[float]], *, row_budget: int,
                          fixed_row_equivalent: float | None = None,
                          row_cost_curve: Sequence[tuple[int, float]] | None = None) -> tuple[int, ...]:
    """One tier per request from ``budget_options`` (draft nodes; a tier of b
    nodes takes b + 1 rows) under ``row_budget`` rows, through the native
    exact-row knapsack.  Exactly one cost model: ``fixed_row_equivalent``
    (cost = fixed + rows) or ``row_cost_curve`` [(rows, cost), ...]."""
    R, T = len(weights), len(budget_options)
    util = np.asarray(utilities, dtype=np.float64)
    if R < 1 or util.shape != (R, T) or (fixed_row_equivalent is None) == (row_cost_curve is None):
        raise ValueError("tier allocation needs one weight and one utility per option for every request, "
                         "and exactly one cost model")
    w = np.ascontiguousarray(weights, dtype=np.float64)
    opts = np.ascontiguousarray(budget_options, dtype=np.int32)
    util = np.ascontiguousarray(util)
    curve = list(row_cost_curve or [])
    c_rows = np.ascontiguousarray([int(r) for r, _ in curve] or [0], dtype=np.int32)
    c_cost = np.ascontiguousarray([float(c) for _, c in curve] or [0.0], dtype=np.float64)
    fixed = math.nan if fixed_row_equivalent is None else float(fixed_row_equivalent)
    out = np.zeros(R, dtype=np.int32)
    lib = _lib.load()
    st = lib.sg_allocate_tiers(R, w.ctypes.data, T, opts.ctypes.data, util.ctypes.data, int(row_budget), fixed,
                               c_rows.ctypes.data, c_cost.ctypes.data, len(curve), out.ctypes.data)
    if st == _lib.SG_ERR_INVALID_ARGUMENT:
        raise ValueError(lib.sg_last_error().decode())
    if st != _lib.SG_OK:
        raise RuntimeError(lib.sg_last_error().decode())
    return tuple(int(v) for v in out)


def allocate_tree_budgets_device(weights: torch.Tensor, budget_options: Sequence[int], utilities: torch.Tensor, *,
                                 row_budget: int, fixed_row_equivalent: float | None = None,
                                 row_cost_curve: Sequence[tuple[int, float]] | None = None,
                                 status: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """``allocate_tree_budgets`` on the device for CUDA fp64 ``weights`` [R]
    and ``utilities`` [R, T] (e.g. from the tree kernels): returns the int32
    tier of each request as a CUDA tensor, enqueued on ``stream`` without a
    host synchronisation.  Device-detected errors (a utility below 1, no
    feasible wave) land in ``status`` (an int32 CUDA word, atomic max of the
    codes) with every tier -1."""
    R, T = weights.shape[0], len(budget_options)
    if (weights.dtype != torch.float64 or utilities.dtype != torch.float64 or not weights.is_cuda
            or utilities.shape != (R, T) or (fixed_row_equivalent is None) == (row_cost_curve is None)):
        raise ValueError("device tier allocation needs CUDA fp64 weights [R] and utilities [R, T], and exactly "
                         "one cost model")
    weights = weights.contiguous()
    utilities = utilities.contiguous()
    opts = np.ascontiguousarray(budget_options, dtype=np.int32)
    curve = list(row_cost_curve or [])
    c_rows = np.ascontiguousarray([int(r) for r, _ in curve] or [0], dtype=np.int32)
    c_cost = np.ascontiguousarray([float(c) for _, c in curve] or [0.0], dtype=np.float64)
    fixed = math.nan if fixed_row_equivalent is None else float(fixed_row_equivalent)
    lib = _lib.load()
    ws_bytes = lib.sg_allocate_tiers_device_workspace_bytes(R, int(row_budget))
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=weights.device)
    out = torch.empty(R, dtype=torch.int32, device=weights.device)
    st = lib.sg_allocate_tiers_device(R, weights.data_ptr(), T, opts.ctypes.data, utilities.data_ptr(),
                                      int(row_budget), fixed, c_rows.ctypes.data, c_cost.ctypes.data, len(curve),
                                      out.data_ptr(), _lib.ptr(status), ws.data_ptr(), ws_bytes,
                                      _lib.stream_ptr(stream))
    if st == _lib.SG_ERR_INVALID_ARGUMENT:
        raise ValueError(lib.sg_last_error().decode())
    _lib.check(st, "sg_allocate_tiers_device")
    return out


@dataclass
class RequestScores:
    """One rank's allocator inputs for its requests."""
    progress: list[int]           # tokens generated so far
    ages: list[int]               # waves since admission
    service_weights: list[float]  # per-request service weight (1 = plain)
    utilities: list[list[float]]  # expected tokens per tier


class ScoreExchange:
    """Fixed-size per-wave allgather of allocator scores.

    Layout per rank: row 0 = [request count, header values (e.g. the rank's
    clock, load and done flag) ...]; rows 1..max_requests = [valid, progress,
    age, service weight, utility_0 .. utility_{T-1}] (fp64).
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

    def pack(self, scores: RequestScores, header: Sequence[float] = ()) -> None:
        n = len(scores.progress)
        if n > self.max_requests:
            raise ValueError("more requests than the exchange was sized for")
        if len(header) > self.width - 1:
            raise ValueError("header wider than a score row")
        host = torch.zeros((self.max_requests + 1, self.width), dtype=torch.float64)
        host[0, 0] = n
        if len(header):
            host[0, 1:1 + len(header)] = torch.tensor([float(v) for v in header], dtype=torch.float64)
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
        if not bool(valid.any()):
            return 0, 0
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
