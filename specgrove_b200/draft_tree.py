"""On-device wave planning from the drafter's logits.

The reference builds each request's draft tree on the host
(``probability_tree``, tree.py:148-212, on ``probabilities(logits, T,
float64)``, sampling.py:29-36), cuts it to tiers (``_prefix_tree``) and
scores them (``_draft_tree_expected_tokens``,
continuous_tree_block_decode.py:560-586), runs the tier knapsack
(``_allocate_global_tree_budgets``, :706-795) and packs the chosen prefixes
into the verify wave (:839-883, :500-546).  Here every step is a kernel of
the library and the whole plan stays on the device:

  sg_proposal_topk         logits -> top-k log masses and ids per depth
  sg_build_draft_trees     best-first trees, tier utilities
  sg_allocate_tiers_device tier per request
  sg_pack_tree_wave        row_offsets / parents / tokens of the wave
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from . import _lib
from .allocator import allocate_tree_budgets_device

SG_DTYPE_F32 = 0
SG_DTYPE_BF16 = 1


def _status(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def proposal_topk(logits: torch.Tensor, temperature: float, k: int, status: torch.Tensor | None = None,
                  stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k fp64 log proposal masses and int64 ids of every row of CUDA
    bf16/fp32 ``logits`` [V], [rows, V] or [groups, rows, V] (unit stride
    over V; the 3-D form may be a strided view, e.g. block rows 1..L of the
    drafter's [R, block, V] logits, read in place)."""
    if logits.dtype not in (torch.bfloat16, torch.float32) or not logits.is_cuda or logits.dim() > 3:
        raise ValueError("proposal logits must be CUDA bf16 or fp32 with at most 3 dims")
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    V = logits.shape[-1]
    view = logits.reshape(1, -1, V) if logits.dim() < 3 else logits
    if view.stride(-1) != 1:
        view = view.contiguous()
    groups, per, _ = view.shape
    rows = groups * per
    log_q = torch.empty((rows, k), dtype=torch.float64, device=logits.device)
    ids = torch.empty((rows, k), dtype=torch.int64, device=logits.device)
    lib = _lib.load()
    st = lib.sg_proposal_topk(view.data_ptr(), SG_DTYPE_BF16 if logits.dtype == torch.bfloat16 else SG_DTYPE_F32,
                              view.stride(1), per, view.stride(0), rows, V, int(k), float(temperature),
                              log_q.data_ptr(), ids.data_ptr(), _lib.ptr(status), _lib.stream_ptr(stream))
    if st == _lib.SG_ERR_INVALID_ARGUMENT:
        raise ValueError(lib.sg_last_error().decode())
    _lib.check(st, "sg_proposal_topk")
    return log_q.reshape(*logits.shape[:-1], k), ids.reshape(*logits.shape[:-1], k)


@dataclass
class DraftTrees:
    tokens: torch.Tensor       # [R, budget] int64; node i >= 1 holds tokens[:, i - 1]
    parents: torch.Tensor      # [R, budget + 1] int64, root -1
    depths: torch.Tensor       # [R, budget + 1] int32
    masses: torch.Tensor       # [R, budget + 1] fp64 prefix log masses
    node_count: torch.Tensor   # [R] int32
    utilities: torch.Tensor | None  # [R, tiers] fp64
    budget: int

    def tree(self, r: int) -> tuple[list[int], list[int], list[int], list[float]]:
        """(tokens, parents, depths, masses) of request r on the host."""
        n = int(self.node_count[r])
        return (self.tokens[r, :n].tolist(), self.parents[r, :n + 1].tolist(), self.depths[r, :n + 1].tolist(),
                self.masses[r, :n + 1].tolist())


def build_draft_trees(log_q: torch.Tensor, ids: torch.Tensor, budget: int, *, budgets: torch.Tensor | None = None,
                      rewards: Sequence[float] | None = None, rank_caps: Sequence[int] | None = None,
                      adaptive_min_budget: int | None = None, confidence_threshold: float | None = None,
                      tiers: Sequence[int] = (), status: torch.Tensor | None = None, stream=None) -> DraftTrees:
    """Best-first trees from ranked log masses [R, length, width]."""
    if log_q.dtype != torch.float64 or ids.dtype != torch.int64 or log_q.shape != ids.shape or log_q.dim() != 3:
        raise ValueError("log_q (fp64) and ids (int64) must both be [trees, length, width]")
    R, L, W = log_q.shape
    dev = log_q.device
    log_q, ids = log_q.contiguous(), ids.contiguous()
    if budgets is not None:
        budgets = budgets.to(device=dev, dtype=torch.int32).contiguous()
    rw = None if rewards is None else np.ascontiguousarray(rewards, dtype=np.float64)
    caps = None if rank_caps is None else np.ascontiguousarray(rank_caps, dtype=np.int32)
    if (rw is not None and rw.shape != (L,)) or (caps is not None and caps.shape != (L,)):
        raise ValueError("rewards and rank caps need one entry per draft depth")
    if adaptive_min_budget is not None and confidence_threshold is None:
        raise ValueError("an adaptive tree budget requires a confidence threshold")
    tier_arr = np.ascontiguousarray(list(tiers), dtype=np.int32)
    T = len(tier_arr)
    out = DraftTrees(torch.empty((R, budget), dtype=torch.int64, device=dev),
                     torch.empty((R, budget + 1), dtype=torch.int64, device=dev),
                     torch.empty((R, budget + 1), dtype=torch.int32, device=dev),
                     torch.empty((R, budget + 1), dtype=torch.float64, device=dev),
                     torch.empty(R, dtype=torch.int32, device=dev),
                     torch.empty((R, T), dtype=torch.float64, device=dev) if T else None, budget)
    lib = _lib.load()
    st = lib.sg_build_draft_trees(
        log_q.data_ptr(), ids.data_ptr(), R, L, W, _lib.ptr(budgets), int(budget),
        None if rw is None else rw.ctypes.data, None if caps is None else caps.ctypes.data,
        -1 if adaptive_min_budget is None else int(adaptive_min_budget),
        math.nan if confidence_threshold is None else float(confidence_threshold),
        tier_arr.ctypes.data if T else None, T, out.tokens.data_ptr(), out.parents.data_ptr(),
        out.depths.data_ptr(), out.masses.data_ptr(), out.node_count.data_ptr(), _lib.ptr(out.utilities),
        _lib.ptr(status), _lib.stream_ptr(stream))
    if st == _lib.SG_ERR_INVALID_ARGUMENT:
        raise ValueError(lib.sg_last_error().decode())
    _lib.check(st, "sg_build_draft_trees")
    return out


def pack_tree_wave(trees: DraftTrees, allocation: torch.Tensor, anchor_tokens: torch.Tensor, max_rows: int,
                   status: torch.Tensor | None = None, stream=None):
    """(row_offsets [R + 1], parents [max_rows], tokens [max_rows]) of the
    verify wave made of each request's chosen tier."""
    R = trees.node_count.shape[0]
    dev = trees.tokens.device
    offsets = torch.empty(R + 1, dtype=torch.int64, device=dev)
    parents = torch.empty(max_rows, dtype=torch.int64, device=dev)
    tokens = torch.empty(max_rows, dtype=torch.int64, device=dev)
    lib = _lib.load()
    st = lib.sg_pack_tree_wave(trees.tokens.data_ptr(), trees.parents.data_ptr(), trees.budget,
                               trees.node_count.data_ptr(), allocation.to(torch.int32).contiguous().data_ptr(),
                               anchor_tokens.to(device=dev, dtype=torch.int64).contiguous().data_ptr(), R,
                               int(max_rows), offsets.data_ptr(), parents.data_ptr(), tokens.data_ptr(),
                               _lib.ptr(status), _lib.stream_ptr(stream))
    if st == _lib.SG_ERR_INVALID_ARGUMENT:
        raise ValueError(lib.sg_last_error().decode())
    _lib.check(st, "sg_pack_tree_wave")
    return offsets, parents, tokens


@dataclass
class WavePlan:
    trees: DraftTrees
    allocation: torch.Tensor   # [R] int32 tier (nodes) per request
    row_offsets: torch.Tensor  # [R + 1]
    parents: torch.Tensor      # [max_rows]
    tokens: torch.Tensor       # [max_rows]
    status: torch.Tensor       # int32 device word (0 = ok)
    log_q: torch.Tensor | None = None  # [R, length, k] ranked log proposal masses
    ids: torch.Tensor | None = None    # [R, length, k] their token ids
    draft_logits: torch.Tensor | None = None  # [R, block, V] when planned by B200Drafter.propose


def plan_wave(draft_logits: torch.Tensor, temperature: float, tiers: Sequence[int], weights: torch.Tensor,
              anchor_tokens: torch.Tensor, *, row_budget: int, fixed_row_equivalent: float | None = None,
              row_cost_curve: Sequence[tuple[int, float]] | None = None, stream=None) -> WavePlan:
    """The next wave from the drafter's logits [R, length, V] (CUDA): one
    canonical tree per request (budget = the largest tier), tier utilities,
    the shared-budget tier knapsack and the packed wave, all enqueued on the
    device without a host synchronisation (the global canonical path of
    continuous_tree_block_decode.py:839-883)."""
    R, L, V = draft_logits.shape
    budget = int(max(tiers))
    status = _status(draft_logits.device)
    k = min(budget, V)
    log_q, ids = proposal_topk(draft_logits, temperature, k, status=status, stream=stream)
    trees = build_draft_trees(log_q, ids, budget, tiers=tiers, status=status, stream=stream)
    allocation = allocate_tree_budgets_device(weights.to(device=draft_logits.device, dtype=torch.float64), tiers,
                                              trees.utilities, row_budget=row_budget,
                                              fixed_row_equivalent=fixed_row_equivalent,
                                              row_cost_curve=row_cost_curve, status=status, stream=stream)
    offsets, parents, tokens = pack_tree_wave(trees, allocation, anchor_tokens, row_budget, status=status,
                                              stream=stream)
    return WavePlan(trees, allocation, offsets, parents, tokens, status, log_q, ids)
