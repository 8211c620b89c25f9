"""CPU oracle for on-device draft-tree construction (test infrastructure only:
imported by tests and never by the product path).

Restates, in float64 Python:

* the proposal masses the tree ranks: q = softmax(logits / T) in float64
  (sampling.py:29-36, ``probabilities``), the top-k of each depth
  (tree.py:183-184) and their logs, here as (x - max) - log(sum exp(x - max));
  ties in q go to the lower vocabulary index;
* the best-first prefix tree ``probability_tree`` (tree.py:148-212): node
  budget, optional per-depth reward schedule, per-depth rank caps and the
  adaptive budget on confident rounds.  Candidates are (score, parent, depth,
  rank) with score = -(prefix log mass + rewards); the smallest is expanded
  next, the tuple order breaking exact score ties (the reference's heap
  order: the tuples are unique).  It is written here as a plain candidate
  list with a minimum search rather than a heap, so it shares no structure
  with the reference's code;
* tier prefixes and their draft expected tokens
  (continuous_tree_block_decode.py:560-586): 1 + the sum of exp(prefix log
  mass) over the prefix's nodes, summed as the reference's ``sum`` does.

Pinned against tests/golden/draft_trees.npz (generated from the reference's
own functions by tests/golden/make_golden.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


def proposal_logs(logits: np.ndarray, temperature: float, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Top-k log proposal masses [L, k] (float64) and their token ids [L, k]
    of fp32/fp64 logits [L, V] at temperature T > 0."""
    x = np.asarray(logits, dtype=np.float64) / float(temperature)
    m = x.max(axis=1, keepdims=True)
    log_total = np.log(np.exp(x - m).sum(axis=1, keepdims=True))
    order = np.argsort(-x, axis=1, kind="stable")[:, :k]   # value desc, index asc
    ids = order.astype(np.int64)
    logs = (np.take_along_axis(x, order, axis=1) - m) - log_total
    return logs, ids


@dataclass
class DraftTree:
    tokens: list[int]      # node i >= 1 carries tokens[i - 1]
    parents: list[int]     # parents[0] = -1 (the root anchor)
    depths: list[int]
    masses: list[float]    # prefix log mass (+ rewards) of every node, root 0.0


def best_first_tree(logs, ids, budget: int, rewards=None, rank_caps=None, adaptive_min_budget=None,
                    confidence_threshold=None) -> DraftTree:
    logs = [[float(v) for v in row] for row in np.asarray(logs, dtype=np.float64)]
    ids = [[int(v) for v in row] for row in np.asarray(ids)]
    length = len(logs)
    width = len(logs[0])
    reward = [0.0] * length if rewards is None else [float(v) for v in rewards]
    caps = [min(width, budget)] * length if rank_caps is None else [min(int(c), budget, width) for c in rank_caps]
    if adaptive_min_budget is not None:
        depths_seen = min(4, length)
        total = 0.0
        for d in range(depths_seen):
            total += logs[d][0]
        if total / depths_seen >= math.log(confidence_threshold):
            budget = adaptive_min_budget
    tree = DraftTree([], [-1], [0], [0.0])
    # candidate: (score, parent, depth, rank, parent prefix log mass)
    candidates = [(-(logs[0][0] + reward[0]), 0, 0, 0, 0.0)]
    while candidates and len(tree.tokens) < budget:
        pick = min(range(len(candidates)), key=lambda j: candidates[j][:4])
        score, parent, depth, rank, parent_mass = candidates.pop(pick)
        node = len(tree.parents)
        tree.tokens.append(ids[depth][rank])
        tree.parents.append(parent)
        tree.depths.append(depth + 1)
        tree.masses.append(-score)
        if rank + 1 < caps[depth]:
            sibling = -((parent_mass + logs[depth][rank + 1]) + reward[depth])
            candidates.append((sibling, parent, depth, rank + 1, parent_mass))
        if depth + 1 < length:
            child = (score - logs[depth + 1][0]) - reward[depth + 1]
            candidates.append((child, node, depth + 1, 0, -score))
    return tree


def neumaier_prefix_sums(values) -> list[float]:
    """Sums of values[:1], values[:2], ... as Python's built-in ``sum`` of
    floats computes each (CPython >= 3.12: Neumaier's compensated summation,
    Z. angew. Math. Mech. 54 (1974) 39-51; the first item enters exactly, the
    compensation is added once at the end)."""
    out = []
    total, comp = 0.0, 0.0
    for i, x in enumerate(values):
        if i == 0:
            total = x
        else:
            t = total + x
            if abs(total) >= abs(x):
                comp += (total - t) + x
            else:
                comp += (x - t) + total
            total = t
        out.append(total + comp if comp != 0.0 and math.isfinite(comp) else total)
    return out


def tier_utility(tree: DraftTree, nodes: int) -> float:
    """Draft expected tokens of the first `nodes` nodes (plus the bonus):
    1 + the sum of exp(prefix log mass) over those nodes."""
    if nodes < 1 or nodes > len(tree.tokens):
        return math.nan
    return 1.0 + neumaier_prefix_sums([math.exp(m) for m in tree.masses[1:nodes + 1]])[-1]
