"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No dataset or checkpoint is used anywhere: trees, logits, prefixes and
weights are generated from fixed seeds with the sizes and value
distributions the configurations name.

Acceptance sweep (64 trees, 4096 packed nodes, vocabulary 151936): tree sizes
in [16, 128] summing to 4096, depth <= 16, branching <= 4, parents drawn from
the seed; each child's token is one of the distinct top-4 tokens of its
parent's draft row (which satisfies the no-duplicate-sibling rule of
sampling.py:925-926); draft logits ~ 4 * N(0, 1), target logits = draft +
0.5 * N(0, 1); target probabilities are the fp32 softmax of the target logits.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class TreeBatch:
    parents: list[list[int]]        # per tree, root parent -1
    tokens: list[list[int]]         # per tree, edge tokens (node j has tokens[j-1])
    depths: list[list[int]]
    row_offsets: list[int]

    @property
    def total_rows(self) -> int:
        return self.row_offsets[-1]

    @property
    def max_depth(self) -> int:
        return max(max(d) for d in self.depths)

    def flat(self):
        """(parents, tokens-with-root--1) flattened over trees, int64 numpy."""
        p = np.asarray([x for ps in self.parents for x in ps], np.int64)
        t = np.asarray([x for ts in self.tokens for x in [-1, *ts]], np.int64)
        return p, t


def tree_sizes(rng: np.random.Generator, count: int, total: int, lo: int, hi: int) -> list[int]:
    if not lo * count <= total <= hi * count:
        raise ValueError("infeasible tree size budget")
    sizes = np.full(count, total // count, dtype=np.int64)
    sizes[: total - sizes.sum()] += 1
    for _ in range(count * 8):  # random transfers keep the sum and the bounds
        a, b = rng.integers(0, count, 2)
        amount = int(rng.integers(0, 32))
        amount = min(amount, sizes[a] - lo, hi - sizes[b])
        if a != b and amount > 0:
            sizes[a] -= amount
            sizes[b] += amount
    return sizes.tolist()


def random_topology(rng: np.random.Generator, n: int, max_depth: int, max_children: int):
    parents, depths, kids = [-1], [0], [0]
    for j in range(1, n):
        while True:
            cand = int(rng.integers(0, j))
            if kids[cand] < max_children and depths[cand] < max_depth:
                break
        parents.append(cand)
        depths.append(depths[cand] + 1)
        kids[cand] += 1
        kids.append(0)
    return parents, depths


def acceptance_sweep(seed: int = 0, trees: int = 64, total_nodes: int = 4096, vocab: int = 151936,
                     min_nodes: int = 16, max_nodes: int = 128, max_depth: int = 16,
                     max_children: int = 4, device="cuda", draft_scale: float = 4.0,
                     noise: float = 0.5, chunk_rows: int = 256):
    """Returns (TreeBatch, probs [total_nodes, vocab] fp32 on device)."""
    rng = np.random.default_rng(seed)
    sizes = tree_sizes(rng, trees, total_nodes, min_nodes, max_nodes)
    topo = [random_topology(rng, n, max_depth, max_children) for n in sizes]
    offsets = [0]
    for n in sizes:
        offsets.append(offsets[-1] + n)
    gen = torch.Generator(device=device).manual_seed(seed)
    probs = torch.empty((total_nodes, vocab), dtype=torch.float32, device=device)
    top = torch.empty((total_nodes, max_children), dtype=torch.long, device=device)
    for r0 in range(0, total_nodes, chunk_rows):
        r1 = min(total_nodes, r0 + chunk_rows)
        draft = torch.randn((r1 - r0, vocab), generator=gen, device=device) * draft_scale
        top[r0:r1] = torch.topk(draft, max_children, dim=-1).indices
        target = draft + torch.randn((r1 - r0, vocab), generator=gen, device=device) * noise
        probs[r0:r1] = torch.softmax(target, dim=-1)
        del draft, target
    top_host = top.cpu().numpy()
    parents_all, tokens_all, depths_all = [], [], []
    for t, (parents, depths) in enumerate(topo):
        seen = [0] * len(parents)
        tokens = []
        for j in range(1, len(parents)):
            p = parents[j]
            tokens.append(int(top_host[offsets[t] + p, seen[p]]))
            seen[p] += 1
        parents_all.append(parents)
        tokens_all.append(tokens)
        depths_all.append(depths)
    return TreeBatch(parents_all, tokens_all, depths_all, offsets), probs


# ---------------------------------------------------------------------------
# Verify-pass waves (configurations 3 and 4)
# ---------------------------------------------------------------------------
def best_first_tree(logs, ids, budget: int, rank_caps=None):
    """Best-first DDTree over per-depth top-k draft tokens (the product-
    probability heap of tree.py:148-212 with depth_reward = 0): returns
    (parents incl. root -1, tokens per node (root -1), depths, prefix log
    masses (root 0))."""
    import heapq
    length = len(logs)
    caps = rank_caps or [len(logs[0])] * length
    parents, tokens, depths, masses = [-1], [-1], [0], [0.0]
    heap = [(-logs[0][0], 0, 0, 0, 0.0)]
    while heap and len(tokens) - 1 < budget:
        neg, parent, depth, rank, parent_log = heapq.heappop(heap)
        node = len(parents)
        tokens.append(int(ids[depth][rank]))
        parents.append(parent)
        depths.append(depth + 1)
        masses.append(-neg)
        if rank + 1 < caps[depth]:
            heapq.heappush(heap, (-(parent_log + logs[depth][rank + 1]), parent, depth, rank + 1, parent_log))
        if depth + 1 < length:
            heapq.heappush(heap, (neg - logs[depth + 1][0], node, depth + 1, 0, -neg))
    return parents, tokens, depths, masses


# (rows incl. root) -> count; each mix sums to the configuration's row budget
TIER_MIX_CONFIG4 = {16: 40, 32: 12, 64: 8, 128: 4}   # 64 requests, 2048 rows
TIER_MIX_CONFIG3 = {16: 8, 32: 4, 64: 4}             # 16 requests, 512 rows


@dataclass
class VerifyWorkload:
    trees: list            # per request (parents, tokens with the root token first)
    cache_lengths: list
    tiers: list
    tier_options: list     # rows incl. root of every tier in the mix
    utilities: list        # per request, draft expected tokens of each tier option


def verify_workload(vocab: int, tier_mix: dict, prefix_range: tuple, seed: int = 0, block: int = 16,
                    draft_scale: float = 4.0, top_k: int = 4, device="cuda") -> VerifyWorkload:
    """One wave: per request a canonical best-first tree (block 16 draft
    positions, top-4 children per depth from softmax(4 N(0,1)) draft logits)
    cut to its tier (ancestor-closed best-first prefix, decode.py:571-586),
    prefix lengths uniform in prefix_range, tokens uniform over the vocab."""
    rng = np.random.default_rng(seed)
    tiers = [t for t, c in sorted(tier_mix.items()) for _ in range(c)]
    rng.shuffle(tiers)
    R = len(tiers)
    gen = torch.Generator(device=device).manual_seed(seed)
    trees, lengths = [], []
    budget = max(tiers) - 1
    options = sorted(tier_mix)
    utilities = []
    for i in range(R):
        draft = torch.randn((block, vocab), generator=gen, device=device) * draft_scale
        logq = torch.log_softmax(draft, -1)
        vals, idx = torch.topk(logq, top_k, dim=-1)
        parents, tokens, _, masses = best_first_tree(vals.tolist(), idx.tolist(), budget, [top_k] * block)
        # expected draft tokens of each tier's prefix (continuous_tree_block_decode.py:560-568)
        utilities.append([1.0 + float(np.exp(np.asarray(masses[1:t])).sum()) for t in options])
        n = tiers[i]
        parents, tokens = parents[:n], tokens[:n]
        tokens[0] = int(rng.integers(0, vocab))        # root row: last committed token
        trees.append((parents, tokens))
        lengths.append(int(rng.integers(prefix_range[0], prefix_range[1] + 1)))
    return VerifyWorkload(trees, lengths, tiers, options, utilities)
