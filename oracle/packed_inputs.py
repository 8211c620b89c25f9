"""TEST INFRASTRUCTURE — restatement of the reference's packed target inputs.

Follows ``_packed_block_inputs`` (continuous_tree_block_decode.py:500-546) and
``_pack_cache_sequence`` (:313-361): packed ids ``[root_token] + tree tokens``
per request, positions ``round_prefix_len + depth``, and the dense additive
mask ``[1, 1, Q, ΣL + Q]`` that is 0 on a row's own cache prefix and on its own
ancestors-or-self (``Tree.visibility``, tree.py:19-26) and -inf elsewhere.
Used by the GPU parity tests to drive HF ``Qwen3Model`` (the reference's
BF16-SDPA target path, engine.py:499-517) with exactly the reference's
inputs.  Pinned to the reference by tests/golden/packed_inputs.npz.
"""
from __future__ import annotations

from typing import Sequence

import torch


def visibility(parents: Sequence[int]) -> torch.Tensor:
    n = len(parents)
    visible = torch.zeros((n, n), dtype=torch.bool)
    visible[0, 0] = True
    for i in range(1, n):
        visible[i] = visible[parents[i]]
        visible[i, i] = True
    return visible


def packed_block_inputs(trees, cache_lengths, round_prefix, dtype=torch.float32, device="cpu"):
    """trees: per request (parents, tokens-with-root-token-first).

    Returns ids [1, Q], positions [1, Q], mask [1, 1, Q, ΣL + Q], query offsets."""
    q_offsets, total_q = [], 0
    for parents, _ in trees:
        q_offsets.append(total_q)
        total_q += len(parents)
    cache_offsets, total_l = [], 0
    for L in cache_lengths:
        cache_offsets.append(total_l)
        total_l += L
    ids = torch.empty((1, total_q), dtype=torch.long)
    positions = torch.empty((1, total_q), dtype=torch.long)
    mask = torch.full((1, 1, total_q, total_l + total_q), float("-inf"), dtype=dtype)
    for (parents, tokens), L, c_off, q_off, base in zip(trees, cache_lengths, cache_offsets, q_offsets, round_prefix):
        n = len(parents)
        depth = [0] * n
        for j in range(1, n):
            depth[j] = depth[parents[j]] + 1
        ids[0, q_off:q_off + n] = torch.tensor(list(tokens))
        positions[0, q_off:q_off + n] = torch.tensor(depth) + base
        mask[0, 0, q_off:q_off + n, c_off:c_off + L] = 0
        block = mask[0, 0, q_off:q_off + n, total_l + q_off:total_l + q_off + n]
        block.masked_fill_(visibility(parents), 0)
    return ids.to(device), positions.to(device), mask.to(device), q_offsets
