"""``torch.ops.specgrove_b200``: the library's kernels as PyTorch operators.

The operators are registered by the in-tree extension ``_torch_ops.so``
(``csrc/torch_ops.cpp``): TORCH_LIBRARY schemas with CUDA kernels that call the
C ABI on the current stream, and Meta kernels for shape propagation.

    tree_accept(probs, row_offsets, parents, tokens, max_nodes, max_depth, rule,
                uniforms?, seed, request_ids?, status?) -> out [trees, max_depth + 2]
    tree_accept_out(..., out)                       in-place variant
    tree_follow(posterior, row_offsets, parents, tokens, max_nodes, max_depth, status?) -> out
    tree_follow_out(..., out)
    kv_commit(dst, src, src_rows, dst_rows, group_offsets, max_group_rows, status?)
    kv_commit_accepted(arena, capacity, slots, lengths_in, lengths_out, accept_out, max_depth, status?)
    lm_head_sample(x, final_norm, lm_head, row_node, row_request, seed, temperature, rms_eps) -> (lse, posterior)
    verify_pass(engine, wave, num_requests, num_rows, max_rows_per_request, max_depth, seed, temperature,
                commit, accept_out, lengths_out?, posterior?, lse?, child_logprob?, hidden_out?, status,
                feature_layers, features_out?, features_kept?, features_kept_offsets?)

There is no fallback: without the built extension, ``load`` raises.
"""
from __future__ import annotations

from pathlib import Path

import torch

from . import _lib

EXTENSION_PATH = Path(__file__).resolve().parent / "_torch_ops.so"
_ops = None


def load():
    """Load the extension once (after the C-ABI library it links to) and
    return the ``torch.ops.specgrove_b200`` namespace."""
    global _ops
    if _ops is None:
        _lib.load()
        if not EXTENSION_PATH.exists():
            raise ImportError(f"{EXTENSION_PATH.name} is not built; run `python -m specgrove_b200.build` "
                              "(the CUDA library is required, there is no CPU fallback)")
        torch.ops.load_library(str(EXTENSION_PATH))
        _ops = torch.ops.specgrove_b200
    return _ops


def seed_arg(seed: int) -> int:
    """A 64-bit unsigned seed as the signed int64 an operator schema takes
    (the C ABI reads the same bits back as uint64)."""
    seed &= (1 << 64) - 1
    return seed - (1 << 64) if seed >= (1 << 63) else seed


def lm_head_sample(x: torch.Tensor, final_norm: torch.Tensor, lm_head: torch.Tensor, row_node: torch.Tensor,
                   row_request: torch.Tensor, *, seed: int, temperature: float = 1.0, rms_eps: float = 1e-6):
    """Final RMSNorm + LM head + softmax sampling of residual rows: returns
    (lse [rows] fp32, posterior [rows] int64).  temperature 0 is greedy."""
    return load().lm_head_sample(x.contiguous(), final_norm, lm_head, row_node.to(torch.int32).contiguous(),
                                 row_request.to(torch.long).contiguous(), seed_arg(seed), float(temperature),
                                 float(rms_eps))
