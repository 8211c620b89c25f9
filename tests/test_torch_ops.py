"""torch.ops.specgrove_b200: the operators load without a GPU, carry their
schemas, propagate shapes through their Meta kernels, and refuse host
tensors (no CPU kernel is registered: there is no fallback)."""
import pytest
import torch

from specgrove_b200 import ops

EXPECTED = ["tree_accept", "tree_accept_out", "tree_follow", "tree_follow_out", "kv_commit",
            "kv_commit_accepted", "lm_head_sample", "verify_pass"]


def test_operators_are_registered_with_schemas():
    ns = ops.load()
    for name in EXPECTED:
        schema = str(getattr(ns, name).default._schema)
        assert schema.startswith(f"specgrove_b200::{name}(")
    assert "Tensor(a!)? status" in str(ns.tree_accept.default._schema)
    assert "int[] feature_layers" in str(ns.verify_pass.default._schema)


def test_meta_kernels_give_output_shapes():
    ns = ops.load()
    m = dict(device="meta")
    probs = torch.empty((40, 151936), **m)
    offsets = torch.empty(5, dtype=torch.long, **m)
    meta_i64 = torch.empty(40, dtype=torch.long, **m)
    out = ns.tree_accept(probs, offsets, meta_i64, meta_i64, 16, 7, 0, None, 3, None, None)
    assert out.shape == (4, 9) and out.dtype == torch.long
    out = ns.tree_follow(meta_i64, offsets, meta_i64, meta_i64, 16, 7, None)
    assert out.shape == (4, 9)
    lse, post = ns.lm_head_sample(torch.empty((40, 4096), **m), torch.empty(4096, dtype=torch.bfloat16, **m),
                                  torch.empty((151936, 4096), dtype=torch.bfloat16, **m),
                                  torch.empty(40, dtype=torch.int32, **m), meta_i64, 0, 1.0, 1e-6)
    assert lse.shape == (40,) and post.dtype == torch.long


def test_host_tensors_are_refused():
    ns = ops.load()
    probs = torch.rand((4, 64))
    offsets = torch.tensor([0, 4])
    parents = torch.tensor([-1, 0, 0, 1])
    with pytest.raises((NotImplementedError, RuntimeError)):
        ns.tree_accept(probs, offsets, parents, parents, 4, 2, 0, None, 0, None, None)


def test_seed_arg_round_trips_64_bits():
    for seed in (0, 1, 2**63 - 1, 2**63, 2**64 - 1):
        s = ops.seed_arg(seed)
        assert -(2**63) <= s < 2**63
        assert s & (2**64 - 1) == seed
