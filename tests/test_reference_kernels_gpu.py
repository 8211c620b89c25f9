"""B200 acceptance kernels against the reference's own CUDA samplers.

The reference kernels (fused_tree_sampling.py:538-627 scan, :688-824 sparse
exit, :120-151 follow) are compiled unmodified into oracle/_ref by
oracle/build_ref.py and fed the same fp32 probabilities and the same uniforms
as the B200 kernels.  Accepted paths must agree bit for bit: integer node ids
and tokens.  (The reference sums in fp64 with a CUB block scan, the B200
kernel in exact fixed point; the two can only differ when u * total lies
within ~1e-16 relative of a CDF boundary, which the seeded cases here do not
hit.)
"""
import pytest
import torch

from oracle.build_ref import load_reference_sampler
from specgrove_b200 import _lib, workloads
from specgrove_b200.sampling import PackedTrees, accept_packed

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    module = load_reference_sampler()
    if module is None:
        pytest.skip("reference sampler not built (oracle/build_ref.py)")
    return module


def test_scan_rule_matches_reference_kernel(cuda_lib, ref):
    batch, probs = workloads.acceptance_sweep(seed=21, trees=16, total_nodes=16 * 48, device="cuda")
    trees = PackedTrees(batch.parents, batch.tokens, "cuda")
    D = trees.max_depth
    gen = torch.Generator(device="cuda").manual_seed(1)
    uniforms = torch.rand((16, D + 1), dtype=torch.float64, device="cuda", generator=gen)
    ours = accept_packed(probs, trees, uniforms=uniforms).cpu()
    for t in range(16):
        r0, r1 = batch.row_offsets[t], batch.row_offsets[t + 1]
        d = max(batch.depths[t])
        edges = torch.tensor([batch.parents[t][1:], batch.tokens[t]], dtype=torch.long, device="cuda")
        packed = ref.fused_tree_sample_scan_cuda(probs[r0:r1].contiguous(), edges[0].contiguous(),
                                                 edges[1].contiguous(), uniforms[t, :d + 1].contiguous(), d).cpu()
        count = int(packed[d])
        assert ours[t, :count].tolist() == packed[:count].tolist(), t
        assert int(ours[t, D]) == count and int(ours[t, D + 1]) == int(packed[d + 1]), t


def test_sparse_exit_matches_reference_kernel(cuda_lib, ref):
    # the reference's batched sparse-exit kernel needs equal-shaped trees of <= 65 nodes
    n, T = 40, 24
    batch, probs = workloads.acceptance_sweep(seed=22, trees=T, total_nodes=T * n, min_nodes=n, max_nodes=n,
                                              device="cuda")
    depth = max(max(d) for d in batch.depths)
    trees = PackedTrees(batch.parents, batch.tokens, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(2)
    uniforms = torch.rand((T, 2 * (depth + 1)), dtype=torch.float64, device="cuda", generator=gen)
    ours = accept_packed(probs, trees, rule=_lib.SG_RULE_SPARSE_EXIT, uniforms=uniforms, max_depth=depth).cpu()
    edges = torch.tensor([[p[1:], tk] for p, tk in zip(batch.parents, batch.tokens)], dtype=torch.long,
                         device="cuda")
    packed = ref.fused_tree_sample_sparse_exit_batched_cuda(
        probs.view(T, n, -1), edges[:, 0].contiguous(), edges[:, 1].contiguous(), uniforms, depth).cpu()
    assert torch.equal(ours, packed)


def test_follow_matches_reference_kernel(cuda_lib, ref):
    batch, probs = workloads.acceptance_sweep(seed=23, trees=8, total_nodes=8 * 32, vocab=4096, device="cuda")
    posterior = torch.multinomial(probs, 1, generator=torch.Generator(device="cuda").manual_seed(3)).reshape(-1)
    trees = PackedTrees(batch.parents, batch.tokens, "cuda")
    from specgrove_b200.sampling import follow_packed
    ours = follow_packed(posterior, trees).cpu()
    D = trees.max_depth
    for t in range(8):
        r0, r1 = batch.row_offsets[t], batch.row_offsets[t + 1]
        d = max(batch.depths[t])
        edges = torch.tensor([batch.parents[t][1:], batch.tokens[t]], dtype=torch.long, device="cuda")
        packed = ref.fused_tree_follow_cuda(posterior[r0:r1].contiguous(), edges[0].contiguous(),
                                            edges[1].contiguous(), d).cpu()
        count = int(packed[d])
        assert ours[t, :count].tolist() == packed[:count].tolist()
        assert int(ours[t, D]) == count and int(ours[t, D + 1]) == int(packed[d + 1])
