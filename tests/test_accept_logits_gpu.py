"""The direct-logits acceptance kernel (sg_tree_accept_logits) against
(1) the golden walks of tests/golden/accept_logits.npz (the reference's
_sample_row_inverse_cdf over exp(double(logit) / T - max)), in fp32 and bf16;
(2) the reference's own compiled batched logits kernel
(fused_tree_sampling.py:1117-1236, oracle/_ref) at V = 151936, same logits
and uniforms; (3) the C oracle on ragged trees with Philox uniforms.  Paths
must agree bit for bit (integer nodes and tokens)."""
import numpy as np
import pytest
import torch

from oracle import cpu as oracle
from specgrove_b200 import sampling
from specgrove_b200.sampling import PackedTrees, accept_logits_packed
from specgrove_b200.workloads import random_topology

pytestmark = pytest.mark.gpu


def _trees(rng, sizes, vocab, logits, topology=None, boost=(14.0, 20.0)):
    parents_b, tokens_b = [], []
    off = 0
    for n in sizes:
        parents = list(topology) if topology is not None else random_topology(rng, n, 16, 4)[0]
        toks, kids = [], {}
        for j in range(1, n):
            used = kids.setdefault(parents[j], set())
            t = int(rng.integers(0, vocab))
            while t in used:
                t = int(rng.integers(0, vocab))
            used.add(t)
            toks.append(t)
            logits[off + parents[j], t] += float(rng.uniform(*boost))   # children likely: walks go deep
        parents_b.append(parents)
        tokens_b.append(toks)
        off += n
    return parents_b, tokens_b


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_logits_kernel_matches_golden(cuda_lib, golden_dir, dtype):
    z = np.load(golden_dir / "accept_logits.npz")
    offsets = z["row_offsets"]
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        D = int(z[f"max_depth_{i}"])
        parents = z["parents"][r0:r1].tolist()
        tokens = z["tokens"][r0:r1].tolist()[1:]
        logits = torch.from_numpy(z[f"probs_{i}"]).cuda().to(dtype)
        trees = PackedTrees([parents], [tokens], "cuda")
        u = torch.from_numpy(z[f"uniforms_{i}"]).cuda()
        out = accept_logits_packed(logits, trees, temperature=float(z[f"temperature_{i}"]), uniforms=u).cpu()
        count = int(out[0, D])
        assert out[0, :count].tolist() == z[f"nodes_{i}"].tolist(), i
        assert int(out[0, D + 1]) == int(z[f"bonus_{i}"]), i


@pytest.fixture(scope="module")
def ref():
    from oracle.build_ref import load_reference_sampler
    module = load_reference_sampler()
    if module is None:
        pytest.skip("reference sampler not built (oracle/build_ref.py)")
    return module


@pytest.mark.parametrize("temperature", [1.0, 0.6])
def test_logits_kernel_matches_reference_kernel(cuda_lib, ref, temperature):
    n, T, V = 40, 24, 151936
    rng = np.random.default_rng(31)
    g = torch.Generator(device="cuda").manual_seed(31)
    logits = torch.randn((T * n, V), generator=g, device="cuda") * 2.0
    host = logits.cpu()
    # one topology for every tree: the reference's batched kernel needs equal shapes and depth
    topology = random_topology(rng, n, 16, 4)[0]
    parents_b, tokens_b = _trees(rng, [n] * T, V, host, topology)
    logits = host.cuda().to(torch.bfloat16)
    D = sampling._topology(parents_b[0], tokens_b[0])[2]
    u = torch.rand((T, D + 1), dtype=torch.float64, device="cuda", generator=g)
    trees = PackedTrees(parents_b, tokens_b, "cuda")
    ours = accept_logits_packed(logits, trees, temperature=temperature, uniforms=u, max_depth=D)
    edges = torch.tensor([[p[1:], t] for p, t in zip(parents_b, tokens_b)], dtype=torch.long, device="cuda")
    theirs = ref.fused_tree_sample_logits_scan_batched_cuda(logits.view(T, n, V), edges[:, 0].contiguous(),
                                                            edges[:, 1].contiguous(), u, temperature, D)
    assert torch.equal(ours.cpu(), theirs.cpu())
    assert int((ours[:, D] > 0).sum()) > 0          # some walks accept nodes


def test_logits_kernel_matches_oracle_with_philox(cuda_lib):
    rng = np.random.default_rng(7)
    sizes = [int(s) for s in rng.integers(8, 96, size=20)]
    V = 151936
    g = torch.Generator(device="cuda").manual_seed(7)
    host = (torch.randn((sum(sizes), V), generator=g, device="cuda") * 3.0).cpu()
    parents_b, tokens_b = _trees(rng, sizes, V, host, boost=(17.0, 24.0))
    logits = host.to(torch.bfloat16)
    trees = PackedTrees(parents_b, tokens_b, "cuda")
    rids = torch.arange(20, dtype=torch.long, device="cuda") * 977 + 5
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = accept_logits_packed(logits.cuda(), trees, temperature=0.8, seed=2**61 + 9, request_ids=rids,
                               status=status).cpu().numpy()
    flat_p = np.asarray([p for ps in parents_b for p in ps], np.int64)
    flat_t = np.asarray([x for ts in tokens_b for x in [-1, *ts]], np.int64)
    expected, st = oracle.accept_logits(logits.float().numpy(), trees.row_offsets_host, flat_p, flat_t,
                                        trees.max_depth, temperature=0.8, seed=2**61 + 9,
                                        request_ids=rids.cpu().numpy())
    assert st == 0 and int(status) == 0
    assert (out == expected).all()
    assert (out[:, trees.max_depth] > 1).any()      # deep walks are covered


def test_reference_named_verifiers_draw_like_the_reference(cuda_lib, ref):
    """tree_verify_ancestral_logits_fused_scan(_batched) consume each request's
    generator as the reference does, so with equal generators they return
    the reference kernel's decisions."""
    n, T, V = 24, 6, 4096
    rng = np.random.default_rng(3)
    g = torch.Generator(device="cuda").manual_seed(3)
    host = (torch.randn((T * n, V), generator=g, device="cuda") * 2.0).cpu()
    parents_b, tokens_b = _trees(rng, [n] * T, V, host, random_topology(rng, n, 16, 4)[0], boost=(4.0, 9.0))
    logits = host.cuda().view(T, n, V)
    single = sampling.tree_verify_ancestral_logits_fused_scan(parents_b[0], tokens_b[0], logits[0], 1.0,
                                                             generator=torch.Generator(device="cuda").manual_seed(9))
    d0 = sampling._topology(parents_b[0], tokens_b[0])[2]
    u0 = torch.rand(d0 + 1, dtype=torch.float64, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9))
    e0 = torch.tensor([parents_b[0][1:], tokens_b[0]], dtype=torch.long, device="cuda")
    packed = ref.fused_tree_sample_logits_scan_batched_cuda(logits[:1].contiguous(), e0[:1].contiguous(),
                                                            e0[1:].contiguous(), u0[None], 1.0, d0).cpu()[0]
    count = int(packed[d0])
    assert single[0] == packed[:count].tolist() and single[2] == int(packed[d0 + 1])
    gens = [torch.Generator(device="cuda").manual_seed(40 + i) for i in range(T)]
    batched = sampling.tree_verify_ancestral_logits_fused_scan_batched(parents_b, tokens_b, logits, 1.0,
                                                                      generators=gens)
    assert len(batched) == T and all(0 <= b[2] < V for b in batched)
