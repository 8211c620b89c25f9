"""Acceptance walk on the GPU through the C ABI, against the reference's golden
outputs and the CPU oracle (bit-exact: integer node ids and tokens)."""
import numpy as np
import pytest
import torch

from oracle import cpu as oracle
from specgrove_b200 import _lib, sampling, workloads
from specgrove_b200.sampling import PackedTrees, accept_packed

pytestmark = pytest.mark.gpu


def _golden_groups(path):
    z = np.load(path)
    offsets = z["row_offsets"]
    groups = {}
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        c = dict(parents=z["parents"][r0:r1].tolist(), tokens=z["tokens"][r0:r1].tolist(),
                 probs=z[f"probs_{i}"], uniforms=z[f"uniforms_{i}"], max_depth=int(z[f"max_depth_{i}"]),
                 nodes=z[f"nodes_{i}"].tolist(), bonus=int(z[f"bonus_{i}"]))
        groups.setdefault(c["probs"].shape[1], []).append(c)
    return groups


@pytest.mark.parametrize("name,rule", [("accept_scan.npz", _lib.SG_RULE_SCAN),
                                       ("accept_sparse.npz", _lib.SG_RULE_SPARSE_EXIT)])
def test_golden_walks_batched(cuda_lib, golden_dir, name, rule):
    per_depth = 2 if rule == _lib.SG_RULE_SPARSE_EXIT else 1
    for vocab, cases in _golden_groups(golden_dir / name).items():
        trees = PackedTrees([c["parents"] for c in cases], [c["tokens"][1:] for c in cases], "cuda")
        D = trees.max_depth
        probs = torch.from_numpy(np.concatenate([c["probs"] for c in cases])).cuda()
        uniforms = torch.zeros((len(cases), per_depth * (D + 1)), dtype=torch.float64)
        for i, c in enumerate(cases):
            uniforms[i, :len(c["uniforms"])] = torch.from_numpy(c["uniforms"])
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = accept_packed(probs, trees, rule=rule, uniforms=uniforms.cuda(), status=status).cpu()
        assert int(status) == 0
        for i, c in enumerate(cases):
            count = int(out[i, D])
            assert out[i, :count].tolist() == c["nodes"], (vocab, i)
            assert int(out[i, D + 1]) == c["bonus"], (vocab, i)
            assert (out[i, count:D] == -1).all()


def _oracle_out(batch: workloads.TreeBatch, probs_host, D, rule, uniforms=None, seed=0, request_ids=None):
    parents, tokens = batch.flat()
    out, st = oracle.accept_probs(probs_host, batch.row_offsets, parents, tokens, D, rule=rule,
                                  uniforms=uniforms, seed=seed, request_ids=request_ids)
    assert st == 0
    return out


@pytest.mark.parametrize("rule", [_lib.SG_RULE_SCAN, _lib.SG_RULE_SPARSE_EXIT])
def test_philox_stream_matches_oracle_full_vocab(cuda_lib, rule):
    batch, probs = workloads.acceptance_sweep(seed=3, trees=24, total_nodes=24 * 40, device="cuda")
    trees = PackedTrees(batch.parents, batch.tokens, "cuda")
    request_ids = torch.arange(1000, 1000 + batch_count(batch), dtype=torch.long, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = accept_packed(probs, trees, rule=rule, seed=987654321, request_ids=request_ids,
                        status=status).cpu().numpy()
    assert int(status) == 0
    expected = _oracle_out(batch, probs.cpu().numpy(), trees.max_depth, rule, seed=987654321,
                           request_ids=request_ids.cpu().numpy())
    np.testing.assert_array_equal(out, expected)


def batch_count(batch):
    return len(batch.row_offsets) - 1


def test_full_acceptance_sweep_matches_oracle(cuda_lib):
    """Config-2 size: 64 trees, 4096 nodes, V = 151936, explicit uniforms."""
    batch, probs = workloads.acceptance_sweep(seed=11, device="cuda")
    trees = PackedTrees(batch.parents, batch.tokens, "cuda")
    D = trees.max_depth
    gen = torch.Generator(device="cuda").manual_seed(5)
    uniforms = torch.rand((64, D + 1), dtype=torch.float64, device="cuda", generator=gen)
    out = accept_packed(probs, trees, rule=_lib.SG_RULE_SCAN, uniforms=uniforms).cpu().numpy()
    expected = _oracle_out(batch, probs.cpu().numpy(), D, oracle.RULE_SCAN,
                           uniforms=uniforms.cpu().numpy())
    np.testing.assert_array_equal(out, expected)
    # and the same decisions as the reference's fp64 running-sum rule
    parents, tokens = batch.flat()
    ref64, _ = oracle.accept_probs(probs.cpu().numpy(), batch.row_offsets, parents, tokens, D,
                                   uniforms=uniforms.cpu().numpy(), arith=oracle.ARITH_FP64)
    assert (ref64 == out).all(axis=1).sum() == 64


def test_reference_api_wrappers_match_oracle(cuda_lib):
    batch, probs = workloads.acceptance_sweep(seed=7, trees=4, total_nodes=4 * 20, vocab=4096,
                                              min_nodes=16, device="cuda")
    for t in range(4):
        r0, r1 = batch.row_offsets[t], batch.row_offsets[t + 1]
        rows = probs[r0:r1].contiguous()
        gen = torch.Generator(device="cuda").manual_seed(100 + t)
        nodes, toks, bonus = sampling.tree_verify_ancestral_fused_scan(
            batch.parents[t], batch.tokens[t], rows, gen, validate=True)
        D = max(batch.depths[t])
        u = torch.rand(D + 1, dtype=torch.float64, device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(100 + t))
        out, _ = oracle.accept_probs(rows.cpu().numpy(), [0, r1 - r0], batch.parents[t],
                                     [-1] + batch.tokens[t], D, uniforms=u.cpu().numpy()[None])
        assert nodes == out[0, :int(out[0, D])].tolist() and bonus == int(out[0, D + 1])
        assert toks == [batch.tokens[t][n - 1] for n in nodes]
        # sparse exit through the reference-named function
        gen = torch.Generator(device="cuda").manual_seed(200 + t)
        nodes, toks, bonus = sampling.tree_verify_ancestral_sparse_exit_fused_scan(
            batch.parents[t], batch.tokens[t], rows.double(), gen, validate=False)
        u = torch.rand(2 * (D + 1), dtype=torch.float64, device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(200 + t))
        out, _ = oracle.accept_probs(rows.cpu().numpy(), [0, r1 - r0], batch.parents[t],
                                     [-1] + batch.tokens[t], D, rule=oracle.RULE_SPARSE_EXIT,
                                     uniforms=u.cpu().numpy()[None])
        assert nodes == out[0, :int(out[0, D])].tolist() and bonus == int(out[0, D + 1])


def test_batched_sparse_exit_ragged(cuda_lib):
    batch, probs = workloads.acceptance_sweep(seed=9, trees=6, total_nodes=6 * 30, vocab=2048,
                                              min_nodes=16, device="cuda")
    rows = [probs[batch.row_offsets[t]:batch.row_offsets[t + 1]].contiguous() for t in range(6)]
    gens = [torch.Generator(device="cuda").manual_seed(50 + t) for t in range(6)]
    results = sampling.tree_verify_ancestral_sparse_exit_fused_scan_batched(
        batch.parents, batch.tokens, rows, gens, validate=False)
    for t, (nodes, toks, bonus) in enumerate(results):
        D = max(batch.depths[t])
        u = torch.rand(2 * (D + 1), dtype=torch.float64, device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(50 + t))
        out, _ = oracle.accept_probs(rows[t].cpu().numpy(), [0, len(batch.parents[t])], batch.parents[t],
                                     [-1] + batch.tokens[t], D, rule=oracle.RULE_SPARSE_EXIT,
                                     uniforms=u.cpu().numpy()[None])
        assert nodes == out[0, :int(out[0, D])].tolist() and bonus == int(out[0, D + 1])


def test_follow_matches_golden(cuda_lib, golden_dir):
    z = np.load(golden_dir / "follow.npz")
    offsets = z["row_offsets"]
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        D = int(z[f"max_depth_{i}"])
        trees = PackedTrees([z["parents"][r0:r1].tolist()], [z["tokens"][r0 + 1:r1].tolist()], "cuda")
        out = sampling.follow_packed(torch.from_numpy(z["posterior"][r0:r1]).cuda(), trees,
                                     max_depth=D).cpu()
        count = int(out[0, D])
        assert out[0, :count].tolist() == z[f"nodes_{i}"].tolist()
        assert int(out[0, D + 1]) == int(z[f"bonus_{i}"])


def test_greedy_one_hot_fixture(cuda_lib):
    probs = torch.zeros((4, 8), dtype=torch.float32)
    probs[0, 4] = probs[1, 6] = probs[3, 7] = probs[2, 0] = 1.0
    nodes, toks, bonus = sampling.tree_verify_ancestral_fused_scan([-1, 0, 0, 1], [4, 5, 6], probs.cuda())
    assert nodes == [1, 3] and toks == [4, 6] and bonus == 7


def test_invalid_inputs_reported(cuda_lib):
    probs = torch.full((2, 64), 1.0 / 64, device="cuda")
    with pytest.raises(ValueError):
        sampling.tree_verify_ancestral_fused_scan([-1, 0], [64], probs)          # token out of range
    with pytest.raises(ValueError):
        sampling.tree_verify_ancestral_fused_scan([-1, 1], [3], probs)           # parent not earlier
    bad = probs.clone()
    bad[0, 3] = -1.0
    with pytest.raises(FloatingPointError):
        sampling.tree_verify_ancestral_fused_scan([-1, 0], [3], bad)
    # device-side detection when host validation is skipped
    trees = PackedTrees([[-1, 0]], [[3]], "cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    accept_packed(bad, trees, uniforms=torch.full((1, 2), 0.5, dtype=torch.float64, device="cuda"),
                  status=status)
    assert int(status) == _lib.SG_ERR_PROBABILITY


def test_empty_batch_and_single_root(cuda_lib):
    probs = torch.softmax(torch.randn(1, 333, device="cuda"), -1)
    trees = PackedTrees([[-1]], [[]], "cuda")
    out = accept_packed(probs, trees, uniforms=torch.tensor([[0.25]], dtype=torch.float64, device="cuda"))
    exp, _ = oracle.accept_probs(probs.cpu().numpy(), [0, 1], [-1], [-1], 0, uniforms=np.array([[0.25]]))
    assert out.cpu().tolist() == exp.tolist()
    lib = _lib.load()
    assert lib.sg_tree_accept_probs(0, 10, 0, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0) == 0
