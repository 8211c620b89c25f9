"""Terminal-mass verifier (sg_tree_verify_terminal_mass) against the
reference-generated fixtures (sampling.py:542-735 at recorded uniforms), the
C oracle bit for bit (explicit uniforms and the Philox stream, vocabularies
of 151936, 4096 and 1001), its output law, and its error reports."""
import numpy as np
import pytest
import torch

from oracle import cpu as oracle
from specgrove_b200.sampling import (PackedTrees, terminal_mass_packed, tree_block_verify_terminal_mass_fused)
from specgrove_b200.workloads import random_topology

pytestmark = pytest.mark.gpu


def _golden_cases(golden_dir):
    z = np.load(golden_dir / "terminal_mass.npz")
    offsets = z["row_offsets"]
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        yield dict(parents=z["parents"][r0:r1].tolist(), tokens=z["tokens"][r0:r1].tolist(), probs=z[f"probs_{i}"],
                   uniforms=z[f"uniforms_{i}"], max_depth=int(z[f"max_depth_{i}"]),
                   nodes=z[f"nodes_{i}"].tolist(), bonus=int(z[f"bonus_{i}"]))


def _run(probs, parents_batch, tokens_batch, uniforms=None, seed=0, request_ids=None, max_depth=None):
    trees = PackedTrees(parents_batch, [t[1:] for t in tokens_batch], "cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    u = None if uniforms is None else torch.as_tensor(uniforms, dtype=torch.float64, device="cuda")
    rid = None if request_ids is None else torch.as_tensor(request_ids, dtype=torch.long, device="cuda")
    out = terminal_mass_packed(torch.as_tensor(probs, device="cuda"), trees, uniforms=u, seed=seed,
                               request_ids=rid, max_depth=max_depth, status=status)
    torch.cuda.synchronize()
    return out.cpu().numpy(), int(status.item()), trees


def test_matches_reference_fixtures(cuda_lib, golden_dir):
    n = 0
    for c in _golden_cases(golden_dir):
        out, st, _ = _run(c["probs"], [c["parents"]], [c["tokens"]], uniforms=c["uniforms"][None],
                          max_depth=c["max_depth"])
        assert st == 0
        D = c["max_depth"]
        assert out[0, :int(out[0, D])].tolist() == c["nodes"]
        assert int(out[0, D + 1]) == c["bonus"]
        n += 1
    assert n >= 12


def _random_batch(rng, sizes, vocab):
    parents_b, tokens_b, rows = [], [], []
    for n in sizes:
        parents, _ = random_topology(rng, n, 16, 4)
        tokens, kids = [-1], {}
        for j in range(1, n):
            used = kids.setdefault(parents[j], set())
            t = int(rng.integers(0, vocab))
            while t in used:
                t = int(rng.integers(0, vocab))
            used.add(t)
            tokens.append(t)
        logits = rng.standard_normal((n, vocab)).astype(np.float32) * 4
        for j in range(1, n):
            logits[parents[j], tokens[j]] += rng.uniform(3, 9)
        p = np.exp(logits - logits.max(axis=1, keepdims=True))
        rows.append((p / p.sum(axis=1, keepdims=True)).astype(np.float32))
        parents_b.append(parents)
        tokens_b.append(tokens)
    return parents_b, tokens_b, np.concatenate(rows)


@pytest.mark.parametrize("vocab,sizes", [(151936, [1, 7, 40, 128]), (4096, [3, 16, 64, 128, 2, 33]),
                                         (1001, [5, 100, 1, 17])])
def test_bit_exact_against_oracle(cuda_lib, vocab, sizes):
    rng = np.random.default_rng(vocab + len(sizes))
    parents_b, tokens_b, probs = _random_batch(rng, sizes, vocab)
    offsets = np.cumsum([0] + sizes)
    flat_p = np.concatenate(parents_b)
    flat_t = np.concatenate(tokens_b)
    D = 16
    uniforms = rng.random((len(sizes), 2))
    out, st, _ = _run(probs, parents_b, tokens_b, uniforms=uniforms, max_depth=D)
    ref, rst = oracle.terminal_mass(probs, offsets, flat_p, flat_t, D, uniforms=uniforms)
    assert st == 0 and rst == 0
    np.testing.assert_array_equal(out, ref)
    # the Philox stream keyed by (seed, request id)
    rids = rng.integers(0, 1 << 40, size=len(sizes))
    out, st, _ = _run(probs, parents_b, tokens_b, seed=1234, request_ids=rids, max_depth=D)
    ref, rst = oracle.terminal_mass(probs, offsets, flat_p, flat_t, D, seed=1234, request_ids=rids)
    assert st == 0 and rst == 0
    np.testing.assert_array_equal(out, ref)


def test_output_law_matches_ancestral_sampling(cuda_lib):
    """20000 Philox draws on one 4-node tree over an 8-token vocabulary: the
    joint law of (terminal node, bonus) is prefix(v) * p_v[b] / total(v) for
    b outside v's children, the law of the ancestral walk."""
    rng = np.random.default_rng(5)
    V, N = 8, 20000
    parents, tokens = [-1, 0, 0, 1], [-1, 2, 5, 1]
    p = rng.random((4, V)).astype(np.float32) + 0.05
    p[0, 2] += 1.5
    p[1, 1] += 1.0
    p /= p.sum(axis=1, keepdims=True)
    pd = p.astype(np.float64)
    law = {}
    prefix = {0: 1.0}
    for j in range(1, 4):
        prefix[j] = prefix[parents[j]] * pd[parents[j], tokens[j]] / pd[parents[j]].sum()
    for v in range(4):
        kids = {tokens[j] for j in range(1, 4) if parents[j] == v}
        for b in range(V):
            if b not in kids:
                law[(v, b)] = prefix[v] * pd[v, b] / pd[v].sum()
    probs = np.tile(p, (N, 1))
    out, st, _ = _run(probs, [parents] * N, [tokens] * N, seed=77, request_ids=np.arange(N), max_depth=2)
    assert st == 0
    counts = {}
    for row in out:
        count = int(row[2])
        v = int(row[count - 1]) if count else 0
        counts[(v, int(row[3]))] = counts.get((v, int(row[3])), 0) + 1
    tv = 0.5 * sum(abs(counts.get(k, 0) / N - q) for k, q in law.items())
    assert sum(counts.values()) == N and set(counts) <= set(law)
    assert tv < 0.02, tv


def test_reports_bad_trees_and_probabilities(cuda_lib):
    probs = np.full((3, 8), 1 / 8, dtype=np.float32)
    u = np.array([[0.3, 0.6]])
    out, st, _ = _run(probs, [[-1, 0, 0]], [[-1, 2, 3]], uniforms=u, max_depth=1)
    assert st == 0 and int(out[0, 2]) >= 0
    bad = probs.copy()
    bad[0, 5] = -0.1
    out, st, _ = _run(bad, [[-1, 0, 0]], [[-1, 2, 3]], uniforms=u, max_depth=1)
    assert st == 4 and (out == -1).all()


def test_reference_named_wrapper(cuda_lib):
    g = torch.Generator(device="cuda").manual_seed(3)
    p = torch.softmax(torch.randn((3, 64), device="cuda") * 3, dim=-1)
    nodes, toks, bonus = tree_block_verify_terminal_mass_fused([-1, 0, 1], [7, 9], p, generator=g)
    assert nodes in ([], [1], [1, 2]) and 0 <= bonus < 64
    assert toks == [[7, 9][n - 1] for n in nodes]


def test_rows_beyond_total_rows_are_reported(cuda_lib):
    """A tree that reaches past `total_rows` (no row sums there) is reported
    as SG_ERR_TREE and its output stays -1; the other trees are drawn."""
    from specgrove_b200 import _lib
    from specgrove_b200._lib import ptr, stream_ptr
    probs = torch.full((5, 16), 1 / 16, device="cuda")
    trees = PackedTrees([[-1, 0], [-1, 0, 1]], [[3], [4, 5]], "cuda")
    out = torch.empty((2, 4), dtype=torch.long, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    u = torch.tensor([[0.5, 0.5], [0.5, 0.5]], dtype=torch.float64, device="cuda")
    lib = _lib.load()
    nbytes = lib.sg_tree_verify_terminal_mass_workspace_bytes(4)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    st = lib.sg_tree_verify_terminal_mass(ptr(probs), 16, ptr(trees.row_offsets), ptr(trees.parents),
                                          ptr(trees.tokens), 2, 4, 2, ptr(u), 2, 0, None, ptr(out), ptr(status),
                                          ptr(ws), nbytes, stream_ptr())
    assert st == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 3
    assert (out[1] == -1).all() and int(out[0, 3]) >= 0
