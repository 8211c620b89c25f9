"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py, which calls the
reference's functions directly.  Both oracle arithmetics must reproduce them:
the exact 64.64 fixed-point sums the CUDA kernels use, and the sequential fp64
running sum of the reference CPU rule.
"""
import math
from fractions import Fraction

import numpy as np
import pytest

from oracle import cpu as oracle


def _cases(path):
    z = np.load(path)
    offsets = z["row_offsets"]
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        yield dict(parents=z["parents"][r0:r1], tokens=z["tokens"][r0:r1], probs=z[f"probs_{i}"],
                   uniforms=z[f"uniforms_{i}"], max_depth=int(z[f"max_depth_{i}"]),
                   nodes=z[f"nodes_{i}"].tolist(), bonus=int(z[f"bonus_{i}"]))


@pytest.mark.parametrize("arith", [oracle.ARITH_EXACT, oracle.ARITH_FP64])
def test_oracle_logits_rule_matches_reference(golden_dir, arith):
    """Direct-logits walk (fused_tree_sampling.py:942-1115) against the
    reference's _sample_row_inverse_cdf over exp(double(logit) / T - max)."""
    z = np.load(golden_dir / "accept_logits.npz")
    offsets = z["row_offsets"]
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        D = int(z[f"max_depth_{i}"])
        out, st = oracle.accept_logits(z[f"probs_{i}"], [0, r1 - r0], z["parents"][r0:r1], z["tokens"][r0:r1], D,
                                       temperature=float(z[f"temperature_{i}"]), uniforms=z[f"uniforms_{i}"][None],
                                       arith=arith)
        assert st == 0
        count = int(out[0, D])
        assert out[0, :count].tolist() == z[f"nodes_{i}"].tolist(), i
        assert int(out[0, D + 1]) == int(z[f"bonus_{i}"]), i


@pytest.mark.parametrize("arith", [oracle.ARITH_EXACT, oracle.ARITH_FP64])
@pytest.mark.parametrize("name,rule", [("accept_scan.npz", oracle.RULE_SCAN),
                                       ("accept_sparse.npz", oracle.RULE_SPARSE_EXIT)])
def test_oracle_matches_reference_walk(golden_dir, name, rule, arith):
    n_cases = 0
    for c in _cases(golden_dir / name):
        out, st = oracle.accept_probs(c["probs"], [0, len(c["parents"])], c["parents"], c["tokens"],
                                      c["max_depth"], rule=rule, uniforms=c["uniforms"][None],
                                      arith=arith)
        assert st == 0
        D = c["max_depth"]
        count = int(out[0, D])
        assert out[0, :count].tolist() == c["nodes"]
        assert int(out[0, D + 1]) == c["bonus"]
        n_cases += 1
    assert n_cases >= 10


def test_oracle_batched_equals_per_tree(golden_dir):
    cases = list(_cases(golden_dir / "accept_scan.npz"))
    cases = [c for c in cases if c["probs"].shape[1] == 256]
    assert len(cases) >= 2
    D = max(c["max_depth"] for c in cases)
    offsets = np.cumsum([0] + [len(c["parents"]) for c in cases])
    parents = np.concatenate([c["parents"] for c in cases])
    tokens = np.concatenate([c["tokens"] for c in cases])
    probs = np.concatenate([c["probs"] for c in cases])
    uniforms = np.zeros((len(cases), D + 1))
    for i, c in enumerate(cases):
        uniforms[i, :len(c["uniforms"])] = c["uniforms"]
    out, st = oracle.accept_probs(probs, offsets, parents, tokens, D, uniforms=uniforms)
    assert st == 0
    for i, c in enumerate(cases):
        count = int(out[i, D])
        assert out[i, :count].tolist() == c["nodes"] and int(out[i, D + 1]) == c["bonus"]


def test_oracle_follow_matches_reference(golden_dir):
    z = np.load(golden_dir / "follow.npz")
    offsets = z["row_offsets"]
    for i in range(int(z["count"])):
        r0, r1 = int(offsets[i]), int(offsets[i + 1])
        D = int(z[f"max_depth_{i}"])
        out = oracle.follow(z["posterior"][r0:r1], [0, r1 - r0], z["parents"][r0:r1],
                            z["tokens"][r0:r1], D)
        count = int(out[0, D])
        assert out[0, :count].tolist() == z[f"nodes_{i}"].tolist()
        assert int(out[0, D + 1]) == int(z[f"bonus_{i}"])


def test_oracle_greedy_fixture():
    # test_continuous_tree_block_decode.py:49-63: one-hot argmax rows walk to
    # nodes [1, 3] with bonus 7 for any uniform.
    parents = [-1, 0, 0, 1]
    tokens = [-1, 4, 5, 6]
    probs = np.zeros((4, 8), np.float32)
    probs[0, 4] = probs[1, 6] = probs[3, 7] = 1.0
    probs[2, 0] = 1.0
    for u in (0.0, 0.3, 0.999999):
        out, st = oracle.accept_probs(probs, [0, 4], parents, tokens, 2, uniforms=np.full((1, 3), u))
        assert out[0, :2].tolist() == [1, 3] and out[0, 2] == 2 and out[0, 3] == 7


def test_oracle_zero_row_falls_back_to_last_token():
    probs = np.zeros((1, 10), np.float32)
    out, st = oracle.accept_probs(probs, [0, 1], [-1], [-1], 0, uniforms=np.array([[0.5]]))
    assert out[0].tolist() == [0, 9]


def test_oracle_kv_commit_matches_reference_pool(golden_dir):
    z = np.load(golden_dir / "kv_commit.npz")
    layers = z["before_k"].shape[0]
    cap = int(z["capacity"])
    lengths = z["lengths"].tolist()
    keep_off = z["keep_offsets"]
    keep = z["keep_flat"]
    src_rows, dst_rows = [], []
    for slot, L in enumerate(lengths):
        rows = keep[keep_off[slot]:keep_off[slot + 1]]
        src_rows += [int(z["packed_old_length"]) + int(z["q_offsets"][slot]) + int(r) for r in rows]
        dst_rows += [slot * cap + L + i for i in range(len(rows))]
    for before, packed, after in (("before_k", "packed_k", "after_k"), ("before_v", "packed_v", "after_v")):
        arena = z[before].copy()       # [layers, H, slots*cap, D]
        src = z[packed].copy()         # [layers, H, T, D]
        H = arena.shape[1]
        dst = arena.reshape(layers * H, arena.shape[2], arena.shape[3])
        st = oracle.kv_commit(dst, src.reshape(layers * H, src.shape[2], src.shape[3]), src_rows, dst_rows)
        assert st == 0
        for slot, L in enumerate(lengths):
            n = int(z["after_lengths"][slot])
            a = arena[:, :, slot * cap: slot * cap + n]
            b = z[after][:, :, slot * cap: slot * cap + n]
            np.testing.assert_array_equal(a, b)


def test_oracle_inplace_compaction_equals_gather():
    rng = np.random.default_rng(0)
    arena = rng.standard_normal((6, 40, 4)).astype(np.float32)
    expected = arena.copy()
    keep = [0, 2, 3, 7]
    base = 10
    for pl in range(6):
        expected[pl, base:base + 4] = arena[pl, [base + k for k in keep]]
    st = oracle.kv_commit(arena, arena, [base + k for k in keep], [base + i for i in range(4)])
    assert st == 0
    np.testing.assert_array_equal(arena, expected)


def test_mass_conversion_is_exact_floor():
    rng = np.random.default_rng(1)
    values = np.concatenate([rng.random(200).astype(np.float32), np.float32([1.0, 0.0, 2**-30, 2**-70, 3.5e11]),
                             (rng.random(50) * 1e-12).astype(np.float32)])
    for v in values:
        m, bad = oracle.mass_of(float(v))
        assert bad == 0
        assert m == int(Fraction(float(v)) * 2**64)  # floor for non-negative
    for bad_value in (-1.0, float("inf"), float("nan"), 2.0**41):
        assert oracle.mass_of(bad_value)[1] == 1
    assert oracle.mass_of(-0.0) == (0, 0)


def test_mass_scale_is_exact_floor():
    rng = np.random.default_rng(2)
    for _ in range(500):
        total = int(rng.integers(1, 2**62)) * int(rng.integers(1, 2**50)) + int(rng.integers(0, 2**63))
        u = float(rng.random())
        assert oracle.mass_scale(u, total) == int(Fraction(u) * total)
    assert oracle.mass_scale(0.0, 12345) == 0


def test_philox_matches_host_restatement():
    from specgrove_b200.sampling import philox_node_uniforms
    for seed, req, node in [(0, 0, 0), (1234567890123, 17, 5), (2**63 + 5, 2**40 + 3, 127)]:
        a = oracle.node_uniforms(seed, req, node)
        b = philox_node_uniforms(seed, req, node)
        assert a == b
        assert 0.0 <= a[0] < 1.0 and 0.0 <= a[1] < 1.0


def test_philox_known_answer():
    # Random123 Philox4x32-10 known-answer vector (counter 0, key 0):
    # 6627e8d5 e169c58d bc57ac4c 9b00dbd8
    from specgrove_b200.sampling import philox_node_uniforms
    u = philox_node_uniforms(0, 0, 0)
    v = ((0xe169c58d << 32) | 0x6627e8d5) >> 11
    assert u[0] == v / 2.0**53


def test_packed_inputs_restatement_matches_reference(golden_dir):
    from oracle.packed_inputs import packed_block_inputs
    z = np.load(golden_dir / "packed_inputs.npz")
    counts = z["row_counts"].tolist()
    offsets = np.cumsum([0] + counts)
    trees = []
    for i, n in enumerate(counts):
        par = z["parents"][offsets[i]:offsets[i + 1]].tolist()
        tok = z["tokens"][offsets[i]:offsets[i + 1]].tolist()
        tok[0] = int(z["roots"][i])
        trees.append((par, tok))
    ids, pos, mask, q_off = packed_block_inputs(trees, z["lengths"].tolist(), z["round_prefix"].tolist())
    np.testing.assert_array_equal(ids.numpy(), z["ids"])
    np.testing.assert_array_equal(pos.numpy(), z["positions"])
    np.testing.assert_array_equal(np.isfinite(mask[0, 0].numpy()), z["visible"])
    assert list(q_off) == z["q_offsets"].tolist()


def test_wave_builder_validates_like_reference():
    from specgrove_b200.engine import Wave
    w = Wave([([-1, 0, 0, 1], [5, 6, 7, 8]), ([-1], [9])], [0, 3], [10, 20], [12, 21], [7, 8])
    assert w.num_rows == 5 and w.max_depth == 2 and w.max_rows_per_request == 4
    assert w.row_offsets == [0, 4, 5]
    with pytest.raises(ValueError, match="precede"):
        Wave([([-1, 1], [1, 2])], [0], [0])
    with pytest.raises(ValueError, match="repeat"):
        Wave([([-1, 0, 0], [1, 2, 2])], [0], [0])


def test_allocator_matches_reference(golden_dir):
    import json
    from specgrove_b200.allocator import allocate_tree_budgets, critical_path_weights, draft_tree_expected_tokens
    z = json.loads((golden_dir / "allocator.json").read_text())
    for p in z["problems"]:
        weights = critical_path_weights(p["progress"], p["ages"], p["criticality"], p["max_new_tokens"])
        curve = [tuple(x) for x in p["curve"]] if p["curve"] else None
        alloc = allocate_tree_budgets(weights, p["options"], p["utilities"], row_budget=p["row_budget"],
                                      fixed_row_equivalent=p["fixed"], row_cost_curve=curve)
        assert list(alloc) == p["allocation"]
    for t in z["trees"]:
        assert draft_tree_expected_tokens(t["masses"]) == pytest.approx(t["expected"], rel=1e-12)


def test_draft_tree_oracle_matches_reference():
    """oracle/draft_tree.py against probability_tree, _prefix_tree and
    _draft_tree_expected_tokens run on the same proposals."""
    from draft_tree_cases import load_cases
    from oracle.draft_tree import best_first_tree, proposal_logs, tier_utility
    for c in load_cases():
        logs, ids = proposal_logs(c["logits"], c["temperature"], c["K"])
        assert np.array_equal(ids, c["ids"])
        assert np.max(np.abs(logs - c["logs"])) < 1e-12
        # the tree is a pure function of the ranked log masses: exact
        t = best_first_tree(c["logs"], c["ids"], c["budget"], c["rewards"], c["caps"], c["adaptive_min"],
                            c["threshold"])
        assert t.tokens == c["tokens"].tolist()
        assert t.parents == c["parents"].tolist()
        assert t.depths == c["depths"].tolist()
        assert t.masses == c["masses"].tolist()
        for b, u in zip(c["tiers"], c["utilities"]):
            got = tier_utility(t, int(b))
            assert (math.isnan(got) and math.isnan(u)) or got == u


def test_dflash_oracle_matches_reference():
    """oracle/draft_forward.py against the reference DFlashDraftModel over two
    cached drafter steps per request: block logits and cached context K/V."""
    import torch
    import dflash_case as case
    from oracle.draft_forward import dflash_step
    c = case.CONFIG
    z = np.load(case.GOLDEN)
    w, features = case.make_weights_and_inputs()
    for r, steps in enumerate(case.UPDATES):
        ck, cv = [], []
        for s_i, _ in enumerate(steps):
            logits, ck, cv = dflash_step(w, c["num_layers"], c["num_q_heads"], c["num_kv_heads"], c["head_dim"],
                                         features[r][s_i], ck, cv, case.ANCHORS[r][s_i], c["mask_token"], c["block"],
                                         case.inv_freq(), c["rms_eps"])
            want = z[f"r{r}_s{s_i}_logits"]
            assert np.max(np.abs(logits.numpy() - want)) < 1e-4 * max(1.0, np.abs(want).max())
        for l in range(c["num_layers"]):
            assert np.max(np.abs(ck[l].numpy() - z[f"r{r}_k{l}"])) < 1e-5
            assert np.max(np.abs(cv[l].numpy() - z[f"r{r}_v{l}"])) < 1e-5


def test_oracle_terminal_mass_matches_reference(golden_dir):
    """Terminal-mass verifier (sampling.py:542-735): the oracle's exact-mass
    restatement picks the reference function's terminal node and bonus token
    at the recorded uniforms, on every case (softmax, sparse-zero and
    unnormalised rows, one-node trees included)."""
    n_cases = 0
    for c in _cases(golden_dir / "terminal_mass.npz"):
        out, st = oracle.terminal_mass(c["probs"], [0, len(c["parents"])], c["parents"], c["tokens"],
                                       c["max_depth"], uniforms=c["uniforms"][None])
        assert st == 0
        D = c["max_depth"]
        count = int(out[0, D])
        assert out[0, :count].tolist() == c["nodes"]
        assert int(out[0, D + 1]) == c["bonus"]
        n_cases += 1
    assert n_cases >= 12


def test_oracle_terminal_mass_rejects_bad_input():
    probs = np.full((3, 8), 1 / 8, dtype=np.float32)
    u = np.array([[0.3, 0.6]])
    _, st = oracle.terminal_mass(probs, [0, 3], [-1, 0, 0], [-1, 2, 2], 2, uniforms=u)
    assert st == 3  # a node repeats a child token
    bad = probs.copy()
    bad[0, 5] = -0.1
    _, st = oracle.terminal_mass(bad, [0, 3], [-1, 0, 0], [-1, 2, 3], 2, uniforms=u)
    assert st == 4
    out, st = oracle.terminal_mass(probs, [0, 3], [-1, 0, 1], [-1, 2, 3], 1, uniforms=u)
    assert st == 3 and (out == -1).all()  # depth 2 > max_depth 1
