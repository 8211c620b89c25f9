"""On-device draft-tree construction against the reference-generated trees
(tests/golden/draft_trees.npz) and the CPU oracle (oracle/draft_tree.py).

* proposal top-k: ids equal, log masses within 1e-12 (fp64; the reference's
  own values come from torch's fp64 softmax + log);
* trees: bit-equal tokens, parents, depths and prefix masses for the same log
  masses (tree.py:148-212, all options: reward schedules, rank caps, the
  adaptive budget, a vocabulary smaller than the budget, exact score ties);
* tier utilities within 4e-16 relative (exp rounding), allocation and packed
  wave equal to the host composition."""
import math

import numpy as np
import pytest
import torch

from draft_tree_cases import load_cases
from oracle.draft_tree import best_first_tree, proposal_logs, tier_utility
from specgrove_b200.allocator import allocate_tree_budgets
from specgrove_b200.draft_tree import build_draft_trees, pack_tree_wave, plan_wave, proposal_topk

pytestmark = pytest.mark.gpu

CASES = load_cases()


def _tree_kwargs(c):
    return dict(rewards=None if c["rewards"] is None else c["rewards"].tolist(),
                rank_caps=None if c["caps"] is None else c["caps"].tolist(),
                adaptive_min_budget=c["adaptive_min"], confidence_threshold=c["threshold"])


@pytest.mark.parametrize("i", range(len(CASES)))
def test_proposal_topk_matches_reference(i):
    c = CASES[i]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    logq, ids = proposal_topk(torch.from_numpy(c["logits"]).cuda(), c["temperature"], c["K"], status=status)
    assert int(status.item()) == 0
    assert np.array_equal(ids.cpu().numpy(), c["ids"])
    assert np.max(np.abs(logq.cpu().numpy() - c["logs"])) < 1e-12


@pytest.mark.parametrize("i", range(len(CASES)))
def test_draft_tree_matches_reference(i):
    c = CASES[i]
    tiers = [int(b) for b in c["tiers"]]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    trees = build_draft_trees(torch.from_numpy(c["logs"])[None].cuda(), torch.from_numpy(c["ids"])[None].cuda(),
                              c["budget"], tiers=tiers, status=status, **_tree_kwargs(c))
    tokens, parents, depths, masses = trees.tree(0)
    assert tokens == c["tokens"].tolist()
    assert parents == c["parents"].tolist()
    assert depths == c["depths"].tolist()
    assert masses == c["masses"].tolist()
    util = trees.utilities[0].cpu().numpy()
    for got, want in zip(util, c["utilities"]):
        if math.isnan(want):
            assert math.isnan(got)
        else:
            assert abs(got - want) <= 4e-16 * want
    expect_status = 3 if np.isnan(c["utilities"]).any() else 0  # SG_ERR_TREE for a tier above the tree
    assert int(status.item()) == expect_status


def test_batched_trees_from_bf16_logits_match_oracle():
    """64 requests x 15 depths at V = 151936 in bf16 (many exactly equal
    logits: ties go to the lower id on both sides)."""
    g = torch.Generator().manual_seed(5)
    R, L, V, budget = 64, 15, 151936, 128
    logits = (torch.randn((R, L, V), generator=g) * 2.5).to(torch.bfloat16)
    logits[:8, :, 17] += 20  # a few confident requests
    dev = logits.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    logq, ids = proposal_topk(dev, 1.0, budget, status=status)
    tiers = [16, 32, 64, 128]
    trees = build_draft_trees(logq, ids, budget, tiers=tiers, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    logq_h, ids_h = logq.cpu().numpy(), ids.cpu().numpy()
    for r in range(0, R, 7):
        want_logs, want_ids = proposal_logs(logits[r].float().numpy(), 1.0, budget)
        assert np.array_equal(ids_h[r], want_ids)
        assert np.max(np.abs(logq_h[r] - want_logs)) < 1e-12
    for r in range(R):
        t = best_first_tree(logq_h[r], ids_h[r], budget)
        tokens, parents, depths, masses = trees.tree(r)
        assert (tokens, parents, depths, masses) == (t.tokens, t.parents, t.depths, t.masses)
        util = trees.utilities[r].cpu().numpy()
        for b, got in zip(tiers, util):
            want = tier_utility(t, b)
            assert abs(got - want) <= 4e-16 * want


def test_plan_wave_matches_host_composition():
    g = torch.Generator().manual_seed(11)
    R, L, V = 24, 15, 4096
    tiers = [15, 31, 63]
    logits = (torch.randn((R, L, V), generator=g) * 3.0).to(torch.bfloat16).cuda()
    weights = torch.rand(R, generator=g, dtype=torch.float64) * 2 + 0.5
    anchors = torch.randint(0, V, (R,), generator=g)
    row_budget = 700
    plan = plan_wave(logits, 1.0, tiers, weights, anchors, row_budget=row_budget, fixed_row_equivalent=24.0)
    torch.cuda.synchronize()
    assert int(plan.status.item()) == 0
    util = plan.trees.utilities.cpu().numpy()
    host_alloc = allocate_tree_budgets(weights.tolist(), tiers, util.tolist(), row_budget=row_budget,
                                       fixed_row_equivalent=24.0)
    assert tuple(plan.allocation.cpu().tolist()) == host_alloc
    offsets = plan.row_offsets.cpu().tolist()
    parents, tokens = plan.parents.cpu().tolist(), plan.tokens.cpu().tolist()
    assert offsets[0] == 0 and offsets[-1] == sum(a + 1 for a in host_alloc) <= row_budget
    for r in range(R):
        t_tokens, t_parents, _, _ = plan.trees.tree(r)
        a = host_alloc[r]
        seg = slice(offsets[r], offsets[r + 1])
        assert parents[seg] == [-1] + t_parents[1:a + 1]
        assert tokens[seg] == [int(anchors[r])] + t_tokens[:a]
        assert all(p < j for j, p in enumerate(parents[seg][1:], start=1))  # ancestor closed


def test_pack_rejects_tier_above_tree():
    log_q = torch.log(torch.tensor([[[0.6, 0.4]], [[0.5, 0.5]]], dtype=torch.float64)).cuda()
    ids = torch.tensor([[[3, 4]], [[5, 6]]], dtype=torch.int64).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    trees = build_draft_trees(log_q, ids, 4, status=status)
    assert trees.node_count.cpu().tolist() == [2, 2]   # one depth, width 2
    offsets, _, _ = pack_tree_wave(trees, torch.tensor([2, 3], dtype=torch.int32, device="cuda"),
                                   torch.tensor([1, 2]), 16, status=status)
    assert int(status.item()) == 3
    assert offsets.cpu().tolist() == [0, 0, 0]
