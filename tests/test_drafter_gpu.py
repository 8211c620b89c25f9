"""The drafter step (sg_draft_pass) against the fp32 DFlash oracle
(oracle/draft_forward.py, pinned to the reference DFlashDraftModel):
block logits of every request over two cached steps (the second reading the
context K/V the first wrote into the draft cache), the cached context K/V
themselves, and the on-device wave plan made from the logits."""
import numpy as np
import pytest
import torch

from oracle.draft_forward import dflash_step
from oracle.draft_tree import best_first_tree, proposal_logs
from specgrove_b200.drafter import B200Drafter, DraftShape, DraftWeights
from specgrove_b200.engine import ModelShape, Weights

pytestmark = pytest.mark.gpu


def oracle_weights(dw: DraftWeights) -> dict:
    s = dw.shape
    H, D, I = s.hidden, s.head_dim, s.intermediate
    nq, nkv = s.num_q_heads, s.num_kv_heads
    f = lambda t: t.float()
    w = {"embed": f(dw.target.embed), "lm_head": f(dw.target.lm_head), "fc": f(dw.fc),
         "hidden_norm": f(dw.hidden_norm), "norm": f(dw.norm)}
    for l, layer in enumerate(dw.layers):
        in_norm, qkv, q_norm, k_norm, o, post, gu, down = layer
        gu = gu.view(I // 128, 2, 128, H)
        w.update({f"layers.{l}.in_norm": f(in_norm), f"layers.{l}.q": f(qkv[:nq * D]),
                  f"layers.{l}.k": f(qkv[nq * D:(nq + nkv) * D]), f"layers.{l}.v": f(qkv[(nq + nkv) * D:]),
                  f"layers.{l}.q_norm": f(q_norm), f"layers.{l}.k_norm": f(k_norm), f"layers.{l}.o": f(o),
                  f"layers.{l}.post_norm": f(post), f"layers.{l}.gate": f(gu[:, 0].reshape(I, H)),
                  f"layers.{l}.up": f(gu[:, 1].reshape(I, H)), f"layers.{l}.down": f(down)})
    return w


def _random_norms(dw: DraftWeights, g):
    # non-trivial norm weights so that every norm is exercised
    for layer in dw.layers:
        for i in (0, 2, 3, 5):
            layer[i].copy_((1 + 0.2 * torch.randn(layer[i].shape, generator=g)).to(layer[i]))
    for t in (dw.hidden_norm, dw.norm):
        t.copy_((1 + 0.2 * torch.randn(t.shape, generator=g)).to(t))


def _check_close(got: torch.Tensor, want: torch.Tensor, max_rel: float, mean_rel: float):
    err = (got.float() - want).abs()
    scale = want.abs().max().item()
    assert err.max().item() <= max_rel * scale, (err.max().item(), scale)
    assert err.mean().item() <= mean_rel * scale, (err.mean().item(), scale)


def run_two_steps(shape: DraftShape, steps: list[list[int]], slots: list[int], std: float, seed: int,
                  capacity: int):
    g = torch.Generator().manual_seed(seed)
    target = Weights.random(ModelShape(1, shape.hidden, shape.num_q_heads, shape.num_kv_heads, shape.head_dim,
                                       shape.intermediate, shape.vocab), seed=seed, std=std)
    dw = DraftWeights.random(shape, target, seed=seed + 1, std=std)
    _random_norms(dw, g)
    R = len(slots)
    max_update = max(sum(s) for s in steps)
    drafter = B200Drafter(dw, num_slots=max(slots) + 1, capacity=capacity, max_requests=R,
                          max_update_rows=max_update)
    w = oracle_weights(dw)
    inv_freq = dw.inv_freq
    F = shape.num_feature_layers * shape.hidden
    caches = [([], []) for _ in range(R)]
    for step in steps:
        feats = [(torch.randn((u, F), generator=g) * 2).to(torch.bfloat16).cuda() for u in step]
        anchors = torch.randint(0, shape.vocab - 1, (R,), generator=g).tolist()
        logits = drafter.draft(slots, feats, anchors)
        torch.cuda.synchronize()
        assert int(drafter.status.item()) == 0
        for r in range(R):
            ck, cv = caches[r]
            want, ck, cv = dflash_step(w, shape.num_layers, shape.num_q_heads, shape.num_kv_heads, shape.head_dim,
                                       feats[r].float(), ck, cv, anchors[r], shape.mask_token_id, shape.block_size,
                                       inv_freq, shape.rms_eps)
            caches[r] = (ck, cv)
            _check_close(logits[r], want, 0.03, 0.004)
    # the draft cache holds every context row's K/V
    arena = drafter.arena
    for r, sl in enumerate(slots):
        n = sum(s[r] for s in steps)
        assert arena.lengths[sl] == n
        for l in range(shape.num_layers):
            k = arena.key_storage[l][:, sl * arena.capacity: sl * arena.capacity + n]
            v = arena.value_storage[l][:, sl * arena.capacity: sl * arena.capacity + n]
            _check_close(k, caches[r][0][l], 0.02, 0.003)
            _check_close(v, caches[r][1][l], 0.02, 0.003)
    return drafter, logits


def test_drafter_small_shape_two_steps():
    shape = DraftShape(2, 256, 4, 2, 64, 768, 4096, num_feature_layers=3, block_size=16, mask_token_id=4095)
    run_two_steps(shape, [[5, 1, 9, 3, 2], [2, 4, 1, 1, 3]], [3, 0, 4, 1, 2], std=0.06, seed=3, capacity=64)


def test_drafter_qwen3_8b_geometry():
    """hidden 4096, 32/8 heads, head_dim 128, intermediate 12288, V = 151936,
    5 feature layers, block 16 (z-lab/Qwen3-8B-DFlash-b16 shapes, 2 of its 5
    layers), draft caches of 300-1100 context rows."""
    shape = DraftShape(2, 4096, 32, 8, 128, 12288, 151936, num_feature_layers=5, block_size=16)
    run_two_steps(shape, [[700, 300, 1100, 450], [3, 1, 5, 2]], [1, 3, 0, 2], std=0.02, seed=8, capacity=1280)


def test_drafter_propose_plans_wave_from_its_logits():
    """propose(): drafter logits -> trees -> tiers -> packed wave, checked
    against the oracle chain on the same logits."""
    from specgrove_b200.allocator import allocate_tree_budgets
    shape = DraftShape(2, 256, 4, 2, 64, 768, 4096, num_feature_layers=3, block_size=16, mask_token_id=4095)
    drafter, _ = run_two_steps(shape, [[4, 6, 2]], [0, 1, 2], std=0.3, seed=21, capacity=64)
    g = torch.Generator().manual_seed(4)
    F = shape.num_feature_layers * shape.hidden
    feats = [(torch.randn((u, F), generator=g) * 2).to(torch.bfloat16).cuda() for u in (1, 2, 1)]
    anchors, tiers, weights = [5, 6, 7], [7, 15, 31], [1.0, 2.0, 1.0]
    plan = drafter.propose([0, 1, 2], feats, anchors, temperature=1.0, tiers=tiers, weights=weights, row_budget=60,
                           fixed_row_equivalent=16.0)
    torch.cuda.synchronize()
    assert int(plan.status.item()) == 0
    logits = plan.draft_logits[:, 1:16].float().cpu().numpy()
    utilities = []
    for r in range(3):
        logs, ids = proposal_logs(logits[r], 1.0, 31)
        assert np.array_equal(ids, plan.ids[r].cpu().numpy())
        assert np.max(np.abs(logs - plan.log_q[r].cpu().numpy())) < 1e-12
        t = best_first_tree(plan.log_q[r].cpu().numpy(), plan.ids[r].cpu().numpy(), 31)
        tokens, parents, depths, masses = plan.trees.tree(r)
        assert (tokens, parents, depths, masses) == (t.tokens, t.parents, t.depths, t.masses)
        utilities.append(plan.trees.utilities[r].cpu().tolist())
    alloc = allocate_tree_budgets(weights, tiers, utilities, row_budget=60, fixed_row_equivalent=16.0)
    assert tuple(plan.allocation.cpu().tolist()) == alloc
    offsets = plan.row_offsets.cpu().tolist()
    assert offsets[-1] == sum(a + 1 for a in alloc) <= 60
    for r in range(3):
        assert plan.tokens[offsets[r]].item() == anchors[r]
        assert plan.parents[offsets[r]].item() == -1
