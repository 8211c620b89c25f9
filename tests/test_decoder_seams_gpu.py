"""The decoder seams (specgrove_b200/decoder_seams.py) driven the way the
reference's wave loop drives them (continuous_tree_block_decode.py:1604-1620
pool, :1748-1789 pack, :1791-1826 target pass, :1933-1964 lazy-projection
verifier, :2121-2129 commit), with HF Qwen3 as the wrapped reference engine.
The dense mask comes from the oracle's restatement of _packed_block_inputs."""
import numpy as np
import pytest
import torch

from oracle.packed_inputs import packed_block_inputs
from specgrove_b200 import decoder_seams as seams
from test_verify_pass_gpu import hf_model, hf_wave_hidden_states, make_trees

pytestmark = pytest.mark.gpu


class _Draft:
    target_layer_ids = (0, 1)


class _BaseEngine:
    """The members of the reference Engine the decoder reads (engine.py)."""

    def __init__(self, model):
        self.target = model
        self.device = torch.device("cuda")
        self.draft = _Draft()

    def target_hidden_forward(self, ids, cache, *, positions=None, mask=None):
        raise AssertionError("a packed arena wave must not reach the wrapped engine")


def _prefill_caches(model, prompts):
    from transformers import DynamicCache
    caches = []
    with torch.no_grad():
        for p in prompts:
            c = DynamicCache()
            model(input_ids=torch.tensor([p], device="cuda"), past_key_values=c, use_cache=True)
            caches.append(c)
    return caches


def test_wave_through_the_seams(cuda_lib):
    model = hf_model(layers=3, hidden=256, nq=4, nkv=2, head_dim=64, inter=512, vocab=1024, logit_scale=1.0)
    rng = np.random.default_rng(17)
    prompts = [rng.integers(0, 1024, size=int(rng.integers(20, 120))).tolist() for _ in range(4)]
    trees = make_trees(rng, 4, 1024, 2, 24)
    hf_hidden = hf_wave_hidden_states(model, prompts, trees)

    pool = seams.arena_pool(_prefill_caches(model, prompts), capacity=256)
    order = [2, 0, 3, 1]                                   # a wave need not follow slot order
    caches = [pool.caches[i] for i in order]
    wave_trees = [trees[i] for i in order]
    packed, lengths, offsets, total = seams.pack_cache_sequence(caches, None, "cuda")
    assert lengths == tuple(len(prompts[i]) for i in order) and total == sum(lengths)
    ids, pos, mask, q_off = packed_block_inputs(wave_trees, list(lengths), list(lengths), dtype=torch.bfloat16,
                                                device="cuda")
    engine = seams.B200VerifyEngine(_BaseEngine(model), max_rows=256)
    out = engine.target_hidden_forward(ids, packed, positions=pos, mask=mask)
    assert [t[0] for t in packed.trees] == [t[0] for t in wave_trees]    # tree structure read from the mask
    # last_hidden_state and the drafter layer's hidden state vs HF, row for row
    hf_rows = torch.cat([torch.arange(sum(len(t[0]) for t in trees[:i]), sum(len(t[0]) for t in trees[:i + 1]))
                         for i in order]).cuda()
    for ours, ref in ((out.last_hidden_state[0], hf_hidden[3][hf_rows]), (out.hidden_states[1][0], hf_hidden[1][hf_rows])):
        err = (ours.float() - ref.float()).abs()
        scale = ref.float().abs().max().item()
        assert err.max().item() < 3e-2 * scale and err.mean().item() < 3e-3 * scale

    # the lazy-projection verifier seam: hidden states + the LM-head module
    lm = model.get_output_embeddings()
    sizes = [len(t[0]) for t in wave_trees]
    rows = list(out.last_hidden_state[0].split(sizes))
    gens = lambda: [torch.Generator(device="cuda").manual_seed(100 + i) for i in range(4)]
    res = seams.tree_verify_ancestral_lazy_projection_fused_scan_batched(
        [t[0] for t in wave_trees], [t[1][1:] for t in wave_trees], rows, lm, 1.0, torch.float64, gens())
    again = seams.tree_verify_ancestral_lazy_projection_fused_scan_batched(
        [t[0] for t in wave_trees], [t[1][1:] for t in wave_trees], rows, lm, 1.0, torch.float64, gens())
    assert [r[:3] for r in res] == [r[:3] for r in again]              # keyed by each request's generator
    for (nodes, toks, bonus, stats), (par, tok) in zip(res, wave_trees):
        assert 0 <= bonus < 1024 and stats["total_tree_rows"] == len(par)
        node = 0
        for n, t in zip(nodes, toks):                                   # a root path of the tree
            assert par[n] == node and tok[n] == t
            node = n
    # greedy (T = 0) walks the argmax of the bf16 logits of the same rows
    greedy = seams.tree_verify_ancestral_lazy_projection_fused_scan_batched(
        [t[0] for t in wave_trees], [t[1][1:] for t in wave_trees], rows, lm, 0.0, torch.float64, gens())
    for (nodes, _, bonus, _), (par, tok), h in zip(greedy, wave_trees, rows):
        logits = (h.float() @ lm.weight.float().t()).to(torch.bfloat16)
        top2 = logits.float().topk(2, dim=-1).values
        if ((top2[:, 0] - top2[:, 1]) < 0.05).any():
            continue                                                    # near-ties: rounding decides
        arg = logits.float().argmax(-1).tolist()
        node, walk = 0, []
        children = {(par[j], tok[j]): j for j in range(1, len(par))}
        while (node, arg[node]) in children:
            node = children[(node, arg[node])]
            walk.append(node)
        assert nodes == walk and bonus == arg[node]

    # the decoder's default verifier seam (terminal mass), called as the
    # decoder calls it, on the same rows' probabilities
    for (par, tok), h in zip(wave_trees, rows):
        probs = torch.softmax(h.float() @ lm.weight.float().t(), dim=-1)
        g = torch.Generator(device="cuda").manual_seed(7)
        nodes, toks, bonus = seams.tree_block_verify_terminal_mass(par, tok[1:], probs, g, validate=False,
                                                                  prefix_mode="batched", exit_mode="internal")
        node = 0
        for n, t in zip(nodes, toks):
            assert par[n] == node and tok[n] == t
            node = n
        assert 0 <= bonus < 1024 and (node, bonus) not in {(par[j], tok[j]) for j in range(1, len(par))}

    # commit: the arena keeps [0] + accepted rows of each request in place
    tail_before = pool.storage.clone()
    keep = [[0] + r[0] for r in res]
    pool.append_packed_sequence(packed, caches, total, q_off, keep)
    torch.cuda.synchronize()
    for c, L, k in zip(caches, lengths, keep):
        assert pool.lengths[c.slot] == L + len(k)
        base = c.slot * pool.capacity + L
        for i, node in enumerate(k):
            assert torch.equal(pool.storage[:, :, :, base + i], tail_before[:, :, :, base + node])
