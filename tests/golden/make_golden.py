"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference source tree is available:

    python tests/golden/make_golden.py --reference <path to specgrove checkout>

Every expected output below is produced by calling the reference's own
functions (no restatement):

  accept_scan.npz    ancestral inverse-CDF walk: fused_tree_sampling._topology,
                     _sample_row_inverse_cdf (fused_tree_sampling.py:2607-2612)
                     on float64 rows, tree_block_skip.child_for_edge, with the
                     stop rule of fused_tree_sampling.py:600-620.
  accept_sparse.npz  sparse-exit walk: child routing by fp64 cumulative child
                     mass (fused_tree_sampling.py:727-746) and the exit draw of
                     _sample_row_inverse_cdf on the row with the children zeroed.
  follow.npz         sampling.tree_verify_ancestral_batched (sampling.py:903-950)
                     with its `sample` replaced by fixed posterior tokens, as the
                     reference's own exact-law test does.
  kv_commit.npz      continuous_tree_block_decode._PersistentRequestCachePool and
                     append_packed_sequence (:176-261) on random small caches.
  packed_inputs.npz  continuous_tree_block_decode._packed_block_inputs (:500-546)
                     on random trees: ids, positions and the additive mask.
  allocator.json     continuous_tree_block_decode._allocate_global_tree_budgets
                     (:706-795) on random problems (linear and measured-curve
                     cost models) and _draft_tree_expected_tokens (:560-568) on
                     probability_tree (tree.py:148-212) outputs.
  draft_trees.npz    tree.probability_tree (tree.py:148-212) on softmax
                     proposals (sampling.probabilities, sampling.py:29-36) of
                     random fp32 logits: the top-k log masses it ranks, the
                     tree, and _prefix_tree / _draft_tree_expected_tokens
                     (continuous_tree_block_decode.py:560-586) per tier.
  terminal_mass.npz  sampling.tree_block_verify_terminal_mass (sampling.py:542-735,
                     default modes) on float64 rows, with its `sample` replaced
                     by an inverse-CDF draw at given uniforms (first index whose
                     running mass exceeds u * total): u[0] draws the terminal
                     node, u[1] the bonus token (a one-node tree's only draw is
                     its bonus, so it gets u[1]).
  dflash_step.npz    third_party/ddtree_official/model/dflash.py
                     DFlashDraftModel (tiny configuration, weights of
                     tests/dflash_case.py) over two drafter steps per request
                     with a DynamicCache cropped to the context rows, as
                     dflash.py:230-241 and the decoder drive it: block logits
                     through the LM head and the cached context K/V.

The fixtures are small (tens of KB) and deterministic (seeded torch CPU RNG).
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def random_tree(gen: torch.Generator, n: int, vocab: int, max_children: int = 4,
                max_depth: int = 8):
    parents, tokens, depths = [-1], [-1], [0]
    kids: dict[int, set[int]] = {0: set()}
    for j in range(1, n):
        while True:
            cand = int(torch.randint(0, j, (1,), generator=gen))
            if len(kids[cand]) < max_children and depths[cand] < max_depth:
                break
        while True:
            tok = int(torch.randint(0, vocab, (1,), generator=gen))
            if tok not in kids[cand]:
                break
        kids[cand].add(tok)
        kids[j] = set()
        parents.append(cand)
        tokens.append(tok)
        depths.append(depths[cand] + 1)
    return parents, tokens, depths


def tree_rows(gen, parents, tokens, vocab, kind: str):
    n = len(parents)
    logits = torch.randn((n, vocab), generator=gen, dtype=torch.float32) * 2.0
    for j in range(1, n):  # make children likely so walks go deep
        logits[parents[j], tokens[j]] += float(torch.empty(1).uniform_(2.0, 6.0, generator=gen))
    probs = torch.softmax(logits, dim=-1)
    if kind == "sparse_zeros":
        probs = probs * (torch.rand((n, vocab), generator=gen) > 0.3)
        probs = probs / probs.sum(-1, keepdim=True)
    elif kind == "unnormalised":
        probs = probs * 7.25
    return probs.to(torch.float32)


def build_accept_cases(ref, gen, rule: str):
    fts = ref.fused
    cases = []
    specs = [(1, 64, "softmax"), (2, 64, "softmax"), (5, 64, "softmax"), (9, 500, "softmax"),
             (17, 300, "softmax"), (8, 1001, "softmax"), (6, 1000, "sparse_zeros"),
             (20, 256, "softmax"), (33, 256, "softmax"), (4, 2048, "softmax"),
             (3, 4096, "sparse_zeros")]
    if rule == "scan":
        specs += [(13, 300, "unnormalised"), (6, 77, "unnormalised")]
    for n, vocab, kind in specs:
        parents, tokens, depths = random_tree(gen, n, vocab)
        probs = tree_rows(gen, parents, tokens, vocab, kind)
        _, _, max_depth = fts._topology(parents, tokens[1:])
        width = (max_depth + 1) * (2 if rule == "sparse" else 1)
        uniforms = torch.rand(width, dtype=torch.float64, generator=gen)
        nodes, toks, bonus = reference_walk(ref, parents, tokens, probs, uniforms, max_depth, rule)
        cases.append(dict(parents=parents, tokens=tokens, probs=probs.numpy(), uniforms=uniforms.numpy(),
                          max_depth=max_depth, nodes=nodes, bonus=bonus, vocab=vocab))
    return cases


def reference_walk(ref, parents, tokens, probs, uniforms, max_depth, rule):
    fts, tbs = ref.fused, ref.tbs
    node, nodes, toks = 0, [], []
    edge_tokens = tokens[1:]
    for depth in range(max_depth + 1):
        row = probs[node].to(torch.float64)
        if rule == "scan":
            token = fts._sample_row_inverse_cdf(row, float(uniforms[depth]))
            child = tbs.child_for_edge(parents, edge_tokens, node, token)
            if child is not None and depth < max_depth:
                nodes.append(child)
                toks.append(token)
                node = child
                continue
            return nodes, toks, token
        # sparse exit
        children = [j for j in range(1, len(parents)) if parents[j] == node]
        cumulative, route = 0.0, None
        for j in children:
            cumulative += float(row[edge_tokens[j - 1]])
            if route is None and float(uniforms[2 * depth]) < cumulative:
                route = j
        if route is not None and depth < max_depth:
            nodes.append(route)
            toks.append(edge_tokens[route - 1])
            node = route
            continue
        masked = row.clone()
        for j in children:
            masked[edge_tokens[j - 1]] = 0.0
        token = fts._sample_row_inverse_cdf(masked, float(uniforms[2 * depth + 1]))
        return nodes, toks, token
    raise AssertionError("walk did not terminate")


def pack_cases(cases):
    offsets = [0]
    parents, tokens, probs, uniforms, expected = [], [], [], [], []
    for c in cases:
        offsets.append(offsets[-1] + len(c["parents"]))
        parents += c["parents"]
        tokens += c["tokens"]
    return np.asarray(offsets, np.int64), np.asarray(parents, np.int64), np.asarray(tokens, np.int64)


def save_accept(name: str, cases):
    offsets, parents, tokens = pack_cases(cases)
    arrays = {"row_offsets": offsets, "parents": parents, "tokens": tokens}
    for i, c in enumerate(cases):
        arrays[f"probs_{i}"] = c["probs"]
        arrays[f"uniforms_{i}"] = c["uniforms"]
        arrays[f"max_depth_{i}"] = np.int64(c["max_depth"])
        arrays[f"nodes_{i}"] = np.asarray(c["nodes"], np.int64)
        arrays[f"bonus_{i}"] = np.int64(c["bonus"])
    arrays["count"] = np.int64(len(cases))
    np.savez_compressed(OUT / name, **arrays)


def build_terminal_mass(ref, gen):
    """Terminal-mass verifier cases: the reference function itself with its
    categorical draws made inverse-CDF draws at recorded uniforms."""
    sampling = ref.sampling
    specs = [(1, 64, "softmax"), (2, 64, "softmax"), (5, 64, "softmax"), (9, 500, "softmax"),
             (17, 300, "softmax"), (8, 1001, "softmax"), (6, 1000, "sparse_zeros"), (20, 256, "softmax"),
             (33, 256, "softmax"), (4, 2048, "softmax"), (13, 300, "unnormalised"), (6, 77, "unnormalised"),
             (12, 128, "softmax"), (3, 4096, "sparse_zeros")]
    cases = []
    original = sampling.sample
    try:
        for n, vocab, kind in specs:
            parents, tokens, depths = random_tree(gen, n, vocab)
            probs = tree_rows(gen, parents, tokens, vocab, kind)
            uniforms = torch.rand(2, dtype=torch.float64, generator=gen)
            queue = [float(uniforms[1])] if n == 1 else [float(uniforms[0]), float(uniforms[1])]

            def inverse_cdf(weights, generator=None, _queue=queue):
                cumulative = weights.reshape(-1).to(torch.float64).cumsum(0)
                u = _queue.pop(0)
                index = torch.searchsorted(cumulative, torch.tensor(u * float(cumulative[-1]), dtype=torch.float64),
                                           right=True)
                return index.clamp_max(cumulative.numel() - 1).reshape(())

            sampling.sample = inverse_cdf
            nodes, _, bonus = sampling.tree_block_verify_terminal_mass(
                parents, tokens[1:], probs.to(torch.float64), generator=None, validate=False)
            cases.append(dict(parents=parents, tokens=tokens, probs=probs.numpy(), uniforms=uniforms.numpy(),
                              max_depth=max(depths), nodes=nodes, bonus=bonus, vocab=vocab))
    finally:
        sampling.sample = original
    save_accept("terminal_mass.npz", cases)
    return cases


def build_accept_logits(ref, gen):
    """Direct-logits walk (the rule of fused_tree_sampling.py:942-1115): the
    reference's own _sample_row_inverse_cdf on the fp64 weights
    exp(double(logit) / T - max), ancestrally with child_for_edge.  Logits
    are bf16-representable so the same rows serve fp32 and bf16 inputs."""
    fts, tbs = ref.fused, ref.tbs
    cases = []
    for n, vocab, temperature in [(1, 64, 1.0), (5, 300, 1.0), (9, 1000, 0.7), (17, 256, 1.6), (8, 4096, 1.0),
                                  (33, 512, 0.35), (12, 2049, 1.0)]:
        parents, tokens, _ = random_tree(gen, n, vocab)
        logits = torch.randn((n, vocab), generator=gen, dtype=torch.float32) * 2.0
        for j in range(1, n):
            logits[parents[j], tokens[j]] += float(torch.empty(1).uniform_(2.0, 6.0, generator=gen))
        logits = logits.to(torch.bfloat16).to(torch.float32)
        _, _, max_depth = fts._topology(parents, tokens[1:])
        uniforms = torch.rand(max_depth + 1, dtype=torch.float64, generator=gen)
        node, nodes, bonus = 0, [], None
        for depth in range(max_depth + 1):
            x = logits[node].to(torch.float64) * (1.0 / temperature)
            weights = torch.exp(x - x.max())
            token = fts._sample_row_inverse_cdf(weights, float(uniforms[depth]))
            child = tbs.child_for_edge(parents, tokens[1:], node, token)
            if child is not None and depth < max_depth:
                nodes.append(child)
                node = child
                continue
            bonus = token
            break
        cases.append(dict(parents=parents, tokens=tokens, probs=logits.numpy(), uniforms=uniforms.numpy(),
                          max_depth=max_depth, nodes=nodes, bonus=bonus, vocab=vocab, temperature=temperature))
    return cases


def build_follow(ref, gen):
    sampling = ref.sampling
    cases = []
    for n, vocab in [(1, 16), (4, 8), (9, 32), (17, 64), (40, 128), (64, 50)]:
        parents, tokens, _ = random_tree(gen, n, vocab)
        # posterior: mostly a child token so the walk descends, sometimes not
        posterior = []
        for j in range(n):
            kids = [tokens[c] for c in range(1, n) if parents[c] == j]
            if kids and float(torch.rand(1, generator=gen)) < 0.8:
                posterior.append(kids[int(torch.randint(0, len(kids), (1,), generator=gen))])
            else:
                posterior.append(int(torch.randint(0, vocab, (1,), generator=gen)))
        fixed = torch.tensor(posterior)
        original = sampling.sample
        sampling.sample = lambda probs, generator=None, _f=fixed: _f.clone()
        try:
            nodes, toks, bonus = sampling.tree_verify_ancestral_batched(
                parents, tokens[1:], torch.ones((n, vocab)) / vocab, None, validate=True)
        finally:
            sampling.sample = original
        depth = [0] * n
        for j in range(1, n):
            depth[j] = depth[parents[j]] + 1
        cases.append(dict(parents=parents, tokens=tokens, posterior=posterior, nodes=nodes,
                          bonus=bonus, max_depth=max(depth)))
    offsets, parents, tokens = pack_cases(cases)
    arrays = {"row_offsets": offsets, "parents": parents, "tokens": tokens,
              "posterior": np.asarray(sum((c["posterior"] for c in cases), []), np.int64),
              "count": np.int64(len(cases))}
    for i, c in enumerate(cases):
        arrays[f"nodes_{i}"] = np.asarray(c["nodes"], np.int64)
        arrays[f"bonus_{i}"] = np.int64(c["bonus"])
        arrays[f"max_depth_{i}"] = np.int64(c["max_depth"])
    np.savez_compressed(OUT / "follow.npz", **arrays)


def build_kv_commit(ref, gen):
    decode = ref.decode
    heads, dim, layers = 2, 8, 3
    lengths = [5, 1, 9, 3]
    capacity = 24
    sources = []
    for L in lengths:
        lay = []
        for _ in range(layers):
            k = torch.randn((1, heads, L, dim), generator=gen)
            v = torch.randn((1, heads, L, dim), generator=gen)
            lay.append(SimpleNamespace(keys=k, values=v))
        sources.append(SimpleNamespace(layers=lay, get_seq_length=(lambda L=L: L)))
    pool = decode._PersistentRequestCachePool(sources, capacity=capacity)
    before_k = torch.stack(pool.key_storage).clone()
    before_v = torch.stack(pool.value_storage).clone()
    rows = [4, 2, 6, 3]
    q_offsets = [0, 4, 6, 12]
    total_prefix = sum(lengths)
    total_q = sum(rows)
    packed_layers = []
    for _ in range(layers):
        k = torch.randn((1, heads, total_prefix + total_q, dim), generator=gen)
        v = torch.randn((1, heads, total_prefix + total_q, dim), generator=gen)
        packed_layers.append(SimpleNamespace(keys=k, values=v))
    packed = SimpleNamespace(layers=packed_layers)
    keep = [[0, 1, 3], [0], [0, 2, 4, 5], [0, 1]]
    pool.append_packed_sequence(packed, pool.caches, total_prefix, q_offsets, keep, "cpu")
    np.savez_compressed(
        OUT / "kv_commit.npz",
        before_k=before_k.numpy(), before_v=before_v.numpy(),
        after_k=torch.stack(pool.key_storage).numpy(), after_v=torch.stack(pool.value_storage).numpy(),
        packed_k=torch.stack([l.keys[0] for l in packed_layers]).numpy(),
        packed_v=torch.stack([l.values[0] for l in packed_layers]).numpy(),
        lengths=np.asarray(lengths, np.int64), capacity=np.int64(capacity),
        q_offsets=np.asarray(q_offsets, np.int64), packed_old_length=np.int64(total_prefix),
        keep_flat=np.asarray(sum(keep, []), np.int64),
        keep_offsets=np.asarray(np.cumsum([0] + [len(k) for k in keep]), np.int64),
        after_lengths=np.asarray(pool.lengths, np.int64))


def build_packed_inputs(ref, gen):
    decode, tbs, tree_mod = ref.decode, ref.tbs, ref.tree
    states, blocks, lengths = [], [], []
    for i, (n, L) in enumerate([(5, 7), (1, 3), (12, 9), (8, 4)]):
        parents, tokens, depths = random_tree(gen, n, 50)
        t = tree_mod.Tree(tokens=tokens[1:], parents=parents, depths=depths, path_nodes=[])
        block = tbs.local_tree_block(t.parents, t.tokens, t.depths, 0, n)
        st = SimpleNamespace(tree=t, generated=[100 + i], block_root=0, round_prefix_len=L + 2 * i)
        states.append(st)
        blocks.append(block)
        lengths.append(L)
    offsets = list(np.cumsum([0] + lengths[:-1]))
    total = sum(lengths)
    ids, positions, mask, q_offsets = decode._packed_block_inputs(
        states, blocks, tuple(lengths), tuple(offsets), total, torch.float32, "cpu")
    np.savez_compressed(
        OUT / "packed_inputs.npz",
        ids=ids.numpy(), positions=positions.numpy(), visible=torch.isfinite(mask[0, 0]).numpy(),
        q_offsets=np.asarray(q_offsets, np.int64), lengths=np.asarray(lengths, np.int64),
        cache_offsets=np.asarray(offsets, np.int64),
        parents=np.asarray(sum((list(b.parents) for b in blocks), []), np.int64),
        tokens=np.asarray(sum(([-1] + list(b.tokens) for b in blocks), []), np.int64),
        depths=np.asarray(sum((list(b.depths) for b in blocks), []), np.int64),
        row_counts=np.asarray([len(b.nodes) for b in blocks], np.int64),
        roots=np.asarray([s.generated[-1] for s in states], np.int64),
        round_prefix=np.asarray([s.round_prefix_len for s in states], np.int64))


def build_allocator(ref, gen):
    import json
    decode, tree_mod = ref.decode, ref.tree
    problems = []
    for case in range(12):
        count = int(torch.randint(2, 9, (1,), generator=gen))
        options = [15, 31, 63] if case % 2 else [11, 23, 45]
        states = [SimpleNamespace(generated=[0] * int(torch.randint(0, 200, (1,), generator=gen)),
                                  age=int(torch.randint(0, 30, (1,), generator=gen)), request_id=i)
                  for i in range(count)]
        utilities = [[1.0 + float(torch.rand(1, generator=gen)) * 3 * (k + 1) for k in range(len(options))]
                     for _ in range(count)]
        row_budget = count * (options[0] + 1) + int(torch.randint(0, count * 40 + 1, (1,), generator=gen))
        curve = [[12, 24.5], [46, 24.6], [96, 24.8], [193, 25.1], [384, 39.0]] if case % 3 == 0 else None
        fixed = None if curve else 20.0 + case
        c = 1.0 if case % 4 else 0.0
        alloc = decode._allocate_global_tree_budgets(
            states, options, utilities, row_budget=row_budget, fixed_row_equivalent=fixed, criticality_weight=c,
            max_new_tokens=256, row_cost_curve=curve)
        problems.append(dict(progress=[len(s.generated) for s in states], ages=[s.age for s in states],
                             options=options, utilities=utilities, row_budget=row_budget, curve=curve,
                             fixed=fixed, criticality=c, max_new_tokens=256, allocation=list(alloc)))
    trees = []
    for case in range(4):
        q = torch.softmax(3 * torch.randn((8, 64), generator=gen, dtype=torch.float64), -1)
        t = tree_mod.probability_tree(q, 15, rank_caps=(4,) * 8)
        trees.append(dict(masses=list(t.draft_prefix_log_masses), parents=list(t.parents),
                          expected=decode._draft_tree_expected_tokens(t)))
    (OUT / "allocator.json").write_text(json.dumps({"problems": problems, "trees": trees}))


def draft_tree_logits(seed: int, L: int, V: int, kind: str) -> torch.Tensor:
    """The fp32 proposal logits of one draft-tree case (regenerated by the
    tests from the stored seed; the fixture keeps a checksum)."""
    logits = torch.randn((L, V), generator=torch.Generator().manual_seed(seed), dtype=torch.float32) * 3.0
    if kind == "spine":
        logits[:, 0] += 30.0
    elif kind == "repeat":  # identical rows: exact ties between heap scores
        logits[:] = logits[0]
    return logits


def build_draft_trees(ref, gen):
    """Cases: (length, vocab, budget, temperature, reward schedule, rank caps,
    adaptive (min budget, threshold), tiers, kind)."""
    tree_mod, decode, sampling = ref.tree, ref.decode, ref.sampling
    specs = [
        (15, 4096, 60, 1.0, None, None, None, (16, 32, 60), "randn"),
        (15, 4096, 128, 0.7, None, None, None, (16, 32, 64, 128), "randn"),
        (15, 2048, 48, 1.0, (0.3,) * 15, None, None, (8, 48), "randn"),
        (6, 1024, 40, 1.5, (0.5, 0.25, 0.0, -0.25, 0.1, 0.2), None, None, (10, 40), "randn"),
        (15, 2048, 64, 1.0, None, (4,) * 15, None, (16, 64), "randn"),
        (8, 512, 64, 1.0, None, (1, 2, 3, 4, 5, 6, 7, 8), None, (20,), "randn"),
        (15, 2048, 64, 1.0, None, None, (16, 0.3), (16,), "spine"),
        (15, 2048, 64, 1.0, None, None, (16, 0.9), (16, 64), "randn"),
        (2, 8, 100, 1.0, None, None, None, (30, 72), "randn"),
        (5, 256, 40, 1.0, None, None, None, (12, 40), "repeat"),
        (15, 151936, 32, 1.0, None, None, None, (16, 32), "randn"),
    ]
    arrays = {"count": np.int64(len(specs))}
    base_seed = int(torch.randint(0, 2**31 - 1, (1,), generator=gen))
    for i, (L, V, budget, T, sched, caps, adaptive, tiers, kind) in enumerate(specs):
        seed = base_seed + i
        logits = draft_tree_logits(seed, L, V, kind)
        q = sampling.probabilities(logits.to(torch.float64), T, torch.float64)
        K = min(budget, V)
        values, indices = torch.topk(q, K, dim=-1, sorted=True)
        kwargs = {}
        if sched is not None:
            kwargs["depth_reward_schedule"] = sched
        if caps is not None:
            kwargs["rank_caps"] = caps
        if adaptive is not None:
            kwargs["adaptive_min_budget"], kwargs["confidence_threshold"] = adaptive
        t = tree_mod.probability_tree(q, budget, **kwargs)
        nodes = len(t.tokens)
        util = [decode._draft_tree_expected_tokens(decode._prefix_tree(t, b)) if b <= nodes else np.nan
                for b in tiers]
        pre = f"c{i}_"
        arrays[pre + "seed"] = np.int64(seed)
        arrays[pre + "kind"] = np.array(kind)
        arrays[pre + "logit_checksum"] = np.array([logits.double().sum().item(), logits.double().abs().max().item()])
        arrays[pre + "meta"] = np.array([L, V, budget, K, -1 if adaptive is None else adaptive[0]], np.int64)
        arrays[pre + "temperature"] = np.float64(T)
        arrays[pre + "threshold"] = np.float64(np.nan if adaptive is None else adaptive[1])
        arrays[pre + "rewards"] = np.array(sched if sched is not None else [], np.float64)
        arrays[pre + "caps"] = np.array(caps if caps is not None else [], np.int64)
        arrays[pre + "logs"] = values.log().numpy()
        arrays[pre + "ids"] = indices.numpy().astype(np.int64)
        arrays[pre + "tokens"] = np.array(t.tokens, np.int64)
        arrays[pre + "parents"] = np.array(t.parents, np.int64)
        arrays[pre + "depths"] = np.array(t.depths, np.int64)
        arrays[pre + "masses"] = np.array(t.draft_prefix_log_masses, np.float64)
        arrays[pre + "tiers"] = np.array(tiers, np.int64)
        arrays[pre + "utilities"] = np.array(util, np.float64)
    np.savez_compressed(OUT / "draft_trees.npz", **arrays)


def build_dflash_step(reference: Path):
    sys.path.insert(0, str(reference / "code" / "natural" / "third_party" / "ddtree_official"))
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from model.dflash import DFlashDraftModel
    from transformers import DynamicCache, Qwen3Config
    import dflash_case as case
    c = case.CONFIG
    cfg = Qwen3Config(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["intermediate"],
                      num_hidden_layers=c["num_layers"], num_attention_heads=c["num_q_heads"],
                      num_key_value_heads=c["num_kv_heads"], head_dim=c["head_dim"], rms_norm_eps=c["rms_eps"],
                      rope_theta=c["rope_theta"], max_position_embeddings=256, attention_bias=False)
    cfg.dflash_config = {"target_layer_ids": list(range(c["feature_layers"])), "mask_token_id": c["mask_token"]}
    cfg.block_size = c["block"]
    cfg.num_target_layers = 8
    cfg._attn_implementation = "eager"
    model = DFlashDraftModel(cfg).float().eval()
    w, features = case.make_weights_and_inputs()
    sd = {"fc.weight": w["fc"], "hidden_norm.weight": w["hidden_norm"], "norm.weight": w["norm"]}
    hf = {"in_norm": "input_layernorm", "q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
          "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm", "o": "self_attn.o_proj",
          "post_norm": "post_attention_layernorm", "gate": "mlp.gate_proj", "up": "mlp.up_proj",
          "down": "mlp.down_proj"}
    for l in range(c["num_layers"]):
        for ours, theirs in hf.items():
            sd[f"layers.{l}.{theirs}.weight"] = w[f"layers.{l}.{ours}"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in k for k in missing), (missing, unexpected)
    embed = torch.nn.Embedding.from_pretrained(w["embed"])
    arrays = {}
    for r, steps in enumerate(case.UPDATES):
        cache = DynamicCache()
        start = 0
        for s_i, u in enumerate(steps):
            feats = features[r][s_i]
            block_ids = torch.tensor([[case.ANCHORS[r][s_i]] + [c["mask_token"]] * (c["block"] - 1)])
            positions = torch.arange(start, start + u + c["block"])[None]
            with torch.no_grad():
                hidden = model(target_hidden=feats[None], noise_embedding=embed(block_ids), position_ids=positions,
                               past_key_values=cache, use_cache=True, is_causal=False)
                logits = hidden[0] @ w["lm_head"].T
            start += u
            cache.crop(start)
            arrays[f"r{r}_s{s_i}_logits"] = logits.numpy()
        for l in range(c["num_layers"]):
            arrays[f"r{r}_k{l}"] = cache.layers[l].keys[0].numpy()
            arrays[f"r{r}_v{l}"] = cache.layers[l].values[0].numpy()
    np.savez_compressed(OUT / "dflash_step.npz", **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the specgrove checkout")
    ap.add_argument("--only", default=None, help="regenerate one fixture builder (e.g. terminal_mass)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "code" / "natural" / "src"))
    from gbv_experiments import continuous_tree_block_decode as decode
    from gbv_experiments import fused_tree_sampling as fused
    from gbv_experiments import sampling, tree, tree_block_skip as tbs
    ref = SimpleNamespace(decode=decode, fused=fused, sampling=sampling, tree=tree, tbs=tbs)
    if args.only == "terminal_mass":
        build_terminal_mass(ref, torch.Generator().manual_seed(20261204))
        return
    gen = torch.Generator().manual_seed(20261201)
    save_accept("accept_scan.npz", build_accept_cases(ref, gen, "scan"))
    save_accept("accept_sparse.npz", build_accept_cases(ref, gen, "sparse"))
    build_follow(ref, gen)
    build_kv_commit(ref, gen)
    build_packed_inputs(ref, gen)
    build_allocator(ref, gen)
    # later fixtures use their own generator, so the ones above stay byte-identical
    logits_cases = build_accept_logits(ref, torch.Generator().manual_seed(20261202))
    save_accept("accept_logits.npz", logits_cases)
    with np.load(OUT / "accept_logits.npz") as z:
        arrays = dict(z)
    for i, c in enumerate(logits_cases):
        arrays[f"temperature_{i}"] = np.float64(c["temperature"])
    np.savez_compressed(OUT / "accept_logits.npz", **arrays)
    build_draft_trees(ref, torch.Generator().manual_seed(20261203))
    build_dflash_step(Path(args.reference))
    build_terminal_mass(ref, torch.Generator().manual_seed(20261204))
    for p in sorted(OUT.glob("*.*")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
