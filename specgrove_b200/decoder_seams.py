"""Drop-in seams for the reference's continuous tree-block decoder.

The reference decoder (``continuous_tree_block_decode.py``) stays unchanged;
its wave loop reaches the target pass, the verifier and the commit through
module attributes and engine members (continuous_tree_block_decode.py:
1748-2129, engine.py:499-517).  This module supplies B200 versions of those
seams and ``install`` swaps them in (the reference's own plugin mechanism is
the same attribute substitution, scripts/paper_dp_allocators.py:59-80):

* ``_PersistentRequestCachePool`` -> ``arena_pool``: the persistent KV arena
  (``PersistentKVArena.from_caches``, one allocation for every layer's K/V);
* ``_pack_cache_sequence`` -> ``pack_cache_sequence``: no gather of the
  prefixes (the module docstring at :5-7 declares it replaceable); the packed
  "cache" names the requests' arena slots and lengths;
* ``engine`` -> ``B200VerifyEngine(engine)``: every member of the reference
  engine is kept (prefill, drafter, ``target``), but ``target_hidden_forward``
  on a packed arena wave runs ``sg_verify_pass``: the tree structure is read
  from the decoder's dense mask, the K/V rows of the tree are written at each
  request's arena tail, and the output carries ``last_hidden_state`` (final
  norm applied) and the drafter's ``hidden_states[l + 1]``;
* ``append_packed_sequence`` of the arena keeps the accepted rows in place;
* ``tree_block_verify_terminal_mass`` (the decoder's default verifier,
  sampling.py:542-735) -> the terminal-mass kernel, same name and arguments;
* the lazy-projection verifiers (``tree_verify_ancestral_lazy_projection_*``,
  fused_tree_sampling.py:2758-3031), which receive hidden states and the
  LM-head module, become one fused LM-head + sampling launch over the
  request's rows followed by the on-device tree walk.  The draw has the law
  of the reference's ancestral sampling; its randomness is Philox keyed by a
  64-bit key drawn from the request's own generator (one draw per call).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from . import ops
from .arena import ArenaRequest, PersistentKVArena
from .engine import B200Engine, Wave, Weights
from .sampling import PackedTrees, _topology, decode_output, follow_packed, tree_block_verify_terminal_mass_fused

# Reference attribute name -> this module's replacement (see ``install``).
VERIFIER_SEAMS = ("tree_verify_ancestral_lazy_projection_fused_scan",
                  "tree_verify_ancestral_lazy_projection_fused_scan_batched",
                  "tree_verify_ancestral_lazy_projection_sparse_exit_batched",
                  "tree_block_verify_terminal_mass")


# --------------------------------------------------------------------------
# The decoder's default verifier (sampling.py:542-735)
# --------------------------------------------------------------------------
def tree_block_verify_terminal_mass(parents, tokens, all_p, generator=None, validate: bool = True, *,
                                    prefix_mode: str = "batched", exit_mode: str = "internal"):
    """``tree_block_verify_terminal_mass`` as the decoder calls it
    (continuous_tree_block_decode.py:2097-2106) on ``sg_tree_verify_terminal_mass``.
    The reference's ablation modes all draw the same law; the kernel computes
    its masses one way (exact row sums, fp64 prefix products), so the modes
    are checked and otherwise ignored.  Rows are read as fp32."""
    if prefix_mode not in {"batched", "serial"} or exit_mode not in {"internal", "dense", "complement", "joint"}:
        raise ValueError("Unknown terminal-mass ablation mode")
    return tree_block_verify_terminal_mass_fused(parents, tokens, all_p, generator, validate)


# --------------------------------------------------------------------------
# KV arena pool and packing
# --------------------------------------------------------------------------
def arena_pool(caches: Sequence, capacity: int) -> PersistentKVArena:
    """``_PersistentRequestCachePool(caches, capacity=...)`` (decode.py:176-213)."""
    return PersistentKVArena.from_caches(caches, capacity)


@dataclass
class PackedArenaWave:
    """What ``pack_cache_sequence`` returns in place of a gathered DynamicCache:
    the requests' arena slots and prefix lengths, in wave order."""
    pool: PersistentKVArena
    slots: tuple
    lengths: tuple
    offsets: tuple
    total: int
    trees: list | None = None        # filled by target_hidden_forward

    def get_seq_length(self) -> int:
        return self.total


def pack_cache_sequence(caches: Sequence, cache_factory=None, device=None):
    """``_pack_cache_sequence`` (decode.py:313-361) without copying: returns
    (packed, lengths, offsets, total) with the reference's meaning."""
    if not caches:
        raise ValueError("At least one cache is required")
    if not all(isinstance(c, ArenaRequest) for c in caches) or len({id(c.pool) for c in caches}) != 1:
        raise ValueError("B200 packing needs request caches of one persistent arena")
    lengths = tuple(int(c.get_seq_length()) for c in caches)
    offsets, total = [], 0
    for length in lengths:
        offsets.append(total)
        total += length
    packed = PackedArenaWave(caches[0].pool, tuple(c.slot for c in caches), lengths, tuple(offsets), total)
    return packed, lengths, tuple(offsets), total


# --------------------------------------------------------------------------
# Engine wrapper
# --------------------------------------------------------------------------
@dataclass
class TargetOutput:
    """The fields of HF's model output that the decoder reads."""
    last_hidden_state: torch.Tensor          # [1, Q, H] bf16, final norm applied
    hidden_states: tuple                     # index l + 1: [1, Q, H] bf16 for the drafter's layers


def trees_from_mask(ids: torch.Tensor, mask: torch.Tensor, packed: PackedArenaWave,
                    query_rows: Sequence[int]) -> list:
    """Per request (parents, tokens) of the wave from the decoder's dense mask
    (``_packed_block_inputs``, decode.py:500-546): in its query block a row
    sees its ancestors and itself, and its parent is the deepest ancestor,
    i.e. the visible row with the largest index below its own."""
    P = packed.total
    vis = mask[0, 0, :, P:] == 0                                 # [Q, Q] query-to-query visibility
    Q = vis.shape[0]
    idx = torch.arange(Q, device=vis.device)
    strict = vis & (idx[None, :] < idx[:, None])
    parent = torch.where(strict.any(-1), (strict * (idx[None, :] + 1)).amax(-1) - 1, torch.full_like(idx, -1))
    parent_h = parent.cpu().tolist()
    tokens_h = ids[0].cpu().tolist()
    trees, q0 = [], 0
    for n in query_rows:
        par = [-1] + [p - q0 for p in parent_h[q0 + 1:q0 + n]]
        trees.append((par, tokens_h[q0:q0 + n]))
        q0 += n
    return trees


class B200VerifyEngine:
    """The reference engine with its packed target pass on the B200 kernels.

    Attribute reads fall through to ``base``; ``target_hidden_forward`` on a
    ``PackedArenaWave`` runs ``sg_verify_pass`` over the wave (no sampling
    decision is committed: the decoder's verifier decides, and the arena's
    ``append_packed_sequence`` keeps the accepted rows)."""

    def __init__(self, base, max_rows: int = 2048, max_requests: int | None = None, weights: Weights | None = None):
        self._base = base
        self._weights = weights if weights is not None else Weights.from_hf(base.target, device=base.device)
        self._max_rows = max_rows
        self._max_requests = max_requests
        self._engines = {}

    def __getattr__(self, name):
        return getattr(self._base, name)

    def _engine_for(self, pool: PersistentKVArena) -> B200Engine:
        key = id(pool)
        if key not in self._engines:
            self._engines[key] = B200Engine(self._weights, num_slots=pool.num_slots, capacity=pool.capacity,
                                            max_rows=self._max_rows, max_requests=self._max_requests or pool.num_slots,
                                            arena=pool)
        return self._engines[key]

    def _feature_layers(self) -> list:
        draft = getattr(self._base, "draft", None)
        return [int(l) for l in getattr(draft, "target_layer_ids", [])]

    def target_hidden_forward(self, ids, cache, *, positions=None, mask=None):
        if not isinstance(cache, PackedArenaWave):
            return self._base.target_hidden_forward(ids, cache, positions=positions, mask=mask)
        if positions is None or mask is None:
            raise ValueError("a packed arena wave needs the decoder's positions and tree mask")
        pool = cache.pool
        engine = self._engine_for(pool)
        # rows per request: query rows of request i see its own prefix
        P = cache.total
        first_rows = (mask[0, 0, :, :P] == 0).float().argmax(-1)        # any visible prefix column
        owner = torch.bucketize(first_rows, torch.tensor(cache.offsets[1:], device=mask.device), right=True)
        counts = torch.bincount(owner, minlength=len(cache.slots)).cpu().tolist()
        trees = trees_from_mask(ids, mask, cache, counts)
        cache.trees = trees
        pos = positions[0].cpu().tolist()
        starts = [0]
        for n in counts:
            starts.append(starts[-1] + n)
        wave = Wave(trees, list(cache.slots), list(cache.lengths), position_base=[pos[s] for s in starts[:-1]])
        L = self._weights.shape.num_layers
        layers = sorted(set(self._feature_layers()) | {L - 1})
        H = self._weights.shape.hidden
        feats = torch.empty((wave.num_rows, len(layers) * H), dtype=torch.bfloat16, device=ids.device)
        engine.verify_device(wave.to(ids.device), seed=0, commit=False, feature_layers=layers, features_out=feats)
        views = {l: feats[:, i * H:(i + 1) * H].unsqueeze(0) for i, l in enumerate(layers)}
        hidden_states = tuple(views.get(l - 1) if l >= 1 else None for l in range(L + 1))
        return TargetOutput(last_hidden_state=views[L - 1], hidden_states=hidden_states)


# --------------------------------------------------------------------------
# Lazy-projection verifiers (hidden states + LM head -> fused sampling)
# --------------------------------------------------------------------------
def _request_key(generator, device) -> torch.Tensor:
    """One 64-bit Philox key per call, drawn from the request's generator."""
    return torch.randint(-(2 ** 63), 2 ** 63 - 1, (1,), dtype=torch.long, device=device, generator=generator)


def _lm_weight(lm_head) -> torch.Tensor:
    w = lm_head.weight if hasattr(lm_head, "weight") else lm_head
    if w.dtype != torch.bfloat16:
        w = w.to(torch.bfloat16)
    return w.contiguous()


def _fused_verify(parents_batch, tokens_batch, hidden_rows, lm_head, temperature, generators):
    topo = [_topology(p, t) for p, t in zip(parents_batch, tokens_batch)]
    sizes = [len(p) for p, _, _ in topo]
    device = hidden_rows.device
    keys = torch.cat([_request_key(g, device) for g in generators])
    row_request = torch.repeat_interleave(keys, torch.tensor(sizes, device=device))
    row_node = torch.cat([torch.arange(n, dtype=torch.int32, device=device) for n in sizes])
    xn = hidden_rows.to(torch.bfloat16).contiguous()
    w = _lm_weight(lm_head)
    if w.shape[1] != xn.shape[1]:
        raise ValueError("Lazy-projection Target hidden states mismatch")
    _, posterior = ops.load().lm_head_sample_normed(xn, w, row_node, row_request, 0, float(temperature))
    trees = PackedTrees([p for p, _, _ in topo], [t for _, t, _ in topo], device, vocab=w.shape[0])
    depth = max(d for _, _, d in topo)
    host = follow_packed(posterior, trees, max_depth=depth).cpu().tolist()
    results = []
    for (par, tok, _), row in zip(topo, host):
        nodes, out_tokens, bonus = decode_output(row, depth, w.shape[0], tok, "B200 fused verifier")
        n = len(par)
        results.append((nodes, out_tokens, bonus, {
            "projected_rows": n, "lm_head_rows": n, "total_tree_rows": n, "probability_rows": 0,
            "fused_lm_head_sampling_rows": n}))
    return results


def _check_temperature(temperature):
    if not isinstance(temperature, (int, float)) or not temperature >= 0 or temperature == float("inf"):
        raise ValueError("temperature must be finite and >= 0")


def tree_verify_ancestral_lazy_projection_fused_scan(parents, tokens, final_hidden, lm_head, temperature: float,
                                                     probability_dtype=torch.float64, generator=None,
                                                     validate: bool = True):
    """fused_tree_sampling.py:2758-2837 on B200: (nodes, tokens, bonus, stats)."""
    _check_temperature(temperature)
    if final_hidden.ndim != 2 or final_hidden.shape[0] != len(parents) or not final_hidden.is_floating_point():
        raise ValueError("Lazy-projection Target hidden states mismatch")
    return _fused_verify([parents], [tokens], final_hidden, lm_head, temperature, [generator])[0]


def tree_verify_ancestral_lazy_projection_fused_scan_batched(parents_batch, tokens_batch, final_hidden, lm_head,
                                                             temperature: float, probability_dtype=torch.float64,
                                                             generators=None, validate: bool = True, *,
                                                             sparse_exit: bool = False):
    """fused_tree_sampling.py:2840-3019 on B200: one fused launch for the batch
    ([B, n, H] hidden states of equally shaped trees, or a list of [n_i, H])."""
    _check_temperature(temperature)
    count = len(parents_batch)
    if count < 1 or len(tokens_batch) != count or generators is None or len(generators) != count:
        raise ValueError("Batched lazy-projection inputs are inconsistent")
    rows = list(final_hidden.unbind(0)) if isinstance(final_hidden, torch.Tensor) else list(final_hidden)
    if len(rows) != count or any(r.ndim != 2 or r.shape[0] != len(p) for r, p in zip(rows, parents_batch)):
        raise ValueError("Batched lazy-projection hidden states mismatch")
    return _fused_verify(parents_batch, tokens_batch, torch.cat(rows, 0), lm_head, temperature, generators)


def tree_verify_ancestral_lazy_projection_sparse_exit_batched(parents_batch, tokens_batch, final_hidden, lm_head,
                                                              temperature: float, probability_dtype=torch.float64,
                                                              generators=None, validate: bool = True):
    """fused_tree_sampling.py:3022-3031 on B200 (same fused draw: the law of
    the sparse-exit walk is the same ancestral law)."""
    return tree_verify_ancestral_lazy_projection_fused_scan_batched(
        parents_batch, tokens_batch, final_hidden, lm_head, temperature, probability_dtype, generators, validate)


# --------------------------------------------------------------------------
# Installation into the reference decoder module
# --------------------------------------------------------------------------
class installed:
    """Context manager: swap the decoder module's seams for the B200 ones
    (and put the originals back on exit).  ``decoder`` is the imported
    ``continuous_tree_block_decode`` module."""

    def __init__(self, decoder):
        self.decoder = decoder
        self.saved = {}

    def __enter__(self):
        replacements = {"_PersistentRequestCachePool": arena_pool, "_pack_cache_sequence": pack_cache_sequence}
        replacements.update({name: globals()[name] for name in VERIFIER_SEAMS})
        for name, fn in replacements.items():
            if not hasattr(self.decoder, name):
                raise AttributeError(f"decoder module has no seam {name}")
            self.saved[name] = getattr(self.decoder, name)
            setattr(self.decoder, name, fn)
        return self

    def __exit__(self, *exc):
        for name, fn in self.saved.items():
            setattr(self.decoder, name, fn)
        self.saved.clear()


def install(decoder):
    """``with install(decoder_module): generate_continuous_tree_blocks(B200VerifyEngine(engine), ...,
    verifier="batched_lazy_projection_fused_scan", layout="packed_sequence", persistent_request_target_cache=True)``"""
    return installed(decoder)
