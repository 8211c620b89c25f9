"""The speculative decoding loop on the device: admission, then steps of
drafter -> wave plan -> verify pass -> commit.

Reference flow (serving ``continuous_tree_block_decode.py``): admission and
prefill of arrivals (:1556-1602), one ``_propose_many`` per wave
(:1686-1705, :889-962 with ``reuse_request_draft_cache``), the packed verify,
verifier and commit (:1748-2129), and the feature gather that becomes each
request's next draft update (:2144-2183).  Here:

* ``admit``: the target prefills each prompt in chain-shaped chunks of at
  most 256 rows, as many chunks per wave as its row budget holds (several
  consecutive chunks of one prompt included; ``sg_verify_pass`` without
  commit, exporting the drafter's feature layers for every prompt row) and
  the drafter appends the same rows to its draft cache (``sg_draft_pass`` in
  context-only mode), so both caches end at the prompt length; the last
  prompt row's sampled posterior is the first generated token.
* ``step``: one ``sg_draft_pass`` over every running request (the kept rows'
  features of its previous verify as the update, its last token as the
  block's anchor), ``plan_wave`` on the device (proposals, trees, tier
  knapsack, packed wave), one ``sg_verify_pass`` on the plan's arrays with
  commit and the kept rows' features, then the host reads the decisions
  (accept_out and the row offsets: two small copies per step).

The invariant of the reference (draft cache + pending update = target cache)
holds after every step.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import torch

from .draft_tree import plan_wave
from .drafter import B200Drafter
from .engine import B200Engine, Wave


@dataclass
class SpecRequest:
    request_id: int
    prompt: list[int]
    max_new_tokens: int
    weight: float = 1.0
    slot: int = -1
    generated: list[int] = field(default_factory=list)
    update: tuple[int, int] = (0, 0)   # rows [start, end) of the kept features awaiting the drafter
    done: bool = False


class _PlannedWave:
    """The host fields the verify pass checks, for a wave planned on the device."""

    def __init__(self, slots, cache_lengths, row_offsets, max_rows_per_request, max_depth):
        self.slots = list(slots)
        self.cache_lengths = list(cache_lengths)
        self.row_offsets = list(row_offsets)
        self.num_requests = len(self.slots)
        self.num_rows = self.row_offsets[-1]
        self.max_rows_per_request = max_rows_per_request
        self.max_depth = max_depth


class _PlannedDeviceWave:
    def __init__(self, wave: _PlannedWave, buf: torch.Tensor):
        self.wave = wave
        self.buf = buf


class SpecDecoder:
    def __init__(self, target: B200Engine, drafter: B200Drafter, feature_layers: Sequence[int], *,
                 tiers: Sequence[int], row_budget: int, temperature: float = 1.0,
                 proposal_temperature: float = 1.0, fixed_row_equivalent: float | None = None,
                 row_cost_curve: Sequence[tuple[int, float]] | None = None, chunk: int = 256, seed: int = 0):
        if drafter.shape.num_feature_layers != len(feature_layers):
            raise ValueError("the drafter's feature width does not match the feature layers")
        if target.arena.num_slots > drafter.arena.num_slots:
            raise ValueError("the draft cache needs a slot for every target slot")
        self.target, self.drafter = target, drafter
        self.feature_layers = [int(l) for l in feature_layers]
        self.tiers = sorted(int(t) for t in tiers)
        self.row_budget = int(row_budget)
        self.temperature = float(temperature)
        self.proposal_temperature = float(proposal_temperature)
        self.fixed_row_equivalent = fixed_row_equivalent
        self.row_cost_curve = row_cost_curve
        self.chunk = min(int(chunk), 256)
        self.seed = int(seed)
        self.depth = drafter.shape.block_size - 1
        dev = target.device
        H, F = target.shape.hidden, len(self.feature_layers)
        rows = target.max_rows
        self.features = torch.empty((rows, F * H), dtype=torch.bfloat16, device=dev)
        self.kept = torch.empty((rows, F * H), dtype=torch.bfloat16, device=dev)
        self.kept_offsets = torch.empty(target.max_requests + 1, dtype=torch.long, device=dev)
        self.posterior = torch.empty(rows, dtype=torch.long, device=dev)
        self.logits = torch.empty((drafter.max_requests, drafter.shape.block_size, drafter.shape.vocab),
                                  dtype=torch.bfloat16, device=dev)
        self.free_slots = list(range(target.arena.num_slots))
        self.running: list[SpecRequest] = []
        self.steps = 0
        self.rows_verified = 0

    # -------------------------------------------------------------- admission
    def admit(self, requests: Sequence[SpecRequest]) -> None:
        """Prefill the target and the draft cache of each request (chain
        chunks of at most ``chunk`` rows, waves of at most ``max_rows`` rows
        and the drafter's update rows) and sample its first token."""
        t, d = self.target, self.drafter
        if len(requests) > len(self.free_slots):
            raise RuntimeError(f"{len(requests)} requests but {len(self.free_slots)} free slots")
        for r in requests:
            if not r.prompt or r.max_new_tokens < 1:
                raise ValueError("a request needs a non-empty prompt and max_new_tokens >= 1")
            need = len(r.prompt) + r.max_new_tokens + max(self.tiers[-1] + 1, d.shape.block_size)
            if need > min(t.arena.capacity, d.arena.capacity):
                raise ValueError("prompt + new tokens + one tree do not fit the slot capacity")
        for r in requests:
            r.slot = self.free_slots.pop(0)
            t.arena.lengths[r.slot] = 0
            d.arena.lengths[r.slot] = 0
        remaining = {r.slot: list(r.prompt) for r in requests}
        by_slot = {r.slot: r for r in requests}
        while any(remaining.values()):
            # A wave takes up to max_rows prompt rows.  A long prompt goes in
            # as several consecutive chain chunks of one slot in the same wave:
            # chunk k's rows sit at cache positions after chunk k - 1's, whose
            # K/V the pass writes into the arena (q/k/v epilogue) before any
            # attention reads them, so chunk k sees them as prefix.
            trees, slots, lens, dlens, rows = [], [], [], [], 0
            limit = min(t.max_rows, d.max_update_rows)
            extra = {}
            for r in requests:
                rem = remaining[r.slot]
                while rem and len(trees) < t.max_requests:
                    take = min(self.chunk, len(rem), limit - rows)
                    if take <= 0:
                        break
                    part = rem[:take]
                    del rem[:take]
                    off = extra.get(r.slot, 0)
                    trees.append(([-1] + list(range(len(part) - 1)), part))
                    slots.append(r.slot)
                    lens.append(t.arena.lengths[r.slot] + off)
                    dlens.append(d.arena.lengths[r.slot] + off)
                    extra[r.slot] = off + take
                    rows += take
            wave = Wave(trees, slots, lens, request_ids=[by_slot[s].request_id for s in slots])
            dw = wave.to(t.device)
            Q = wave.num_rows
            t.verify_device(dw, seed=self.seed, temperature=self.temperature, commit=False,
                            posterior=self.posterior, feature_layers=self.feature_layers,
                            features_out=self.features)
            d.append_context(dw.slots, torch.tensor(dlens, dtype=torch.long, device=t.device), dw.row_offsets,
                             self.features[:Q], Q)
            for s, n in extra.items():
                t.arena.lengths[s] += n
                d.arena.lengths[s] += n
            last = {}
            for i, s in enumerate(slots):
                if not remaining[s]:
                    last[s] = wave.row_offsets[i + 1] - 1      # the slot's last chunk in this wave
            if last:
                picks = self.posterior[torch.tensor(list(last.values()), device=t.device)].cpu().tolist()
                for s, tok in zip(last, picks):
                    by_slot[s].generated = [int(tok)]
        self._check_status("admission")
        for r in requests:
            if len(r.generated) >= r.max_new_tokens:   # the first token was the last
                r.done = True
                self.free_slots.append(r.slot)
            else:
                self.running.append(r)

    # ------------------------------------------------------------------ step
    def step(self) -> int:
        """One speculative step over every running request; returns the
        tokens generated (accepted + bonus) across requests."""
        reqs = [r for r in self.running if not r.done]
        if not reqs:
            return 0
        t, d = self.target, self.drafter
        dev = t.device
        R = len(reqs)
        slots = [r.slot for r in reqs]
        # the drafter's update: each request's kept rows of the previous verify
        starts, offs = [], [0]
        for r in reqs:
            a, b = r.update
            starts.append((a, b))
            offs.append(offs[-1] + (b - a))
        U = offs[-1]
        feats = None
        if U:
            idx = torch.tensor([i for a, b in starts for i in range(a, b)], dtype=torch.long).to(dev)
            feats = self.kept.index_select(0, idx)
        dlens = [d.arena.lengths[s] for s in slots]
        meta = torch.tensor(slots + dlens + offs + [r.generated[-1] for r in reqs] +
                            [t.arena.lengths[s] for s in slots] + [r.request_id for r in reqs],
                            dtype=torch.long).to(dev, non_blocking=True)
        slots_t, dlen_t = meta[:R], meta[R:2 * R]
        offs_t, anchors_t = meta[2 * R:3 * R + 1], meta[3 * R + 1:4 * R + 1]
        tlen_t, rid_t = meta[4 * R + 1:5 * R + 1], meta[5 * R + 1:6 * R + 1]
        logits = d.draft_device(slots_t, dlen_t, offs_t, feats, anchors_t, U, logits_out=self.logits[:R])
        for r, (a, b) in zip(reqs, starts):
            d.arena.lengths[r.slot] += b - a
            r.update = (0, 0)
        weights = torch.tensor([r.weight for r in reqs], dtype=torch.float64, device=dev)
        plan = plan_wave(logits[:, 1:self.depth + 1], self.proposal_temperature, self.tiers, weights, anchors_t,
                         row_budget=self.row_budget, fixed_row_equivalent=self.fixed_row_equivalent,
                         row_cost_curve=self.row_cost_curve)
        offsets = plan.row_offsets.cpu().tolist()
        Q = offsets[-1]
        self.rows_verified += Q
        tlens = [t.arena.lengths[s] for s in slots]
        buf = torch.cat([plan.row_offsets, plan.parents[:Q], plan.tokens[:Q], slots_t, tlen_t, tlen_t, rid_t])
        wave = _PlannedWave(slots, tlens, offsets, self.tiers[-1] + 1, self.depth)
        accept = t.verify_device(_PlannedDeviceWave(wave, buf), seed=self.seed + 1 + self.steps,
                                 temperature=self.temperature, commit=True, max_depth=self.depth,
                                 feature_layers=self.feature_layers, features_out=self.features,
                                 features_kept=self.kept, features_kept_offsets=self.kept_offsets)
        host = accept.cpu().tolist()
        kept = self.kept_offsets[:R + 1].cpu().tolist()
        tokens = plan.tokens[:Q].cpu().tolist()
        self._check_status("step")
        produced = 0
        for i, r in enumerate(reqs):
            count, bonus = host[i][self.depth], host[i][self.depth + 1]
            new = [tokens[offsets[i] + n] for n in host[i][:count]] + [int(bonus)]
            room = r.max_new_tokens - len(r.generated)
            r.generated.extend(new[:room])
            produced += min(len(new), room)
            t.arena.lengths[r.slot] = tlens[i] + count + 1
            r.update = (kept[i], kept[i + 1])
            if len(r.generated) >= r.max_new_tokens:
                r.done = True
                self.free_slots.append(r.slot)
        self.running = [r for r in self.running if not r.done]
        self.steps += 1
        return produced

    def _check_status(self, where: str) -> None:
        for eng in (self.target, self.drafter):
            st = int(eng.status.item())
            if st != 0:
                eng.status.zero_()
                raise RuntimeError(f"{where}: device status {st}")
