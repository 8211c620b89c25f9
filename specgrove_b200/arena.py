"""Persistent per-request KV arena with on-device accepted-path commit.

Mirrors ``_PersistentRequestCachePool`` / ``_PersistentRequestCache`` /
``_PersistentRequestCacheLayer`` of ``continuous_tree_block_decode.py:126-261``:
same per-layer ``key_storage[l]`` / ``value_storage[l]`` shape
``[H_kv, slots * capacity, D]``, same ``lengths`` list, same request views
(``layers[i].keys/values`` of shape ``[1, H_kv, length, D]``,
``get_seq_length()``), and the same ``append_packed_sequence`` signature and
capacity error.  The difference is the memory layout and the commit: all
layers' K and V live in ONE allocation ``[layers, 2, H_kv, slots*capacity, D]``
(plane = (layer, K|V, kv head)), so a wave's commit is one ``sg_kv_commit``
launch over every plane instead of four launches per layer.
"""
from __future__ import annotations

from contextlib import nullcontext
from typing import Sequence

import torch

from . import ops


class ArenaLayer:
    """Request-local view of one layer (reference :126-150)."""

    def __init__(self, cache: "ArenaRequest", layer_index: int):
        self._cache = cache
        self._layer_index = layer_index

    @property
    def keys(self):
        pool = self._cache.pool
        start = self._cache.slot * pool.capacity
        return pool.key_storage[self._layer_index][:, start:start + pool.lengths[self._cache.slot]].unsqueeze(0)

    @property
    def values(self):
        pool = self._cache.pool
        start = self._cache.slot * pool.capacity
        return pool.value_storage[self._layer_index][:, start:start + pool.lengths[self._cache.slot]].unsqueeze(0)


class ArenaRequest:
    """Cache-compatible request view (reference :153-165)."""

    def __init__(self, pool: "PersistentKVArena", slot: int):
        self.pool = pool
        self.slot = slot
        self.layers = [ArenaLayer(self, i) for i in range(pool.num_layers)]

    def get_seq_length(self):
        return self.pool.lengths[self.slot]


class PersistentKVArena:
    """Slot-strided KV arena: ``storage[layer, kv, head, slot*capacity + t, :]``."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_slots: int,
                 capacity: int, dtype=torch.bfloat16, device="cuda"):
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.num_slots = int(num_slots)
        self.capacity = int(capacity)
        self.storage = torch.empty(
            (self.num_layers, 2, self.num_kv_heads, self.num_slots * self.capacity, self.head_dim),
            dtype=dtype, device=device)
        self.lengths = [0] * self.num_slots
        self.key_storage = [self.storage[l, 0] for l in range(self.num_layers)]
        self.value_storage = [self.storage[l, 1] for l in range(self.num_layers)]
        self.caches = tuple(ArenaRequest(self, s) for s in range(self.num_slots))
        self._status = torch.zeros(1, dtype=torch.int32, device=device)

    @classmethod
    def from_caches(cls, caches: Sequence, capacity: int) -> "PersistentKVArena":
        """Reference constructor semantics (:176-213): copy each request's prefix."""
        if not caches:
            raise ValueError("At least one cache is required")
        lengths = [int(c.get_seq_length()) for c in caches]
        if capacity < max(lengths):
            raise ValueError("Persistent cache capacity is below the prefix")
        layer_count = len(caches[0].layers)
        if any(len(c.layers) != layer_count for c in caches):
            raise ValueError("Target caches have different layer counts")
        example = caches[0].layers[0].keys
        if example.shape[0] != 1:
            raise ValueError("Expected one request per source cache")
        arena = cls(layer_count, example.shape[1], example.shape[-1], len(caches), capacity,
                    dtype=example.dtype, device=example.device)
        for slot, (cache, length) in enumerate(zip(caches, lengths)):
            start = slot * capacity
            for l, layer in enumerate(cache.layers):
                arena.storage[l, 0, :, start:start + length].copy_(layer.keys[0])
                arena.storage[l, 1, :, start:start + length].copy_(layer.values[0])
        arena.lengths = list(lengths)
        return arena

    @property
    def num_planes(self) -> int:
        return self.num_layers * 2 * self.num_kv_heads

    @property
    def plane_rows(self) -> int:
        return self.num_slots * self.capacity

    @property
    def row_bytes(self) -> int:
        return self.head_dim * self.storage.element_size()

    def _commit(self, src_base: torch.Tensor, src_plane_rows: int, src_rows, dst_rows, group_sizes,
                stream=None):
        offsets = [0]
        for g in group_sizes:
            offsets.append(offsets[-1] + g)
        meta = torch.tensor([*src_rows, *dst_rows, *offsets], dtype=torch.long)
        meta = meta.pin_memory().to(self.storage.device, non_blocking=True)
        n = len(src_rows)
        self._status.zero_()
        src = src_base.view(-1, src_plane_rows, self.head_dim)
        with torch.cuda.stream(stream) if stream is not None else nullcontext():
            ops.load().kv_commit(self.storage, src, meta[:n], meta[n:2 * n], meta[2 * n:],
                                 max(group_sizes) if group_sizes else 0, self._status)

    def commit_tail(self, slots: Sequence[int], keep_rows: Sequence[Sequence[int]], stream=None):
        """In-place commit: the wave wrote its tree rows at ``old_length + j``
        of each slot; keep rows ``[0] + accepted`` move to ``old_length + i``."""
        src_rows, dst_rows, groups, increments = [], [], [], []
        for slot, rows in zip(slots, keep_rows):
            old = self.lengths[slot]
            if old + len(rows) > self.capacity:
                raise RuntimeError("Persistent request KV capacity exhausted")
            base = slot * self.capacity + old
            src_rows += [base + int(r) for r in rows]
            dst_rows += [base + i for i in range(len(rows))]
            groups.append(len(rows))
            increments.append((slot, len(rows)))
        self._commit(self.storage, self.plane_rows, src_rows, dst_rows, groups, stream)
        for slot, inc in increments:
            self.lengths[slot] += inc

    def append_packed_sequence(self, packed, caches: Sequence[ArenaRequest], packed_old_length: int,
                               query_offsets: Sequence[int], keep_query_rows: Sequence[Sequence[int]],
                               device=None):
        """Reference :215-261: scatter kept packed query rows into the arena.

        ``packed`` is a DynamicCache-like object whose ``layers[l].keys/values``
        are ``[1, H_kv, packed_old_length + Q, D]``.  One launch per layer and
        tensor moves every kv head (the packed layers are separate tensors).
        """
        if not (len(caches) == len(query_offsets) == len(keep_query_rows) and caches):
            raise ValueError("Persistent cache append metadata disagree")
        if getattr(packed, "pool", None) is self:
            # a wave packed without copying (decoder_seams.pack_cache_sequence):
            # the pass wrote its tree rows at each slot's tail, keep them in place
            if any(cache.pool is not self for cache in caches):
                raise ValueError("Persistent cache belongs to another pool")
            self.commit_tail([cache.slot for cache in caches], keep_query_rows)
            return
        src_rows, dst_rows, groups, increments = [], [], [], []
        for cache, q_off, rows in zip(caches, query_offsets, keep_query_rows):
            if cache.pool is not self:
                raise ValueError("Persistent cache belongs to another pool")
            old = self.lengths[cache.slot]
            if old + len(rows) > self.capacity:
                raise RuntimeError("Persistent request KV capacity exhausted")
            src_rows += [packed_old_length + q_off + int(r) for r in rows]
            dst_rows += [cache.slot * self.capacity + old + i for i in range(len(rows))]
            groups.append(len(rows))
            increments.append((cache.slot, len(rows)))
        offsets = [0]
        for g in groups:
            offsets.append(offsets[-1] + g)
        meta = torch.tensor([*src_rows, *dst_rows, *offsets], dtype=torch.long)
        if self.storage.is_cuda:
            meta = meta.pin_memory()
        meta = meta.to(self.storage.device, non_blocking=True)
        n = len(src_rows)
        commit = ops.load().kv_commit
        for l, layer in enumerate(packed.layers):
            for kv, src in ((0, layer.keys), (1, layer.values)):
                src = src.contiguous()
                if src.dtype != self.storage.dtype or src.shape[-1] != self.head_dim:
                    raise ValueError("Packed cache dtype/head_dim differ from the arena")
                dst = self.storage[l, kv]
                commit(dst, src.view(-1, src.shape[-2], self.head_dim), meta[:n], meta[n:2 * n], meta[2 * n:],
                       max(groups), self._status)
        for slot, inc in increments:
            self.lengths[slot] += inc
