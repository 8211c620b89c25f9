"""B200 drafter step: the DFlash block drafter over a persistent draft cache.

The reference proposes each wave's trees with one padded DFlash forward
(``_propose_many`` with ``reuse_request_draft_cache``,
continuous_tree_block_decode.py:889-962, model
third_party/ddtree_official/model/dflash.py:147-200): per request the target
features of the rows committed since the last proposal (the ``draft_update``)
become context K/V in the draft cache, and a block of ``block_size`` rows (the
last generated token, then mask tokens) attends bidirectionally to the whole
draft cache and to itself; the target's LM head turns block rows
1..length into proposal logits.  ``B200Drafter.draft`` runs that as ONE
``sg_draft_pass`` (packed requests, no padding, the draft cache in a KV
arena), and ``B200Drafter.propose`` continues on the device into the wave
plan (``draft_tree.plan_wave``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib
from ._lib import check
from .arena import PersistentKVArena
from .draft_tree import WavePlan, plan_wave
from .engine import ModelShape, Weights, _ArenaDesc, _ModelDesc, interleave_gate_up, rope_inv_freq


@dataclass(frozen=True)
class DraftShape:
    """The drafter's layer stack (Qwen3 decoder layers) and its block."""
    num_layers: int
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int               # the target's vocabulary (shared embedding and LM head)
    num_feature_layers: int  # target layers concatenated per context row
    block_size: int = 16
    mask_token_id: int = 151669
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6

    def layer_shape(self) -> ModelShape:
        return ModelShape(self.num_layers, self.hidden, self.num_q_heads, self.num_kv_heads, self.head_dim,
                          self.intermediate, self.vocab, self.rope_theta, self.rms_eps)


# z-lab/Qwen3-8B-DFlash-b16 (runtime_model.py:50-66 of the reference): 5
# layers of the target's width, features of target layers [1, 9, 17, 25, 33].
QWEN3_8B_DFLASH = DraftShape(5, 4096, 32, 8, 128, 12288, 151936, 5, 16, 151669)
QWEN3_8B_DFLASH_FEATURE_LAYERS = (1, 9, 17, 25, 33)


class _DraftDesc(ctypes.Structure):
    _fields_ = [("fc", ctypes.c_void_p), ("hidden_norm", ctypes.c_void_p), ("num_feature_layers", ctypes.c_int32),
                ("block_size", ctypes.c_int32), ("mask_token_id", ctypes.c_int64),
                ("max_update_rows", ctypes.c_int32)]


class _DraftWave(ctypes.Structure):
    _fields_ = [("num_requests", ctypes.c_int32), ("num_update_rows", ctypes.c_int32), ("slots", ctypes.c_void_p),
                ("cache_lengths", ctypes.c_void_p), ("update_offsets", ctypes.c_void_p),
                ("features", ctypes.c_void_p), ("anchor_tokens", ctypes.c_void_p), ("logits_out", ctypes.c_void_p),
                ("lengths_out", ctypes.c_void_p), ("status", ctypes.c_void_p), ("context_only", ctypes.c_int32)]


def _bind(lib):
    if getattr(lib, "_sg_draft_bound", False):
        return lib
    lib.sg_draft_engine_create.restype = ctypes.c_int
    lib.sg_draft_engine_create.argtypes = [ctypes.POINTER(_ModelDesc), ctypes.POINTER(_DraftDesc),
                                           ctypes.POINTER(_ArenaDesc), ctypes.c_int32,
                                           ctypes.POINTER(ctypes.c_void_p)]
    lib.sg_draft_pass.restype = ctypes.c_int
    lib.sg_draft_pass.argtypes = [ctypes.c_void_p, ctypes.POINTER(_DraftWave), ctypes.c_void_p]
    lib.sg_engine_destroy.restype = ctypes.c_int
    lib.sg_engine_destroy.argtypes = [ctypes.c_void_p]
    lib._sg_draft_bound = True
    return lib


class DraftWeights:
    """The drafter's bf16 weights in the engine's packed layer layout, plus
    fc and hidden_norm; embedding and LM head are the target's."""

    def __init__(self, shape: DraftShape, target: Weights):
        if target.shape.hidden != shape.hidden or target.shape.vocab != shape.vocab:
            raise ValueError("the drafter shares the target's hidden size and vocabulary")
        self.shape = shape
        self.target = target
        self.device = target.device
        self.layers: list[list[torch.Tensor]] = []
        self.fc = None
        self.hidden_norm = None
        self.norm = None
        self.inv_freq = rope_inv_freq(shape.layer_shape()).to(self.device)

    @classmethod
    def random(cls, shape: DraftShape, target: Weights, seed: int = 1, std: float = 0.02) -> "DraftWeights":
        w = cls(shape, target)
        dev = target.device
        g = torch.Generator(device=dev).manual_seed(seed)
        H, D, I = shape.hidden, shape.head_dim, shape.intermediate
        nq, nkv = shape.num_q_heads, shape.num_kv_heads

        def normal(*size):
            t = torch.empty(size, dtype=torch.bfloat16, device=dev)
            t.normal_(0.0, std, generator=g)
            return t

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)
        w.fc = normal(H, shape.num_feature_layers * H)
        w.hidden_norm = ones(H)
        w.norm = ones(H)
        for _ in range(shape.num_layers):
            w.layers.append([ones(H), normal((nq + 2 * nkv) * D, H), ones(D), ones(D), normal(H, nq * D), ones(H),
                             normal(2 * I, H), normal(H, I)])
        return w

    @classmethod
    def from_module(cls, draft, target: Weights, block_size: int, mask_token_id: int) -> "DraftWeights":
        """Pack a DFlash draft module (dflash.py:147-170: ``layers``, ``fc``,
        ``hidden_norm``, ``norm``)."""
        cfg = draft.config
        n_feat = draft.fc.weight.shape[1] // cfg.hidden_size
        theta = getattr(cfg, "rope_theta", None) or cfg.rope_parameters["rope_theta"]
        shape = DraftShape(cfg.num_hidden_layers, cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads,
                           cfg.head_dim, cfg.intermediate_size, target.shape.vocab, n_feat, block_size,
                           mask_token_id, float(theta), float(cfg.rms_norm_eps))
        w = cls(shape, target)
        bf = lambda t: t.detach().to(device=target.device, dtype=torch.bfloat16).contiguous()
        w.fc = bf(draft.fc.weight)
        w.hidden_norm = bf(draft.hidden_norm.weight)
        w.norm = bf(draft.norm.weight)
        for layer in draft.layers:
            at, mlp = layer.self_attn, layer.mlp
            qkv = torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight], dim=0)
            w.layers.append([bf(layer.input_layernorm.weight), bf(qkv), bf(at.q_norm.weight), bf(at.k_norm.weight),
                             bf(at.o_proj.weight), bf(layer.post_attention_layernorm.weight),
                             bf(interleave_gate_up(mlp.gate_proj.weight, mlp.up_proj.weight)),
                             bf(mlp.down_proj.weight)])
        return w


class B200Drafter:
    """Drafter weights + the draft cache (a KV arena of the drafter's layers)
    + the C engine handle."""

    def __init__(self, weights: DraftWeights, num_slots: int, capacity: int, max_requests: int,
                 max_update_rows: int, arena: PersistentKVArena | None = None):
        s = weights.shape
        self.weights = weights
        self.shape = s
        self.device = weights.device
        self.lib = _bind(_lib.load())
        self.arena = arena or PersistentKVArena(s.num_layers, s.num_kv_heads, s.head_dim, num_slots, capacity,
                                                dtype=torch.bfloat16, device=self.device)
        self.max_requests = max_requests
        self.max_update_rows = max_update_rows
        ptrs = [t.data_ptr() for layer in weights.layers for t in layer]
        self._layer_array = (ctypes.c_void_p * len(ptrs))(*ptrs)
        t = weights.target
        self._model = _ModelDesc(s.num_layers, s.hidden, s.num_q_heads, s.num_kv_heads, s.head_dim, s.intermediate,
                                 s.vocab, s.rms_eps, t.embed.data_ptr(), weights.norm.data_ptr(), t.lm_head.data_ptr(),
                                 weights.inv_freq.data_ptr(),
                                 ctypes.cast(self._layer_array, ctypes.POINTER(ctypes.c_void_p)))
        self._draft = _DraftDesc(weights.fc.data_ptr(), weights.hidden_norm.data_ptr(), s.num_feature_layers,
                                 s.block_size, s.mask_token_id, max_update_rows)
        self._arena_desc = _ArenaDesc(self.arena.storage.data_ptr(), self.arena.num_slots, self.arena.capacity)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(self.lib.sg_draft_engine_create(ctypes.byref(self._model), ctypes.byref(self._draft),
                                                  ctypes.byref(self._arena_desc), max_requests, ctypes.byref(handle)),
                  "sg_draft_engine_create")
        self.handle = handle
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.sg_engine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def draft_device(self, slots: torch.Tensor, cache_lengths: torch.Tensor, update_offsets: torch.Tensor,
                     features: torch.Tensor | None, anchor_tokens: torch.Tensor, num_update_rows: int, *,
                     logits_out: torch.Tensor | None = None, lengths_out: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor:
        """Enqueue one drafter step (no host synchronisation): device int64
        slots / cache_lengths / anchor_tokens [R], update_offsets [R + 1],
        bf16 features [U, F * hidden] (U = num_update_rows, the host copy of
        update_offsets[R]).  Returns bf16 logits [R, block_size, vocab]."""
        s = self.shape
        R = int(slots.shape[0])
        if logits_out is None:
            logits_out = torch.empty((R, s.block_size, s.vocab), dtype=torch.bfloat16, device=self.device)
        if features is not None and (features.dtype != torch.bfloat16 or not features.is_contiguous()):
            raise ValueError("features must be contiguous bf16 [U, F * hidden]")
        wave = _DraftWave(R, int(num_update_rows), slots.data_ptr(), cache_lengths.data_ptr(),
                          update_offsets.data_ptr(), None if features is None else features.data_ptr(),
                          anchor_tokens.data_ptr(), logits_out.data_ptr(),
                          None if lengths_out is None else lengths_out.data_ptr(), self.status.data_ptr(), 0)
        check(self.lib.sg_draft_pass(self.handle, ctypes.byref(wave), _lib.stream_ptr(stream)), "sg_draft_pass")
        return logits_out

    def append_context(self, slots: torch.Tensor, cache_lengths: torch.Tensor, update_offsets: torch.Tensor,
                       features: torch.Tensor, num_update_rows: int, *, lengths_out: torch.Tensor | None = None,
                       stream=None) -> None:
        """Append context rows to the draft caches without running the block
        (the draft cache's prefill, chunk by chunk with the target's)."""
        if num_update_rows == 0:
            return
        if features.dtype != torch.bfloat16 or not features.is_contiguous():
            raise ValueError("features must be contiguous bf16 [U, F * hidden]")
        R = int(slots.shape[0])
        wave = _DraftWave(R, int(num_update_rows), slots.data_ptr(), cache_lengths.data_ptr(),
                          update_offsets.data_ptr(), features.data_ptr(), None, None,
                          None if lengths_out is None else lengths_out.data_ptr(), self.status.data_ptr(), 1)
        check(self.lib.sg_draft_pass(self.handle, ctypes.byref(wave), _lib.stream_ptr(stream)), "sg_draft_pass")

    def draft(self, slots: Sequence[int], features: Sequence[torch.Tensor], anchor_tokens: Sequence[int],
              stream=None) -> torch.Tensor:
        """Host-list convenience: appends each request's feature rows to its
        draft cache (the arena's lengths advance) and returns the logits."""
        dev = self.device
        counts = [int(f.shape[0]) for f in features]
        offsets = [0]
        for c in counts:
            offsets.append(offsets[-1] + c)
        lengths = [self.arena.lengths[int(sl)] for sl in slots]
        meta = torch.tensor(list(slots) + lengths + offsets + list(anchor_tokens), dtype=torch.int64).to(dev)
        R = len(slots)
        feats = torch.cat([f.to(device=dev, dtype=torch.bfloat16) for f in features]).contiguous() \
            if offsets[-1] else None
        lengths_out = torch.empty(R, dtype=torch.int64, device=dev)
        logits = self.draft_device(meta[:R], meta[R:2 * R], meta[2 * R:3 * R + 1], feats, meta[3 * R + 1:],
                                   offsets[-1], lengths_out=lengths_out, stream=stream)
        for sl, c in zip(slots, counts):
            self.arena.lengths[int(sl)] += c
        return logits

    def propose(self, slots: Sequence[int], features: Sequence[torch.Tensor], anchor_tokens: Sequence[int], *,
                temperature: float, tiers: Sequence[int], weights: Sequence[float], row_budget: int,
                length: int | None = None, fixed_row_equivalent: float | None = None,
                row_cost_curve: Sequence[tuple[int, float]] | None = None, stream=None) -> WavePlan:
        """Drafter step, then the wave plan on the device: block rows
        1..length of the logits (the proposal depths, variant.length in the
        reference) -> trees -> tier allocation -> packed wave."""
        logits = self.draft(slots, features, anchor_tokens, stream=stream)
        L = self.shape.block_size - 1 if length is None else int(length)
        anchors = torch.tensor(list(anchor_tokens), dtype=torch.int64, device=self.device)
        w = torch.tensor(list(weights), dtype=torch.float64, device=self.device)
        plan = plan_wave(logits[:, 1:L + 1], temperature, tiers, w, anchors, row_budget=row_budget,
                         fixed_row_equivalent=fixed_row_equivalent, row_cost_curve=row_cost_curve, stream=stream)
        plan.draft_logits = logits
        return plan
