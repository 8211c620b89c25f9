"""B200 target engine: weights, KV arena and the packed verify pass.

``B200Engine.verify`` runs ONE ``sg_verify_pass`` over a wave of request
trees: the stage the reference runs as pack -> ``engine.target_hidden_forward``
-> lm_head -> ``probabilities`` -> per-request verifier -> ``append_packed_sequence``
(continuous_tree_block_decode.py:1748-2129).  Inputs follow the reference's
``_packed_block_inputs`` contract (:500-546): per request a local tree
(parents, tokens, depths) whose root row carries the last committed token,
positions = round_prefix_len + depth, and attention restricted to the
request's own cache prefix plus the row's tree ancestors.

Weights are either random-initialised with the Qwen3 architecture shapes
(synthetic benchmark models; no checkpoints exist here) or packed from an HF
``Qwen3ForCausalLM`` (parity tests).
"""
from __future__ import annotations

import ctypes
from contextlib import nullcontext
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from . import _lib, ops
from ._lib import check, ptr, stream_ptr
from .arena import PersistentKVArena
from .sampling import _topology

LAYER_WEIGHTS = 8


@dataclass(frozen=True)
class ModelShape:
    num_layers: int
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6

    @property
    def kv_bytes_per_token(self) -> int:
        return self.num_layers * 2 * self.num_kv_heads * self.head_dim * 2

    def gemm_flops_per_row(self) -> int:
        H, D = self.hidden, self.head_dim
        per_layer = H * (self.num_q_heads + 2 * self.num_kv_heads) * D + self.num_q_heads * D * H \
            + 3 * H * self.intermediate
        return 2 * (self.num_layers * per_layer + H * self.vocab)

    def attention_flops(self, context: int) -> int:
        """QK^T and PV flops of one query row attending to `context` keys."""
        return 4 * self.num_q_heads * self.head_dim * self.num_layers * context


# Configurations of the benchmark (random-init, bf16).
CONFIG1_TINY = ModelShape(2, 256, 4, 2, 64, 768, 4096)
QWEN3_4B = ModelShape(36, 2560, 32, 8, 128, 9728, 151936)
QWEN3_8B = ModelShape(36, 4096, 32, 8, 128, 12288, 151936)


class _ModelDesc(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("num_q_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("rms_eps", ctypes.c_float), ("embed", ctypes.c_void_p),
                ("final_norm", ctypes.c_void_p), ("lm_head", ctypes.c_void_p), ("inv_freq", ctypes.c_void_p),
                ("layers", ctypes.POINTER(ctypes.c_void_p))]


class _ArenaDesc(ctypes.Structure):
    _fields_ = [("storage", ctypes.c_void_p), ("num_slots", ctypes.c_int64), ("capacity", ctypes.c_int64)]


class _WaveDesc(ctypes.Structure):
    _fields_ = [("num_requests", ctypes.c_int32), ("num_rows", ctypes.c_int32),
                ("max_rows_per_request", ctypes.c_int32), ("max_depth", ctypes.c_int32),
                ("row_offsets", ctypes.c_void_p), ("parents", ctypes.c_void_p), ("tokens", ctypes.c_void_p),
                ("slots", ctypes.c_void_p), ("cache_lengths", ctypes.c_void_p), ("position_base", ctypes.c_void_p),
                ("request_ids", ctypes.c_void_p), ("seed", ctypes.c_uint64), ("temperature", ctypes.c_float),
                ("commit", ctypes.c_int32), ("accept_out", ctypes.c_void_p), ("lengths_out", ctypes.c_void_p),
                ("posterior", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("child_logprob", ctypes.c_void_p),
                ("hidden_out", ctypes.c_void_p), ("status", ctypes.c_void_p),
                ("trace_events", ctypes.POINTER(ctypes.c_void_p)),
                ("num_feature_layers", ctypes.c_int32), ("feature_layers", ctypes.POINTER(ctypes.c_int32)),
                ("features_out", ctypes.c_void_p), ("features_kept", ctypes.c_void_p),
                ("features_kept_offsets", ctypes.c_void_p)]

TRACE_EVENTS = 16
TRACE_STAGES = ["meta+embed", "L0 in-norm", "L0 qkv gemm", "L0 qk-norm+rope+kv", "L0 attention", "L0 o gemm",
                "L0 post-norm", "L0 gate/up gemm", "L0 down gemm", "layers 1..", "final norm", "lm head+sample",
                "combine", "tree walk", "commit"]


def _bind_engine_symbols(lib):
    if getattr(lib, "_sg_engine_bound", False):
        return lib
    lib.sg_engine_create.restype = ctypes.c_int
    lib.sg_engine_create.argtypes = [ctypes.POINTER(_ModelDesc), ctypes.POINTER(_ArenaDesc), ctypes.c_int32,
                                     ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p)]
    lib.sg_engine_destroy.restype = ctypes.c_int
    lib.sg_engine_destroy.argtypes = [ctypes.c_void_p]
    lib.sg_engine_workspace_bytes.restype = ctypes.c_size_t
    lib.sg_engine_workspace_bytes.argtypes = [ctypes.c_void_p]
    lib.sg_verify_pass.restype = ctypes.c_int
    lib.sg_verify_pass.argtypes = [ctypes.c_void_p, ctypes.POINTER(_WaveDesc), ctypes.c_void_p]
    lib._sg_engine_bound = True
    return lib


def rope_inv_freq(shape: ModelShape) -> torch.Tensor:
    """HF default rotary inverse frequencies (computed in fp32 exactly as
    transformers' _compute_default_rope_parameters does)."""
    D = shape.head_dim
    return 1.0 / (shape.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    I, H = gate.shape
    if I % 128:
        raise ValueError("intermediate size must be a multiple of 128")
    return torch.stack([gate.reshape(I // 128, 128, H), up.reshape(I // 128, 128, H)], dim=1).reshape(2 * I, H)


class Weights:
    """Device-resident bf16 weights in the engine's packed layout."""

    def __init__(self, shape: ModelShape, device="cuda"):
        self.shape = shape
        self.device = torch.device(device)
        self.embed = None
        self.final_norm = None
        self.lm_head = None
        self.layers: list[list[torch.Tensor]] = []
        self.inv_freq = rope_inv_freq(shape).to(self.device)

    @classmethod
    def random(cls, shape: ModelShape, seed: int = 0, std: float = 0.02, device="cuda") -> "Weights":
        """Random init with HF Qwen3 conventions (normal(0, initializer_range)
        linear/embedding weights, unit RMSNorm weights)."""
        w = cls(shape, device)
        g = torch.Generator(device=device).manual_seed(seed)
        H, D, I = shape.hidden, shape.head_dim, shape.intermediate
        nq, nkv = shape.num_q_heads, shape.num_kv_heads

        def normal(*size):
            t = torch.empty(size, dtype=torch.bfloat16, device=device)
            t.normal_(0.0, std, generator=g)
            return t

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=device)
        w.embed = normal(shape.vocab, H)
        w.lm_head = normal(shape.vocab, H)
        w.final_norm = ones(H)
        for _ in range(shape.num_layers):
            w.layers.append([ones(H), normal((nq + 2 * nkv) * D, H), ones(D), ones(D), normal(H, nq * D), ones(H),
                             normal(2 * I, H), normal(H, I)])
        return w

    @classmethod
    def from_hf(cls, model, device="cuda") -> "Weights":
        """Pack an HF Qwen3ForCausalLM (any dtype) into bf16 engine weights."""
        cfg = model.config
        shape = ModelShape(cfg.num_hidden_layers, cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads,
                           cfg.head_dim, cfg.intermediate_size, cfg.vocab_size,
                           float(getattr(cfg, "rope_theta", None) or cfg.rope_parameters["rope_theta"]),
                           float(cfg.rms_norm_eps))
        w = cls(shape, device)
        bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()
        w.embed = bf(model.model.embed_tokens.weight)
        w.lm_head = bf(model.get_output_embeddings().weight)
        w.final_norm = bf(model.model.norm.weight)
        for layer in model.model.layers:
            at, mlp = layer.self_attn, layer.mlp
            qkv = torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight], dim=0)
            w.layers.append([bf(layer.input_layernorm.weight), bf(qkv), bf(at.q_norm.weight), bf(at.k_norm.weight),
                             bf(at.o_proj.weight), bf(layer.post_attention_layernorm.weight),
                             bf(interleave_gate_up(mlp.gate_proj.weight, mlp.up_proj.weight)),
                             bf(mlp.down_proj.weight)])
        return w

    def nbytes(self) -> int:
        total = self.embed.nbytes + self.lm_head.nbytes + self.final_norm.nbytes
        return total + sum(t.nbytes for layer in self.layers for t in layer)


class Wave:
    """Host description of one wave, staged to the device with ONE copy.

    ``trees``: per request ``(parents, tokens)`` where ``parents[0] == -1``
    and ``tokens`` has one entry per row: the root row's entry is the input
    token at the root (the last committed token), the others the tree tokens
    (``[root_token] + block.tokens`` of the reference, :527-529).
    """

    FIELDS = 6  # row_offsets, parents, tokens, slots, cache_lengths, position_base (+ request ids)

    def __init__(self, trees: Sequence[tuple[Sequence[int], Sequence[int]]], slots: Sequence[int],
                 cache_lengths: Sequence[int], position_base: Sequence[int] | None = None,
                 request_ids: Sequence[int] | None = None):
        R = len(trees)
        offsets = [0]
        parents, tokens = [], []
        max_rows, max_depth = 1, 0
        for par, tok in trees:
            if len(par) != len(tok) or len(par) < 1:
                raise ValueError("each tree needs one token per row (the root row's input token first)")
            _, _, depth = _topology(par, list(tok)[1:])
            max_rows = max(max_rows, len(par))
            max_depth = max(max_depth, depth)
            parents += list(par)
            tokens += list(tok)
            offsets.append(len(parents))
        self.num_requests = R
        self.num_rows = offsets[-1]
        self.max_rows_per_request = max_rows
        self.max_depth = max_depth
        self.row_offsets = offsets
        pos = list(cache_lengths) if position_base is None else list(position_base)
        rid = list(range(R)) if request_ids is None else list(request_ids)
        self.host = torch.tensor(offsets + parents + tokens + list(slots) + list(cache_lengths) + pos + rid,
                                 dtype=torch.long)
        self.cache_lengths = list(cache_lengths)
        self.slots = list(slots)

    def to(self, device) -> "DeviceWave":
        return DeviceWave(self, device)


class DeviceWave:
    def __init__(self, wave: Wave, device):
        self.wave = wave
        host = wave.host.pin_memory() if torch.device(device).type == "cuda" else wave.host
        self.buf = host.to(device, non_blocking=True)
        R, Q = wave.num_requests, wave.num_rows
        o = 0
        self.row_offsets = self.buf[o:o + R + 1]; o += R + 1
        self.parents = self.buf[o:o + Q]; o += Q
        self.tokens = self.buf[o:o + Q]; o += Q
        self.slots = self.buf[o:o + R]; o += R
        self.cache_lengths = self.buf[o:o + R]; o += R
        self.position_base = self.buf[o:o + R]; o += R
        self.request_ids = self.buf[o:o + R]; o += R


class B200Engine:
    """Weights + persistent KV arena + the C engine handle."""

    def __init__(self, weights: Weights, num_slots: int, capacity: int, max_rows: int, max_requests: int | None = None,
                 arena: PersistentKVArena | None = None):
        self.weights = weights
        self.shape = s = weights.shape
        self.device = weights.device
        self.lib = _bind_engine_symbols(_lib.load())
        self.arena = arena or PersistentKVArena(s.num_layers, s.num_kv_heads, s.head_dim, num_slots, capacity,
                                                dtype=torch.bfloat16, device=self.device)
        self.max_rows = max_rows
        self.max_requests = max_requests or num_slots
        ptrs = [t.data_ptr() for layer in weights.layers for t in layer]
        self._layer_array = (ctypes.c_void_p * len(ptrs))(*ptrs)
        self._model = _ModelDesc(s.num_layers, s.hidden, s.num_q_heads, s.num_kv_heads, s.head_dim, s.intermediate,
                                 s.vocab, s.rms_eps, weights.embed.data_ptr(), weights.final_norm.data_ptr(),
                                 weights.lm_head.data_ptr(), weights.inv_freq.data_ptr(),
                                 ctypes.cast(self._layer_array, ctypes.POINTER(ctypes.c_void_p)))
        self._arena_desc = _ArenaDesc(self.arena.storage.data_ptr(), self.arena.num_slots, self.arena.capacity)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(self.lib.sg_engine_create(ctypes.byref(self._model), ctypes.byref(self._arena_desc), max_rows,
                                            self.max_requests, ctypes.byref(handle)), "sg_engine_create")
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

    @property
    def workspace_bytes(self) -> int:
        return int(self.lib.sg_engine_workspace_bytes(self.handle))

    def verify_device(self, dw: DeviceWave, *, seed: int, temperature: float = 1.0, commit: bool = True,
                      accept_out: torch.Tensor | None = None, lengths_out: torch.Tensor | None = None,
                      posterior: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                      child_logprob: torch.Tensor | None = None, hidden_out: torch.Tensor | None = None,
                      feature_layers: Sequence[int] = (), features_out: torch.Tensor | None = None,
                      features_kept: torch.Tensor | None = None, features_kept_offsets: torch.Tensor | None = None,
                      max_depth: int | None = None, stream=None, trace=None) -> torch.Tensor:
        """Enqueue one verify pass (no host synchronisation).

        ``feature_layers`` / ``features_out`` (bf16 [rows, len(layers) * hidden])
        export HF's ``hidden_states[l + 1]`` of those layers for every packed
        row; ``features_kept`` / ``features_kept_offsets`` also gather each
        request's rows [0] + accepted nodes (the drafter's next input)."""
        w = dw.wave
        for s, L, (r0, r1) in zip(w.slots, w.cache_lengths, zip(w.row_offsets, w.row_offsets[1:])):
            if not 0 <= s < self.arena.num_slots:
                raise ValueError("arena slot out of range")
            if L < 0 or L + (r1 - r0) > self.arena.capacity:
                raise RuntimeError("Persistent request KV capacity exhausted")
        if w.num_rows > self.max_rows or w.num_requests > self.max_requests:
            raise ValueError("wave exceeds the engine's max_rows / max_requests")
        D = w.max_depth if max_depth is None else max_depth
        if accept_out is None:
            accept_out = torch.empty((w.num_requests, D + 2), dtype=torch.long, device=self.device)
        if commit and lengths_out is None:
            lengths_out = torch.empty(w.num_requests, dtype=torch.long, device=self.device)
        if feature_layers:
            H = self.shape.hidden
            if (features_out is None or features_out.dtype != torch.bfloat16 or not features_out.is_contiguous()
                    or features_out.shape[0] < w.num_rows or features_out.shape[-1] != len(feature_layers) * H):
                raise ValueError("features_out must be contiguous bf16 [rows, len(feature_layers) * hidden]")
            if features_kept is not None and (features_kept_offsets is None
                                              or features_kept_offsets.numel() < w.num_requests + 1):
                raise ValueError("features_kept needs features_kept_offsets [requests + 1]")
        if trace is None:
            with torch.cuda.stream(stream) if stream is not None else nullcontext():
                ops.load().verify_pass(self.handle.value, dw.buf, w.num_requests, w.num_rows,
                                       w.max_rows_per_request, D, ops.seed_arg(seed), float(temperature),
                                       bool(commit), accept_out, lengths_out, posterior, lse, child_logprob,
                                       hidden_out, self.status, [int(l) for l in feature_layers],
                                       features_out if feature_layers else None,
                                       features_kept if feature_layers else None,
                                       features_kept_offsets if feature_layers else None)
        else:
            # profiling: the C descriptor also takes the stage-boundary events
            desc = _WaveDesc(w.num_requests, w.num_rows, w.max_rows_per_request, D, ptr(dw.row_offsets),
                             ptr(dw.parents), ptr(dw.tokens), ptr(dw.slots), ptr(dw.cache_lengths),
                             ptr(dw.position_base), ptr(dw.request_ids), seed & ((1 << 64) - 1), float(temperature),
                             int(bool(commit)), ptr(accept_out), ptr(lengths_out), ptr(posterior), ptr(lse),
                             ptr(child_logprob), ptr(hidden_out), ptr(self.status), None)
            layers = (ctypes.c_int32 * max(1, len(feature_layers)))(*[int(l) for l in feature_layers])
            if feature_layers:
                desc.num_feature_layers = len(feature_layers)
                desc.feature_layers = ctypes.cast(layers, ctypes.POINTER(ctypes.c_int32))
                desc.features_out = ptr(features_out)
                desc.features_kept = ptr(features_kept)
                desc.features_kept_offsets = ptr(features_kept_offsets)
            arr = (ctypes.c_void_p * TRACE_EVENTS)(*[e.cuda_event for e in trace])
            desc.trace_events = ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))
            check(self.lib.sg_verify_pass(self.handle, ctypes.byref(desc), stream_ptr(stream)), "sg_verify_pass")
        self._last_lengths_out = lengths_out
        return accept_out

    def verify(self, wave: Wave, *, seed: int, temperature: float = 1.0, commit: bool = True, **outputs):
        """Stage the wave, run the pass, read the decisions back.

        Returns ``[(nodes, tokens, bonus)]`` per request in the reference
        verifier's format and updates ``arena.lengths`` when committing."""
        dw = wave.to(self.device)
        out = self.verify_device(dw, seed=seed, temperature=temperature, commit=commit, **outputs)
        host = out.cpu().tolist()
        if int(self.status) != 0:
            st = int(self.status)
            self.status.zero_()
            raise _lib.SpecgroveError(st, "sg_verify_pass (device status)")
        D = wave.max_depth
        R, Q = wave.num_requests, wave.num_rows
        tokens = wave.host[R + 1 + Q: R + 1 + 2 * Q].tolist()
        decoded = []
        for i in range(R):
            count, bonus = host[i][D], host[i][D + 1]
            nodes = host[i][:count]
            r0 = wave.row_offsets[i]
            decoded.append((nodes, [tokens[r0 + n] for n in nodes], bonus))
            if commit:
                self.arena.lengths[wave.slots[i]] = wave.cache_lengths[i] + len(nodes) + 1
        return decoded

    def prefill(self, prompts: Sequence[Sequence[int]], slots: Sequence[int], chunk: int = 256):
        """Write each prompt's KV into its slot by running chain-shaped waves
        (a chain's ancestor mask is the causal mask), without committing any
        sampled decision.  A request contributes at most one chunk per wave
        and a wave holds at most ``max_rows`` rows."""
        chunk = min(chunk, 256, self.max_rows)
        pos = {s: self.arena.lengths[s] for s in slots}
        remaining = {s: list(p) for s, p in zip(slots, prompts)}
        while any(remaining.values()):
            trees, wslots, lens, rows = [], [], [], 0
            for s in slots:
                rem = remaining[s]
                if not rem or rows + min(chunk, len(rem)) > self.max_rows or len(trees) >= self.max_requests:
                    continue
                part = rem[:chunk]
                del rem[:chunk]
                trees.append(([-1] + list(range(len(part) - 1)), part))
                wslots.append(s)
                lens.append(pos[s])
                rows += len(part)
            wave = Wave(trees, wslots, lens)
            self.verify_device(wave.to(self.device), seed=0, commit=False)
            for s, (_, part) in zip(wslots, trees):
                pos[s] += len(part)
                self.arena.lengths[s] = pos[s]
        torch.cuda.current_stream().synchronize()
        if int(self.status) != 0:
            raise _lib.SpecgroveError(int(self.status), "prefill (device status)")
