"""Tree-sampling acceptance through the C ABI, with the reference's verifier API.

The per-request functions keep the names, arguments, return values and error
types of the reference verifiers in
``gbv_experiments/fused_tree_sampling.py`` (``tree_verify_ancestral_fused_scan`` :2172-2202,
``tree_verify_ancestral_sparse_exit_fused_scan`` :2205-2259,
``..._batched`` :2262-2373, ``tree_verify_ancestral_same_draw_fused``
:2376-2414; ``tree_block_verify_terminal_mass_fused`` follows
``sampling.py:542-735``), so the decoder's verifier dispatch
(``continuous_tree_block_decode.py:1965-2107``) can call them unchanged.  They
draw their uniforms from the request's ``torch.Generator`` exactly as the
reference does (``torch.rand(max_depth + 1)`` or ``2 * (max_depth + 1)``
float64 values on the rows' device).

``accept_packed`` is the batched, packed-row entry the B200 engine uses: one
launch for every tree of a wave, uniforms either explicit or drawn on device
from Philox4x32-10 keyed by (seed, request, node).
"""
from __future__ import annotations

from contextlib import nullcontext as _nullcontext

import torch

from . import ops
from ._lib import SG_RULE_SCAN, SG_RULE_SPARSE_EXIT


def _topology(parents, tokens):
    """Check one probability tree and return (parents, edge tokens, depth).

    The rules a tree must satisfy (the reference validates the same ones,
    fused_tree_sampling.py:2089-2102, sampling.py:922-926): node 0 is the root
    (parent -1), every other node's parent is an earlier node, there is one
    edge token per non-root node, and no node has two children with the same
    token.  A violation raises ValueError."""
    parents = [int(p) for p in parents]
    tokens = [int(t) for t in tokens]
    n = len(parents)
    if n == 0 or parents[0] != -1 or len(tokens) != n - 1:
        raise ValueError("Invalid probability-tree topology: need a root with parent -1 and one token per edge")
    depth = [0] * n
    edges = set()
    for node in range(1, n):
        parent = parents[node]
        if not 0 <= parent < node:
            raise ValueError(f"Invalid probability-tree topology: node {node} has parent {parent}, "
                             "which does not precede it")
        edge = (parent, tokens[node - 1])
        if edge in edges:
            raise ValueError(f"Invalid probability-tree topology: node {parent} repeats child token {edge[1]}")
        edges.add(edge)
        depth[node] = depth[parent] + 1
    return parents, tokens, max(depth)


def _check_rows(all_p, node_count, what):
    if (not all_p.is_cuda or all_p.ndim != 2 or all_p.shape[0] != node_count
            or all_p.shape[1] < 1 or not all_p.is_floating_point()):
        raise ValueError(f"{what} probability tensor mismatch")


def _validate_probabilities(all_p, normalised: bool):
    """Every row must be finite and non-negative with positive mass; the
    sparse-exit rule also needs rows that already sum to one (it routes on
    child masses without normalising).  Violations raise FloatingPointError."""
    row_sums = all_p.sum(dim=-1, dtype=torch.float64)
    bad = (~torch.isfinite(all_p)).any() | (all_p < 0).any()
    if normalised:
        bad = bad | ((row_sums - 1.0).abs() > 1e-12 + 1e-10).any()
    else:
        bad = bad | (row_sums <= 0).any()
    if bool(bad):
        kind = "normalised, " if normalised else ""
        raise FloatingPointError(f"Target probabilities must be finite, non-negative, {kind}with positive row mass")


def _as_fp32_rows(all_p: torch.Tensor) -> torch.Tensor:
    if all_p.dtype != torch.float32:
        all_p = all_p.to(torch.float32)
    return all_p.contiguous()


class PackedTrees:
    """Device metadata of a batch of trees packed row after row.

    ``parents``/``tokens`` hold one entry per node (root parent -1, root token
    -1); tree ``t`` owns rows ``row_offsets[t]:row_offsets[t+1]``.
    """

    def __init__(self, parents_batch, tokens_batch, device, vocab: int | None = None):
        offsets = [0]
        flat_parents: list[int] = []
        flat_tokens: list[int] = []
        depth = 0
        max_nodes = 1
        for parents, tokens in zip(parents_batch, tokens_batch):
            parents, tokens, d = _topology(parents, tokens)
            if vocab is not None and any(t < 0 or t >= vocab for t in tokens):
                raise ValueError("Tree token is outside the Target vocabulary")
            depth = max(depth, d)
            max_nodes = max(max_nodes, len(parents))
            flat_parents += parents
            flat_tokens += [-1] + tokens
            offsets.append(len(flat_parents))
        meta = torch.tensor([flat_parents, flat_tokens], dtype=torch.long)
        self.count = len(offsets) - 1
        self.max_depth = depth
        self.max_nodes = max_nodes
        self.total_rows = offsets[-1]
        self.row_offsets_host = offsets
        pinned = torch.cat([torch.tensor(offsets, dtype=torch.long), meta.reshape(-1)])
        if torch.device(device).type == "cuda":
            pinned = pinned.pin_memory()
        dev = pinned.to(device, non_blocking=True)
        n = len(offsets)
        self.row_offsets = dev[:n]
        self.parents = dev[n:n + self.total_rows]
        self.tokens = dev[n + self.total_rows:]


def accept_packed(probs: torch.Tensor, trees: PackedTrees, *, rule: int = SG_RULE_SCAN,
                  uniforms: torch.Tensor | None = None, seed: int = 0,
                  request_ids: torch.Tensor | None = None, max_depth: int | None = None,
                  out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
    """One launch of ``sg_tree_accept_probs`` over packed rows; returns the
    device ``[trees, max_depth + 2]`` int64 output (reference layout)."""
    if probs.dtype != torch.float32 or not probs.is_cuda or probs.ndim != 2:
        raise ValueError("accept_packed expects a CUDA float32 [rows, vocab] tensor")
    probs = probs.contiguous()
    if probs.shape[0] < trees.total_rows:
        raise ValueError("fewer probability rows than packed tree nodes")
    depth = trees.max_depth if max_depth is None else int(max_depth)
    if depth < trees.max_depth:
        raise ValueError("max_depth is below the depth of a packed tree")
    stride = 0
    if uniforms is not None:
        if uniforms.dtype != torch.float64 or uniforms.device != probs.device:
            raise ValueError("uniforms must be float64 on the probabilities' device")
        uniforms = uniforms.reshape(trees.count, -1).contiguous()
        stride = uniforms.shape[1]
    if out is None:
        out = torch.empty((trees.count, depth + 2), dtype=torch.long, device=probs.device)
    with torch.cuda.stream(stream) if stream is not None else _nullcontext():
        ops.load().tree_accept_out(probs, trees.row_offsets, trees.parents, trees.tokens, trees.max_nodes, depth,
                                   rule, uniforms, ops.seed_arg(seed), request_ids, status, out)
    return out


def decode_output(packed_row, max_depth: int, vocab: int, tokens, what: str):
    """(nodes, tokens, bonus) of one row of the kernels' [max_depth + 2]
    layout: slots [0, count) hold the accepted nodes, slot max_depth the
    count, slot max_depth + 1 the bonus token."""
    count, bonus = int(packed_row[max_depth]), int(packed_row[max_depth + 1])
    if count < 0 or count > max_depth or bonus < 0 or bonus >= vocab:
        raise RuntimeError(f"{what}: kernel output out of range (count {count}, bonus {bonus})")
    nodes = [int(v) for v in packed_row[:count]]
    return nodes, [tokens[v - 1] for v in nodes], bonus


def tree_verify_ancestral_fused_scan(parents, tokens, all_p, generator=None, validate: bool = True):
    """Reference fused_tree_sampling.py:2172-2202 on the B200 kernel."""
    parents, tokens, max_depth = _topology(parents, tokens)
    node_count = len(parents)
    _check_rows(all_p, node_count, "Scan-fused DDTree")
    if any(token < 0 or token >= all_p.shape[1] for token in tokens):
        raise ValueError("Tree token is outside the Target vocabulary")
    if validate:
        _validate_probabilities(all_p, normalised=False)
    uniforms = torch.rand(max_depth + 1, dtype=torch.float64, device=all_p.device, generator=generator)
    trees = PackedTrees([parents], [tokens], all_p.device)
    out = accept_packed(_as_fp32_rows(all_p), trees, rule=SG_RULE_SCAN, uniforms=uniforms,
                        max_depth=max_depth)
    return decode_output(out[0].tolist(), max_depth, all_p.shape[1], tokens,
                         "Scan-fused tree sampler")


def tree_verify_ancestral_sparse_exit_fused_scan(parents, tokens, all_p, generator=None,
                                                 validate: bool = True):
    """Reference fused_tree_sampling.py:2205-2259 on the B200 kernel."""
    parents, tokens, max_depth = _topology(parents, tokens)
    node_count = len(parents)
    if not all_p.is_contiguous():
        raise ValueError("Sparse-exit Target probability tensor mismatch")
    _check_rows(all_p, node_count, "Sparse-exit Target")
    if any(token < 0 or token >= all_p.shape[1] for token in tokens):
        raise ValueError("Tree token is outside the Target vocabulary")
    if validate:
        _validate_probabilities(all_p, normalised=True)
    uniforms = torch.rand(2 * (max_depth + 1), dtype=torch.float64, device=all_p.device,
                          generator=generator)
    trees = PackedTrees([parents], [tokens], all_p.device)
    out = accept_packed(_as_fp32_rows(all_p), trees, rule=SG_RULE_SPARSE_EXIT, uniforms=uniforms,
                        max_depth=max_depth)
    return decode_output(out[0].tolist(), max_depth, all_p.shape[1], tokens,
                         "Sparse-exit sampler")


def tree_verify_ancestral_sparse_exit_fused_scan_batched(parents_batch, tokens_batch,
                                                         probability_batch, generators,
                                                         validate: bool = True):
    """Reference fused_tree_sampling.py:2262-2373: ragged or equal-shaped
    batches both run as ONE launch over packed rows with one host transfer."""
    count = len(parents_batch)
    if (count < 1 or len(tokens_batch) != count or len(probability_batch) != count
            or len(generators) != count):
        raise ValueError("Sparse-exit batch inputs have different lengths")
    rows = (list(probability_batch.unbind(0)) if isinstance(probability_batch, torch.Tensor)
            else list(probability_batch))
    topologies = []
    for parents, tokens, all_p in zip(parents_batch, tokens_batch, rows):
        parents, tokens, max_depth = _topology(parents, tokens)
        _check_rows(all_p, len(parents), "Sparse-exit Target")
        if any(token < 0 or token >= all_p.shape[1] for token in tokens):
            raise ValueError("Tree token is outside the Target vocabulary")
        if validate:
            _validate_probabilities(all_p, normalised=True)
        topologies.append((parents, tokens, max_depth, all_p.shape[1]))
    if len({vocab for *_, vocab in topologies}) != 1 or len({r.device for r in rows}) != 1:
        raise ValueError("Sparse-exit batch rows must share vocabulary and device")
    device = rows[0].device
    depth = max(t[2] for t in topologies)
    # Each request consumes 2 * (its max_depth + 1) uniforms from its own
    # generator, as in the reference; the kernel reads them at stride 2*(depth+1).
    uniforms = torch.zeros((count, 2 * (depth + 1)), dtype=torch.float64, device=device)
    for i, ((_, _, d, _), gen) in enumerate(zip(topologies, generators)):
        uniforms[i, :2 * (d + 1)] = torch.rand(2 * (d + 1), dtype=torch.float64, device=device,
                                               generator=gen)
    trees = PackedTrees([t[0] for t in topologies], [t[1] for t in topologies], device)
    probs = torch.cat([_as_fp32_rows(r) for r in rows], dim=0)
    out = accept_packed(probs, trees, rule=SG_RULE_SPARSE_EXIT, uniforms=uniforms, max_depth=depth)
    host = out.tolist()
    return [decode_output(host[i], depth, topologies[i][3], topologies[i][1], "Sparse-exit sampler")
            for i in range(count)]


def tree_verify_ancestral_same_draw_fused(parents, tokens, all_p, generator=None,
                                          validate: bool = True):
    """Reference fused_tree_sampling.py:2376-2414: the reference's multinomial
    draws (same primitive, shape and order), walked on device."""
    parents, tokens, max_depth = _topology(parents, tokens)
    node_count = len(parents)
    _check_rows(all_p, node_count, "Same-draw DDTree")
    if any(token < 0 or token >= all_p.shape[1] for token in tokens):
        raise ValueError("Tree token is outside the Target vocabulary")
    if validate:
        _validate_probabilities(all_p, normalised=False)
    posterior = torch.multinomial(all_p, 1, generator=generator).reshape(-1)
    trees = PackedTrees([parents], [tokens], all_p.device)
    out = follow_packed(posterior, trees, max_depth=max_depth)
    return decode_output(out[0].tolist(), max_depth, all_p.shape[1], tokens,
                         "Same-draw fused tree walk")


def follow_packed(posterior: torch.Tensor, trees: PackedTrees, *, max_depth: int | None = None,
                  out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
    depth = trees.max_depth if max_depth is None else int(max_depth)
    posterior = posterior.to(torch.long).contiguous()
    if out is None:
        out = torch.empty((trees.count, depth + 2), dtype=torch.long, device=posterior.device)
    with torch.cuda.stream(stream) if stream is not None else _nullcontext():
        ops.load().tree_follow_out(posterior, trees.row_offsets, trees.parents, trees.tokens, trees.max_nodes,
                                   depth, status, out)
    return out


def accept_logits_packed(logits: torch.Tensor, trees: PackedTrees, *, temperature: float = 1.0,
                         uniforms: torch.Tensor | None = None, seed: int = 0,
                         request_ids: torch.Tensor | None = None, max_depth: int | None = None,
                         out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                         stream=None) -> torch.Tensor:
    """One launch of the direct-logits walk (``sg_tree_accept_logits``) over
    packed fp32 or bf16 logit rows; returns the device [trees, max_depth + 2]
    output (reference layout)."""
    if not logits.is_cuda or logits.ndim != 2 or logits.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("accept_logits_packed expects a CUDA float32 or bfloat16 [rows, vocab] tensor")
    logits = logits.contiguous()
    if logits.shape[0] < trees.total_rows:
        raise ValueError("fewer logit rows than packed tree nodes")
    depth = trees.max_depth if max_depth is None else int(max_depth)
    if uniforms is not None:
        uniforms = uniforms.reshape(trees.count, -1).contiguous()
    if out is None:
        out = torch.empty((trees.count, depth + 2), dtype=torch.long, device=logits.device)
    with torch.cuda.stream(stream) if stream is not None else _nullcontext():
        ops.load().tree_accept_logits_out(logits, trees.row_offsets, trees.parents, trees.tokens, trees.max_nodes,
                                          depth, float(temperature), uniforms, ops.seed_arg(seed), request_ids,
                                          status, out)
    return out


def _check_logit_temperature(temperature, probability_dtype):
    if (not isinstance(temperature, (float, int)) or not temperature > 0
            or temperature == float("inf")):
        raise ValueError("Direct-logits temperature must be finite and positive")
    if probability_dtype != torch.float64:
        raise ValueError("Direct-logits verifier requires FP64 probability arithmetic")


def _logit_stats(count, node_count):
    return {"visited_probability_rows": count + 1, "total_tree_rows": node_count, "lm_head_rows": node_count}


def tree_verify_ancestral_logits_fused_scan(parents, tokens, all_logits, temperature: float,
                                            probability_dtype=torch.float64, generator=None,
                                            validate: bool = True):
    """Reference fused_tree_sampling.py:2417-2465 on the B200 kernel:
    (nodes, tokens, bonus, stats); uniforms drawn from ``generator`` as the
    reference draws them (``torch.rand(max_depth + 1)`` float64)."""
    parents, tokens, max_depth = _topology(parents, tokens)
    node_count = len(parents)
    if (not all_logits.is_cuda or all_logits.ndim != 2 or all_logits.shape[0] != node_count
            or all_logits.shape[1] < 1 or not all_logits.is_floating_point()):
        raise ValueError("Direct-logits Target tensor mismatch")
    _check_logit_temperature(temperature, probability_dtype)
    if any(t < 0 or t >= all_logits.shape[1] for t in tokens):
        raise ValueError("Tree token is outside the Target vocabulary")
    if validate and not bool(torch.isfinite(all_logits).all()):
        raise FloatingPointError("Target logits must be finite")
    uniforms = torch.rand(max_depth + 1, dtype=torch.float64, device=all_logits.device, generator=generator)
    rows = all_logits if all_logits.dtype in (torch.float32, torch.bfloat16) else all_logits.float()
    trees = PackedTrees([parents], [tokens], all_logits.device)
    out = accept_logits_packed(rows, trees, temperature=temperature, uniforms=uniforms, max_depth=max_depth)
    nodes, toks, bonus = decode_output(out[0].tolist(), max_depth, all_logits.shape[1], tokens,
                                       "Direct-logits sampler")
    return nodes, toks, bonus, _logit_stats(len(nodes), node_count)


def tree_verify_ancestral_logits_fused_scan_batched(parents_batch, tokens_batch, all_logits, temperature: float,
                                                    probability_dtype=torch.float64, generators=None,
                                                    validate: bool = True):
    """Reference fused_tree_sampling.py:2468-2533: equally shaped trees
    ([B, n, V] logits), one launch, one uniform draw per request generator.
    Ragged batches (a list of [n_i, V]) run as one launch too."""
    count = len(parents_batch)
    if (count < 1 or len(tokens_batch) != count or generators is None or len(generators) != count):
        raise ValueError("Batched direct-logits inputs are inconsistent")
    _check_logit_temperature(temperature, probability_dtype)
    rows = list(all_logits.unbind(0)) if isinstance(all_logits, torch.Tensor) else list(all_logits)
    topo = [_topology(p, t) for p, t in zip(parents_batch, tokens_batch)]
    if len(rows) != count or any(r.ndim != 2 or r.shape[0] != len(p) or not r.is_cuda
                                 for r, (p, _, _) in zip(rows, topo)):
        raise ValueError("Batched direct-logits tensor shape mismatch")
    vocab = rows[0].shape[1]
    if any(t < 0 or t >= vocab for _, toks, _ in topo for t in toks):
        raise ValueError("Tree token is outside the Target vocabulary")
    if validate and not all(bool(torch.isfinite(r).all()) for r in rows):
        raise FloatingPointError("Target logits must be finite")
    depth = max(d for _, _, d in topo)
    device = rows[0].device
    uniforms = torch.zeros((count, depth + 1), dtype=torch.float64, device=device)
    for i, ((_, _, d), gen) in enumerate(zip(topo, generators)):
        uniforms[i, :d + 1] = torch.rand(d + 1, dtype=torch.float64, device=device, generator=gen)
    flat = torch.cat([r if r.dtype in (torch.float32, torch.bfloat16) else r.float() for r in rows], 0)
    trees = PackedTrees([p for p, _, _ in topo], [t for _, t, _ in topo], device)
    host = accept_logits_packed(flat, trees, temperature=temperature, uniforms=uniforms, max_depth=depth).tolist()
    results = []
    for (par, toks, _), row in zip(topo, host):
        nodes, out_toks, bonus = decode_output(row, depth, vocab, toks, "Batched direct-logits sampler")
        results.append((nodes, out_toks, bonus, _logit_stats(len(nodes), len(par))))
    return results


def terminal_mass_packed(probs: torch.Tensor, trees: PackedTrees, *, uniforms: torch.Tensor | None = None,
                         seed: int = 0, request_ids: torch.Tensor | None = None, max_depth: int | None = None,
                         out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                         stream=None) -> torch.Tensor:
    """One call of ``sg_tree_verify_terminal_mass`` (two launches) over packed
    rows; returns the device ``[trees, max_depth + 2]`` int64 output
    (reference layout).  ``uniforms``: ``[trees, 2]`` float64 (terminal node,
    bonus token) or None for the Philox stream keyed by (seed, request)."""
    from . import _lib
    if probs.dtype != torch.float32 or not probs.is_cuda or probs.ndim != 2:
        raise ValueError("terminal_mass_packed expects a CUDA float32 [rows, vocab] tensor")
    probs = probs.contiguous()
    if probs.shape[0] < trees.total_rows:
        raise ValueError("fewer probability rows than packed tree nodes")
    depth = trees.max_depth if max_depth is None else int(max_depth)
    if depth < trees.max_depth:
        raise ValueError("max_depth is below the depth of a packed tree")
    stride = 0
    if uniforms is not None:
        if uniforms.dtype != torch.float64 or uniforms.device != probs.device:
            raise ValueError("uniforms must be float64 on the probabilities' device")
        uniforms = uniforms.reshape(trees.count, -1).contiguous()
        stride = uniforms.shape[1]
        if stride < 2:
            raise ValueError("terminal-mass draws need two uniforms per tree")
    if out is None:
        out = torch.empty((trees.count, depth + 2), dtype=torch.long, device=probs.device)
    lib = _lib.load()
    nbytes = lib.sg_tree_verify_terminal_mass_workspace_bytes(trees.total_rows)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=probs.device)
    st = lib.sg_tree_verify_terminal_mass(
        _lib.ptr(probs), probs.shape[1], _lib.ptr(trees.row_offsets), _lib.ptr(trees.parents),
        _lib.ptr(trees.tokens), trees.count, trees.total_rows, depth, _lib.ptr(uniforms), stride, seed,
        _lib.ptr(request_ids), _lib.ptr(out), _lib.ptr(status), _lib.ptr(ws), nbytes, _lib.stream_ptr(stream))
    _lib.check(st, "sg_tree_verify_terminal_mass")
    return out


def tree_block_verify_terminal_mass_fused(parents, tokens, all_p, generator=None, validate: bool = True):
    """Reference sampling.py:542-735 (``tree_block_verify_terminal_mass``, the
    decoder's default verifier) on the B200 kernel: (nodes, tokens, bonus)
    with the same output law, its two draws taken from ``torch.rand(2)`` on
    the request's generator (terminal node, then bonus token)."""
    parents, tokens, max_depth = _topology(parents, tokens)
    node_count = len(parents)
    _check_rows(all_p, node_count, "Terminal-mass tree")
    if any(token < 0 or token >= all_p.shape[1] for token in tokens):
        raise ValueError("Tree token is outside the Target vocabulary")
    if validate:
        _validate_probabilities(all_p, normalised=False)
    uniforms = torch.rand(2, dtype=torch.float64, device=all_p.device, generator=generator)
    trees = PackedTrees([parents], [tokens], all_p.device)
    status = torch.zeros(1, dtype=torch.int32, device=all_p.device)
    out = terminal_mass_packed(_as_fp32_rows(all_p), trees, uniforms=uniforms, max_depth=max_depth,
                               status=status)
    row, st = out[0].tolist(), int(status.item())
    if st != 0:
        raise FloatingPointError(f"Terminal-mass tree sampler: device status {st}")
    return decode_output(row, max_depth, all_p.shape[1], tokens, "Terminal-mass tree sampler")


def philox_node_uniforms(seed: int, request: int, node: int) -> tuple[float, float]:
    """Host restatement of the kernel's per-node uniforms (for reproducibility
    checks): Philox4x32-10, key = seed, counter = (node, request lo, request hi, 0)."""
    M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
    mask = 0xFFFFFFFF
    c = [node & mask, request & mask, (request >> 32) & mask, 0]
    k0, k1 = seed & mask, (seed >> 32) & mask
    for r in range(10):
        if r:
            k0, k1 = (k0 + W0) & mask, (k1 + W1) & mask
        p0, p1 = M0 * c[0], M1 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & mask, p1 & mask, ((p0 >> 32) ^ c[3] ^ k1) & mask, p0 & mask]
    u = lambda a, b: (((b << 32) | a) >> 11) * (1.0 / 9007199254740992.0)
    return u(c[0], c[1]), u(c[2], c[3])


__all__ = [
    "PackedTrees", "accept_packed", "accept_logits_packed", "follow_packed", "decode_output",
    "tree_verify_ancestral_logits_fused_scan", "tree_verify_ancestral_logits_fused_scan_batched",
    "tree_verify_ancestral_fused_scan", "tree_verify_ancestral_sparse_exit_fused_scan",
    "tree_verify_ancestral_sparse_exit_fused_scan_batched", "tree_verify_ancestral_same_draw_fused",
    "philox_node_uniforms", "SG_RULE_SCAN", "SG_RULE_SPARSE_EXIT",
]
