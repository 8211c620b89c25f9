"""TEST INFRASTRUCTURE — CPU restatement of the packed verify pass (torch fp32).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
It restates the reference's target step for one wave
(continuous_tree_block_decode.py:1748-1824 calling HF Qwen3Model through
engine.py:499-517): embedding, 36 x {RMSNorm, q/k/v projections, per-head
q/k RMSNorm, rotate-half RoPE at positions round_prefix_len + depth, GQA
attention over the request's own cache prefix plus its tree ancestors (the
mask of :500-546), o projection + residual, RMSNorm, SwiGLU MLP + residual},
final RMSNorm, LM head, fp32 softmax (sampling.py:29-36); then the acceptance
walk of the C oracle over those probabilities.  Weights and cache prefixes
are plain fp32 tensors (the engine's packed layout: fused q|k|v, gate/up
interleaved in 128-row blocks).
"""
from __future__ import annotations

import numpy as np
import torch


def rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """x [rows, heads, D]; rotate-half convention of HF Qwen3."""
    ang = pos.float()[:, None] * inv_freq[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], -1)
    return x * cos + rot * sin


class CpuWeights:
    """CPU copy of engine weights (specgrove_b200.engine.Weights).

    Kept in fp32 when host memory allows; otherwise kept in bf16 and widened
    to fp32 one layer at a time (``lazy``)."""

    def __init__(self, w, lazy: bool | None = None, device="cpu"):
        if lazy is None:
            try:
                import psutil
                lazy = psutil.virtual_memory().available < 3 * 2 * w.nbytes()
            except ImportError:
                lazy = True
        self.lazy = lazy
        f = lambda t: t.detach().float().to(device)
        keep = (lambda t: t.detach().to(device)) if lazy else f
        self.shape = w.shape
        self.embed = f(w.embed)
        self.lm_head = keep(w.lm_head)
        self.final_norm = f(w.final_norm)
        self.inv_freq = f(w.inv_freq)
        self.layers = [[keep(t) for t in layer] for layer in w.layers]

    def layer(self, l: int):
        return [t.float() for t in self.layers[l]] if self.lazy else self.layers[l]

    def head(self):
        return self.lm_head.float() if self.lazy else self.lm_head


def verify_logits(cw: CpuWeights, prefixes, trees, cache_lengths, return_kv: bool = False):
    """prefixes: per request per layer (K [nkv, L, D], V [nkv, L, D]) fp32;
    trees: per request (parents, tokens-with-root-token-first).
    Returns logits [Q, V] fp32 and the packed row offsets (and, with
    return_kv, every layer's post-RoPE keys and values of the packed rows)."""
    s = cw.shape
    nq, nkv, D, H, I = s.num_q_heads, s.num_kv_heads, s.head_dim, s.hidden, s.intermediate
    G = nq // nkv
    offsets, tokens, positions, parents_all = [0], [], [], []
    for (par, tok), L in zip(trees, cache_lengths):
        depth = [0] * len(par)
        for j in range(1, len(par)):
            depth[j] = depth[par[j]] + 1
        tokens += list(tok)
        positions += [L + d for d in depth]
        parents_all.append(par)
        offsets.append(offsets[-1] + len(par))
    Q = offsets[-1]
    dev = cw.embed.device
    x = cw.embed[torch.tensor(tokens, device=dev)]
    pos = torch.tensor(positions, device=dev)
    kv = []
    vis = []
    for par in parents_all:
        n = len(par)
        v = torch.zeros((n, n), dtype=torch.bool, device=dev)
        v[0, 0] = True
        for i in range(1, n):
            v[i] = v[par[i]]
            v[i, i] = True
        vis.append(v)
    for l in range(len(cw.layers)):
        in_norm, wqkv, qn, kn, wo, post_norm, wgu, wdown = cw.layer(l)
        xn = rms(x, in_norm, s.rms_eps)
        qkv = xn @ wqkv.t()
        q = qkv[:, :nq * D].view(Q, nq, D)
        k = qkv[:, nq * D:(nq + nkv) * D].view(Q, nkv, D)
        v = qkv[:, (nq + nkv) * D:].view(Q, nkv, D)
        q = rope(rms(q, qn, s.rms_eps), pos, cw.inv_freq)
        k = rope(rms(k, kn, s.rms_eps), pos, cw.inv_freq)
        kv.append((k, v))
        attn = torch.empty((Q, nq, D), device=dev)
        for i, (r0, r1) in enumerate(zip(offsets, offsets[1:])):
            Kp, Vp = prefixes[i][l]
            keys = torch.cat([Kp, k[r0:r1].transpose(0, 1)], dim=1)      # [nkv, L+n, D]
            vals = torch.cat([Vp, v[r0:r1].transpose(0, 1)], dim=1)
            L = Kp.shape[1]
            mask = torch.cat([torch.ones((r1 - r0, L), dtype=torch.bool, device=dev), vis[i]], dim=1)
            qh = q[r0:r1].transpose(0, 1).reshape(nkv, G, r1 - r0, D)  # query head h*G+g
            sc = torch.einsum("hgnd,hkd->hgnk", qh, keys) / (D ** 0.5)
            sc = sc.masked_fill(~mask[None, None], float("-inf"))
            p = torch.softmax(sc, dim=-1)
            o = torch.einsum("hgnk,hkd->hgnd", p, vals)                  # [nkv, G, n, D]
            attn[r0:r1] = o.reshape(nq, r1 - r0, D).transpose(0, 1)
        x = x + attn.reshape(Q, nq * D) @ wo.t()
        xn = rms(x, post_norm, s.rms_eps)
        gu = xn @ wgu.t()
        g = gu.view(Q, I // 128, 2, 128)[:, :, 0].reshape(Q, I)
        u = gu.view(Q, I // 128, 2, 128)[:, :, 1].reshape(Q, I)
        x = x + (torch.nn.functional.silu(g) * u) @ wdown.t()
    xn = rms(x, cw.final_norm, s.rms_eps)
    logits = xn @ cw.head().t()
    return (logits, offsets, kv) if return_kv else (logits, offsets)


def verify_step(cw: CpuWeights, prefixes, trees, cache_lengths, uniforms=None, seed: int = 0,
                temperature: float = 1.0):
    """Full CPU step: logits -> fp32 softmax -> acceptance walk (C oracle).
    Returns (per-request (nodes, bonus), offsets)."""
    from . import cpu as oracle
    logits, offsets = verify_logits(cw, prefixes, trees, cache_lengths)
    probs = torch.softmax(logits / temperature, dim=-1).numpy()
    parents = np.asarray([p for par, _ in trees for p in par], np.int64)
    tokens = np.asarray([t if j else -1 for par, tok in trees for j, t in enumerate(tok)], np.int64)
    depth = 0
    for par, _ in trees:
        d = [0] * len(par)
        for j in range(1, len(par)):
            d[j] = d[par[j]] + 1
        depth = max(depth, max(d))
    out, st = oracle.accept_probs(probs, offsets, parents, tokens, depth, uniforms=uniforms, seed=seed,
                                  arith=oracle.ARITH_FP64)
    res = []
    for i in range(len(trees)):
        count = int(out[i, depth])
        res.append((out[i, :count].tolist(), int(out[i, depth + 1])))
    return res, offsets
