"""CPU/fp32 oracle of the DFlash drafter step (test infrastructure only:
imported by tests, never by the product path).

Restates third_party/ddtree_official/model/dflash.py:22-200 for one request
with a draft cache, the way the decoder drives it
(continuous_tree_block_decode.py:889-962):

* target_hidden = hidden_norm(fc(features)) for the request's new context
  rows (its draft update);
* block rows = [last token, mask, ..., mask] embedded with the target's
  embedding, positions prefix .. prefix + block - 1 after the context rows'
  positions cache_len .. prefix - 1;
* per layer: q from the input-normed block rows; k and v from the context
  rows (target_hidden, no input norm) and the block rows; per-head RMSNorm on
  q and k, RoPE (rotate-half form) at the rows' positions; attention of the
  block rows over [cache, context, block], all visible (non-causal); o
  projection and residual; post-attention norm, SwiGLU MLP, residual;
* the drafter's final norm and the target's LM head on every block row.

The cache keeps the context rows' K/V (the reference crops the block rows'
K/V after the call).  Weights are a dict of fp32 tensors with HF shapes:
embed, lm_head, fc, hidden_norm, norm and per layer in_norm, q, k, v, q_norm,
k_norm, o, post_norm, gate, up, down.  Pinned against
tests/golden/dflash_step.npz (the reference DFlashDraftModel run with the same
weights by tests/golden/make_golden.py).
"""
from __future__ import annotations

import torch


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def _rope(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """x [n, heads, D] rotated at positions pos [n] (fp32 angles)."""
    ang = pos.to(torch.float32)[:, None] * inv_freq[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], -1)
    return x * cos + rot * sin


def dflash_step(w: dict, num_layers: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                features: torch.Tensor, cache_k: list, cache_v: list, anchor: int, mask_token: int, block: int,
                inv_freq: torch.Tensor, eps: float) -> tuple[torch.Tensor, list, list]:
    """One request's drafter step.  features [u, F * H]; cache_k/v per layer
    [nkv, c, D] (c = rows already cached).  Returns the block rows' logits
    [block, V] and the caches with the u context rows appended."""
    D, nq, nkv = head_dim, num_q_heads, num_kv_heads
    G = nq // nkv
    dev = features.device
    u = features.shape[0]
    c = cache_k[0].shape[1] if cache_k else 0
    th = _rms(features.float() @ w["fc"].T, w["hidden_norm"], eps)
    tokens = torch.tensor([anchor] + [mask_token] * (block - 1), device=dev)
    x = w["embed"][tokens].float()
    pos_ctx = torch.arange(c, c + u, device=dev)
    pos_blk = torch.arange(c + u, c + u + block, device=dev)
    new_k, new_v = [], []
    for l in range(num_layers):
        p = lambda name: w[f"layers.{l}.{name}"]
        h = _rms(x, p("in_norm"), eps)
        q = _rope(_rms((h @ p("q").T).view(block, nq, D), p("q_norm"), eps), pos_blk, inv_freq)
        kc = _rope(_rms((th @ p("k").T).view(u, nkv, D), p("k_norm"), eps), pos_ctx, inv_freq)
        vc = (th @ p("v").T).view(u, nkv, D)
        kb = _rope(_rms((h @ p("k").T).view(block, nkv, D), p("k_norm"), eps), pos_blk, inv_freq)
        vb = (h @ p("v").T).view(block, nkv, D)
        k_all = torch.cat([cache_k[l].permute(1, 0, 2), kc, kb]) if c else torch.cat([kc, kb])
        v_all = torch.cat([cache_v[l].permute(1, 0, 2), vc, vb]) if c else torch.cat([vc, vb])
        new_k.append(torch.cat([cache_k[l], kc.permute(1, 0, 2)], 1) if c else kc.permute(1, 0, 2).contiguous())
        new_v.append(torch.cat([cache_v[l], vc.permute(1, 0, 2)], 1) if c else vc.permute(1, 0, 2).contiguous())
        out = torch.empty(block, nq, D, device=dev)
        for hq in range(nq):
            kv = hq // G
            s = (q[:, hq] @ k_all[:, kv].T) / D ** 0.5
            out[:, hq] = torch.softmax(s, -1) @ v_all[:, kv]
        x = x + out.reshape(block, nq * D) @ p("o").T
        h2 = _rms(x, p("post_norm"), eps)
        x = x + (torch.nn.functional.silu(h2 @ p("gate").T) * (h2 @ p("up").T)) @ p("down").T
    logits = _rms(x, w["norm"], eps) @ w["lm_head"].T
    return logits, new_k, new_v
