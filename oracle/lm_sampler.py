"""TEST INFRASTRUCTURE — float64 restatement of the fused LM-head sampler.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
it.  It restates, from the logits, what the LM-head GEMM epilogue of the
CUDA library draws for each packed row (the law of the reference's
``probabilities`` + ``sample``, sampling.py:29-42, used by
``tree_verify_ancestral_batched``, sampling.py:903-950; greedy rows follow
``tree_verify_greedy_block``, continuous_tree_block_decode.py:45-71, whose
argmax runs over the bf16 logits of continuous_tree_block_decode.py:1809-1811):

* x = logits / T, cut into 256-column vocabulary tiles (the last one may be
  narrower);
* per tile t: m_t = max x, S_t = sum exp(x - m_t), and one Philox4x32-10 draw
  keyed by the seed with counter (t, node, request lo, 0x80000000 | request
  hi): words (x, y) give an Exp(1) variate E_t, word z a 24-bit uniform U_t;
* the row's tile is argmax_t (m_t + log S_t - log E_t) (a Gumbel race over
  the tile masses), its token the first column of that tile whose running sum
  of exp(x - m_t) exceeds U_t * S_t (inverse CDF);
* greedy rows (T = 0): the first column whose bf16-rounded logit is maximal.

Everything is evaluated in float64 from the same random words, so the CUDA
path must agree except where a decision sits within fp32 rounding of a
boundary; ``sample_rows`` reports each row's margin to such a boundary.
"""
from __future__ import annotations

import numpy as np
import torch

TILE = 256
_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, seed: int):
    """Philox4x32-10 (Salmon et al., SC 2011) over broadcast uint32 counter
    words; returns the four output words as uint64 arrays holding 32 bits."""
    c = [np.asarray(v, dtype=np.uint64) & _MASK for v in (c0, c1, c2, c3)]
    c = list(np.broadcast_arrays(*c))
    c = [v.copy() for v in c]
    k0 = np.uint64(seed & 0xFFFFFFFF)
    k1 = np.uint64((seed >> 32) & 0xFFFFFFFF)
    for r in range(10):
        if r:
            k0 = (k0 + _W0) & _MASK
            k1 = (k1 + _W1) & _MASK
        p0 = _M0 * c[0]
        p1 = _M1 * c[2]
        c = [((p1 >> np.uint64(32)) ^ c[1] ^ k0) & _MASK, p1 & _MASK,
             ((p0 >> np.uint64(32)) ^ c[3] ^ k1) & _MASK, p0 & _MASK]
    return c


def exp_variate(lo, hi) -> np.ndarray:
    """E = -ln(1 - V), V = (2k + 1) / 2^53, k = (hi:lo) >> 12, in float64."""
    w = (np.asarray(hi, np.uint64) << np.uint64(32)) | np.asarray(lo, np.uint64)
    k = w >> np.uint64(12)
    v = (2.0 * k.astype(np.float64) + 1.0) * 2.0 ** -53   # exact: k < 2^52
    low = v < 0.5
    comp = (2.0 * ((np.uint64((1 << 52) - 1) - k).astype(np.float64)) + 1.0) * 2.0 ** -53
    return np.where(low, -np.log1p(-np.where(low, v, 0.0)), -np.log(np.where(low, 1.0, comp)))


def tile_draws(seed: int, nodes, requests, n_tiles: int):
    """(E [rows, tiles], U [rows, tiles]) of the sampler's Philox draws."""
    nodes = np.asarray(nodes, np.int64).reshape(-1, 1)
    req = np.asarray(requests, np.int64).astype(np.uint64).reshape(-1, 1)
    t = np.arange(n_tiles, dtype=np.uint64).reshape(1, -1)
    hi_word = np.uint64(0x80000000) | ((req >> np.uint64(32)) & np.uint64(0x7FFFFFFF))
    x, y, z, _ = philox4x32_10(t, nodes.astype(np.uint64), req & _MASK, hi_word, seed)
    E = exp_variate(x, y)
    U = ((z >> np.uint64(8)).astype(np.float64) + 0.5) / 16777216.0
    return E, U


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    """Round to bfloat16 (nearest even) through float32, returned as float64."""
    return x.to(torch.float32).to(torch.bfloat16).to(torch.float64)


def sample_rows(logits: torch.Tensor, nodes, requests, seed: int, temperature: float):
    """Tokens, lse and decision margins of every row.

    logits: float64 [rows, vocab] (any device).  Returns numpy arrays
    (tokens int64, lse float64 of logits / T (T = 1 for greedy), key_gap,
    cdf_margin).  key_gap is the distance of the row's tile choice to a tie
    in logit units: the gap between the two largest tile keys (greedy rows:
    the distance of any logit to a rounding boundary next to the top bf16
    value).  cdf_margin is the distance of U * S to the nearest cumulative
    boundary of the chosen column, relative to S (inf for greedy rows)."""
    logits = logits.to(torch.float64)
    rows, vocab = logits.shape
    n_tiles = (vocab + TILE - 1) // TILE
    greedy = temperature == 0
    x = logits if greedy else logits / temperature
    lse = torch.logsumexp(x, dim=-1).cpu().numpy()
    if greedy:
        b = bf16_round(logits)
        top = b.max(dim=-1).values
        tokens = (b == top[:, None]).to(torch.int8).argmax(dim=-1).cpu().numpy()
        # the two bf16 neighbours of the top value (adjacent bit patterns) and
        # the rounding boundaries half-way to them
        bits = top.to(torch.float32).view(torch.int32) >> 16
        nb = [((bits + d) << 16).view(torch.float32).to(torch.float64) for d in (-1, 1)]
        dist = torch.stack([(logits - ((top + n) / 2)[:, None]).abs() for n in nb]).amin(dim=(0, 2))
        return tokens.astype(np.int64), lse, dist.cpu().numpy(), np.full(rows, np.inf)
    pad = n_tiles * TILE - vocab
    xt = torch.nn.functional.pad(x, (0, pad), value=float("-inf")).view(rows, n_tiles, TILE)
    m = xt.max(dim=-1).values                                   # [rows, tiles]
    w = torch.exp(xt - m[..., None])                            # [rows, tiles, 256]
    S = w.sum(dim=-1)
    E, U = tile_draws(seed, nodes, requests, n_tiles)
    key = (m + torch.log(S)).cpu().numpy() - np.log(E)
    order = np.argsort(-key, axis=1, kind="stable")
    best = order[:, 0]
    gap = key[np.arange(rows), best] - key[np.arange(rows), order[:, 1]] if n_tiles > 1 else np.full(rows, np.inf)
    ridx = torch.arange(rows, device=logits.device)
    bt = torch.as_tensor(best, device=logits.device)
    cum = torch.cumsum(w[ridx, bt], dim=-1)                      # [rows, 256]
    Sb = S[ridx, bt]
    thr = torch.as_tensor(U[np.arange(rows), best], device=logits.device) * Sb
    width = torch.full((rows,), TILE, device=logits.device)
    width[bt == n_tiles - 1] = vocab - (n_tiles - 1) * TILE
    col = torch.searchsorted(cum, thr[:, None], right=True)[:, 0]
    col = torch.minimum(col, width - 1)
    prev = torch.where(col > 0, cum[ridx, (col - 1).clamp_min(0)], torch.zeros_like(thr))
    cdf_margin = torch.minimum(thr - prev, cum[ridx, col] - thr) / Sb
    tokens = (bt * TILE + col).cpu().numpy()
    return tokens.astype(np.int64), lse, gap, cdf_margin.cpu().numpy()
