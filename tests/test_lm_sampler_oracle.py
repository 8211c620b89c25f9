"""The float64 restatement of the fused LM-head sampler (oracle/lm_sampler.py)
against the law it must draw from: the reference's per-row softmax sampling
(``probabilities`` + ``sample``, sampling.py:29-42) and, at T = 0, the argmax
of the bf16 logits (continuous_tree_block_decode.py:45-71).  CPU only."""
import math

import numpy as np
import pytest
import torch

from oracle import lm_sampler


def test_philox_known_answers():
    # Random123 Philox4x32-10 known-answer vectors (counter, key -> output).
    cases = [((0, 0, 0, 0), 0, (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
             ((0xffffffff,) * 4, 0xffffffffffffffff, (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
             ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0x299f31d0 << 32) | 0xa4093822,
              (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]
    for ctr, seed, want in cases:
        got = lm_sampler.philox4x32_10(*ctr, seed)
        assert tuple(int(w) for w in got) == want


def test_exp_variate_tails():
    # V near 0 and near 1 keep full precision: E ~ V for small V, -log(1-V) near 1.
    k_small = np.uint64(5)                       # V = 11 / 2^53
    lo, hi = (k_small << np.uint64(12)) & np.uint64(0xFFFFFFFF), (k_small << np.uint64(12)) >> np.uint64(32)
    e = lm_sampler.exp_variate(lo, hi)
    assert e == pytest.approx(11 * 2.0 ** -53, rel=1e-15)
    k_big = np.uint64((1 << 52) - 3)             # 1 - V = 5 / 2^53
    w = k_big << np.uint64(12)
    e = lm_sampler.exp_variate(w & np.uint64(0xFFFFFFFF), w >> np.uint64(32))
    assert e == pytest.approx(-math.log(5 * 2.0 ** -53), rel=1e-15)


@pytest.mark.parametrize("temperature", [1.0, 0.6])
def test_two_level_draw_has_the_softmax_law(temperature):
    """N independent rows with one logit vector spanning five tiles (the last
    one 32 columns wide): the empirical law must match softmax(l / T)."""
    vocab, n = 1056, 40000
    g = torch.Generator().manual_seed(0)
    base = torch.randn(vocab, generator=g, dtype=torch.float64) * 1.5
    base[1030] += 3.0                            # mass in the narrow last tile
    logits = base.expand(n, vocab)
    tokens, lse, gap, cdf = lm_sampler.sample_rows(logits, np.arange(n), np.full(n, 7), seed=12345,
                                                   temperature=temperature)
    p = torch.softmax(base / temperature, -1).numpy()
    assert lse[0] == pytest.approx(float(torch.logsumexp(base / temperature, -1)), abs=1e-12)
    emp = np.bincount(tokens, minlength=vocab) / n
    # cells with enough mass: standardised deviations stay within 5 sigma
    big = p * n > 30
    z = (emp[big] - p[big]) / np.sqrt(p[big] * (1 - p[big]) / n)
    assert np.abs(z).max() < 5.0, np.abs(z).max()
    # chi-square over the pooled law (big cells + the rest pooled)
    obs = np.append(emp[big] * n, emp[~big].sum() * n)
    exp = np.append(p[big] * n, p[~big].sum() * n)
    chi2 = ((obs - exp) ** 2 / exp).sum()
    dof = len(obs) - 1
    assert chi2 < dof + 6 * math.sqrt(2 * dof), (chi2, dof)
    assert (gap > 0).all() and (cdf > 0).all()
    # how often a decision sits within the GPU's rounding of a boundary
    assert (gap < 1e-4).mean() < 0.002 and (cdf < 1e-5).mean() < 0.008


def test_draws_are_keyed_by_request_node_and_seed():
    vocab = 512
    logits = torch.zeros(4, vocab, dtype=torch.float64)
    a = lm_sampler.sample_rows(logits, [0, 1, 0, 0], [3, 3, 4, 3], seed=1, temperature=1.0)[0]
    b = lm_sampler.sample_rows(logits, [0, 1, 0, 0], [3, 3, 4, 3], seed=1, temperature=1.0)[0]
    c = lm_sampler.sample_rows(logits, [0, 1, 0, 0], [3, 3, 4, 3], seed=2, temperature=1.0)[0]
    assert (a == b).all()
    assert a[0] == a[3]                     # same (seed, request, node): same draw
    assert len({int(a[0]), int(a[1]), int(a[2])}) == 3 or (a != c).any()


def test_greedy_is_first_argmax_of_bf16_logits():
    logits = torch.tensor([[0.1, 2.0, 2.001, -1.0, 2.0],      # 2.0 and 2.001 round to one bf16 value
                           [5.0, 1.0, 7.5, 7.5, 0.0]], dtype=torch.float64)
    tokens, lse, gap, _ = lm_sampler.sample_rows(logits, [0, 1], [0, 0], seed=0, temperature=0.0)
    assert tokens.tolist() == [1, 2]
    assert lse[1] == pytest.approx(float(torch.logsumexp(logits[1], -1)))
    assert gap[0] > 1e-4
