"""How often the exact 64.64 fixed-point acceptance rule (the CUDA kernels'
and the C oracle's arithmetic) picks a different token than the reference's
fp64 running-sum rule (fused_tree_sampling.py:2607-2612: cumsum of the fp32
probabilities in fp64, first index whose running sum exceeds u * total).

The two rules can only disagree when u * total falls within fp64 rounding of
a CDF boundary.  The count is measured over 10^6 draws on configuration-2
rows (V = 151936, target logits = 4 N(0,1) + 0.5 N(0,1), softmax in fp32):
both rules are restated here with numpy (the fp64 rule by a sequential
cumsum, the fixed-point rule by exact integer prefix sums) and a subsample
is checked against the C oracle's two arithmetics."""
import numpy as np

from oracle import cpu

V = 151936
ROWS = 100
DRAWS_PER_ROW = 10_000   # 10^6 draws in all


def _softmax_rows(rng, rows):
    logits = (4.0 * rng.standard_normal((rows, V)) + 0.5 * rng.standard_normal((rows, V))).astype(np.float32)
    z = logits - logits.max(axis=1, keepdims=True)
    e = np.exp(z, dtype=np.float32)
    return (e / e.sum(axis=1, dtype=np.float32, keepdims=True)).astype(np.float32)


def _exact_prefix(row):
    """Exact prefix sums of floor(p * 2^64) as (hi, lo) uint64 halves of 2^32."""
    mass = np.floor(row.astype(np.float64) * 2.0 ** 64)      # exact: a power-of-two scaling, then floor
    hi = np.floor(mass / 2.0 ** 32)
    lo = mass - hi * 2.0 ** 32
    return np.cumsum(hi.astype(np.uint64)), np.cumsum(lo.astype(np.uint64))


def _count_row(row, us):
    cdf = np.cumsum(row.astype(np.float64))                   # sequential fp64 running sum
    pick64 = np.searchsorted(cdf, us * cdf[-1], side="right")  # first t with u * total < run(t)
    hi, lo = _exact_prefix(row)
    P = lambda t: (int(hi[t]) << 32) + int(lo[t])
    total = P(V - 1)
    bad, margin = 0, float("inf")
    for u, t in zip(us.tolist(), pick64.tolist()):
        num, den = u.as_integer_ratio()
        thr = num * total // den                              # floor(u * total), exact
        hit = t < V and P(t) > thr and (t == 0 or P(t - 1) <= thr)
        bad += not hit
        if t < V:
            lo_gap = thr - (P(t - 1) if t else 0)
            margin = min(margin, min(lo_gap, P(t) - thr) / total)
    return bad, pick64, margin


def test_fixed_point_vs_fp64_rule_disagreement_count():
    rng = np.random.default_rng(20261202)
    rows = _softmax_rows(rng, ROWS)
    disagreements, margin = 0, float("inf")
    checked = 0
    for i in range(ROWS):
        us = (rng.integers(0, 1 << 53, size=DRAWS_PER_ROW, dtype=np.int64) * 2.0 ** -53)
        bad, pick64, m = _count_row(rows[i], us)
        disagreements += bad
        margin = min(margin, m)
        if i < 4:
            # the restatements pick what the C oracle picks, in both arithmetics
            for j in range(3):
                u = np.array([[us[j]]])
                outs = [cpu.accept_probs(rows[i:i + 1], [0, 1], [-1], [0], 0, uniforms=u, arith=a)[0][0, 1]
                        for a in (cpu.ARITH_EXACT, cpu.ARITH_FP64)]
                assert outs[0] == outs[1] == pick64[j]
                checked += 1
    print(f"fixed-point vs fp64 rule: {disagreements} of {ROWS * DRAWS_PER_ROW} draws disagree; "
          f"closest threshold to a CDF boundary {margin:.3e} of the row total")
    assert checked == 12
    # Disagreement needs u * total within ~1e-16 (relative) of a boundary:
    # expected count << 1 over 10^6 draws.
    assert disagreements == 0
