"""CPU model checks of the persistent tree-attention barrier protocol
(tests/attention_protocol_model.py mirrors csrc/attention.cu's warp roles)."""
import random

import pytest

from attention_protocol_model import Hazard, random_items, run


@pytest.mark.parametrize("kst,vst", [(4, 3), (3, 3), (6, 6), (2, 2)])
def test_protocol_has_no_deadlock_overflow_or_hazard(kst, vst):
    rng = random.Random(kst * 10 + vst)
    for trial in range(300):
        run(random_items(rng), kst=kst, vst=vst, seed=trial)


def test_short_items_with_idle_quarters():
    """Prefill-like waves: many one- or two-tile items, lane quarters going
    idle and active again (the case that once broke the kernel)."""
    rng = random.Random(3)
    for trial in range(300):
        items = [(rng.randint(1, 2), rng.choice([1, 4])) for _ in range(12)]
        run(items, seed=trial)


@pytest.mark.parametrize("bug", ["skip_idle", "no_v_wait"])
def test_model_catches_planted_bugs(bug):
    """The model must flag the historical mistakes, or it proves nothing."""
    rng = random.Random(11)
    caught = 0
    for trial in range(300):
        try:
            run(random_items(rng), seed=trial, bugs=frozenset({bug}))
        except Hazard:
            caught += 1
    assert caught > 0
