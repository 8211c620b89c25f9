"""Device tier allocator (sg_allocate_tiers_device) against the host knapsack
and the reference-generated allocator fixtures: identical allocations,
including exact and within-1e-12 reward ties (continuous_tree_block_decode.py
:706-795)."""
import json

import numpy as np
import pytest
import torch

from specgrove_b200.allocator import allocate_tree_budgets, allocate_tree_budgets_device, critical_path_weights

pytestmark = pytest.mark.gpu


def _device(weights, options, utilities, **kw):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = allocate_tree_budgets_device(torch.tensor(weights, dtype=torch.float64, device="cuda"), options,
                                       torch.tensor(utilities, dtype=torch.float64, device="cuda"), status=status,
                                       **kw)
    return tuple(int(v) for v in out.cpu()), int(status.item())


def test_device_allocator_matches_reference_fixtures(golden_dir):
    z = json.loads((golden_dir / "allocator.json").read_text())
    for p in z["problems"]:
        weights = critical_path_weights(p["progress"], p["ages"], p["criticality"], p["max_new_tokens"])
        curve = [tuple(x) for x in p["curve"]] if p["curve"] else None
        alloc, st = _device(weights, p["options"], p["utilities"], row_budget=p["row_budget"],
                            fixed_row_equivalent=p["fixed"], row_cost_curve=curve)
        assert st == 0
        assert list(alloc) == p["allocation"]


@pytest.mark.parametrize("seed", range(12))
def test_device_allocator_matches_host_with_ties(seed):
    rng = np.random.default_rng(7000 + seed)
    R = int(rng.choice([1, 3, 8, 24, 64]))
    options = sorted(rng.choice(np.arange(1, 160), size=int(rng.integers(1, 6)), replace=False).tolist())
    R = min(R, 4096 // (options[0] + 1))  # the device knapsack takes row budgets up to 4096
    lo = R * (options[0] + 1)
    budget = int(min(4096, lo + rng.integers(0, R * (options[-1] + 1) - lo + 2)))
    if seed % 3 == 0:
        # few distinct values: many exact reward ties between allocations
        utilities = rng.choice([1.0, 1.5, 2.0, 3.0], size=(R, len(options)))
        weights = np.ones(R)
    elif seed % 3 == 1:
        # near-ties inside the 1e-12 tolerance
        base = rng.choice([1.25, 2.5], size=(R, len(options)))
        utilities = base + rng.choice([0.0, 2e-13, 4e-13], size=base.shape)
        weights = rng.choice([1.0, 2.0], size=R)
    else:
        utilities = 1.0 + rng.random((R, len(options))) * 8
        weights = rng.random(R) * 3
    utilities = np.sort(utilities, axis=1)
    if seed % 2 == 0:
        kw = dict(fixed_row_equivalent=float(rng.uniform(4, 64)))
    else:
        rows = np.cumsum(rng.integers(8, 400, size=5)).tolist()
        cost = np.cumsum(rng.uniform(0.5, 10, size=5)).tolist()
        kw = dict(row_cost_curve=list(zip(rows, cost)))
    host = allocate_tree_budgets(weights.tolist(), options, utilities.tolist(), row_budget=budget, **kw)
    dev, st = _device(weights.tolist(), options, utilities.tolist(), row_budget=budget, **kw)
    assert st == 0
    assert dev == host


def test_device_allocator_reports_bad_utilities():
    alloc, st = _device([1.0, 1.0], [3, 7], [[1.0, 2.0], [0.5, 2.0]], row_budget=40, fixed_row_equivalent=8.0)
    assert st == 1  # SG_ERR_INVALID_ARGUMENT
    assert alloc == (-1, -1)


def test_device_allocator_rejects_bad_shapes_on_host():
    with pytest.raises(ValueError, match="strictly increasing"):
        _device([1.0], [7, 3], [[1.0, 2.0]], row_budget=40, fixed_row_equivalent=8.0)
    with pytest.raises(ValueError, match="row budget"):
        _device([1.0, 1.0], [7], [[1.0], [1.0]], row_budget=10, fixed_row_equivalent=8.0)
