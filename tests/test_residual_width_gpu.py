"""The verify pass with its residual (O and down) projections on 160- and
256-column tiles (SG_RESIDUAL_BN pins the width the pass would otherwise
pick per wave) gives the same per-node log-probs, lse and residual stream:
the tile width changes which CTA computes an output column, not the order
of its k-accumulation.  The switch is read once per process, so each width
runs in its own child process."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import json, sys, torch
sys.path.insert(0, sys.argv[1])
from specgrove_b200.engine import B200Engine, ModelShape, Wave, Weights
shape = ModelShape(2, 512, 8, 2, 128, 1024, 4096)
w = Weights.random(shape, seed=5, std=0.05)
eng = B200Engine(w, num_slots=4, capacity=640, max_rows=512, max_requests=4)
eng.arena.storage.normal_(0.0, 1.0, generator=torch.Generator(device="cuda").manual_seed(2))
trees = [([-1, 0, 0, 1], [5, 6, 7, 8]), ([-1, 0], [9, 10]), ([-1] + list(range(199)), list(range(100, 300))),
         ([-1, 0, 1, 1, 2], [1, 2, 3, 4, 5])]
wave = Wave(trees, [2, 0, 3, 1], [100, 313, 37, 250])
Q = wave.num_rows
lse = torch.empty(Q, device="cuda"); child = torch.empty(Q, device="cuda")
hidden = torch.empty((Q, 512), device="cuda")
eng.verify(wave, seed=3, lse=lse, child_logprob=child, hidden_out=hidden, commit=False)
torch.cuda.synchronize()
assert int(eng.status.item()) == 0
print(json.dumps({"lse": lse.tolist(), "child": child.tolist(), "hidden": hidden.flatten()[::7].tolist()}))
"""


def _run(width: str):
    env = dict(os.environ, SG_RESIDUAL_BN=width)
    out = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_residual_tile_widths_agree():
    a, b = _run("160"), _run("256")
    for key in ("lse", "child", "hidden"):
        x, y = np.array(a[key]), np.array(b[key])
        assert np.allclose(x, y, rtol=1e-6, atol=1e-6), (key, np.abs(x - y).max())
