"""The folded-RMSNorm form of the verify pass (SG_NORM_FUSED=1: input and
post-attention norms inside the neighbouring GEMM epilogues) against the
default form on the same wave: per-node log-probs, lse and the last residual
stream agree within bf16 rounding.  The switch is read once per process, so
each form runs in its own child process."""
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
eng = B200Engine(w, num_slots=4, capacity=640, max_rows=256, max_requests=4)
eng.arena.storage.normal_(0.0, 1.0, generator=torch.Generator(device="cuda").manual_seed(2))
trees = [([-1, 0, 0, 1], [5, 6, 7, 8]), ([-1, 0], [9, 10]), ([-1] + list(range(39)), list(range(100, 140))),
         ([-1, 0, 1, 1, 2], [1, 2, 3, 4, 5])]
wave = Wave(trees, [2, 0, 3, 1], [100, 513, 37, 250])
Q = wave.num_rows
lse = torch.empty(Q, device="cuda"); child = torch.empty(Q, device="cuda")
hidden = torch.empty((Q, 512), device="cuda")
eng.verify(wave, seed=3, lse=lse, child_logprob=child, hidden_out=hidden, commit=False)
torch.cuda.synchronize()
assert int(eng.status.item()) == 0
print(json.dumps({"lse": lse.tolist(), "child": child.tolist(), "hidden": hidden.flatten()[::37].tolist()}))
"""


def _run(fused: str):
    env = dict(os.environ, SG_NORM_FUSED=fused)
    out = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_folded_norms_match_norm_kernels():
    a, b = _run("0"), _run("1")
    # two bf16 forms (activations rounded before vs after the norm's row
    # scale): their gap is the sum of their roundings, each about 1e-2 of a
    # log-prob at this shape, so twice the per-path bound on the maximum
    for key in ("child", "lse"):
        gap = np.abs(np.array(a[key]) - np.array(b[key]))
        assert gap.max() < 4e-2 and gap.mean() < 1e-2, (key, gap.max(), gap.mean())
    ha, hb = np.array(a["hidden"]), np.array(b["hidden"])
    assert np.max(np.abs(ha - hb)) < 3e-2 * np.max(np.abs(ha))
