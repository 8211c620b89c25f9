"""The draft-tree cases of tests/golden/draft_trees.npz, with their proposal
logits regenerated from the stored seeds (as tests/golden/make_golden.py
made them) and checked against the stored checksum."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden" / "draft_trees.npz"


def regenerate_logits(seed: int, L: int, V: int, kind: str) -> torch.Tensor:
    logits = torch.randn((L, V), generator=torch.Generator().manual_seed(seed), dtype=torch.float32) * 3.0
    if kind == "spine":
        logits[:, 0] += 30.0
    elif kind == "repeat":
        logits[:] = logits[0]
    return logits


def load_cases(with_logits: bool = True) -> list[dict]:
    z = np.load(GOLDEN)
    cases = []
    for i in range(int(z["count"])):
        p = f"c{i}_"
        L, V, budget, K, adaptive_min = (int(v) for v in z[p + "meta"])
        c = dict(L=L, V=V, budget=budget, K=K, temperature=float(z[p + "temperature"]),
                 adaptive_min=None if adaptive_min < 0 else adaptive_min,
                 threshold=None if adaptive_min < 0 else float(z[p + "threshold"]),
                 rewards=None if z[p + "rewards"].size == 0 else z[p + "rewards"],
                 caps=None if z[p + "caps"].size == 0 else z[p + "caps"],
                 logs=z[p + "logs"], ids=z[p + "ids"], tokens=z[p + "tokens"], parents=z[p + "parents"],
                 depths=z[p + "depths"], masses=z[p + "masses"], tiers=z[p + "tiers"],
                 utilities=z[p + "utilities"], kind=str(z[p + "kind"]))
        if with_logits:
            logits = regenerate_logits(int(z[p + "seed"]), L, V, c["kind"])
            checksum = [logits.double().sum().item(), logits.double().abs().max().item()]
            assert np.allclose(checksum, z[p + "logit_checksum"], rtol=0, atol=1e-6), "regenerated logits drifted"
            c["logits"] = logits.numpy()
        cases.append(c)
    return cases
