"""The drafter-step case of tests/golden/dflash_step.npz: a tiny DFlash
configuration, its weights and inputs regenerated from a seed (the same
recipe tests/golden/make_golden.py loads into the reference model)."""
from __future__ import annotations

from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden" / "dflash_step.npz"

CONFIG = dict(vocab=96, hidden=64, intermediate=128, num_layers=2, num_q_heads=4, num_kv_heads=2, head_dim=16,
              rms_eps=1e-6, rope_theta=10000.0, block=4, feature_layers=3, mask_token=95)
SEED = 20261204
# per request: context rows of the first and second drafter step
UPDATES = [(5, 2), (3, 4)]
ANCHORS = [(7, 11), (42, 3)]


def weight_names() -> list[tuple[str, tuple[int, ...], str]]:
    c = CONFIG
    H, I, D = c["hidden"], c["intermediate"], c["head_dim"]
    nq, nkv, V, F = c["num_q_heads"], c["num_kv_heads"], c["vocab"], c["feature_layers"]
    names = [("embed", (V, H), "emb"), ("lm_head", (V, H), "emb"), ("fc", (H, F * H), "mat"),
             ("hidden_norm", (H,), "norm"), ("norm", (H,), "norm")]
    for l in range(c["num_layers"]):
        names += [(f"layers.{l}.in_norm", (H,), "norm"), (f"layers.{l}.q", (nq * D, H), "mat"),
                  (f"layers.{l}.k", (nkv * D, H), "mat"), (f"layers.{l}.v", (nkv * D, H), "mat"),
                  (f"layers.{l}.q_norm", (D,), "norm"), (f"layers.{l}.k_norm", (D,), "norm"),
                  (f"layers.{l}.o", (H, nq * D), "mat"), (f"layers.{l}.post_norm", (H,), "norm"),
                  (f"layers.{l}.gate", (I, H), "mat"), (f"layers.{l}.up", (I, H), "mat"),
                  (f"layers.{l}.down", (H, I), "mat")]
    return names


def make_weights_and_inputs():
    g = torch.Generator().manual_seed(SEED)
    w = {}
    for name, shape, kind in weight_names():
        t = torch.randn(shape, generator=g, dtype=torch.float32)
        w[name] = {"emb": 0.5 * t, "mat": 0.15 * t, "norm": 1.0 + 0.1 * t}[kind]
    F, H = CONFIG["feature_layers"], CONFIG["hidden"]
    features = [[torch.randn((u, F * H), generator=g, dtype=torch.float32) for u in steps] for steps in UPDATES]
    return w, features


def inv_freq() -> torch.Tensor:
    D, theta = CONFIG["head_dim"], CONFIG["rope_theta"]
    return 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
