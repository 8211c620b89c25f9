"""Per-node log-prob parity of the packed verify pass at the Qwen3-8B
geometry (hidden 4096, 32 q / 8 kv heads, head_dim 128, intermediate 12288,
vocab 151936; 2 layers so the models fit in a few GB) with prefixes up to 4096
tokens (32 key tiles) and the benchmark's tiers of 16, 32, 64 and 128 rows
(up to 4 query blocks per kv head).

References, as in the north-star bound "per-node fp32 log-probs within 2e-2
max abs of the reference's BF16-SDPA path":
* the reference's target path: HF ``Qwen3Model`` in bf16 with SDPA, loaded
  the way the reference loads its target (bf16 weights, fp32 rotary
  frequencies; engine.py:270-282), fed the packed DynamicCache and dense tree
  mask of ``_packed_block_inputs`` (continuous_tree_block_decode.py:500-546),
  then ``log_softmax(lm_head(h).float())`` (:1809-1824);
* the fp32 truth: the oracle's torch fp32 restatement of the same pass.
The audit follows serving scripts/audit_bf16_posterior_paths_h20.py:179-220
(both paths against a common exact reference, max and mean gaps).
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from specgrove_b200 import _lib
from specgrove_b200._lib import ptr, stream_ptr
from specgrove_b200.engine import B200Engine, Wave, Weights
from specgrove_b200.workloads import random_topology
from test_verify_pass_gpu import fp32_truth_logprobs, hf_wave_logprobs, node_index

pytestmark = pytest.mark.gpu

TOL = 2e-2          # north-star bound on per-node log-probs (max abs)
VOCAB = 151936


@pytest.fixture(scope="module")
def model8b():
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=VOCAB, hidden_size=4096, intermediate_size=12288, num_hidden_layers=2,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1.0e6,
                      max_position_embeddings=40960, tie_word_embeddings=False, rms_norm_eps=1e-6,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM._from_config(cfg, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(8)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.uniform_(0.8, 1.2, generator=g)
            elif "embed" in name:
                p.normal_(0.0, 1.0, generator=g)
            else:
                p.normal_(0.0, 1.0 / math.sqrt(p.shape[1]), generator=g)
    return model.eval()


def tier_trees(rng, sizes, vocab):
    trees = []
    for n in sizes:
        parents, _ = random_topology(rng, n, 16, 4)
        tokens, kids = [int(rng.integers(0, vocab))], {}
        for j in range(1, n):
            used = kids.setdefault(parents[j], set())
            t = int(rng.integers(0, vocab))
            while t in used:
                t = int(rng.integers(0, vocab))
            used.add(t)
            tokens.append(t)
        trees.append((parents, tokens))
    return trees


def test_logprobs_at_qwen3_8b_geometry(cuda_lib, model8b):
    rng = np.random.default_rng(21)
    lengths = [4096, 1024, 2600, 512]
    prompts = [rng.integers(0, VOCAB, size=L).tolist() for L in lengths]
    trees = tier_trees(rng, [128, 64, 32, 16], VOCAB)
    hf_lp, _ = hf_wave_logprobs(model8b, prompts, trees)
    weights = Weights.from_hf(model8b)
    truth_lp, truth_lse = fp32_truth_logprobs(weights, prompts, trees)

    cap = 4096 + 256
    engine = B200Engine(weights, num_slots=4, capacity=cap, max_rows=512)
    slots = [2, 0, 3, 1]
    engine.prefill(prompts, slots)
    wave = Wave(trees, slots, lengths, request_ids=[11, 12, 13, 14])
    Q = wave.num_rows
    lse = torch.empty(Q, device="cuda")
    child = torch.empty(Q, device="cuda")
    post = torch.empty(Q, dtype=torch.long, device="cuda")
    hidden = torch.empty((Q, 4096), device="cuda")
    engine.verify(wave, seed=99, lse=lse, child_logprob=child, posterior=post, hidden_out=hidden, commit=False)
    torch.cuda.synchronize()
    pr, tk, rows = node_index(trees)
    ours, hf, truth = child[rows], hf_lp[pr, tk], truth_lp[pr, tk]
    err_ours = (ours - truth).abs()
    err_ref = (hf - truth).abs()
    gap = (ours - hf).abs()
    print(f"\n8B geometry, {len(rows)} nodes: B200 vs fp32 truth max {err_ours.max():.4f} mean {err_ours.mean():.5f}; "
          f"reference BF16-SDPA vs truth max {err_ref.max():.4f} mean {err_ref.mean():.5f}; "
          f"B200 vs reference max {gap.max():.4f} mean {gap.mean():.5f}; "
          f"lse vs truth max {(lse - truth_lse).abs().max():.5f}")
    assert err_ours.max().item() <= TOL                      # the bound, against the exact path
    assert err_ours.max().item() <= err_ref.max().item()     # at least as accurate as the reference path
    assert gap.mean().item() <= TOL / 2
    if err_ref.max().item() <= TOL / 2:                      # the reference path's own rounding leaves room
        assert gap.max().item() <= TOL
    assert (lse - truth_lse).abs().max().item() < TOL

    # the pass's sampler at the benchmark vocabulary equals the stand-alone
    # sampler on the same residual rows (same kernels, same keys)
    lib = _lib.load()
    nodes = torch.tensor([j for par, _ in trees for j in range(len(par))], dtype=torch.int32, device="cuda")
    reqs = torch.tensor([11 + i for i, (par, _) in enumerate(trees) for _ in par], dtype=torch.long, device="cuda")
    nbytes = lib.sg_lm_head_sample_workspace_bytes(Q, 4096, VOCAB)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    lse2 = torch.empty(Q, device="cuda")
    post2 = torch.empty(Q, dtype=torch.long, device="cuda")
    st = lib.sg_lm_head_sample(ptr(hidden), ptr(weights.final_norm), ptr(weights.lm_head), Q, 4096, VOCAB,
                               ctypes.c_float(weights.shape.rms_eps), ptr(nodes), ptr(reqs), 99, ctypes.c_float(1.0),
                               ptr(lse2), ptr(post2), ptr(ws), nbytes, stream_ptr())
    assert st == 0, lib.sg_last_error()
    torch.cuda.synchronize()
    assert torch.equal(post, post2)
    assert torch.equal(lse, lse2)
