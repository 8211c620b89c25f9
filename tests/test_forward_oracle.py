"""Pin the CPU restatement of the verify pass (oracle/forward.py) against HF
Qwen3 (fp32, CPU) fed the reference's packed cache and dense tree mask."""
import math

import numpy as np
import torch

from oracle.forward import CpuWeights, verify_logits, verify_step
from oracle.packed_inputs import packed_block_inputs


def _model(seed=0):
    from transformers import DynamicCache, Qwen3Config, Qwen3ForCausalLM  # noqa: F401
    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=1.0e6,
                      max_position_embeddings=4096, tie_word_embeddings=False, attn_implementation="sdpa")
    m = Qwen3ForCausalLM(cfg).eval()
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "norm" in name:
                p.uniform_(0.8, 1.2)
            elif "embed" in name:
                p.normal_(0, 1)
            else:
                p.normal_(0, 1 / math.sqrt(p.shape[1]))
            p.copy_(p.bfloat16().float())  # bf16-representable, as engine weights are
    return m


def test_cpu_forward_matches_hf_packed_mask():
    from transformers import DynamicCache
    from specgrove_b200.engine import Weights
    model = _model()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 512, size=n).tolist() for n in (20, 35, 9)]
    trees = [([-1, 0, 0, 1, 3], [7, 8, 9, 10, 11]), ([-1], [5]), ([-1, 0, 1, 1], [1, 2, 3, 4])]
    caches = []
    with torch.no_grad():
        for p in prompts:
            c = DynamicCache()
            model(input_ids=torch.tensor([p]), past_key_values=c, use_cache=True)
            caches.append(c)
        packed = DynamicCache()
        for l in range(2):
            packed.update(torch.cat([c.layers[l].keys for c in caches], -2),
                          torch.cat([c.layers[l].values for c in caches], -2), l)
        lengths = [len(p) for p in prompts]
        ids, pos, mask, _ = packed_block_inputs(trees, lengths, lengths)
        ref = model(input_ids=ids, past_key_values=packed, position_ids=pos, attention_mask=mask).logits[0]
    cw = CpuWeights(Weights.from_hf(model, device="cpu"))
    prefixes = [[(c.layers[l].keys[0], c.layers[l].values[0]) for l in range(2)] for c in caches]
    ours, offsets = verify_logits(cw, prefixes, trees, lengths)
    torch.testing.assert_close(ours, ref, rtol=1e-4, atol=2e-4)
    res, _ = verify_step(cw, prefixes, trees, lengths, uniforms=np.full((3, 4), 0.5))
    assert len(res) == 3 and all(0 <= bonus < 512 for _, bonus in res)
