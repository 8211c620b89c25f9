"""The on-device speculative loop (SpecDecoder): admission (chunked target
prefill + draft-cache prefill), then steps of drafter -> wave plan -> verify
-> commit.  Checks the caches' invariant (draft cache + pending update =
target cache = prompt + generated - 1), the first token against the target's
own prefill sampling, and that a second run with the same seeds generates the
same tokens."""
import pytest
import torch

from specgrove_b200.drafter import B200Drafter, DraftShape, DraftWeights
from specgrove_b200.engine import B200Engine, ModelShape, Wave, Weights
from specgrove_b200.speculative import SpecDecoder, SpecRequest

pytestmark = pytest.mark.gpu

SHAPE = ModelShape(4, 256, 4, 2, 64, 768, 4096)
DSHAPE = DraftShape(2, 256, 4, 2, 64, 768, 4096, num_feature_layers=3, block_size=8, mask_token_id=4095)
FEATURES = [0, 2, 3]


def build(seed=0):
    target_w = Weights.random(SHAPE, seed=11, std=0.08)
    draft_w = DraftWeights.random(DSHAPE, target_w, seed=12, std=0.08)
    target = B200Engine(target_w, num_slots=4, capacity=1024, max_rows=512, max_requests=4)
    drafter = B200Drafter(draft_w, num_slots=4, capacity=1024, max_requests=4, max_update_rows=512)
    dec = SpecDecoder(target, drafter, FEATURES, tiers=[3, 7], row_budget=32, temperature=1.0,
                      fixed_row_equivalent=8.0, seed=seed)
    return dec


def prompts():
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, 4000, (n,), generator=g).tolist() for n in (20, 300, 70)]


def run(steps=6):
    dec = build(seed=5)
    reqs = [SpecRequest(100 + i, p, max_new_tokens=40) for i, p in enumerate(prompts())]
    dec.admit(reqs)
    for r in reqs:
        assert dec.target.arena.lengths[r.slot] == len(r.prompt)
        assert dec.drafter.arena.lengths[r.slot] == len(r.prompt)
        assert len(r.generated) == 1
    first = [r.generated[0] for r in reqs]
    for _ in range(steps):
        produced = dec.step()
        assert produced >= len(dec.running)
        for r in reqs:
            if r.done:
                continue
            t_len = dec.target.arena.lengths[r.slot]
            assert t_len == len(r.prompt) + len(r.generated) - 1
            a, b = r.update
            assert dec.drafter.arena.lengths[r.slot] + (b - a) == t_len
            assert all(0 <= tok < SHAPE.vocab for tok in r.generated)
    return reqs, first, dec


def test_speculative_loop_invariants_and_determinism():
    reqs, first, dec = run()
    again, first2, _ = run()
    assert first == first2
    assert [r.generated for r in reqs] == [r.generated for r in again]
    # every request advanced by at least one token per step
    assert all(len(r.generated) >= 1 + 6 for r in reqs)


def test_first_token_is_the_prefill_draw():
    """The first generated token is the target's posterior draw at the last
    prompt row, the same draw a plain chain wave over the whole prompt makes."""
    dec = build(seed=5)
    p = prompts()[0]
    req = SpecRequest(100, p, max_new_tokens=4)
    dec.admit([req])
    engine = B200Engine(dec.target.weights, num_slots=1, capacity=1024, max_rows=512, max_requests=1)
    post = torch.empty(len(p), dtype=torch.long, device="cuda")
    wave = Wave([([-1] + list(range(len(p) - 1)), p)], [0], [0], request_ids=[100])
    engine.verify_device(wave.to("cuda"), seed=5, temperature=1.0, commit=False, posterior=post)
    torch.cuda.synchronize()
    assert req.generated[0] == int(post[-1])


def test_spec_server_serves_every_request():
    """One rank's open-loop server on the speculative loop: every arrival is
    admitted (real prefill), served to exactly max_new_tokens and releases its
    slot; the score exchange runs once per loop iteration."""
    from specgrove_b200.allocator import ScoreExchange
    from specgrove_b200.serving import SpecServer, make_prompts, make_requests
    dec = build(seed=9)
    requests = make_requests(7, 2000.0, (16, 200), [4, 8], SHAPE.vocab, seed=4)
    prompts = make_prompts(requests, SHAPE.vocab, seed=8)
    server = SpecServer(requests, dec, prompts, rank=0, world=1, exchange=ScoreExchange(4, 2, "cuda"), num_tiers=2,
                        max_new_tokens=24, max_admit_per_wave=3)
    stats = server.run()
    assert stats.requests == 7
    assert stats.tokens == 7 * 24
    assert all(r.generated == 24 and r.finish is not None for r in requests)
    assert sorted(dec.free_slots) == [0, 1, 2, 3]
    assert not dec.running
    assert stats.exchanges >= stats.waves


def test_multi_chunk_prefill_wave_matches_chunk_per_wave():
    """A 700-token prompt prefilled as three chain chunks of one slot in a
    single wave writes the same target and draft-cache K/V (bf16 rounding of
    a different attention tiling aside) and samples the same greedy first
    token as one chunk per wave."""
    prompt = torch.randint(0, 4000, (700,), generator=torch.Generator().manual_seed(9)).tolist()

    def run(max_rows):
        target_w = Weights.random(SHAPE, seed=11, std=0.08)
        draft_w = DraftWeights.random(DSHAPE, target_w, seed=12, std=0.08)
        target = B200Engine(target_w, num_slots=2, capacity=1024, max_rows=max_rows, max_requests=4)
        drafter = B200Drafter(draft_w, num_slots=2, capacity=1024, max_requests=4, max_update_rows=1024)
        dec = SpecDecoder(target, drafter, FEATURES, tiers=[3, 7], row_budget=32, temperature=0.0,
                          fixed_row_equivalent=8.0, seed=3)
        req = SpecRequest(7, prompt, max_new_tokens=4)
        dec.admit([req])
        torch.cuda.synchronize()
        s = req.slot
        cap = target.arena.capacity
        kv_t = target.arena.storage[:, :, :, s * cap:s * cap + 700].float().cpu()
        kv_d = drafter.arena.storage[:, :, :, s * cap:s * cap + 700].float().cpu()
        return req.generated[0], kv_t, kv_d, target.arena.lengths[s], drafter.arena.lengths[s]

    one_wave = run(1024)      # 256 + 256 + 188 rows in one wave
    per_wave = run(256)       # one 256-row chunk per wave
    assert one_wave[3] == per_wave[3] == 700 and one_wave[4] == per_wave[4] == 700
    for a, b in ((one_wave[1], per_wave[1]), (one_wave[2], per_wave[2])):
        assert (a - b).abs().max().item() <= 2e-2 * b.abs().max().item()
    assert one_wave[0] == per_wave[0]
