"""sg_lm_head_sample_static: the sampling head for callers that cannot call
cudaMalloc (a host whose device memory belongs to its own pool allocator, or
an FFI caller that only hands over its own buffers).  Its scratch is a
library-owned static device array, so the test checks, through the C ABI,
that two calls in a row reproduce the sampling stage of sg_verify_pass (the
existing entry point) on the same residual rows: identical posterior tokens
and log-normalisers within the tests' tolerance.  It must pass alone in a
fresh process (the first call resolves the array's device address) and
after the rest of the suite."""
import ctypes

import numpy as np
import pytest
import torch

from specgrove_b200 import _lib
from specgrove_b200._lib import ptr, stream_ptr
from specgrove_b200.engine import B200Engine, ModelShape, Wave, Weights
from specgrove_b200.workloads import random_topology

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _wave(rng, vocab, count, lo, hi):
    trees, lengths = [], []
    for _ in range(count):
        n = int(rng.integers(lo, hi + 1))
        parents, _ = random_topology(rng, n, 8, 4)
        tokens, seen = [int(rng.integers(0, vocab))], set()
        for j in range(1, n):
            t = int(rng.integers(0, vocab))
            while (parents[j], t) in seen:
                t = int(rng.integers(0, vocab))
            seen.add((parents[j], t))
            tokens.append(t)
        trees.append((parents, tokens))
        lengths.append(int(rng.integers(8, 64)))
    return trees, lengths


def _row_keys(trees, request_ids):
    nodes, reqs = [], []
    for (parents, _), rid in zip(trees, request_ids):
        nodes += list(range(len(parents)))
        reqs += [rid] * len(parents)
    return (torch.tensor(nodes, dtype=torch.int32, device="cuda"),
            torch.tensor(reqs, dtype=torch.long, device="cuda"))


def test_static_scratch_sampler_matches_verify_pass(cuda_lib):
    shape = ModelShape(2, 512, 8, 2, 128, 1024, 4096)
    weights = Weights.random(shape, seed=7, std=0.05)
    engine = B200Engine(weights, num_slots=6, capacity=128, max_rows=256)
    engine.arena.storage.normal_(0.0, 1.0)
    lib = _lib.load()
    rng = np.random.default_rng(11)
    for call, (count, seed, temperature) in enumerate([(6, 1234, 1.0), (3, 98765, 0.7), (5, 4321, 0.0)]):
        trees, lengths = _wave(rng, shape.vocab, count, 4, 40)
        request_ids = [100 * call + i for i in range(count)]
        wave = Wave(trees, list(range(count)), lengths, request_ids=request_ids)
        Q = wave.num_rows
        lse_ref = torch.empty(Q, device="cuda")
        post_ref = torch.empty(Q, dtype=torch.long, device="cuda")
        hidden = torch.empty((Q, shape.hidden), device="cuda")
        engine.verify_device(wave.to("cuda"), seed=seed, temperature=temperature, commit=False, lse=lse_ref,
                             posterior=post_ref, hidden_out=hidden)
        nodes, reqs = _row_keys(trees, request_ids)
        lse = torch.full((Q,), float("nan"), device="cuda")
        post = torch.full((Q,), -1, dtype=torch.long, device="cuda")
        torch.cuda.synchronize()
        if call > 0:   # everything this call needs is allocated by now
            free_before, reserved_before = torch.cuda.mem_get_info()[0], torch.cuda.memory_reserved()
        st = lib.sg_lm_head_sample_static(ptr(hidden), ptr(weights.final_norm), ptr(weights.lm_head), Q, shape.hidden,
                                          shape.vocab, ctypes.c_float(shape.rms_eps), ptr(nodes), ptr(reqs), seed,
                                          ctypes.c_float(temperature), ptr(lse), ptr(post), stream_ptr())
        assert st == 0, lib.sg_last_error()
        torch.cuda.synchronize()
        if call > 0:
            # the call itself allocated nothing: device free memory and the
            # caching allocator's reservation are unchanged across it
            assert torch.cuda.mem_get_info()[0] == free_before
            assert torch.cuda.memory_reserved() == reserved_before
        assert int(engine.status) == 0
        assert torch.equal(post, post_ref), call
        torch.testing.assert_close(lse, lse_ref, rtol=0.0, atol=TOL)


def test_static_scratch_rejects_misaligned_rows(cuda_lib):
    """A residual-row pointer that is not 16-byte aligned (a row slice at an
    odd float offset) is refused before any launch instead of faulting."""
    lib = _lib.load()
    x = torch.zeros((4, 512), device="cuda")
    small = torch.zeros(16384, device="cuda")   # covers a 32 x 512 bf16 LM head
    nodes = torch.zeros(4, dtype=torch.int32, device="cuda")
    reqs = torch.zeros(4, dtype=torch.long, device="cuda")
    lse = torch.empty(4, device="cuda")
    post = torch.empty(4, dtype=torch.long, device="cuda")
    st = lib.sg_lm_head_sample_static(x.data_ptr() + 4, ptr(small), ptr(small), 3, 512, 32, ctypes.c_float(1e-6),
                                      ptr(nodes), ptr(reqs), 0, ctypes.c_float(1.0), ptr(lse), ptr(post),
                                      stream_ptr())
    assert st == _lib.SG_ERR_INVALID_ARGUMENT
    assert b"misaligned" in lib.sg_last_error()
    torch.cuda.synchronize()


def test_static_scratch_rejects_oversized_requests(cuda_lib):
    lib = _lib.load()
    rows, hidden, vocab = 4096, 4096, 151936  # ~72 MB of scratch, above the static array
    dummy = torch.empty(16, device="cuda")
    st = lib.sg_lm_head_sample_static(ptr(dummy), ptr(dummy), ptr(dummy), rows, hidden, vocab, ctypes.c_float(1e-6),
                                      ptr(dummy), ptr(dummy), 0, ctypes.c_float(1.0), ptr(dummy), ptr(dummy),
                                      stream_ptr())
    assert st == _lib.SG_ERR_WORKSPACE
    assert b"static" in lib.sg_last_error()
