"""Accepted-path KV commit on the GPU through the C ABI (bit-exact copies)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import cpu as oracle
from specgrove_b200.arena import PersistentKVArena

pytestmark = pytest.mark.gpu


def test_append_packed_sequence_matches_reference_pool(cuda_lib, golden_dir):
    z = np.load(golden_dir / "kv_commit.npz")
    layers, heads, rows, dim = z["before_k"].shape
    cap = int(z["capacity"])
    lengths = z["lengths"].tolist()
    sources = []
    for slot, L in enumerate(lengths):
        lay = [SimpleNamespace(keys=torch.from_numpy(z["before_k"][l, :, slot * cap:slot * cap + L])[None].cuda(),
                               values=torch.from_numpy(z["before_v"][l, :, slot * cap:slot * cap + L])[None].cuda())
               for l in range(layers)]
        sources.append(SimpleNamespace(layers=lay, get_seq_length=(lambda L=L: L)))
    arena = PersistentKVArena.from_caches(sources, capacity=cap)
    packed = SimpleNamespace(layers=[
        SimpleNamespace(keys=torch.from_numpy(z["packed_k"][l])[None].cuda(),
                        values=torch.from_numpy(z["packed_v"][l])[None].cuda()) for l in range(layers)])
    ko = z["keep_offsets"]
    keep = [z["keep_flat"][ko[i]:ko[i + 1]].tolist() for i in range(len(lengths))]
    arena.append_packed_sequence(packed, arena.caches, int(z["packed_old_length"]),
                                 z["q_offsets"].tolist(), keep, "cuda")
    torch.cuda.synchronize()
    assert arena.lengths == z["after_lengths"].tolist()
    assert int(arena._status) == 0
    for slot in range(len(lengths)):
        n = arena.lengths[slot]
        for l in range(layers):
            got_k = arena.caches[slot].layers[l].keys[0].cpu().numpy()
            got_v = arena.caches[slot].layers[l].values[0].cpu().numpy()
            np.testing.assert_array_equal(got_k, z["after_k"][l, :, slot * cap:slot * cap + n])
            np.testing.assert_array_equal(got_v, z["after_v"][l, :, slot * cap:slot * cap + n])


def _random_keep(rng, rows):
    depth = int(rng.integers(0, min(rows, 17)))
    accepted = sorted(rng.choice(np.arange(1, rows), size=depth, replace=False).tolist()) if depth else []
    return [0] + accepted


@pytest.mark.parametrize("layers,heads,dim", [(36, 8, 128), (2, 2, 64), (3, 1, 8)])
def test_commit_tail_matches_oracle(cuda_lib, layers, heads, dim):
    rng = np.random.default_rng(layers * 100 + dim)
    slots, cap = 64 if layers == 36 else 5, 300
    arena = PersistentKVArena(layers, heads, dim, slots, cap, dtype=torch.bfloat16)
    arena.storage.copy_(torch.randn(arena.storage.shape, dtype=torch.bfloat16, device="cuda"))
    arena.lengths = [int(rng.integers(1, 150)) for _ in range(slots)]
    keep = [_random_keep(rng, int(rng.integers(1, 129))) for _ in range(slots)]
    before = arena.storage.view(torch.int16).cpu().numpy()
    expected = before.copy().reshape(layers * 2 * heads, slots * cap, dim)
    src_rows, dst_rows = [], []
    for slot, k in enumerate(keep):
        base = slot * cap + arena.lengths[slot]
        src_rows += [base + r for r in k]
        dst_rows += [base + i for i in range(len(k))]
    assert oracle.kv_commit(expected, expected, src_rows, dst_rows) == 0
    old = list(arena.lengths)
    arena.commit_tail(list(range(slots)), keep)
    torch.cuda.synchronize()
    got = arena.storage.view(torch.int16).cpu().numpy().reshape(expected.shape)
    np.testing.assert_array_equal(got, expected)
    assert arena.lengths == [o + len(k) for o, k in zip(old, keep)]
    assert int(arena._status) == 0


def test_capacity_exhaustion_raises(cuda_lib):
    arena = PersistentKVArena(1, 1, 8, 2, 4, dtype=torch.float32)
    arena.lengths = [3, 0]
    with pytest.raises(RuntimeError, match="capacity exhausted"):
        arena.commit_tail([0], [[0, 1]])
    assert arena.lengths == [3, 0]


def test_unaligned_rows_use_scalar_path(cuda_lib):
    # row of 3 fp32 = 12 bytes: not a multiple of 16 -> 4-byte units
    arena = PersistentKVArena(2, 2, 3, 2, 10, dtype=torch.float32)
    arena.storage.copy_(torch.arange(arena.storage.numel(), dtype=torch.float32,
                                     device="cuda").reshape(arena.storage.shape))
    arena.lengths = [2, 4]
    ref = arena.storage.cpu().numpy().reshape(8, 20, 3).copy()
    oracle.kv_commit(ref, ref, [2 + 0, 2 + 3, 14 + 0, 14 + 1], [2, 3, 14, 15])
    arena.commit_tail([0, 1], [[0, 3], [0, 1]])
    np.testing.assert_array_equal(arena.storage.cpu().numpy().reshape(8, 20, 3), ref)


def test_commit_from_accept_output_matches_oracle(cuda_lib):
    from specgrove_b200 import _lib
    from specgrove_b200._lib import ptr, stream_ptr
    rng = np.random.default_rng(4)
    layers, heads, dim, slots, cap, D = 4, 8, 128, 16, 200, 6
    arena = PersistentKVArena(layers, heads, dim, slots, cap, dtype=torch.bfloat16)
    arena.storage.copy_(torch.randn(arena.storage.shape, dtype=torch.bfloat16, device="cuda"))
    order = rng.permutation(slots)[:12]                       # trees -> slots
    lengths = rng.integers(10, 150, size=12)
    out = np.full((12, D + 2), -1, np.int64)
    keeps = []
    for t in range(12):
        keep = _random_keep(rng, 40)[:D + 1]
        out[t, :len(keep) - 1] = keep[1:]
        out[t, D] = len(keep) - 1
        out[t, D + 1] = 7
        keeps.append(keep)
    expected = arena.storage.view(torch.int16).cpu().numpy().reshape(layers * 2 * heads, slots * cap, dim).copy()
    src_rows, dst_rows = [], []
    for t, keep in enumerate(keeps):
        base = int(order[t]) * cap + int(lengths[t])
        src_rows += [base + r for r in keep]
        dst_rows += [base + i for i in range(len(keep))]
    oracle.kv_commit(expected, expected, src_rows, dst_rows)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int64)).cuda()
    slots_d, len_in, len_out, out_d = dev(order), dev(lengths), torch.empty(12, dtype=torch.long, device="cuda"), dev(out)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _lib.load().sg_kv_commit_accepted(
        ptr(arena.storage), arena.plane_rows, arena.num_planes, arena.row_bytes, cap, ptr(slots_d),
        ptr(len_in), ptr(len_out), ptr(out_d), 12, D, ptr(status), stream_ptr())
    assert st == 0
    torch.cuda.synchronize()
    assert int(status) == 0
    np.testing.assert_array_equal(arena.storage.view(torch.int16).cpu().numpy().reshape(expected.shape), expected)
    assert len_out.cpu().tolist() == [int(l) + len(k) for l, k in zip(lengths, keeps)]


def test_commit_rejects_a_non_root_path_without_moving_rows(cuda_lib):
    """A path whose node at depth r lies below r (not a root path of the
    slot's tail) is reported as SG_ERR_TREE and leaves that tree's rows as
    they were; the other trees of the launch commit normally."""
    from specgrove_b200 import _lib
    from specgrove_b200._lib import SG_ERR_TREE, ptr, stream_ptr
    layers, heads, dim, slots, cap, D = 2, 4, 128, 4, 64, 4
    arena = PersistentKVArena(layers, heads, dim, slots, cap, dtype=torch.bfloat16)
    arena.storage.copy_(torch.randn(arena.storage.shape, dtype=torch.bfloat16, device="cuda"))
    before = arena.storage.view(torch.int16).cpu().numpy().reshape(layers * 2 * heads, slots * cap, dim).copy()
    out = np.full((2, D + 2), -1, np.int64)
    out[0, :3] = [3, 1, 5]          # depth 2 holds node 1 < 2: not a root path
    out[0, D], out[0, D + 1] = 3, 9
    out[1, :2] = [2, 4]             # a valid path in slot 1
    out[1, D], out[1, D + 1] = 2, 9
    lengths = np.array([10, 20], np.int64)
    expected = before.copy()
    base = 1 * cap + 20
    oracle.kv_commit(expected, expected, [base + r for r in (0, 2, 4)], [base + i for i in range(3)])
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int64)).cuda()
    # device arrays stay bound until the kernel has run
    slots_d, len_in, out_d = dev([0, 1]), dev(lengths), dev(out)
    len_out = torch.empty(2, dtype=torch.long, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _lib.load().sg_kv_commit_accepted(
        ptr(arena.storage), arena.plane_rows, arena.num_planes, arena.row_bytes, cap, ptr(slots_d),
        ptr(len_in), ptr(len_out), ptr(out_d), 2, D, ptr(status), stream_ptr())
    assert st == 0
    torch.cuda.synchronize()
    assert int(status) == SG_ERR_TREE
    got = arena.storage.view(torch.int16).cpu().numpy().reshape(expected.shape)
    np.testing.assert_array_equal(got, expected)
