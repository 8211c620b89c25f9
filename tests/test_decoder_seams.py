"""The B200 seams fit the reference decoder's own attributes: every name that
``decoder_seams.install`` swaps exists in the reference's
``continuous_tree_block_decode`` module, with the same leading parameters, and
is restored on exit.  Runs where the reference checkout is present (the build
container); CPU only, nothing is executed on a device."""
import inspect
import sys
from pathlib import Path

import pytest

REFERENCE_SRC = Path("/root/reference/code/natural/src")
pytestmark = pytest.mark.skipif(not REFERENCE_SRC.is_dir(), reason="reference checkout not present")


@pytest.fixture(scope="module")
def decoder():
    sys.path.insert(0, str(REFERENCE_SRC))
    try:
        import gbv_experiments.continuous_tree_block_decode as module
    finally:
        sys.path.remove(str(REFERENCE_SRC))
    return module


def _params(fn):
    return [p.name for p in inspect.signature(fn).parameters.values()
            if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]


def test_seams_exist_with_matching_signatures(decoder):
    from specgrove_b200 import decoder_seams as seams
    for name in seams.VERIFIER_SEAMS:
        ref = _params(getattr(decoder, name))
        ours = _params(getattr(seams, name))
        assert ours[:len(ref)] == ref, (name, ref, ours)
    assert _params(decoder._pack_cache_sequence) == ["caches", "cache_factory", "device"]
    assert _params(seams.pack_cache_sequence) == ["caches", "cache_factory", "device"]
    pool_params = _params(decoder._PersistentRequestCachePool.__init__)[1:]
    assert _params(seams.arena_pool) == pool_params
    # the arena exposes what the decoder reads from the reference pool
    from specgrove_b200.arena import PersistentKVArena
    for member in ("caches", "lengths", "key_storage", "value_storage", "capacity"):
        assert member in PersistentKVArena.__init__.__code__.co_names or hasattr(PersistentKVArena, member)
    ref_append = _params(decoder._PersistentRequestCachePool.append_packed_sequence)
    assert _params(PersistentKVArena.append_packed_sequence)[:len(ref_append)] == ref_append


def test_install_swaps_and_restores(decoder):
    from specgrove_b200 import decoder_seams as seams
    names = ["_PersistentRequestCachePool", "_pack_cache_sequence", *seams.VERIFIER_SEAMS]
    before = {n: getattr(decoder, n) for n in names}
    with seams.install(decoder):
        assert decoder._pack_cache_sequence is seams.pack_cache_sequence
        assert decoder._PersistentRequestCachePool is seams.arena_pool
        for n in seams.VERIFIER_SEAMS:
            assert getattr(decoder, n) is getattr(seams, n)
    assert {n: getattr(decoder, n) for n in names} == before


def test_engine_wrapper_forwards_other_members():
    from specgrove_b200.decoder_seams import B200VerifyEngine

    class Base:
        device = "cpu"
        draft = object()

        def cache_factory(self):
            return "cache"

        def target_hidden_forward(self, ids, cache, *, positions=None, mask=None):
            return ("base", ids, cache)

    w = object.__new__(B200VerifyEngine)
    w._base = Base()
    w._engines = {}
    assert w.cache_factory() == "cache" and w.draft is Base.draft
    assert w.target_hidden_forward(1, "prefill-cache") == ("base", 1, "prefill-cache")
