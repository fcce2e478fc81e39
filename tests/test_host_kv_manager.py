"""Host KVManager vs the reference KVManager (miniprefix/src/kv/kv_manager.cpp).

Random operation sequences (reservations, create/fork/reuse/publish, Append
transactions with commit, rollback and a failing copier, reset, release, clear)
run on both; after EVERY operation the result, the exception class and message,
the 16 KvStats fields and every sequence's (used, pages) must be identical.
The fixed scenarios of miniprefix/tests/kv_manager_test.cpp and cow_test.cpp
metadata() follow.
"""
import numpy as np
import pytest

from oracle.oracle import RefKV
from tinyinfer_b200.host import KVManager

IDS = ["a", "b", "c", "d", "e"]


def message(impl, rc):
    if rc >= 0:
        return None
    return impl.ref.error() if isinstance(impl, RefKV) else impl.error()


def compare(mine, theirs):
    assert mine.stats() == theirs.stats()
    for i in IDS:
        assert mine.sequence(i) == theirs.sequence(i), i


def random_op(rng, vocabulary, context):
    kind = int(rng.integers(0, 14))
    i = IDS[int(rng.integers(0, len(IDS)))]
    j = IDS[int(rng.integers(0, len(IDS)))]

    def tokens(lo=0, hi=6):
        n = int(rng.integers(lo, hi))
        # mostly a small alphabet so that prefixes collide; now and then an invalid token
        return [int(rng.integers(0, 3)) if rng.random() < 0.9 else int(rng.integers(-1, vocabulary + 2))
                for _ in range(n)]

    if kind == 0:
        return ("reserve", i, int(rng.integers(0, context + 3)))
    if kind == 1:
        return ("release_reservation", i)
    if kind in (2, 3):
        return ("create", i)
    if kind == 4:
        return ("fork", i, j)
    if kind == 5:
        return ("reuse_prefix", i, tokens(0, 10))
    if kind == 6:
        return ("cache_prefix", i)
    if kind == 7:
        return ("clear_prefix_cache",)
    if kind in (8, 9, 10):
        return ("append", i, tokens(0, 6), int(rng.choice([0, 0, 0, 1, 2])))
    if kind == 11:
        return ("reset_sequence", i)
    if kind == 12:
        return ("release", i)
    return ("clear",) if rng.random() < 0.2 else ("cache_prefix", i)


@pytest.mark.parametrize("seed", range(12))
def test_random_transactions_match_reference(built, ref, seed):
    rng = np.random.default_rng(1000 + seed)
    bt = int(rng.integers(1, 5))
    max_blocks = int(rng.integers(2, 13))
    cache = int(rng.integers(0, max_blocks + 1))
    context, vocabulary = 16, 8
    args = (bt, max_blocks, cache, 2, 3, context, vocabulary)
    mine, theirs = KVManager(*args), RefKV(ref, *args)
    for step in range(1500):
        op = random_op(rng, vocabulary, context)
        a = mine.call(*op)
        b = theirs.call(*op)
        assert a == b, (step, op, a, b, message(mine, a[0]), message(theirs, b[0]))
        assert message(mine, a[0]) == message(theirs, b[0]), (step, op)
        compare(mine, theirs)
    mine.close()
    theirs.close()


def run(impl, ops):
    out = []
    for op in ops:
        rc, res = impl.call(*op)
        out.append((rc, res))
    return out


def test_reservations_scenario(built, ref):
    """kv_manager_test.cpp:14-29"""
    for impl in (KVManager(2, 3, 3, 1, 1, 16, 100), RefKV(ref, 2, 3, 3, 1, 1, 16, 100)):
        assert impl.call("reserve", "too-big", 7)[1] == "Impossible"
        assert impl.call("reserve", "a", 4)[1] == "Ready"
        assert impl.call("reserve", "b", 4)[1] == "Wait"
        assert impl.stats()["kv_live_blocks"] == 0
        impl.call("create", "external")
        assert impl.call("append", "external", [1, 2], 0)[0] == 0
        assert impl.call("append", "external", [3], 0)[0] < 0
        impl.call("create", "a")
        assert impl.call("append", "a", [1, 2, 3, 4], 0)[0] == 0
        impl.call("cache_prefix", "a")
        assert impl.call("append", "a", [5], 0)[0] < 0
        impl.call("release", "a")
        assert impl.call("reserve", "b", 4)[1] == "Ready"
        impl.call("create", "b")
        assert impl.call("append", "b", [5, 6, 7, 8], 0)[0] == 0
        impl.call("clear")
        assert impl.call("reserve", "all", 6)[1] == "Ready"
        impl.call("release_reservation", "all")
        assert impl.call("reserve", "again", 6)[1] == "Ready"
        impl.call("clear")
        assert impl.stats()["kv_live_blocks"] == 0


def test_exhaustion_message_and_eviction_effects(built, ref):
    """kv_manager_test.cpp:119-150: validation precedes eviction; a rolled-back append
    keeps its eviction side effects; the exhaustion message is exact."""
    for impl in (KVManager(2, 2, 2, 1, 1, 8, 100), RefKV(ref, 2, 2, 2, 1, 1, 8, 100)):
        impl.call("create", "source")
        impl.call("append", "source", [1, 2, 3, 4], 0)
        impl.call("cache_prefix", "source")
        impl.call("release", "source")
        impl.call("create", "next")
        assert impl.call("append", "next", [100], 0)[0] == -1
        assert impl.call("append", "next", [1] * 9, 0)[0] == -1
        assert impl.stats()["prefix_evictions"] == 0 and impl.stats()["kv_cached_blocks"] == 2
        assert impl.call("append", "next", [5], 1)[0] == 0  # prepare then roll back
        st = impl.stats()
        assert st["prefix_evictions"] == 1 and st["kv_cached_blocks"] == 1 and st["kv_live_blocks"] == 1
        assert impl.call("append", "next", [5], 0)[0] == 0
        assert impl.stats()["prefix_evictions"] == 1
    for cache in (0, 2):
        impl = KVManager(2, 2, cache, 1, 1, 8, 100)
        impl.call("create", "source")
        impl.call("append", "source", [1, 2, 3, 4], 0)
        impl.call("cache_prefix", "source")
        impl.call("release", "source")
        impl.call("create", "next")
        rc, _ = impl.call("append", "next", [1, 2, 3, 4, 5], 0)
        assert rc == -3 and impl.error() == "paged KV block pool exhausted"
        assert impl.stats()["prefix_evictions"] == cache


def test_cow_metadata_scenario(built, ref):
    """cow_test.cpp:14-54: a forked partial tail copies on write; a failing copier
    blocks commit; rollback restores the shared page."""
    for impl in (KVManager(4, 4, 0, 2, 3, 16, 100), RefKV(ref, 4, 4, 0, 2, 3, 16, 100)):
        assert impl.call("reserve", "a", 8)[1] == "Ready"
        assert impl.call("reserve", "b", 8)[1] == "Ready"
        impl.call("create", "a")
        impl.call("create", "b")
        impl.call("append", "a", [1, 2, 3], 0)
        impl.call("fork", "a", "b")
        original = impl.sequence("b")
        assert impl.stats()["kv_live_blocks"] == 1
        assert impl.call("reserve", "third", 1)[1] == "Wait"
        rc, (tail, region) = impl.call("append", "b", [4, 5], 1)
        assert tail[2] == 3 and region == (tail[1] * 2 * 12, tail[0] * 2 * 12, 12, 9, 2)
        assert impl.sequence("b") == original
        rc, (tail, region) = impl.call("append", "b", [4, 5], 2)  # copier throws: commit refused
        assert rc == 0 and impl.sequence("b") == original and impl.stats()["kv_live_blocks"] == 1
        assert impl.call("append", "b", [4, 5], 0)[0] == 0
        assert impl.sequence("a") == original
        rc, (tail, _) = impl.call("append", "a", [6, 7], 0)
        assert tail == (-1, -1, -1)
        assert impl.stats()["kv_live_blocks"] == 4
        impl.call("clear")
        assert impl.stats()["kv_live_blocks"] == 0
