"""Host page pool + exact prefix cache vs the reference's, decision by decision.

The reference's own differential test (miniprefix/tests/prefix_cache_test.cpp:22-52)
compares its trie with a flat full-history model over 3000 random operations for 5
capacities; here the same operation mix runs on the product cache AND the
reference cache, and every result, counter and page reference count must agree
after every operation. The fixed scenarios of prefix_cache_test.cpp:53-171 follow.
"""
import numpy as np
import pytest

from oracle.oracle import RefCache, RefError
from tinyinfer_b200.host import HostError, PrefixCache


def both(ref, *args):
    return PrefixCache(*args), RefCache(ref, *args)


def same_state(a, b, pages):
    assert a.stats() == b.stats()
    assert a.references() == b.references()


@pytest.mark.parametrize("capacity", [0, 1, 2, 5, 16])
def test_random_operations_match_reference(built, ref, capacity):
    a, b = both(ref, 2, 128, capacity)
    rng = np.random.default_rng(7341 + capacity)
    for step in range(3000):
        action = int(rng.integers(0, 7))
        if action == 0:
            assert a.evict_one() == b.evict_one()
        elif action == 1:
            a.clear()
            b.clear()
        else:
            length = 1 + int(rng.integers(0, 23))
            tokens = [int(rng.integers(0, 2)) if i < 4 else int(rng.integers(0, 5)) for i in range(length)]
            if action < 4:
                a.append("s", tokens)
                b.append("s", tokens)
                a.publish("s")
                b.publish("s")
            else:
                assert a.reuse("s", tokens) == b.reuse("s", tokens)
            assert a.sequence("s") == b.sequence("s")
            if step % 3 == 0:
                assert a.evict_one() == b.evict_one()
            same_state(a, b, 128)
            a.release("s")
            b.release("s")
        same_state(a, b, 128)
    a.clear()
    b.clear()
    same_state(a, b, 128)
    assert a.stats()["live_blocks"] == 0


@pytest.mark.parametrize("capacity", [1, 3, 16, 48])
def test_publication_churn_matches_reference(built, ref, capacity):
    a, b = both(ref, 4, 128, capacity)
    for step in range(500):
        tokens = [7] * (1 + step % 63)
        if step % 5 == 0:
            tokens[0] = 9
        tokens[-1] = step % 17
        for c in (a, b):
            c.append("s", tokens)
            c.publish("s")
            c.publish("s")
        if step % 3 == 0:
            assert a.evict_one() == b.evict_one()
        for c in (a, b):
            c.publish("s")
        probe = tokens + [99]
        assert a.reuse("p", probe) == b.reuse("p", probe)
        assert a.sequence("p") == b.sequence("p")
        same_state(a, b, 128)
        for c in (a, b):
            c.release("p")
            c.release("s")
        if step % 19 == 0:
            a.clear()
            b.clear()
            assert a.stats()["live_blocks"] == 0
    same_state(a, b, 128)


def test_invalid_page_leaves_no_node(built, ref):
    """publish() of a sequence naming a page outside the pool throws
    std::out_of_range and leaves neither a lease nor an index node
    (prefix_cache_test.cpp:79-86, 96-98)."""
    for impl in both(ref, 4, 8, 1):
        impl.append("source", [1, 2])
        impl.publish("source")
        impl.evict_one()
        impl.define("invalid", 3, [4, 5, 6], [99])
        with pytest.raises((HostError, RefError)) as e:
            impl.publish("invalid")
        assert e.value.code == -5
        assert impl.stats()["size"] == 0 and impl.stats()["index_nodes"] == 0
        impl.publish("source")
        assert impl.reuse("probe", [1, 2, 3]) == 2
        impl.release("source")
        impl.release("probe")
        impl.clear()
        assert impl.stats()["live_blocks"] == 0
    for impl in both(ref, 2, 8, 2):
        impl.append("a", [1, 2, 3, 4])
        impl.publish("a")
        impl.evict_one()
        impl.append("b", [7, 8])
        impl.publish("b")  # LRU is the sole descendant of the missing [1, 2]
        impl.publish("a")  # eviction must not prune the ancestor being republished
        assert impl.reuse("probe", [1, 2, 3, 4, 5]) == 4


def test_deep_path(built, ref):
    depth = 8192
    a, b = both(ref, 1, depth, depth)
    for c in (a, b):
        c.append("s", [1] * depth)
        c.publish("s")
        c.release("s")
    assert a.stats()["index_nodes"] == depth
    for _ in range(depth):
        assert a.evict_one() and b.evict_one()
    assert a.stats()["index_nodes"] == 0 and a.stats()["live_blocks"] == 0
    same_state(a, b, depth)


def test_reference_scenarios(built, ref):
    """prefix_cache_test.cpp:119-170, each run on both implementations."""
    for impl in both(ref, 4, 4, 4):
        impl.append("source", [1, 2, 3, 4])
        impl.publish("source")
        assert impl.reuse("shorter", [1, 2, 9]) == 2
        impl.publish("shorter")
        impl.release("source")
        impl.release("shorter")
        st = impl.stats()
        assert st["size"] == 2 and st["live_blocks"] == 1 and st["cache_only_blocks"] == 1
        assert impl.evict_one()
        assert impl.reuse("probe", [1, 2, 8]) == 2
        impl.clear()
        assert impl.stats()["live_blocks"] == 1
        impl.release("probe")
        assert impl.stats()["live_blocks"] == 0
    for impl in both(ref, 2, 8, 3, 2, 4):
        impl.append("source", [1, 2, 3, 4, 5])
        impl.publish("source")
        assert impl.stats()["size"] == 3 and impl.stats()["live_blocks"] == 3
        shared = impl.sequence("source")[1][0]
        assert impl.references()[shared] == 2
        assert impl.reuse("a", [1, 2, 3, 4, 5]) == 4 and impl.references()[shared] == 3
        assert impl.reuse("b", [9, 9, 3, 4, 5]) == 0
        impl.release("b")
        assert impl.reuse("b", [1, 2, 3, 4]) == 3
        impl.clear()
        assert impl.stats()["size"] == 0 and impl.references()[shared] == 3
    for impl in both(ref, 2, 6, 2):
        impl.append("a", [1, 2, 3, 4])
        impl.publish("a")
        impl.release("a")
        assert impl.reuse("b", [1, 2, 9]) == 2
        impl.release("b")
        impl.append("c", [7, 8])
        impl.publish("c")
        impl.release("c")
        assert impl.stats()["evictions"] == 1 and impl.stats()["size"] == 2
        assert impl.reuse("a", [1, 2, 3, 4, 5]) == 2  # LRU evicted the second page, not the first
    for impl in both(ref, 2, 4, 0):
        impl.append("a", [1, 2, 3])
        impl.publish("a")
        assert impl.stats()["size"] == 0 and impl.reuse("b", [1, 2, 3]) == 0


def test_pool_free_list_order(built, ref):
    """paged_kv_test.cpp:7-31: pages {0,2,3} after interleaved growth, then the
    released hole and the next page {1,4}."""
    for impl in both(ref, 3, 5, 0, 2, 4):
        impl.append("a", [1, 1, 1])
        impl.append("b", [1, 1, 1])
        impl.append("a", [1, 1, 1, 1])
        assert impl.sequence("a")[1] == [0, 2, 3]
        impl.release("b")
        impl.append("c", [1] * 6)
        assert impl.sequence("c")[1] == [1, 4]
        assert impl.stats()["live_blocks"] == 5


@pytest.mark.parametrize("capacity", [3, 12, 64])
def test_undo_window_restores_exact_state(built, ref, capacity):
    """The batched engine's step checkpoint: operations inside an undo window that
    is rolled back leave no trace (the reference cache never sees them and every
    later result, counter, LRU decision and page reference still agrees); a window
    that is kept equals the reference applying the same operations. Sequences grow
    and republish, so publish() runs on its path hints, stale ones included."""
    a, b = both(ref, 4, 256, capacity)
    rng = np.random.default_rng(91 + capacity)
    live = []
    counter = [0]

    def random_ops(n):
        ops, names = [], list(live)
        for _ in range(n):
            k = int(rng.integers(0, 10))
            if k < 4 and names:
                s = names[int(rng.integers(0, len(names)))]
                ops.append(("append", s, [int(t) for t in rng.integers(0, 3, size=int(rng.integers(1, 9)))]))
            elif k < 6 and names:
                ops.append(("publish", names[int(rng.integers(0, len(names)))]))
            elif k < 8 or not names:
                counter[0] += 1
                prompt = [int(t) for t in rng.integers(0, 3, size=int(rng.integers(1, 30)))]
                ops.append(("reuse", f"s{counter[0]}", prompt))
                names.append(f"s{counter[0]}")
            elif k < 9:
                ops.append(("release", names.pop(int(rng.integers(0, len(names))))))
            else:
                ops.append(("evict",))
        return ops

    def apply(c, ops, names):
        out = []
        for op in ops:
            if op[0] == "append":
                c.append(op[1], op[2])
                c.publish(op[1])
            elif op[0] == "publish":
                c.publish(op[1])
            elif op[0] == "reuse":
                out.append(c.reuse(op[1], op[2]))
                names.append(op[1])
            elif op[0] == "release":
                c.release(op[1])
                names.remove(op[1])
            else:
                out.append(c.evict_one())
        return out

    for window in range(150):
        before = list(live)
        ops = random_ops(int(rng.integers(1, 12)))
        a.journal("begin")
        names_a = list(live)
        out_a = apply(a, ops, names_a)
        if rng.random() < 0.5:
            a.journal("rollback")
            live[:] = before
        else:
            a.journal("end")
            names_b = list(live)
            assert apply(b, ops, names_b) == out_a
            assert names_a == names_b
            live[:] = names_b
        same_state(a, b, 256)
        for s in live:
            assert a.sequence(s) == b.sequence(s), s
    for s in list(live):
        a.release(s)
        b.release(s)
    a.clear()
    b.clear()
    same_state(a, b, 256)
