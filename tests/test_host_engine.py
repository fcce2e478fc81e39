"""The batched host Engine vs the reference Engine (miniprefix/src/engine/engine.cpp).

Both engines drive a scripted runner that keeps the real KV manager of its side
and returns, for each successful append of a request, the next token of that
request's script; appends that contain a poisoned token fail as a nonfinite
forward does. The product engine runs every step as a staged batch (one device
forward per step on a real runner); the reference runs requests one by one.
After every step the events (ids, tokens, finish reasons, messages), step stats,
25 runner stats, cost counters, engine state and every sequence's pages must be
identical -- including steps that fail and poison the engine.
"""
import numpy as np
import pytest

from oracle.oracle import RefEngine, RefError, RefRunner
from tinyinfer_b200.host import Engine, HostError, Runner


def pair(ref, vocab, context, bt, max_blocks, cache, batch, budget, chunk):
    mr = Runner.scripted(vocab, context, 1, 1, bt, max_blocks, cache)
    rr = RefRunner.scripted_runner(ref, vocab, context, 1, 1, bt, max_blocks, cache)
    return Engine(mr, batch, budget, chunk, context), RefEngine(rr, batch, budget, chunk, context), mr, rr


def same(me, re, ids):
    assert me.poll_events() == re.poll_events()
    assert me.last_step_stats() == re.last_step_stats()
    assert me.runner_stats() == re.runner_stats()
    assert me.cost_stats() == re.cost_stats()
    assert me.failed() == re.failed() and me.idle() == re.idle()
    for i in ids:
        assert me.sequence(i) == re.sequence(i), i


def call(f, *a):
    try:
        return ("ok", f(*a))
    except (HostError, RefError) as e:
        return ("err", e.code, e.message)


@pytest.mark.parametrize("seed", range(40))
def test_random_workloads_match_reference(built, ref, seed):
    rng = np.random.default_rng(seed)
    vocab, context = 8, 48
    bt = int(rng.choice([1, 2, 4]))
    max_blocks = int(rng.integers(6, 40))
    cache = int(rng.integers(0, max_blocks + 1))
    batch, budget, chunk = int(rng.integers(1, 7)), int(rng.integers(1, 24)), int(rng.integers(1, 9))
    me, re, mr, rr = pair(ref, vocab, context, bt, max_blocks, cache, batch, budget, chunk)
    roots = [list(rng.integers(0, 3, size=int(rng.integers(1, 12)))) for _ in range(3)]
    ids = []
    poisoned = seed % 4 == 3
    for step in range(120):
        if rng.random() < 0.35 or not ids:
            rid = f"r{len(ids)}"
            root = roots[int(rng.integers(0, len(roots)))]
            prompt = [int(t) for t in root[:int(rng.integers(1, len(root) + 1))]]
            prompt += [int(t) for t in rng.integers(0, vocab, size=int(rng.integers(0, 6)))]
            max_new = int(rng.integers(1, 7))
            eos = int(rng.integers(0, vocab)) if rng.random() < 0.3 else None
            script = [int(t) for t in rng.integers(0, vocab, size=30)]
            mr.script(rid, script)
            rr.script(rid, script)
            a = call(me.submit, rid, prompt, max_new, eos)
            b = call(re.submit, rid, prompt, max_new, eos)
            assert a == b
            ids.append(rid)
        if poisoned and step == 25:
            t = int(rng.integers(0, vocab))
            mr.poison(t)
            rr.poison(t)
        if ids and rng.random() < 0.08:
            victim = ids[int(rng.integers(0, len(ids)))]
            assert call(me.cancel, victim) == call(re.cancel, victim)
        a = call(me.step)
        b = call(re.step)
        assert a == b, (step, a, b)
        same(me, re, ids)
        if me.failed():
            break
    assert call(me.shutdown) == call(re.shutdown)
    same(me, re, ids)


def test_same_step_publish_reuse_and_cow(built, ref):
    """A decoder publishes its partial tail page and a follower admitted in the same
    step reuses it and copies it on write (engine_history_test.cpp:105-115)."""
    for cache in (0, 16):
        me, re, mr, rr = pair(ref, 128, 128, 4, 32, cache, 2, 8, 8)
        for r in (mr, rr):
            r.script("source", [4, 5, 6, 7, 8])
            r.script("fork", [51])
        for e in (me, re):
            e.submit("source", [1, 2, 3], 5)
            e.step()
        same(me, re, ["source"])
        for e in (me, re):
            e.submit("fork", [1, 2, 3, 4, 50], 1)
            e.step()
        same(me, re, ["source", "fork"])
        assert mr.regions() == rr.regions()


def test_failed_step_poisons_like_reference(built, ref):
    """A nonfinite forward in the middle of a batched step: earlier requests keep
    their events, every request ends in Error with the runner's message, and the
    cumulative counters equal the reference's."""
    me, re, mr, rr = pair(ref, 16, 64, 2, 64, 8, 4, 64, 8)
    for r in (mr, rr):
        for i in range(4):
            r.script(f"q{i}", [3, 4, 5, 6, 7, 8])
    for e in (me, re):
        for i in range(4):
            e.submit(f"q{i}", [1, 2, 9 + i], 6)
        e.step()
    same(me, re, [f"q{i}" for i in range(4)])
    for r in (mr, rr):
        r.poison(4)  # the second decode input of every request
    for _ in range(3):
        assert call(me.step) == call(re.step)
        same(me, re, [f"q{i}" for i in range(4)])
    assert me.failed()
