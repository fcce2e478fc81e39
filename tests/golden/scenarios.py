"""Seeded scenarios shared by the golden-fixture generator (make_golden.py) and the
tests that replay them: each scenario is a plain list of operations that runs
unchanged on the reference's objects (oracle/_ref through oracle/oracle.py) and on
the product's (tinyinfer_b200.host), so a fixture recorded from the reference
can be checked against the product without the reference present.

Runner scripts follow miniprefix/tests/cow_test.cpp:142-229 (fork, copy-on-write
of a shared partial tail, failing appends that roll back, prefix reuse of a
partial and an interior page, eviction of a cache-only lease); engine workloads
are random request streams over prefix trees, with cancels and a poisoned token
(a nonfinite forward) in every fourth seed, as in
miniprefix/tests/engine_history_test.cpp and engine_prefill_test.cpp.
"""
from __future__ import annotations

import numpy as np

# Model of the runner scripts: the 135M attention geometry (hidden 576, 9/3 heads
# of 64) with 2 layers and a 64-token vocabulary; appending POISON fails (its
# embedding row is NaN, cow_test.cpp:135).
MINI = dict(layers=2, intermediate=128, vocabulary=64, context=32, tied=False)
MINI_SEED = 5
POISON = 15
# stats fields that the CPU and device runners share (the device-table and byte
# counters differ by design between a CPU and a device backend)
STAT_FIELDS = ("live_sequences", "kv_live_blocks", "kv_cached_blocks", "forward_tokens", "prefix_hits",
               "prefix_reused_tokens")


def mini_weights(seed: int = MINI_SEED):
    from tinyinfer_b200.synthetic import ModelConfig, random_weights

    cfg = ModelConfig(**MINI)
    w = random_weights(cfg, seed=seed)
    w["model.embed_tokens.weight"][POISON, :] = np.nan
    return cfg, w


def runner_scripts() -> dict[str, tuple[tuple[int, int, int], list[tuple]]]:
    """name -> ((block_tokens, max_blocks, prefix_blocks), operations).
    Operations: (method, *args) on a runner built with context 16."""
    out = {}
    ops = []
    for length in (3, 4, 7):
        for fail in (False, True):
            history = list(range(1, length + 1))
            ops += [("reserve_request", "a", 8), ("reserve_request", "b", 8), ("create", "a"), ("create", "b"),
                    ("append", "a", history), ("fork_sequence", "a", "b"), ("stats",)]
            if fail:
                ops += [("append", "b", [POISON, 9] if length == 3 else [POISON]), ("stats",), ("release", "a")]
            ops.append(("append", "b", [9, 8] if length == 3 else [9]))
            if not fail:
                ops += [("append", "a", [10]), ("release", "a")]
            ops += [("release", "b"), ("stats",)]
    ops += [("clear",), ("stats",)]
    out["fork_cow_failure"] = ((4, 4, 0), ops)

    ops = []
    for length in (1, 3, 4, 7, 8):
        history = list(range(1, length + 1))
        ops += [("create", "source"), ("append", "source", history), ("cache_prefix", "source")]
        for common in (1, length):
            prompt = history[:common] + [10]
            ops += [("create", "target"), ("reuse_prefix", "target", prompt), ("stats",),
                    ("append", "target", [POISON]), ("stats",), ("append", "target", [10]), ("release", "target")]
        ops += [("create", "identical"), ("reuse_prefix", "identical", history),
                ("append", "identical", [history[-1]]), ("clear",), ("stats",)]
    out["partial_prefix_reuse"] = ((4, 8, 8), ops)

    out["evict_cache_only_lease"] = ((4, 1, 1), [
        ("create", "seed"), ("append", "seed", [1, 2, 3]), ("cache_prefix", "seed"), ("release", "seed"),
        ("reserve_request", "next", 4), ("create", "next"), ("reuse_prefix", "next", [1, 2, 3, 4]),
        ("append", "next", [4]), ("stats",), ("release", "next"), ("stats",)])
    return out


def run_runner_script(runner, ops, errors) -> list:
    """Applies ops; returns one record per op: ("ok", value) or ("err", code).
    `errors` is the tuple of exception types that carry a reference error code."""
    rec = []
    for op in ops:
        name, args = op[0], op[1:]
        try:
            if name == "stats":
                s = runner.stats()
                rec.append(("ok", {k: int(s[k]) for k in STAT_FIELDS}))
                continue
            v = getattr(runner, name)(*args)
            if name == "append":
                v = np.asarray(v, dtype=np.float32)
            elif name == "reuse_prefix":
                v = int(v)
            elif name == "reserve_request":
                v = str(v)
            else:
                v = None
            rec.append(("ok", v))
        except errors as e:
            rec.append(("err", int(e.code)))
    return rec


def engine_workload(seed: int):
    """(engine parameters, operations) of one random engine workload.
    Parameters: vocab, context, block_tokens, max_blocks, prefix_blocks, max_batch,
    token_budget, prefill_chunk. Operations: ("submit", id, prompt, max_new, eos,
    script), ("poison", token), ("cancel", id), ("step",)."""
    rng = np.random.default_rng(1000 + seed)
    vocab, context = 8, 48
    bt = int(rng.choice([1, 2, 4]))
    max_blocks = int(rng.integers(6, 40))
    cache = int(rng.integers(0, max_blocks + 1))
    if seed >= 8:
        # copy-on-write heavy: pages of 4 tokens, a roomy cache, and requests that
        # extend a published history in the middle of its last page
        bt, max_blocks, cache = 4, int(rng.integers(24, 48)), int(rng.integers(8, 24))
    batch, budget, chunk = int(rng.integers(1, 7)), int(rng.integers(1, 24)), int(rng.integers(1, 9))
    params = dict(vocab=vocab, context=context, block_tokens=bt, max_blocks=max_blocks, prefix_blocks=cache,
                  max_batch=batch, token_budget=budget, prefill_chunk=chunk)
    root_len = (1, 12) if seed < 8 else (5, 15)
    roots = [[int(t) for t in rng.integers(0, 3, size=int(rng.integers(*root_len)))] for _ in range(3)]
    ids, ops = [], []
    for step in range(100):
        if rng.random() < 0.35 or not ids:
            rid = f"r{len(ids)}"
            root = roots[int(rng.integers(0, len(roots)))]
            prompt = root[:int(rng.integers(1, len(root) + 1))]
            if seed >= 8 and len(ids) % 2 == 1:
                prompt = list(root)
            prompt += [int(t) for t in rng.integers(0, vocab, size=int(rng.integers(0, 6)))]
            max_new = int(rng.integers(1, 7))
            eos = int(rng.integers(0, vocab)) if rng.random() < 0.3 else None
            script = [int(t) for t in rng.integers(0, vocab, size=30)]
            ops.append(("submit", rid, prompt, max_new, eos, script))
            ids.append(rid)
        if seed % 4 == 3 and step == 25:
            ops.append(("poison", int(rng.integers(0, vocab))))
        if rng.random() < 0.08:
            ops.append(("cancel", ids[int(rng.integers(0, len(ids)))]))
        ops.append(("step",))
    return params, ops


def run_engine_workload(engine, runner, ops, errors) -> list:
    """Applies a workload; after every op records its outcome, and after every step
    the events, step stats, runner stats, cost counters and engine state. Stops
    after the step that leaves the engine failed, then shuts down."""
    rec = []
    ids = []

    def call(f, *a):
        try:
            r = f(*a)
            return ["ok", r if isinstance(r, (bool, int, str)) or r is None else None]
        except errors as e:
            return ["err", int(e.code), str(e.message)]

    for op in ops:
        kind = op[0]
        if kind == "submit":
            _, rid, prompt, max_new, eos, script = op
            runner.script(rid, script)
            rec.append(call(engine.submit, rid, prompt, max_new, eos))
            ids.append(rid)
        elif kind == "poison":
            runner.poison(op[1])
            rec.append(["ok", None])
        elif kind == "cancel":
            rec.append(call(engine.cancel, op[1]))
        else:
            rec.append(call(engine.step))
            rec.append(_snapshot(engine, ids))
            if engine.failed():
                break
    rec.append(call(engine.shutdown))
    rec.append(_snapshot(engine, ids))
    # every copy-on-write region the runner was asked to copy, in order
    rec.append({"regions": [list(map(int, r)) for r in runner.regions()]})
    return rec


def _snapshot(engine, ids) -> dict:
    return {
        "events": [list(e) for e in engine.poll_events()],
        "step": dict(engine.last_step_stats()),
        "runner": dict(engine.runner_stats()),
        "cost": dict(engine.cost_stats()),
        "failed": bool(engine.failed()),
        "idle": bool(engine.idle()),
        "sequences": {i: _plain(engine.sequence(i)) for i in ids},
    }


def _plain(x):
    if isinstance(x, dict):
        return {k: _plain(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_plain(v) for v in x]
    if isinstance(x, (np.integer,)):
        return int(x)
    return x
