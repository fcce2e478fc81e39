"""The bookkeeping replay checker (oracle/replay.py) on CPU: a product Engine run
over the scripted runner, recorded as a trace, replays through the reference
engine without a difference; a trace with one event missing, one finish reason,
one page id or one stat changed is reported. (The replay takes the product's
tokens as given -- their values are checked against the C oracle's logits
elsewhere -- so it checks what the reference engine decides from them.)"""
import numpy as np
import pytest

from oracle.replay import Mismatch, Trace, replay
from tinyinfer_b200.host import Engine, Runner

GEOM = dict(vocabulary=16, context=64, layers=2, width=8, block_tokens=4, max_blocks=96, prefix_blocks=12,
            max_batch=6, token_budget=40, prefill_chunk=8)


def record(seed):
    g = GEOM
    rng = np.random.default_rng(seed)
    runner = Runner.scripted(g["vocabulary"], g["context"], g["layers"], g["width"], g["block_tokens"],
                             g["max_blocks"], g["prefix_blocks"])
    engine = Engine(runner, g["max_batch"], g["token_budget"], g["prefill_chunk"], g["context"])
    trace = Trace()
    shared = [int(t) for t in rng.integers(0, 16, 9)]
    ids = []
    for step in range(60):
        if len(ids) < 12 and (rng.random() < 0.4 or not ids):
            rid = f"q{len(ids)}"
            runner.script(rid, [int(t) for t in rng.integers(1, 16, 12)])
            prompt = shared[:int(rng.integers(1, 10))] + [int(t) for t in rng.integers(0, 16, int(rng.integers(0, 5)))]
            max_new = int(rng.integers(1, 8))
            engine.submit(rid, prompt, max_new)
            trace.submit(rid, prompt, max_new)
            ids.append(rid)
        if engine.idle():
            break
        engine.step()
        live = [r for r in ids if engine.sequence(r) is not None]
        trace.step(engine, events=engine.poll_events(), sequences=live)
    engine.shutdown()
    engine.close()
    return trace


@pytest.mark.parametrize("seed", range(4))
def test_replay_of_a_product_run_matches(built, ref, seed):
    trace = record(seed)
    counted = replay(trace, ref=ref, cow=False, **GEOM)
    assert counted["steps"] > 5 and counted["tables"] > 0 and counted["stats_checks"] == counted["steps"]


def test_replay_reports_a_changed_event_page_or_stat(built, ref):
    import copy

    trace = record(1)
    steps = [op[1] for op in trace.ops if op[0] == "step"]
    # an event the product did not emit
    t = copy.deepcopy(trace)
    s = next(op[1] for op in t.ops if op[0] == "step" and len(op[1].events) > 1)
    del s.events[-1]
    with pytest.raises(Mismatch, match="events differ"):
        replay(t, ref=ref, cow=False, **GEOM)
    # a finish reason
    t = copy.deepcopy(trace)
    s = next(op[1] for op in t.ops if op[0] == "step" and any(e[2] is not None for e in op[1].events))
    i = next(i for i, e in enumerate(s.events) if e[2] is not None)
    s.events[i] = (s.events[i][0], s.events[i][1], 2)
    with pytest.raises(Mismatch, match="events differ"):
        replay(t, ref=ref, cow=False, **GEOM)
    # a page id
    t = copy.deepcopy(trace)
    s = next(op[1] for op in t.ops if op[0] == "step" and op[1].sequences)
    rid, (used, blocks) = next(iter(s.sequences.items()))
    s.sequences[rid] = (used, [blocks[0] + 1] + blocks[1:])
    with pytest.raises(Mismatch, match="page table"):
        replay(t, ref=ref, cow=False, **GEOM)
    # a KV stat
    t = copy.deepcopy(trace)
    s = [op[1] for op in t.ops if op[0] == "step"][-1]
    s.kv["prefix_hits"] += 1
    with pytest.raises(Mismatch, match="KV stats"):
        replay(t, ref=ref, cow=False, **GEOM)
    assert len(steps) > 5


def test_bench_record_format_replays(built, ref):
    """bench.py records its run as plain lists (setup steps with stats, timed steps
    as poll_compact arrays, final stats and page tables); replay_parity turns that
    into a trace and replays it. Here the same recording runs over the scripted
    runner on CPU."""
    import bench

    g = dict(GEOM, max_batch=8, token_budget=64)
    runner = Runner.scripted(g["vocabulary"], g["context"], g["layers"], g["width"], g["block_tokens"],
                             g["max_blocks"], g["prefix_blocks"])
    engine = Engine(runner, g["max_batch"], g["token_budget"], g["prefill_chunk"], g["context"])
    rng = np.random.default_rng(5)
    shared = [int(t) for t in rng.integers(0, 16, 10)]
    ids = [f"r{i}" for i in range(8)]
    record = {"ops": [], "ids": ids}
    for i, rid in enumerate(ids):
        runner.script(rid, [int(t) for t in rng.integers(1, 16, 40)])
        prompt = shared + [int(t) for t in rng.integers(0, 16, 3)]
        engine.submit(rid, prompt, 30)
        record["ops"].append(("submit", rid, np.array(prompt, dtype=np.int32), 30))
        if i == 0:
            for _ in range(3):
                engine.step()
                evs = engine.poll_events()
                record["ops"].append(("step", [(e[0], e[1], e[2]) for e in evs], engine.last_step_stats(),
                                      engine.runner_stats(), engine.cost_stats()))
    for _ in range(12):
        engine.step()
        record["ops"].append(("compact", engine.poll_compact()))
    record["final"] = {"step_stats": engine.last_step_stats(), "runner_stats": engine.runner_stats(),
                       "costs": engine.cost_stats(), "sequences": {rid: engine.sequence(rid) for rid in ids}}
    record["geometry"] = g
    out = bench.replay_parity(record, cow=False)
    assert out["bookkeeping"] == "identical", out
    assert out["compared"]["tables"] == 8
    record["final"]["sequences"]["r3"] = (record["final"]["sequences"]["r3"][0] + 1,
                                          record["final"]["sequences"]["r3"][1])
    assert bench.replay_parity(record, cow=False)["bookkeeping"] == "MISMATCH"
    engine.close()


def test_copy_on_write_counts_compare_with_reference_regions(built, ref):
    """A device runner counts its copy-on-write pages and bytes; the replay compares
    them with the regions the reference engine produced. Here the product scripted
    runner's own regions stand in for a device runner's counters."""
    import copy

    g = GEOM
    rng = np.random.default_rng(11)
    runner = Runner.scripted(g["vocabulary"], g["context"], g["layers"], g["width"], g["block_tokens"],
                             g["max_blocks"], g["prefix_blocks"])
    engine = Engine(runner, g["max_batch"], g["token_budget"], g["prefill_chunk"], g["context"])
    trace = Trace()
    shared = [int(t) for t in rng.integers(0, 16, 9)]  # a partial shared page at 4 tokens per page
    cow = [0, 0]  # the product runner's regions so far (each read drains them)

    def step():
        engine.step()
        trace.step(engine, events=engine.poll_events())
        regions = runner.regions()
        cow[0] += len(regions)
        cow[1] += sum(2 * r[3] * r[4] * 4 for r in regions)
        trace.ops[-1][1].costs.update(cow_pages=cow[0], cow_bytes=cow[1])

    for i in range(6):
        rid = f"c{i}"
        runner.script(rid, [int(t) for t in rng.integers(1, 16, 8)])
        prompt = shared + [int(t) for t in rng.integers(0, 16, 2)]
        engine.submit(rid, prompt, 4)
        trace.submit(rid, prompt, 4)
        if i == 0:  # the seed runs first and publishes the shared pages
            for _ in range(4):
                step()
    while not engine.idle():
        step()
    engine.close()
    counted = replay(trace, ref=ref, **GEOM)
    assert counted["cow_pages"] >= 1
    t = copy.deepcopy(trace)
    t.ops[-1][1].costs["cow_pages"] += 1
    with pytest.raises(Mismatch, match="copy-on-write"):
        replay(t, ref=ref, **GEOM)
