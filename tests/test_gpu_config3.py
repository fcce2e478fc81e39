"""BASELINE config 3's geometry at full model size on the GPU: the batched decode
that bench.py times, checked against the C oracle and the reference engine.

The 135M-shape model (30 layers, vocabulary 49152, tied head, page size 16). A
seed request prefills a 1032-token shared prefix plus 8 tokens of its own in
512-token chunks and is published; 255 followers then reuse the 1032 shared
tokens (64 full pages and 8 tokens of a partial page, which each follower copies
on write), prefill short unique suffixes, and decode together with the seed:
every decode step is one device forward over 256 rows at contexts of about 1.05k,
which runs the M = 256 cluster split-K GEMMs with their RoPE, SwiGLU and residual
epilogues, the decode attention over the shared pages, and the tied LM head.

Checks:
  * logits: for a seeded sample of 8 followers and the seed, the FULL logits of
    every emitted token (the prefill's and each decode step's) against the C
    oracle recomputing that request over its own pages,
    |gpu - oracle| <= 1e-3 + 1e-4 |oracle| (the north star's bar);
  * greedy tokens: each sampled token is the oracle's argmax (a token within the
    tolerance of the oracle's maximum is counted as a tie, at most one allowed);
  * bookkeeping: the whole run's emitted tokens replayed through the unmodified
    reference Engine over its scripted runner gives the same events, step stats,
    KV stats, copy-on-write and reuse counters after every step, and the same
    page table for every live request (oracle/replay.py).
Reference: miniprefix/src/backend/cpu/llama_runner.cpp:60-104 (the oracle's
algorithm), miniprefix/src/engine/engine.cpp:56-125 (the replayed engine).
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from oracle.replay import Trace, replay
from tinyinfer_b200.synthetic import ModelConfig, random_weights

BT, N, SHARED, SEED_OWN = 16, 256, 1032, 8
SEED_NEW, FOLLOWER_NEW = 8, 5
CHUNK, BUDGET, PREFIX_BLOCKS = 512, 8192, 66


def tolerance_ok(gpu, ref):
    return np.abs(gpu - ref) <= 1e-3 + 1e-4 * np.abs(ref)


@pytest.mark.gpu
def test_config3_geometry_against_oracle_and_reference_engine(built, ref):
    from tinyinfer_b200.host import Engine, Runner

    cfg = ModelConfig(context=1152)
    w = random_weights(cfg, seed=3)
    rng = np.random.default_rng(33)
    V = cfg.vocabulary
    shared = [int(t) for t in rng.integers(0, V, SHARED)]
    seed_prompt = shared + [int(t) for t in rng.integers(0, V, SEED_OWN)]
    prompts = {"seed": seed_prompt}
    for i in range(1, N):
        suffix = [int(t) for t in rng.integers(0, V, int(rng.integers(1, 25)))]
        if suffix[0] == seed_prompt[SHARED]:
            suffix[0] = (suffix[0] + 1) % V  # diverge from the seed right after the shared part
        prompts[f"f{i}"] = shared + suffix
    sample = ["seed"] + [f"f{i}" for i in sorted(rng.choice(np.arange(1, N), 8, replace=False))]

    longest = max(len(p) for p in prompts.values()) + SEED_NEW
    max_blocks = (N + 1) * -(-longest // BT) + 64
    geom = dict(vocabulary=V, context=cfg.context, layers=cfg.layers, width=cfg.kv_width, block_tokens=BT,
                max_blocks=max_blocks, prefix_blocks=PREFIX_BLOCKS, max_batch=N, token_budget=BUDGET,
                prefill_chunk=CHUNK)
    runner = Runner.b200(cfg, w, context=cfg.context, block_tokens=BT, max_blocks=max_blocks,
                         prefix_blocks=PREFIX_BLOCKS, max_sequences=N + 8, max_step_tokens=BUDGET,
                         max_step_sequences=N + 8)
    engine = Engine(runner, N, BUDGET, CHUNK, cfg.context)
    engine.capture_logits(True)
    trace = Trace()
    captured = {rid: [] for rid in sample}
    decode_256 = 0

    def step():
        nonlocal decode_256
        engine.step()
        events = engine.poll_events()
        for rid, tok, reason, err in events:
            assert reason in (None, 1), (rid, reason, err)  # 1 = Length
            if tok is not None and rid in captured:
                captured[rid].append((engine.logits(rid), tok))
        if engine.last_step_stats()["decode_tokens"] == N:
            decode_256 += 1
        live = [rid for rid in trace.ids if engine.sequence(rid) is not None]
        trace.step(engine, events=events, sequences=live)

    engine.submit("seed", seed_prompt, SEED_NEW)
    trace.submit("seed", seed_prompt, SEED_NEW)
    while not captured["seed"]:
        step()
    for i in range(1, N):
        engine.submit(f"f{i}", prompts[f"f{i}"], FOLLOWER_NEW)
        trace.submit(f"f{i}", prompts[f"f{i}"], FOLLOWER_NEW)
    while not engine.idle():
        step()
    st = engine.runner_stats()
    costs = engine.cost_stats()
    engine.capture_logits(False)
    engine.shutdown()
    engine.close()
    assert decode_256 >= 3, decode_256
    assert st["prefix_reused_tokens"] == (N - 1) * SHARED
    assert costs["cow_pages"] >= N - 1
    tokens = trace.tokens()
    assert all(len(tokens[r]) == (SEED_NEW if r == "seed" else FOLLOWER_NEW) for r in tokens)

    # --- bookkeeping: the reference engine on the GPU's tokens
    counted = replay(trace, ref=ref, **geom)
    assert counted["steps"] == sum(1 for op in trace.ops if op[0] == "step")

    # --- logits and tokens of the sampled requests: the C oracle over own pages
    o = Oracle(cfg, w, BT)
    seed_pages = -(-(len(seed_prompt) + SEED_NEW) // BT)
    own = 3  # pages a follower writes: its copy of page 64 and at most two more
    keys, values = o.new_pools(seed_pages + own * (len(sample) - 1))
    page_floats = cfg.layers * BT * cfg.kv_width
    ties, worst = 0, 0.0

    def check(rid, tables, start, tokens_in):
        nonlocal ties, worst
        used = start
        feed = list(tokens_in)
        for k, (gpu, tok) in enumerate(captured[rid]):
            expect, finite = o.append(keys, values, tables, used, feed)
            assert finite
            used += len(feed)
            ok = tolerance_ok(gpu, expect)
            worst = max(worst, float(np.abs(gpu - expect).max()))
            assert ok.all(), (rid, k, float(np.abs(gpu - expect).max()))
            best = int(np.argmax(expect))
            if tok != best:
                assert expect[best] - expect[tok] <= 1e-3 + 1e-4 * abs(expect[best]), (rid, k, tok, best)
                ties += 1
            feed = [tok]

    seed_table = list(range(seed_pages))
    check("seed", seed_table, 0, seed_prompt)
    partial = SHARED // BT  # page 64: 8 shared tokens, copied on write by every follower
    for j, rid in enumerate(sample[1:]):
        base = seed_pages + own * j
        keys[base * page_floats:(base + 1) * page_floats] = keys[partial * page_floats:(partial + 1) * page_floats]
        values[base * page_floats:(base + 1) * page_floats] = values[partial * page_floats:(partial + 1) * page_floats]
        table = seed_table[:partial] + [base + i for i in range(own)]
        check(rid, table, SHARED, prompts[rid][SHARED:])
    assert ties <= 1, ties
    print(f"config-3 geometry: {sum(len(v) for v in captured.values())} logits vectors checked, worst abs err "
          f"{worst:.3g}, {ties} near-ties; replay {counted}")
