"""Shared-prefix decode attention (attention_shared.cu) through the batched engine.

A seed request publishes a prompt; followers reuse its full pages through the
prefix cache (and copy its partial page on write), so their decode rows start
with the same physical pages and the forward serves those tokens once for the
whole group. Every follower's greedy stream must equal the C oracle's, which
recomputes each history from an empty pool; the device counters must show that
the shared-prefix path ran. Cases cover token chunks that end inside a 32-token
tile, query blocks past 64 vectors, and page sizes 8 and 16. The path is opt-in
(mp_set_shared_prefix); by default every row reads the shared pages itself, and
the last case checks that the default leaves it unused with the same streams.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200.synthetic import ModelConfig, random_weights


@pytest.mark.gpu
@pytest.mark.parametrize("shared,followers,bt,enabled", [(300, 24, 16, True), (136, 8, 16, True), (523, 12, 8, True),
                                                         (300, 24, 16, False)])
def test_shared_prefix_streams_match_oracle(built, shared, followers, bt, enabled):
    from tinyinfer_b200.host import Engine, Runner

    context = 640
    cfg = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=context, tied=True)
    w = random_weights(cfg, seed=23)
    o = Oracle(cfg, w, bt)

    def greedy(seq):
        keys, values = o.new_pools(context // bt + 2)
        out, ok = o.append(keys, values, list(range(context // bt + 2)), 0, list(seq))
        assert ok
        return int(np.argmax(out))

    pages = context // bt + 1
    runner = Runner.b200(cfg, w, context=context, block_tokens=bt, max_blocks=(followers + 2) * pages,
                         prefix_blocks=pages, max_sequences=followers + 4, max_step_tokens=2048,
                         max_step_sequences=followers + 4)
    engine = Engine(runner, followers + 1, 2048, 512, context)
    rng = np.random.default_rng(shared + followers)
    prefix = [int(t) for t in rng.integers(0, 64, shared)]
    engine.submit("seed", prefix + [1], 2)
    while not engine.idle():
        engine.step()
    engine.poll_events()
    prompts = {}
    for i in range(followers):
        prompts[f"f{i}"] = prefix + [int(t) for t in rng.integers(0, 64, int(rng.integers(1, 20)))]
        engine.submit(f"f{i}", prompts[f"f{i}"], 6)
    dev = engine.device()
    if enabled:
        dev.shared_prefix(8, 128)
    dev.counters(reset=True)
    outputs = {}
    while not engine.idle():
        engine.step()
        for rid, tok, reason, err in engine.poll_events():
            assert reason in (None, 1), err
            if tok is not None:
                outputs.setdefault(rid, []).append(tok)
    counters = dev.counters(reset=True)
    if enabled:
        assert counters["shared_prefix_rows"] > 0, counters
        assert counters["shared_prefix_tokens"] >= (shared // bt) * bt * followers
    else:
        assert counters["shared_prefix_rows"] == 0 and counters["shared_prefix_tokens"] == 0, counters
    for rid, p in prompts.items():
        seq = list(p)
        assert len(outputs[rid]) == 6
        for t in outputs[rid]:
            assert t == greedy(seq), rid
            seq.append(t)
    assert engine.runner_stats()["prefix_hits"] >= followers
    engine.shutdown()
