"""B200 runner and engine on the GPU vs the C oracle.

Ports of miniprefix/tests/cow_test.cpp runner()/partial_cache()/costs() (fork,
copy-on-write of a shared partial tail, failed appends that must roll back and
repair the device table, prefix reuse, cost counters) on a 2-layer model of the
135M attention geometry. The oracle recomputes a sequence's whole history from
scratch; logits tolerance |gpu - oracle| <= 1e-3 + 1e-4 |oracle| and identical
argmax (the north star's bar; cow_test's own CUDA check is 2e-5 on its tiny model).
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200.synthetic import ModelConfig, random_weights

MINI = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=32, tied=False)
POISON = 15


def weights(seed=5):
    w = random_weights(MINI, seed=seed)
    w["model.embed_tokens.weight"][POISON, :] = np.nan  # appending token 15 fails (cow_test.cpp:135)
    return w


class History:
    """Oracle logits of a full history, recomputed from an empty pool."""

    def __init__(self, w):
        self.o = Oracle(MINI, w, 4)

    def logits(self, tokens):
        keys, values = self.o.new_pools(16)
        out, ok = self.o.append(keys, values, list(range(16)), 0, list(tokens))
        return out


def same(gpu, ref):
    err = np.abs(gpu - ref)
    assert np.isfinite(gpu).all()
    assert (err <= 1e-3 + 1e-4 * np.abs(ref)).all(), float(err.max())
    assert int(np.argmax(gpu)) == int(np.argmax(ref))


def make_runner(w, kv, **kw):
    from tinyinfer_b200.host import Runner

    return Runner.b200(MINI, w, context=16, block_tokens=kv[0], max_blocks=kv[1], prefix_blocks=kv[2],
                       max_sequences=8, max_step_tokens=64, max_step_sequences=8, **kw)


@pytest.mark.gpu
def test_fork_cow_failure_retry(built):
    """cow_test.cpp:142-169"""
    from tinyinfer_b200.host import HostError

    w = weights()
    h = History(w)
    r = make_runner(w, (4, 4, 0))
    for length in (3, 4, 7):
        for fail in (False, True):
            assert r.reserve_request("a", 8) == "Ready" and r.reserve_request("b", 8) == "Ready"
            r.create("a")
            r.create("b")
            history = list(range(1, length + 1))
            r.append("a", history)
            r.fork_sequence("a", "b")
            before = r.stats()
            if fail:
                with pytest.raises(HostError):
                    r.append("b", [POISON, 9] if length == 3 else [POISON])
                after = r.stats()
                assert after["forward_tokens"] == before["forward_tokens"]
                assert after["kv_live_blocks"] == before["kv_live_blocks"]
                r.release("a")  # the retry must repair the device table without COW
            suffix = [9, 8] if length == 3 else [9]
            same(r.append("b", suffix), h.logits(history + suffix))
            if not fail:
                same(r.append("a", [10]), h.logits(history + [10]))
                r.release("a")
            r.release("b")
            st = r.stats()
            assert st["kv_live_blocks"] == 0 and st["block_table_device_bytes"] == 0
    r.clear()
    assert r.stats()["live_sequences"] == 0
    r.close()


@pytest.mark.gpu
def test_partial_prefix_reuse(built):
    """cow_test.cpp:170-202"""
    from tinyinfer_b200.host import HostError

    w = weights()
    h = History(w)
    r = make_runner(w, (4, 8, 8))
    for length in (1, 3, 4, 7, 8):
        history = list(range(1, length + 1))
        r.create("source")
        r.append("source", history)
        r.cache_prefix("source")
        for common in (1, length):
            prompt = history[:common] + [10]
            r.create("target")
            assert r.reuse_prefix("target", prompt) == common
            before = r.stats()
            with pytest.raises(HostError):
                r.append("target", [POISON])
            assert r.stats()["forward_tokens"] == before["forward_tokens"]
            assert r.stats()["kv_live_blocks"] == before["kv_live_blocks"]
            same(r.append("target", [10]), h.logits(prompt))
            r.release("target")
        r.create("identical")
        assert r.reuse_prefix("identical", history) == length - 1
        same(r.append("identical", [history[-1]]), h.logits(history))
        r.clear()
        assert r.stats()["kv_live_blocks"] == 0 and r.stats()["block_table_device_bytes"] == 0
    r.close()
    # All capacity reserved: a cache-only shared tail becomes exclusive on eviction.
    r = make_runner(w, (4, 1, 1))
    r.create("seed")
    r.append("seed", [1, 2, 3])
    r.cache_prefix("seed")
    r.release("seed")
    assert r.reserve_request("next", 4) == "Ready"
    r.create("next")
    assert r.reuse_prefix("next", [1, 2, 3, 4]) == 3
    same(r.append("next", [4]), h.logits([1, 2, 3, 4]))
    assert r.stats()["kv_live_blocks"] == 1 and r.stats()["kv_cached_blocks"] == 0
    r.close()


@pytest.mark.gpu
def test_cost_counters(built):
    """cow_test.cpp:203-229 (cow_bytes for this model: 2 pools x 3 tokens x 192 floats x 2 layers x 4 B)."""
    from tinyinfer_b200.host import HostError

    w = weights()
    per_cow = 2 * 3 * MINI.kv_width * MINI.layers * 4
    for timed in (False, True):
        r = make_runner(w, (4, 8, 8))
        r.set_cost_timing(timed)
        r.create("a")
        r.append("a", [1, 2, 3])
        r.cache_prefix("a")
        r.create("b")
        assert r.reuse_prefix("b", [1, 2, 3, 4]) == 3
        r.append("b", [4])
        c = r.cost_stats()
        assert c["lookup_calls"] == 1 and c["publish_calls"] == 1
        assert c["cow_pages"] == 1 and c["cow_bytes"] == per_cow and c["cow_timed_copies"] == int(timed)
        if not timed:
            assert c["lookup_ns"] == 0 and c["publish_ns"] == 0 and c["cow_copy_ns"] == 0
        r.create("failed")
        r.fork_sequence("a", "failed")
        with pytest.raises(HostError):
            r.append("failed", [POISON])
        c = r.cost_stats()
        assert c["cow_pages"] == 2 and c["cow_bytes"] == 2 * per_cow
        assert c["cow_timed_copies"] == (2 if timed else 0)
        r.clear()
        assert r.cost_stats()["cow_bytes"] == 2 * per_cow and r.stats()["kv_live_blocks"] == 0
        r.close()


def greedy_stream(h, prompt, steps):
    seq = list(prompt)
    out = []
    for _ in range(steps):
        t = int(np.argmax(h.logits(seq)))
        out.append(t)
        seq.append(t)
    return out


@pytest.mark.gpu
def test_batched_engine_streams_match_oracle(built, ref):
    """Requests sharing a prefix (reuse + COW of the partial shared page), chunked
    prefill and batched decode in one engine: every greedy stream equals the
    oracle's, and the run's bookkeeping equals the reference engine replayed with
    the GPU's tokens (oracle/replay.py: events, step stats, KV stats, copy-on-write
    counts and every live page table after each step)."""
    from oracle.replay import Trace, replay
    from tinyinfer_b200.host import Engine, Runner

    cfg = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=64, tied=True)
    w = random_weights(cfg, seed=17)
    o = Oracle(cfg, w, 4)

    def logits(seq):
        keys, values = o.new_pools(32)
        out, _ = o.append(keys, values, list(range(32)), 0, list(seq))
        return out

    geom = dict(vocabulary=64, context=64, layers=cfg.layers, width=cfg.kv_width, block_tokens=4, max_blocks=256,
                prefix_blocks=32, max_batch=6, token_budget=24, prefill_chunk=8)
    runner = Runner.b200(cfg, w, context=64, block_tokens=4, max_blocks=256, prefix_blocks=32, max_sequences=16,
                         max_step_tokens=128, max_step_sequences=16)
    engine = Engine(runner, 6, 24, 8, 64)
    trace = Trace()
    rng = np.random.default_rng(4)
    shared = [int(t) for t in rng.integers(0, 64, 9)]  # 9 tokens: a partial shared page at block_tokens 4
    prompts = {"seed": shared + [1]}
    for i in range(5):
        prompts[f"f{i}"] = shared + [int(t) for t in rng.integers(0, 64, int(rng.integers(1, 6)))]
    outputs = {}

    def step():
        engine.step()
        events = engine.poll_events()
        live = [r for r in trace.ids if engine.sequence(r) is not None]
        trace.step(engine, events=events, sequences=live)
        for rid, tok, reason, err in events:
            assert reason in (None, 1), err
            if tok is not None:
                outputs.setdefault(rid, []).append(tok)

    engine.submit("seed", prompts["seed"], 4)
    trace.submit("seed", prompts["seed"], 4)
    while not engine.idle():
        step()
    for k, p in prompts.items():
        if k != "seed":
            engine.submit(k, p, 5)
            trace.submit(k, p, 5)
    while not engine.idle():
        step()
    for rid, p in prompts.items():
        seq = list(p)
        for t in outputs[rid]:
            assert t == int(np.argmax(logits(seq))), rid
            seq.append(t)
    st = engine.runner_stats()
    assert st["prefix_hits"] >= 5 and engine.cost_stats()["cow_pages"] >= 1
    engine.shutdown()
    assert engine.runner_stats()["kv_live_blocks"] == 0
    counted = replay(trace, ref=ref, **geom)
    assert counted["cow_pages"] >= 1 and counted["tables"] > 0


@pytest.mark.gpu
def test_decode_steps_run_as_one_forward(built):
    """The engine publishes every request's pages after each append (engine.cpp:
    93-98), so every decode append copies its shared partial tail, and the page it
    copied away from is freed and handed to the next request's copy in the same
    step. Those copies read their sources before any destination is written, so a
    pure decode step is one device forward with no hazard flush, and every stream
    still equals the oracle's."""
    from tinyinfer_b200.host import Engine, Runner

    cfg = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=64, tied=True)
    w = random_weights(cfg, seed=19)
    o = Oracle(cfg, w, 4)

    def token(seq):
        keys, values = o.new_pools(32)
        out, _ = o.append(keys, values, list(range(32)), 0, list(seq))
        return int(np.argmax(out))

    runner = Runner.b200(cfg, w, context=64, block_tokens=4, max_blocks=256, prefix_blocks=64, max_sequences=16,
                         max_step_tokens=128, max_step_sequences=16)
    engine = Engine(runner, 8, 128, 32, 64)
    rng = np.random.default_rng(9)
    prompts = {f"r{i}": [int(t) for t in rng.integers(0, 64, int(rng.integers(5, 15)))] for i in range(8)}
    for rid, p in prompts.items():
        engine.submit(rid, p, 9)
    outputs, decode_steps = {}, 0
    while not engine.idle():
        f0, h0 = engine.flushes()
        engine.step()
        f1, h1 = engine.flushes()
        st = engine.last_step_stats()
        if st["prefill_tokens"] == 0 and st["decode_tokens"] > 1:
            decode_steps += 1
            assert (f1 - f0, h1 - h0) == (1, 0), st
        for rid, tok, reason, err in engine.poll_events():
            assert reason in (None, 1), err
            if tok is not None:
                outputs.setdefault(rid, []).append(tok)
    assert decode_steps >= 6
    assert engine.cost_stats()["cow_pages"] >= 8 * 4
    for rid, p in prompts.items():
        seq = list(p)
        assert len(outputs[rid]) == 9
        for t in outputs[rid]:
            assert t == token(seq), rid
            seq.append(t)
    engine.shutdown()


@pytest.mark.gpu
def test_runner_from_mpfx_file_equals_uploaded_weights(built, tmp_path):
    """Runner.b200_from_file (make_cuda_runner(ModelWeights::load(path), ...)) gives
    the same logits, bit for bit, as the same weights uploaded tensor by tensor."""
    from tinyinfer_b200 import mpfx
    from tinyinfer_b200.host import Runner

    cfg = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=64, tied=False)
    w = random_weights(cfg, seed=29)
    path = str(tmp_path / "model.mpfx")
    mpfx.write(path, cfg, w)
    kw = dict(context=64, block_tokens=4, max_blocks=64, prefix_blocks=0, max_sequences=4, max_step_tokens=64,
              max_step_sequences=4)
    a = Runner.b200(cfg, w, **kw)
    b = Runner.b200_from_file(path, **kw)
    assert b.config.layers == 2 and not b.config.tied
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, 64, 11)]
    outs = []
    for r in (a, b):
        r.create("s")
        first = r.append("s", prompt)
        second = r.append("s", [int(np.argmax(first))])
        outs.append((first, second))
        r.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
