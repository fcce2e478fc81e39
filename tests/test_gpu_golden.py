"""The B200 path against the golden fixtures recorded from the reference's own CPU
runner and engine (tests/golden/make_golden.py).

Bar (the north star's): logits within max-abs 1e-3 / rel 1e-4 of the reference's,
identical greedy tokens, identical bookkeeping (admissions, reuse lengths, error
codes, page and sequence counters).
"""
import json
import os
import sys

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)

import scenarios  # noqa: E402


def close(gpu, ref):
    gpu = np.asarray(gpu, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(gpu - ref)
    assert np.isfinite(gpu).all()
    assert (err <= 1e-3 + 1e-4 * np.abs(ref)).all(), float(err.max())


@pytest.mark.gpu
def test_config1_full_matches_reference(built):
    """256-token prompt + 64 greedy decode appends of the
    135M-shape model through the B200 runner, every step against the reference's
    logits; then the same request through the batched Engine gives the
    reference Engine's token stream."""
    from tinyinfer_b200.host import Engine, Runner
    from tinyinfer_b200.synthetic import SMOLLM2_135M, random_weights

    g = np.load(os.path.join(GOLDEN, "config1_135m.npz"))
    meta = json.loads(str(g["meta"]))
    w = random_weights(SMOLLM2_135M, seed=meta["weights_seed"])
    prompt = [int(t) for t in g["prompt"]]

    def runner():
        return Runner.b200(SMOLLM2_135M, w, context=meta["context"], block_tokens=meta["block_tokens"],
                           max_blocks=meta["max_blocks"], prefix_blocks=0, max_sequences=4, max_step_tokens=256,
                           max_step_sequences=4)

    r = runner()
    r.create("config1")
    out = r.append("config1", prompt)
    close(out, g["first_logits"])
    worst = 0.0
    for step in range(meta["decode_steps"] + 1):
        assert int(np.argmax(out)) == int(g["tokens"][step]), step
        top = g["top_index"][step]
        close(out[top], g["top_value"][step])
        worst = max(worst, float(np.abs(out[top] - g["top_value"][step]).max()))
        assert abs(float(np.sum(out, dtype=np.float64)) - float(g["sum"][step])) <= 1e-3 * out.size ** 0.5
        if step == meta["decode_steps"]:
            break
        out = r.append("config1", [int(g["tokens"][step])])
    close(out, g["last_logits"])
    r.close()
    print(f"config 1: worst top-8 logit error {worst:.2e}")

    r = runner()
    e = Engine(r, 1, 256, 256, meta["context"])
    e.submit("config1", prompt, meta["decode_steps"])
    while not e.idle():
        e.step()
    stream = [t for _, t, _, _ in e.poll_events() if t is not None]
    assert stream == [int(t) for t in g["engine_stream"]]
    e.shutdown()


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(scenarios.runner_scripts()))
def test_runner_scripts_match_reference(built, name):
    """cow_test.cpp's runner / partial-cache scenarios through the B200 runner vs
    the reference CpuRunner's recorded outcomes."""
    from tinyinfer_b200.host import HostError, Runner

    cfg, w = scenarios.mini_weights()
    kv, ops = scenarios.runner_scripts()[name]
    d = np.load(os.path.join(GOLDEN, "runner_scripts.npz"))
    golden = json.loads(str(d["index"]))[name]
    r = Runner.b200(cfg, w, context=16, block_tokens=kv[0], max_blocks=kv[1], prefix_blocks=kv[2], max_sequences=8,
                    max_step_tokens=64, max_step_sequences=8)
    rec = scenarios.run_runner_script(r, ops, (HostError,))
    r.close()
    assert len(rec) == len(golden)
    for op, (status, value), (gstatus, gvalue) in zip(ops, rec, golden):
        if gstatus == "logits":
            assert status == "ok", (op, value)
            close(value, d[gvalue])
            assert int(np.argmax(value)) == int(np.argmax(d[gvalue])), op
        else:
            assert [status, value] == [gstatus, gvalue], op
