"""The committed golden fixtures (tests/golden/, recorded from the reference's own
CPU runner and engine by tests/golden/make_golden.py) against the C oracle and the
product's host layer -- no reference library needed.

* config 1 (135M-shape model, 256-token prompt, 64 greedy decode appends): the
  oracle's logits are bit-identical to the reference's at every step (SHA-256 of
  the float32 bytes), so its greedy stream is too;
* runner scripts (fork / COW / failure / prefix reuse on the MINI model): the
  oracle recomputing each sequence's whole history from an empty pool gives the
  reference's logits bit for bit;
* engine traces: the batched host Engine over the scripted runner reproduces the
  reference Engine's events, stats, counters, state, page tables and
  copy-on-write regions exactly.
"""
import gzip
import hashlib
import json
import os
import sys

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)

import scenarios  # noqa: E402


def load_runner_scripts():
    d = np.load(os.path.join(GOLDEN, "runner_scripts.npz"))
    index = json.loads(str(d["index"]))
    out = {}
    for name, rows in index.items():
        out[name] = [("ok", d[v]) if s == "logits" else (s, v) for s, v in rows]
    return out


class Histories:
    """Token history of every sequence of a runner script, as the reference's
    ModelRunner would hold it (appends that fail leave it unchanged)."""

    def __init__(self):
        self.h = {}

    def apply(self, op, outcome):
        name, args = op[0], op[1:]
        status, value = outcome
        if status != "ok":
            return None
        if name == "create":
            self.h[args[0]] = []
        elif name == "append":
            self.h[args[0]] = self.h[args[0]] + list(args[1])
            return list(self.h[args[0]])
        elif name == "fork_sequence":
            self.h[args[1]] = list(self.h[args[0]])
        elif name == "reuse_prefix":
            self.h[args[0]] = list(args[1][:value])
        elif name == "release":
            self.h.pop(args[0], None)
        elif name == "clear":
            self.h.clear()
        return None


def test_oracle_config1_bit_exact_to_golden():
    from oracle.oracle import Oracle
    from tinyinfer_b200.synthetic import SMOLLM2_135M, random_weights

    g = np.load(os.path.join(GOLDEN, "config1_135m.npz"))
    meta = json.loads(str(g["meta"]))
    w = random_weights(SMOLLM2_135M, seed=meta["weights_seed"])
    o = Oracle(SMOLLM2_135M, w, meta["block_tokens"])
    keys, values = o.new_pools(meta["max_blocks"])
    pages = list(range(meta["max_blocks"]))
    prompt = [int(t) for t in g["prompt"]]
    out, ok = o.append(keys, values, pages, 0, prompt)
    used = len(prompt)
    assert ok and np.array_equal(out, g["first_logits"])
    for step in range(meta["decode_steps"] + 1):
        assert hashlib.sha256(out.astype(np.float32).tobytes()).hexdigest() == str(g["sha256"][step]), step
        assert int(np.argmax(out)) == int(g["tokens"][step])
        if step == meta["decode_steps"]:
            break
        out, ok = o.append(keys, values, pages, used, [int(g["tokens"][step])])
        used += 1
        assert ok
    assert np.array_equal(out, g["last_logits"])
    # the reference Engine's stream is the runner's greedy stream
    assert list(g["engine_stream"]) == list(g["tokens"][:meta["decode_steps"]])


def test_oracle_replays_runner_scripts_bit_exact():
    from oracle.oracle import Oracle

    cfg, w = scenarios.mini_weights()
    o = Oracle(cfg, w, 4)
    golden = load_runner_scripts()
    checked = 0
    for name, (kv, ops) in scenarios.runner_scripts().items():
        hist = Histories()
        assert len(golden[name]) == len(ops)
        for op, outcome in zip(ops, golden[name]):
            seq = hist.apply(op, outcome)
            if seq is None:
                continue
            keys, values = o.new_pools(16)
            out, ok = o.append(keys, values, list(range(16)), 0, seq)
            assert ok and np.array_equal(out, outcome[1]), (name, op)
            checked += 1
    assert checked >= 30


def test_runner_script_failures_are_recorded():
    """Every append of the poisoned token failed in the reference with
    runtime_error (-4) and left no trace in the shared stats."""
    golden = load_runner_scripts()
    for name, (kv, ops) in scenarios.runner_scripts().items():
        for op, (status, value) in zip(ops, golden[name]):
            if op[0] == "append" and scenarios.POISON in op[2]:
                assert (status, value) == ("err", -4), (name, op)


@pytest.mark.parametrize("seed", range(12))
def test_host_engine_matches_golden_trace(built, seed):
    from tinyinfer_b200.host import Engine, HostError, Runner

    with gzip.open(os.path.join(GOLDEN, "engine_traces.json.gz"), "rt") as f:
        golden = json.load(f)[str(seed)]
    p, ops = scenarios.engine_workload(seed)
    r = Runner.scripted(p["vocab"], p["context"], 1, 1, p["block_tokens"], p["max_blocks"], p["prefix_blocks"])
    e = Engine(r, p["max_batch"], p["token_budget"], p["prefill_chunk"], p["context"])
    rec = json.loads(json.dumps(scenarios.run_engine_workload(e, r, ops, (HostError,))))
    assert len(rec) == len(golden)
    for i, (a, b) in enumerate(zip(rec, golden)):
        assert a == b, (seed, i)
