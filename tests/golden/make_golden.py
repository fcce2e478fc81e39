"""Generates the golden fixtures in this folder from the REFERENCE itself: the
MiniPrefix CPU runner and engine of TinyInfer compiled from its own sources into
oracle/_ref/libmpref.so (recipe: oracle/Makefile), driven through
oracle/oracle.py. Run from the repository root with the reference present:

    python tests/golden/make_golden.py            # all fixtures
    python tests/golden/make_golden.py config1    # one of: config1 runner engine

Fixtures (all inputs are regenerated from the recorded seeds, so only outputs
are stored):

* config1_135m.npz -- BASELINE config 1 on the 135M-shape model (weights
  N(0, 0.02) from PCG64 seed 1, tied head): 256 prompt tokens (seed 1), then 64
  greedy decode appends through CpuRunner (miniprefix/src/backend/cpu/
  llama_runner.cpp), context 320, KvCacheConfig{16, 20, 0}. Per step (prefill +
  64 decodes): the greedy token (first index of the maximum), the top-8 logits,
  sum / sum of squares in float64, and the SHA-256 of the float32 logits bytes;
  the full logits of the prefill and of the last decode step. The token stream of
  the same request through the reference Engine (max_batch 1, token budget 256,
  prefill chunk 256, 64 new tokens) is stored too.
* runner_scripts.npz -- the scenarios.runner_scripts() operation lists on the
  MINI model through CpuRunner: per operation its outcome (logits, reuse length,
  admission, error code, shared stats).
* engine_traces.json.gz -- scenarios.engine_workload(seed) for 12 seeds (8-11 copy-on-write
  heavy) through the
  reference Engine over its scripted runner (a real KVManager): per operation its
  outcome and after every step events, step stats, runner stats, cost counters,
  engine state and every sequence's pages.
"""
from __future__ import annotations

import gzip
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
if HERE not in sys.path:
    sys.path.insert(0, HERE)

import scenarios  # noqa: E402

CONFIG1 = dict(weights_seed=1, prompt_seed=1, prompt_tokens=256, decode_steps=64, context=320, block_tokens=16,
               max_blocks=20, top=8)
ENGINE_SEEDS = tuple(range(12))


def logits_summary(rows: list[np.ndarray], top: int) -> dict:
    arr = np.stack(rows).astype(np.float32)
    idx = np.argsort(-arr, axis=1, kind="stable")[:, :top]
    return {
        "tokens": np.array([int(np.argmax(r)) for r in arr], dtype=np.int32),
        "top_index": idx.astype(np.int32),
        "top_value": np.take_along_axis(arr, idx, axis=1),
        "sum": arr.astype(np.float64).sum(axis=1),
        "sumsq": (arr.astype(np.float64) ** 2).sum(axis=1),
        "sha256": np.array([hashlib.sha256(r.tobytes()).hexdigest() for r in arr]),
    }


def make_config1(ref):
    from oracle.oracle import RefEngine, RefRunner
    from tinyinfer_b200.synthetic import SMOLLM2_135M, random_tokens, random_weights

    c = CONFIG1
    w = random_weights(SMOLLM2_135M, seed=c["weights_seed"])
    prompt = random_tokens(c["prompt_tokens"], SMOLLM2_135M.vocabulary, seed=c["prompt_seed"])
    r = RefRunner.cpu(ref, SMOLLM2_135M, w, c["context"], c["block_tokens"], c["max_blocks"], 0)
    r.create("config1")
    rows = [r.append("config1", prompt)]
    for _ in range(c["decode_steps"]):
        rows.append(r.append("config1", [int(np.argmax(rows[-1]))]))
    r.close()
    s = logits_summary(rows, c["top"])
    # the same request through the reference Engine
    r = RefRunner.cpu(ref, SMOLLM2_135M, w, c["context"], c["block_tokens"], c["max_blocks"], 0)
    e = RefEngine(r, 1, 256, 256, c["context"])
    e.submit("config1", prompt, c["decode_steps"])
    while not e.idle():
        e.step()
    stream = [t for _, t, _, _ in e.poll_events() if t is not None]
    e.close()
    r.close()
    np.savez_compressed(os.path.join(HERE, "config1_135m.npz"), prompt=np.array(prompt, dtype=np.int32),
                        engine_stream=np.array(stream, dtype=np.int32), first_logits=rows[0].astype(np.float32),
                        last_logits=rows[-1].astype(np.float32), meta=json.dumps(c), **s)


def make_runner_scripts(ref):
    from oracle.oracle import RefError, RefRunner

    cfg, w = scenarios.mini_weights()
    out = {}
    for name, (kv, ops) in scenarios.runner_scripts().items():
        r = RefRunner.cpu(ref, cfg, w, 16, *kv)
        rec = scenarios.run_runner_script(r, ops, (RefError,))
        r.close()
        out[name] = rec
    arrays, index = {}, {}
    for name, rec in out.items():
        rows = []
        for i, (status, v) in enumerate(rec):
            if status == "ok" and isinstance(v, np.ndarray):
                arrays[f"{name}/{i}"] = v
                rows.append(["logits", f"{name}/{i}"])
            else:
                rows.append([status, v])
        index[name] = rows
    np.savez_compressed(os.path.join(HERE, "runner_scripts.npz"), index=json.dumps(index), **arrays)


def make_engine_traces(ref):
    from oracle.oracle import RefEngine, RefError, RefRunner

    traces = {}
    for seed in ENGINE_SEEDS:
        p, ops = scenarios.engine_workload(seed)
        r = RefRunner.scripted_runner(ref, p["vocab"], p["context"], 1, 1, p["block_tokens"], p["max_blocks"],
                                      p["prefix_blocks"])
        e = RefEngine(r, p["max_batch"], p["token_budget"], p["prefill_chunk"], p["context"])
        rec = scenarios.run_engine_workload(e, r, ops, (RefError,))
        e.close()
        r.close()
        traces[str(seed)] = json.loads(json.dumps(rec))
    with gzip.open(os.path.join(HERE, "engine_traces.json.gz"), "wt") as f:
        json.dump(traces, f, separators=(",", ":"))


def main(which):
    from oracle import oracle

    if not (os.path.exists(oracle.REF_SO) or oracle.build_ref()):
        raise SystemExit("the reference library oracle/_ref/libmpref.so is not built and cannot be")
    ref = oracle.RefLib()
    for name, fn in (("config1", make_config1), ("runner", make_runner_scripts), ("engine", make_engine_traces)):
        if not which or name in which:
            t = time.time()
            fn(ref)
            print(f"{name}: {time.time() - t:.1f} s")


if __name__ == "__main__":
    main(sys.argv[1:])
