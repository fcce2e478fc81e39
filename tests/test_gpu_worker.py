"""The protocol worker and the lifecycle stress harness on a B200.

* mpb200_worker: an MPFX0001 model served over stdin/stdout with protocol v3
  (miniprefix/apps/worker.cpp); the READY line, the events of a short run and a
  FORWARD diagnostic must match the C oracle's greedy tokens and logits.
* mpb200_stress: the reference's 8-request wave harness (benchmarks/stress.cpp)
  for a few waves: tokens equal the no-cache stream, no sequence, table or page
  leaks, bounded pool, exit status 0.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200 import mpfx
from tinyinfer_b200.synthetic import ModelConfig, random_weights

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(HERE, "tinyinfer_b200", "mpb200_worker")
STRESS = os.path.join(HERE, "tinyinfer_b200", "mpb200_stress")
CFG = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=128, tied=True)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    w = random_weights(CFG, seed=31)
    path = str(tmp_path_factory.mktemp("mpfx") / "model.mpfx")
    mpfx.write(path, CFG, w)
    return path, w


@pytest.mark.gpu
def test_worker_serves_protocol(built, model):
    path, w = model
    o = Oracle(CFG, w, 4)

    def greedy(seq):
        keys, values = o.new_pools(40)
        out, _ = o.append(keys, values, list(range(40)), 0, list(seq))
        return out

    prompt = [int(t) for t in np.random.default_rng(2).integers(0, 64, 9)]
    lines = [f"SUBMIT 1 4 -1 {len(prompt)} " + " ".join(map(str, prompt))] + ["STEP"] * 6 + \
            [f"FORWARD 3 {len(prompt)} " + " ".join(map(str, prompt)), "STATS", "QUIT"]
    proc = subprocess.run([WORKER, path, "b200", "64", "4", "32", "16", "4", "64", "8"],
                          input="\n".join(lines) + "\n", capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr
    out = proc.stdout.splitlines()
    assert out[0] == "READY MINIPREFIX 3 64 0 64 b200"
    replies = out[1:]
    assert len(replies) == len(lines)  # one response line per command
    tokens, finished = [], None
    for cmd, reply in zip(lines, replies):
        if cmd != "STEP":
            continue
        f = reply.split()
        assert f[0] == "OK" and len(f) == 2 + 3 * int(f[1])
        for i in range(int(f[1])):
            rid, tok, reason = f[2 + 3 * i: 5 + 3 * i]
            assert rid == "1"
            if int(tok) >= 0:
                tokens.append(int(tok))
            if int(reason) >= 0:
                finished = int(reason)
    seq = list(prompt)
    for t in tokens:
        assert t == int(np.argmax(greedy(seq)))
        seq.append(t)
    assert len(tokens) == 4 and finished == 1  # length
    forward = replies[lines.index(next(c for c in lines if c.startswith("FORWARD")))].split()
    assert forward[0] == "OK" and len(forward) == 1 + CFG.vocabulary
    logits = np.array([float(v) for v in forward[1:]], dtype=np.float32)
    ref = greedy(prompt)
    assert (np.abs(logits - ref) <= 1e-3 + 1e-4 * np.abs(ref)).all()
    assert out[-1] == "OK"


@pytest.mark.gpu
def test_stress_waves(built, model):
    path, _ = model
    proc = subprocess.run([STRESS, path, "b200", "1", "3"], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr
    records = [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]
    summary = records[-1]
    assert summary["passed"] and summary["waves"] >= 3 and summary["requests"] == 8 * summary["waves"]
    for r in records[:-1]:
        assert r["tokens"] > 0 and r["cached_pages"] <= 12
