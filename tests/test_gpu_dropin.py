"""The reference-side drop-in (tinyinfer_b200/dropin/b200_model_runner.cpp):
miniprefix::make_cuda_runner backed by the B200 runner, compiled against the
reference's own headers and linked into the reference's own, unmodified sources
by oracle/Makefile's `dropin` target:

* miniprefix/apps/worker.cpp -> oracle/_ref/miniprefix_worker_b200. Its `cuda`
  backend is make_cuda_runner (the B200 runner behind the reference's ModelRunner
  virtuals, model.h:35-62), its `cpu` backend the reference CPU runner. The GPU
  test serves one protocol v3 session on an MPFX0001 file of the 135M geometry
  (2 layers) through both and compares the transcripts: events, step stats and
  prefix-reuse counts identical, FORWARD logits within |gpu - cpu| <= 1e-3 +
  1e-4 |cpu| with the same argmax, the KV fields of STATS and the counting fields
  of COST_STATS identical.
* miniprefix/tests/cow_test.cpp -> oracle/_ref/cow_test_b200, linked against the
  drop-in. Its --cuda scenarios build the regression model of cow_test.cpp:118-137
  (hidden 8, head dim 4), which is outside the B200 kernels' specialisation (9 q /
  3 kv heads of dim 64): make_cuda_runner rejects it, so only its CPU scenarios run
  here, as a check that the reference's test compiles and links against the file.
"""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle

RUNNER_FIELDS = oracle.RUNNER_STATS_FIELDS
KV_STATS = set(oracle.KV_STATS_FIELDS)
COUNTS = (0, 2, 4, 5)  # lookup_calls, publish_calls, cow_pages, cow_bytes
WORKER = os.path.join(os.path.dirname(oracle.DROPIN_TEST), "miniprefix_worker_b200")


def binary(path):
    if not os.path.exists(path):
        oracle.build_ref()
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not built and the reference sources are absent")
    return path


def test_reference_cow_test_links_against_the_dropin(built):
    r = subprocess.run([binary(oracle.DROPIN_TEST)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Publication snapshot churn, rollback and release passed" in r.stdout


def session(rng, vocab):
    shared = [int(t) for t in rng.integers(1, vocab, 17)]  # a partial shared page at 16 tokens per page
    own = lambda n: [int(t) for t in rng.integers(1, vocab, n)]

    def submit(i, new, prompt):
        return f"SUBMIT {i} {new} -1 {len(prompt)} " + " ".join(map(str, prompt))

    lines = [submit(1, 6, shared + own(3))] + ["STEP"] * 3
    lines += [submit(2, 5, shared + own(2)), submit(3, 5, shared + own(4))] + ["STEP", "STEP_STATS"] * 8
    lines += ["FORWARD 7 5 " + " ".join(map(str, own(5))), "REUSE 8 18 " + " ".join(map(str, shared + own(1))),
              "FORWARD 8 1 " + str(own(1)[0]), "CACHE 7", "STATS", "COST_STATS", "RELEASE 7", "RELEASE 8",
              "CLEAR_PREFIX", "STATS", "QUIT"]
    return "\n".join(lines) + "\n"


def serve(path, backend, model, text):
    args = [path, model, backend, "256", "4", "64", "16", "16", "64", "16"]
    r = subprocess.run(args, input=text, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return r.stdout.splitlines()


@pytest.mark.gpu
def test_reference_worker_serves_on_the_b200_runner(built, tmp_path):
    from tinyinfer_b200 import mpfx
    from tinyinfer_b200.synthetic import ModelConfig, random_weights

    worker = binary(WORKER)
    cfg = ModelConfig(layers=2, context=512)
    model = str(tmp_path / "m135_2layer.mpfx")
    mpfx.write(model, cfg, random_weights(cfg, seed=23))
    text = session(np.random.default_rng(6), cfg.vocabulary)
    gpu = serve(worker, "cuda", model, text)
    cpu = serve(worker, "cpu", model, text)
    assert len(gpu) == len(cpu) and gpu[0].endswith(" cuda") and cpu[0].endswith(" cpu")
    commands = text.splitlines()
    forwards = stats_seen = 0
    for cmd, g, c in zip(commands, gpu[1:], cpu[1:]):
        verb = cmd.split()[0]
        assert g.startswith("OK") and c.startswith("OK"), (cmd, g[:80], c[:80])
        if verb == "FORWARD":
            a = np.array(g.split()[1:], dtype=np.float64)
            b = np.array(c.split()[1:], dtype=np.float64)
            assert a.shape == b.shape == (cfg.vocabulary,)
            assert (np.abs(a - b) <= 1e-3 + 1e-4 * np.abs(b)).all(), float(np.abs(a - b).max())
            assert int(np.argmax(a)) == int(np.argmax(b))
            forwards += 1
        elif verb == "STATS":
            a, b = g.split()[1:], c.split()[1:]
            assert len(a) == len(b) == 25
            for name, x, y in zip(RUNNER_FIELDS, a, b):
                if name in KV_STATS:
                    assert x == y, (name, x, y)
            stats_seen += 1
        elif verb == "COST_STATS":
            a, b = g.split()[1:], c.split()[1:]
            assert [a[i] for i in COUNTS] == [b[i] for i in COUNTS], (a, b)
        else:
            assert g == c, (cmd, g, c)
    assert forwards == 2 and stats_seen == 2
