"""The reference-side drop-in: the reference's own regression
miniprefix/tests/cow_test.cpp, compiled UNMODIFIED with MINIPREFIX_ENABLE_CUDA and
linked against tinyinfer_b200/dropin/b200_model_runner.cpp, so that its
make_cuda_runner(weights, context, kv) returns the B200 runner behind the
reference's ModelRunner virtuals (miniprefix/include/miniprefix/model.h:35-62).
With --cuda its runner / partial_cache / costs / publication scenarios
(cow_test.cpp:138-256) compare the B200 runner with the reference CPU runner
(abs < 2e-5 and argmax, its own bar) through fork, copy-on-write, failed appends
that roll back and retry, partial prefix reuse and cost counters.
Built by oracle/Makefile's `dropin` target (oracle.build_ref())."""
import os
import subprocess

import pytest

from oracle import oracle

PASSED = ["COW metadata passed", "COW payload passed", "COW copy, capacity, rollback, retry and release passed",
          "Partial prefix cache, COW and capacity passed", "Cost counters and opt-in timing passed",
          "Publication snapshot churn, rollback and release passed"]


def binary():
    if not os.path.exists(oracle.DROPIN_TEST):
        oracle.build_ref()
    if not os.path.exists(oracle.DROPIN_TEST):
        pytest.skip("oracle/_ref/cow_test_b200 not built and the reference sources are absent")
    return oracle.DROPIN_TEST


def test_reference_cow_test_links_against_the_dropin(built):
    """Without --cuda the binary runs the reference's CPU scenarios: it loads, links
    the drop-in and the product host library, and passes."""
    r = subprocess.run([binary()], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    for line in PASSED:
        assert line in r.stdout


@pytest.mark.gpu
def test_reference_cow_test_on_the_b200_runner(built):
    r = subprocess.run([binary(), "--cuda", "--require-device"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    for line in PASSED:
        assert line in r.stdout
