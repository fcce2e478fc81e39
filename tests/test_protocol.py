"""Worker protocol v3 (miniprefix/apps/protocol/*): this engine's serve loop vs the
reference's own protocol code, transcript against transcript.

Both sides run a scripted runner that keeps the real KV manager of its side and
answers each append with the next token of the request's script (one-hot
logits), so every response line -- events, stats, diagnostics, errors -- must be
byte-identical. The command streams are the reference test's own scripts
(worker_protocol_test.cpp: parse errors, a full transcript, recovery after bad
lines and end of input, diagnostics after a failed engine) and seeded random
streams that mix valid and malformed commands.
"""
import numpy as np
import pytest

from oracle.oracle import RefEngine, RefRunner
from tinyinfer_b200.host import Engine, Runner


def pair(ref, *, vocab=8, context=16, bt=4, max_blocks=32, cache=8, batch=2, budget=8, chunk=4):
    mr = Runner.scripted(vocab, context, 1, 1, bt, max_blocks, cache)
    rr = RefRunner.scripted_runner(ref, vocab, context, 1, 1, bt, max_blocks, cache)
    return Engine(mr, batch, budget, chunk, context), RefEngine(rr, batch, budget, chunk, context), mr, rr


def script(runners, rid, tokens):
    for r in runners:
        r.script(rid, tokens)


PARSE_ERRORS = ["COST_TIMING 2", "COST_TIMING", "", "step", "UNKNOWN 1", "CANCEL", "CANCEL 2147483648",
                "SUBMIT 0 0 -2 0", "SUBMIT 0 0 -2", "SUBMIT 1 1 -2 0", "SUBMIT 1 1 -2 1", "SUBMIT 1 1 -2 1 0",
                "FORWARD 0 0", "REUSE 0 1", "REUSE 0 1 0", "FORWARD 1 131073", "FORWARD 1 -1",
                " \tSUBMIT +1 2 -1 2 0 3 trailing ignored\r", "CACHE -2", "RELEASE 0", "STEP junk", "CANCEL 1x"]


def test_parse_errors_and_lenient_forms(built, ref):
    me, re, mr, rr = pair(ref)
    script((mr, rr), "1", [5, 6, 7])
    text = "\n".join(PARSE_ERRORS) + "\n"
    a, b = me.serve(text), re.serve(text)
    assert a == b
    assert "ERROR invalid timing flag\nERROR missing integer\nERROR unknown command\n" in a


def test_reference_scripts(built, ref):
    for text in (
        "FORWARD 1 1 1\nSUBMIT 1 1 -1 1 1\nCACHE 1\nREUSE 2 2 1 1\nSTEP\nSTEP_STATS\nFORWARD 1 1 8\n"
        "FORWARD 1 1 1\nRELEASE 1\nRELEASE 1\nCACHE -2\nCANCEL 0\nCLEAR_PREFIX\nQUIT\nUNKNOWN\n",
        "\nSUBMIT 1 2 -1 2 1\nSUBMIT 1 2 -1 2 1 1\nSUBMIT 2 1 -1 1 1\nSTEP\nCANCEL 2\nCANCEL 1\nSTEP\n"
        "FORWARD 7 1 8\nFORWARD 7 1 1\nREUSE 7 1 1\nRELEASE 7\nFORWARD 7 1 1",
    ):
        me, re, mr, rr = pair(ref, batch=1, budget=2, chunk=2)
        script((mr, rr), "1", [3, 4, 5])
        script((mr, rr), "2", [6])
        a, b = me.serve(text), re.serve(text)
        assert a == b, (a, b)
        assert me.idle() == re.idle() and me.failed() == re.failed()


def test_failed_engine_rejects_diagnostics(built, ref):
    me, re, mr, rr = pair(ref, batch=1, budget=1, chunk=1)
    for r in (mr, rr):
        r.script("1", [2])
        r.poison(1)  # the first append fails as a nonfinite forward
    text = "SUBMIT 1 1 -1 1 1\nSTEP\nFORWARD 2 1 1\nREUSE 2 1 1\nCACHE 1\nRELEASE 1\nCLEAR_PREFIX\nSTEP_STATS\nSTATS\n"
    a, b = me.serve(text), re.serve(text)
    assert a == b
    assert a.count("ERROR engine failed; create a new engine") == 5
    assert me.failed() and re.failed()


@pytest.mark.parametrize("seed", range(12))
def test_random_streams_match_reference(built, ref, seed):
    rng = np.random.default_rng(900 + seed)
    vocab, context = 8, 24
    me, re, mr, rr = pair(ref, vocab=vocab, context=context, bt=int(rng.choice([2, 4])),
                          max_blocks=int(rng.integers(10, 40)), cache=int(rng.integers(0, 12)),
                          batch=int(rng.integers(1, 4)), budget=int(rng.integers(2, 12)), chunk=int(rng.integers(1, 6)))
    poisoned = seed % 4 == 3
    lines = []
    for rid in range(1, 9):
        script((mr, rr), str(rid), [int(t) for t in rng.integers(0, vocab, 20)])
    if poisoned:
        token = int(rng.integers(0, vocab))
        for r in (mr, rr):
            r.poison(token)
    roots = [[int(t) for t in rng.integers(0, 3, int(rng.integers(1, 10)))] for _ in range(3)]
    for _ in range(80):
        k = int(rng.integers(0, 16))
        rid = int(rng.integers(1, 9))
        if k < 4:
            p = roots[int(rng.integers(0, 3))][: int(rng.integers(1, 9))] + \
                [int(t) for t in rng.integers(0, vocab, int(rng.integers(0, 5)))]
            eos = int(rng.integers(0, vocab)) if rng.random() < 0.3 else -1
            lines.append(f"SUBMIT {rid} {int(rng.integers(1, 6))} {eos} {len(p)} " + " ".join(map(str, p)))
        elif k < 8:
            lines.append("STEP")
        elif k == 8:
            lines.append(f"CANCEL {rid}")
        elif k == 9:
            toks = [int(t) for t in rng.integers(0, vocab + 1, int(rng.integers(1, 4)))]
            lines.append(f"FORWARD {int(rng.integers(1, 4))} {len(toks)} " + " ".join(map(str, toks)))
        elif k == 10:
            p = roots[int(rng.integers(0, 3))]
            lines.append(f"REUSE {int(rng.integers(1, 4))} {len(p)} " + " ".join(map(str, p)))
        elif k == 11:
            lines.append(f"{['CACHE', 'RELEASE'][int(rng.integers(0, 2))]} {int(rng.integers(-1, 4))}")
        elif k == 12:
            lines.append(["STATS", "STEP_STATS", "COST_STATS", "COST_TIMING 0"][int(rng.integers(0, 4))])
        elif k == 13:
            lines.append("CLEAR_PREFIX")
        else:
            lines.append(["", "BOGUS", "SUBMIT 1", "FORWARD 0 1 1", "STEP extra fields", "CANCEL x"][int(rng.integers(0, 6))])
    lines.append("STATS")
    text = "\n".join(lines) + "\n"
    a, b = me.serve(text), re.serve(text)
    assert a.splitlines() == b.splitlines()
    tail = "STATS\nQUIT\nSTATS\n"
    assert me.serve(tail) == re.serve(tail)
