"""Pins the C oracle (oracle/mp_oracle.c) to the reference CPU runner (oracle/_ref):
logits must be bit-identical, on the reference's own regression model
(miniprefix/tests/cow_test.cpp:118-137 shape, 2 layers, hidden 8) and on
135M-geometry models."""
import numpy as np
import pytest

from oracle.oracle import Oracle, RefRunner
from tinyinfer_b200.synthetic import ModelConfig, random_weights, sine_weights, random_tokens

TINY = ModelConfig(layers=2, hidden=8, heads=2, kv_heads=1, intermediate=12, vocabulary=16, context=32, eos=0,
                   rms_epsilon=1e-5, rope_theta=10000, tied=False)


def run_pair(ref, config, weights, block_tokens, appends):
    """Append the same chunks through both; the oracle gets the pages the reference's
    LIFO free list hands out for a fresh pool (0, 1, 2, ...)."""
    r = RefRunner.cpu(ref, config, weights, config.context, block_tokens, 64, 0)
    o = Oracle(config, weights, block_tokens)
    keys, values = o.new_pools(64)
    r.create("s")
    used = 0
    out = []
    for chunk in appends:
        pages = list(range(-(-(used + len(chunk)) // block_tokens)))
        a = r.append("s", chunk)
        b, ok = o.append(keys, values, pages, used, chunk)
        assert ok
        out.append((a, b))
        used += len(chunk)
    r.close()
    return out


def test_tiny_model_bit_exact(ref):
    w = sine_weights(TINY)
    for a, b in run_pair(ref, TINY, w, 4, [[1, 2, 3], [4, 5], [6], [7, 8, 9, 10, 11]]):
        assert np.array_equal(a, b)


def test_135m_geometry_bit_exact(ref):
    c = ModelConfig(layers=2, vocabulary=2048, context=256)
    w = random_weights(c, seed=11)
    toks = random_tokens(50, c.vocabulary, seed=3)
    for a, b in run_pair(ref, c, w, 16, [toks[:37], toks[37:38], toks[38:50]]):
        assert np.array_equal(a, b)


def test_tied_head_bit_exact(ref):
    c = ModelConfig(layers=1, vocabulary=1024, context=64, tied=True)
    w = random_weights(c, seed=5)
    for a, b in run_pair(ref, c, w, 16, [random_tokens(20, c.vocabulary, 9)]):
        assert np.array_equal(a, b)


def test_nonfinite_is_reported(ref):
    w = sine_weights(TINY)
    w["model.embed_tokens.weight"][15, :] = np.nan
    o = Oracle(TINY, w, 4)
    k, v = o.new_pools(8)
    _, ok = o.append(k, v, [0], 0, [15])
    assert not ok
    r = RefRunner.cpu(ref, TINY, w, 16, 4, 8, 0)
    r.create("a")
    from oracle.oracle import RefError
    with pytest.raises(RefError):
        r.append("a", [15])
