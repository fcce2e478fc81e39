"""Chunked prefill on the tensor-core attention kernel vs the C oracle.

The 135M widths (hidden 576, 9 q / 3 kv heads, head dim 64, vocabulary 49152) with
4 layers so the oracle stays fast. Two sequences prefill 1100 and 700-token
prompts in 512-token chunks -- several in one forward, tiles of 42 rows that end
mid-chunk, contexts past 1024 tokens -- then decode two tokens together. The
logits of every forward's last row per sequence must be within
|gpu - oracle| <= 1e-3 + 1e-4 |oracle| of the oracle appending the same chunks
(miniprefix/src/backend/cpu/llama_runner.cpp:60-104), and the greedy tokens equal.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200.synthetic import ModelConfig, random_tokens, random_weights


def close(gpu, ref):
    err = np.abs(gpu - ref)
    assert np.isfinite(gpu).all()
    assert (err <= 1e-3 + 1e-4 * np.abs(ref)).all(), float(err.max())
    assert int(np.argmax(gpu)) == int(np.argmax(ref))
    return float(err.max())


@pytest.mark.gpu
def test_chunked_prefill_two_sequences_against_oracle(built):
    from tinyinfer_b200.device import DeviceContext

    cfg = ModelConfig(layers=4, context=2048)
    w = random_weights(cfg, seed=41)
    o = Oracle(cfg, w, 16)
    lengths = {0: 1100, 1: 700}
    prompts = {s: random_tokens(n, cfg.vocabulary, 50 + s) for s, n in lengths.items()}
    pages = {0: list(range(0, 72)), 1: list(range(72, 118))}  # enough for the prompt + 2 decode tokens
    ctx = DeviceContext(cfg, device=0, block_tokens=16, max_blocks=128, max_sequences=2, max_step_tokens=1024,
                        max_step_sequences=2)
    ctx.load_weights(w)
    for s, tbl in pages.items():
        ctx.table_write(s, 0, tbl)
    pools = {s: o.new_pools(128) for s in pages}
    used = {0: 0, 1: 0}
    worst = 0.0

    def step(parts):
        nonlocal worst
        seqs = [(s, used[s], len(toks)) for s, toks in parts]
        t, f, logits, rc = ctx.forward(seqs, np.concatenate([np.asarray(toks, dtype=np.int32) for _, toks in parts]))
        assert rc == 0 and f.all()
        out = {}
        for i, (s, toks) in enumerate(parts):
            ref, ok = o.append(*pools[s], pages[s], used[s], list(toks))
            assert ok
            worst = max(worst, close(logits[i], ref))
            used[s] += len(toks)
            out[s] = int(t[i])
        return out

    step([(0, prompts[0][0:512]), (1, prompts[1][0:512])])
    second = step([(0, prompts[0][512:1024]), (1, prompts[1][512:700])])
    last = step([(0, prompts[0][1024:1100])])
    last[1] = second[1]  # sequence 1's prompt ended in the second forward
    for _ in range(2):
        last = step([(0, [last[0]]), (1, [last[1]])])
    ctx.close()
    print(f"chunked prefill: worst abs err {worst:.3g}")


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [3, 4])
def test_prefill_operator_against_oracle(built, seed):
    """mp_paged_attention_prefill on random N(0,1) Q/K/V: chunks at positions 0 and
    deep into a context, tiles that end mid-chunk, single-row chunks, page tables
    that are a random permutation of the pool. Each row equals the oracle's decode
    attention of that row over the tokens up to its position, within the attention
    tests' tolerance |gpu - oracle| <= 1e-5 + 1e-4 |oracle|."""
    import torch
    from tinyinfer_b200 import device

    rng = np.random.default_rng(seed)
    bt, pool = 16, 2048
    chunks = [(0, 50), (100, 42), (1000, 300), (3584, 512), (7, 1), (64, 43)]
    stride = max(-(-(s + c) // bt) for s, c in chunks)
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((len(chunks), stride), dtype=np.int32)
    at = 0
    for i, (s, c) in enumerate(chunks):
        n = -(-(s + c) // bt)
        tables[i, :n] = perm[at:at + n]
        at += n
    keys = rng.standard_normal(pool * bt * 192, dtype=np.float32)
    values = rng.standard_normal(pool * bt * 192, dtype=np.float32)
    rows = sum(c for _, c in chunks)
    q = rng.standard_normal((rows, 576), dtype=np.float32)
    dev = torch.device("cuda:0")
    tq, tk, tv, tt = (torch.from_numpy(a).to(dev) for a in (q, keys, values, tables))
    out = torch.full_like(tq, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    device.paged_attention_prefill(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), 1, 0, bt, pool, tt.data_ptr(), stride,
                                   [s for s, _ in chunks], [c for _, c in chunks], out.data_ptr(), stream)
    assert device.paged_attention_status(stream) == 0
    got = out.cpu().numpy()
    lengths = np.concatenate([np.arange(s + 1, s + c + 1) for s, c in chunks]).astype(np.int32)
    row_tables = np.concatenate([np.repeat(tables[i:i + 1], c, axis=0) for i, (_, c) in enumerate(chunks)])
    expect = Oracle.decode_attention(q, lengths, row_tables, keys, values, 9, 3, 64, bt)
    assert np.isfinite(got).all()
    err = np.abs(got - expect)
    assert (err <= 1e-5 + 1e-4 * np.abs(expect)).all(), float(err.max())
