"""Paged-attention decode operator vs the C oracle (BASELINE config 2 and edge cases).

Config 2: 64 sequences, lengths U[1, 4096], 9 q / 3 kv heads, head_dim 64, page 16,
block tables a random permutation of a 32768-page pool, Q/K/V ~ N(0, 1) (seeded).
Every pool row the kernel must NOT read (unused pages, slots past a sequence's
length) holds NaN, so any stray read shows up as NaN in the output.
Tolerance (fp32 with a different summation order): |gpu - oracle| <= 1e-5 + 1e-4 |oracle|.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle

HEADS, KVH, DIM = 9, 3, 64
KVW = KVH * DIM


def make_case(seed, count, max_len, block_tokens, pool_pages, lengths=None):
    rng = np.random.default_rng(seed)
    if lengths is None:
        lengths = rng.integers(1, max_len + 1, size=count)
    lengths = np.asarray(lengths, dtype=np.int32)
    pages = (lengths + block_tokens - 1) // block_tokens
    stride = int(pages.max())
    perm = rng.permutation(pool_pages).astype(np.int32)
    assert pages.sum() <= pool_pages
    tables = np.full((len(lengths), stride), -1, dtype=np.int32)
    at = 0
    for i, p in enumerate(pages):
        tables[i, :p] = perm[at:at + p]
        at += p
    keys = np.full((pool_pages, block_tokens, KVW), np.nan, dtype=np.float32)
    values = np.full_like(keys, np.nan)
    for i, L in enumerate(lengths):
        for t in range(0, L, block_tokens):
            n = min(block_tokens, L - t)
            blk = tables[i, t // block_tokens]
            keys[blk, :n] = rng.standard_normal((n, KVW), dtype=np.float32)
            values[blk, :n] = rng.standard_normal((n, KVW), dtype=np.float32)
    q = rng.standard_normal((len(lengths), HEADS * DIM), dtype=np.float32)
    return q, keys.reshape(-1), values.reshape(-1), tables, lengths


def run_gpu(q, keys, values, tables, lengths, block_tokens, pool_pages, pps):
    import torch
    from tinyinfer_b200 import device

    dev = torch.device("cuda:0")
    tq = torch.from_numpy(q).to(dev)
    tk = torch.from_numpy(keys).to(dev)
    tv = torch.from_numpy(values).to(dev)
    tt = torch.from_numpy(np.ascontiguousarray(tables)).to(dev)
    out = torch.full_like(tq, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    device.paged_attention_decode(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), 1, 0, block_tokens, pool_pages,
                                  tt.data_ptr(), tables.shape[1], lengths, out.data_ptr(), pps, stream)
    status = device.paged_attention_status(stream)
    torch.cuda.synchronize()
    return out.cpu().numpy(), status


def check_close(gpu, ref):
    assert np.isfinite(gpu).all()
    err = np.abs(gpu - ref)
    bound = 1e-5 + 1e-4 * np.abs(ref)
    assert (err <= bound).all(), f"max abs err {err.max():.3e}"
    return float(err.max())


@pytest.mark.gpu
def test_config2_matches_oracle(built):
    q, k, v, tables, lengths = make_case(2, 64, 4096, 16, 32768)
    ref = Oracle.decode_attention(q, lengths, tables, k, v, HEADS, KVH, DIM, 16)
    gpu, status = run_gpu(q, k, v, tables, lengths, 16, 32768, 0)
    assert status == 0
    print("config2 max abs err", check_close(gpu, ref))


@pytest.mark.gpu
@pytest.mark.parametrize("block_tokens,pps", [(16, 1), (16, 3), (4, 5), (12, 2), (32, 0), (1, 40), (16, 0), (4, 0),
                                               (1, 0)])
def test_edge_lengths_and_splits(built, block_tokens, pps):
    lengths = [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 100, 255, 256, 257, 1000]
    pool = sum(-(-L // block_tokens) for L in lengths) + 7
    q, k, v, tables, lengths = make_case(5, 0, 0, block_tokens, pool, lengths)
    ref = Oracle.decode_attention(q, lengths, tables, k, v, HEADS, KVH, DIM, block_tokens)
    gpu, status = run_gpu(q, k, v, tables, lengths, block_tokens, pool, pps)
    assert status == 0
    check_close(gpu, ref)


@pytest.mark.gpu
def test_repeated_launches_reuse_counters(built):
    """Arrival counters reset themselves: back-to-back launches give identical results."""
    q, k, v, tables, lengths = make_case(9, 16, 700, 16, 2048)
    a, _ = run_gpu(q, k, v, tables, lengths, 16, 2048, 2)
    b, _ = run_gpu(q, k, v, tables, lengths, 16, 2048, 2)
    assert np.array_equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("count,max_len", [(300, 40), (3, 5000), (444, 16), (7, 1)])
def test_static_runs_match_oracle(built, count, max_len):
    """pages_per_split 0: the pages of all sequences, concatenated, cut into one
    equal run per CTA (fewer runs than CTAs when there are fewer pages; a run
    spanning several sequences; a sequence spanning many runs); two launches give
    identical results."""
    pool = count * (-(-max_len // 16)) + 5
    q, k, v, tables, lengths = make_case(13 + count, count, max_len, 16, pool)
    ref = Oracle.decode_attention(q, lengths, tables, k, v, HEADS, KVH, DIM, 16)
    a, status = run_gpu(q, k, v, tables, lengths, 16, pool, 0)
    assert status == 0
    check_close(a, ref)
    b, _ = run_gpu(q, k, v, tables, lengths, 16, pool, 0)
    assert np.array_equal(a, b)


@pytest.mark.gpu
def test_out_of_range_page_is_reported(built):
    """A block-table entry outside the pool is caught on the device (no fault) and
    reported as MP_ERR_BOUNDS."""
    from tinyinfer_b200 import device

    q, k, v, tables, lengths = make_case(3, 4, 60, 16, 64)
    tables = tables.copy()
    tables[1, 0] = 64 + 5
    _, status = run_gpu(q, k, v, tables, lengths, 16, 64, 0)
    assert status == device.MP_ERR_BOUNDS
    _, status = run_gpu(*make_case(3, 4, 60, 16, 64), 16, 64, 0)
    assert status == 0
