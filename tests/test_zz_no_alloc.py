"""mp_paged_attention_decode_noalloc through the C ABI: the allocation-free
variant of the decode operator, for callers that cannot call cudaMalloc (a host
embedding this library in a runtime that owns all GPU memory, or a path where an
allocation would synchronise the device). Its scratch is a fixed device array, so
this file runs last and must pass both alone and after every other test: the
array keeps the previous call's contents, and results must not depend on them.

Two calls in a row must each match the allocating operator
(mp_paged_attention_decode) within the attention tests' tolerance
|a - b| <= 1e-5 + 1e-4 |b|, and match each other exactly.
"""
import ctypes as C
import os

import numpy as np
import pytest

HEADS, KVH, DIM = 9, 3, 64


def case(seed, count, max_len, bt, pool):
    rng = np.random.default_rng(seed)
    lengths = rng.integers(1, max_len + 1, size=count).astype(np.int32)
    pages = (lengths + bt - 1) // bt
    stride = int(pages.max())
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((count, stride), dtype=np.int32)
    at = 0
    for i, p in enumerate(pages):
        tables[i, :p] = perm[at:at + p]
        at += p
    keys = rng.standard_normal((pool, bt, KVH * DIM), dtype=np.float32).reshape(-1)
    values = rng.standard_normal((pool, bt, KVH * DIM), dtype=np.float32).reshape(-1)
    q = rng.standard_normal((count, HEADS * DIM), dtype=np.float32)
    return q, keys, values, tables, lengths


@pytest.mark.gpu
def test_noalloc_matches_allocating_operator_twice(built):
    import torch
    from tinyinfer_b200 import device

    lib = device.library()
    lib.mp_paged_attention_decode_noalloc.argtypes = [C.c_void_p] * 3 + [C.c_int32] * 4 + [
        C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]
    bt, pool = 16, 12000
    q, k, v, tables, lengths = case(11, 64, 2500, bt, pool)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    tt = torch.from_numpy(tables).to(dev)
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.full_like(tq, float("nan"))
    device.paged_attention_decode(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), 1, 0, bt, pool, tt.data_ptr(),
                                  tables.shape[1], lengths, ref.data_ptr(), 0, stream)
    assert device.paged_attention_status(stream) == 0
    lens = np.ascontiguousarray(lengths)
    outs = []
    for _ in range(2):
        out = torch.full_like(tq, float("nan"))
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        rc = lib.mp_paged_attention_decode_noalloc(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), 1, 0, bt, pool,
                                                    tt.data_ptr(), tables.shape[1], lens.ctypes.data_as(C.c_void_p),
                                                    len(lens), out.data_ptr(), 0, stream, err.data_ptr())
        assert rc == 0, device.last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append(out.cpu().numpy())
    expect = ref.cpu().numpy()
    for got in outs:
        assert np.isfinite(got).all()
        assert (np.abs(got - expect) <= 1e-5 + 1e-4 * np.abs(expect)).all()
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.gpu
def test_noalloc_rejects_too_many_sequences(built):
    from tinyinfer_b200 import device

    lib = device.library()
    lib.mp_paged_attention_decode_noalloc.argtypes = [C.c_void_p] * 3 + [C.c_int32] * 4 + [
        C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]
    lens = np.ones(513, dtype=np.int32)
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = lib.mp_paged_attention_decode_noalloc(dummy, dummy, dummy, 1, 0, 16, 8, dummy, 1,
                                                lens.ctypes.data_as(C.c_void_p), 513, dummy, 0, None, None)
    assert rc == device.MP_ERR_INVALID
    assert "512" in device.last_error()
