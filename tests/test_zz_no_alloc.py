"""mp_paged_attention_decode_noalloc through the C ABI: the allocation-free
variant of the decode operator, for callers that cannot call cudaMalloc (a host
embedding this library in a runtime that owns all GPU memory, or a path where an
allocation would synchronise the device). Its scratch is a fixed device array, so
this file runs last and must pass both alone and after every other test: the
array keeps the previous call's contents, and results must not depend on them.

Two calls in a row must each equal the allocating operator
(mp_paged_attention_decode) bit for bit -- both build the same work list and
schedule -- and match the C oracle within the attention tests' tolerance
|a - b| <= 1e-5 + 1e-4 |b|. A planted out-of-range page id must be reported
whether the caller passes a device error word or not.
"""
import ctypes as C

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


def noalloc(lib):
    f = lib.mp_paged_attention_decode_noalloc
    f.argtypes = [C.c_void_p] * 3 + [C.c_int32] * 4 + [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                                       C.c_int32, C.c_void_p, C.c_void_p]
    return f


class Case:
    """One operator input on cuda:0 and the two ways of calling the operator."""

    def __init__(self, seed, count, max_len, bt, pool):
        import torch

        self.q, self.k, self.v, self.tables, self.lengths = case(seed, count, max_len, bt, pool)
        self.bt, self.pool = bt, pool
        dev = torch.device("cuda:0")
        self.tq, self.tk, self.tv = (torch.from_numpy(a).to(dev) for a in (self.q, self.k, self.v))
        self.tt = torch.from_numpy(self.tables).to(dev)
        self.stream = torch.cuda.current_stream().cuda_stream
        self.lens = np.ascontiguousarray(self.lengths)

    def allocating(self, pps):
        import torch
        from tinyinfer_b200 import device

        out = torch.full_like(self.tq, float("nan"))
        device.paged_attention_decode(self.tq.data_ptr(), self.tk.data_ptr(), self.tv.data_ptr(), 1, 0, self.bt,
                                      self.pool, self.tt.data_ptr(), self.tables.shape[1], self.lengths,
                                      out.data_ptr(), pps, self.stream)
        assert device.paged_attention_status(self.stream) == 0
        return out.cpu().numpy()

    def noalloc(self, pps, error_word=True):
        """(rc, output, device error word or None)."""
        import torch
        from tinyinfer_b200 import device

        out = torch.full_like(self.tq, float("nan"))
        err = torch.zeros(1, dtype=torch.int32, device=self.tq.device) if error_word else None
        rc = noalloc(device.library())(self.tq.data_ptr(), self.tk.data_ptr(), self.tv.data_ptr(), 1, 0, self.bt,
                                       self.pool, self.tt.data_ptr(), self.tables.shape[1],
                                       self.lens.ctypes.data_as(C.c_void_p), len(self.lens), out.data_ptr(), pps,
                                       self.stream, err.data_ptr() if error_word else None)
        torch.cuda.synchronize()
        return rc, out.cpu().numpy(), (int(err.item()) if error_word else None)


@pytest.mark.gpu
@pytest.mark.parametrize("pps", [0, 4])
def test_noalloc_matches_allocating_operator_and_oracle_twice(built, pps):
    from oracle.oracle import Oracle
    from tinyinfer_b200 import device

    c = Case(11, 64, 2500, 16, 12000)
    expect = Oracle.decode_attention(c.q, c.lengths, c.tables, c.k, c.v, HEADS, KVH, DIM, c.bt)
    allocating = c.allocating(pps)
    outs = []
    for _ in range(2):
        rc, got, err = c.noalloc(pps)
        assert rc == 0, device.last_error()
        assert err == 0
        assert np.isfinite(got).all()
        assert (np.abs(got - expect) <= 1e-5 + 1e-4 * np.abs(expect)).all(), float(np.abs(got - expect).max())
        assert np.array_equal(got, allocating)
        outs.append(got)
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.gpu
def test_noalloc_reports_a_bad_page_with_and_without_an_error_word(built):
    from tinyinfer_b200 import device

    c = Case(12, 16, 300, 16, 1024)
    good = c.tables.copy()
    c.tables[3, 0] = c.pool + 5  # row 3's first page lies outside the pool
    import torch

    c.tt = torch.from_numpy(c.tables).to(c.tq.device)
    rc, out, err = c.noalloc(0, error_word=True)
    assert rc == 0 and err & 1, err
    assert device.paged_attention_status(c.stream) == device.MP_OK  # the bits went to the caller's word
    rc, out, err = c.noalloc(0, error_word=False)
    assert rc == 0
    assert device.paged_attention_status(c.stream) == device.MP_ERR_BOUNDS
    assert device.paged_attention_status(c.stream) == device.MP_OK  # read and cleared
    # the next call with valid tables is unaffected
    c.tables = good
    c.tt = torch.from_numpy(good).to(c.tq.device)
    rc, out, err = c.noalloc(0, error_word=False)
    assert rc == 0 and device.paged_attention_status(c.stream) == device.MP_OK
    assert np.array_equal(out, c.allocating(0))


def test_noalloc_rejects_too_many_sequences(built):
    """Checked before any CUDA call: runs without a GPU."""
    from tinyinfer_b200 import device

    lens = np.ones(513, dtype=np.int32)
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = noalloc(device.library())(dummy, dummy, dummy, 1, 0, 16, 8, dummy, 1, lens.ctypes.data_as(C.c_void_p),
                                   513, dummy, 0, None, None)
    assert rc == device.MP_ERR_INVALID
    assert "512" in device.last_error()


def test_noalloc_rejects_too_many_slices(built):
    """An explicit pages_per_split whose slices exceed the fixed work list (2048) is
    rejected before anything is queued: runs without a GPU."""
    from tinyinfer_b200 import device

    lens = np.full(300, 16 * 8, dtype=np.int32)  # 8 pages per row, 1 page per slice: 2400 slices
    dummy = C.c_void_p(16)
    rc = noalloc(device.library())(dummy, dummy, dummy, 1, 0, 16, 4096, dummy, 8, lens.ctypes.data_as(C.c_void_p),
                                   300, dummy, 1, None, None)
    assert rc == device.MP_ERR_INVALID
    assert "2048" in device.last_error()
    rc = noalloc(device.library())(dummy, dummy, dummy, 1, 0, 16, 4096, dummy, 8, lens.ctypes.data_as(C.c_void_p),
                                   300, dummy, -1, None, None)
    assert rc == device.MP_ERR_INVALID
