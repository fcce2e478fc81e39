"""The split-precision tcgen05 GEMM alone vs float64 numpy: C = A . B^T.

Every operand value x goes to the tensor cores as two FP16 halves, hi = fp16(x) and
lo = fp16((x - hi) * 2^11), and the GEMM forms A_hi.B_hi + 2^-11 (A_hi.B_lo +
A_lo.B_hi). Two checks per shape, on the worst element's
|gpu - exact| / sum_k |a_k b_k|:
  * absolute: at most 2^-18 (about 4e-6);
  * against a single FP16 product (both operands rounded to FP16, computed in
    float64 here): the split's error must be at least 8x smaller -- the split must
    buy back the precision one FP16 pass drops. (The remaining error is dominated
    by the tensor core's FP32 accumulation, and grows slowly with K.)
"""
import numpy as np
import pytest


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 64, 32), (7, 128, 576), (128, 960, 576), (130, 576, 576), (256, 1536, 576),
                                   (256, 576, 1536), (300, 64, 64), (1000, 192, 128), (256, 4096, 576),
                                   (3, 64, 160), (5, 64, 1536), (33, 3072, 576)])
def test_tc_gemm_matches_float64(built, m, n, k):
    import torch
    from tinyinfer_b200 import device

    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    dev = torch.device("cuda:0")
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tc = torch.full((m, n), float("nan"), device=dev)
    device.gemm_f32(ta.data_ptr(), tb.data_ptr(), tc.data_ptr(), m, n, k, torch.cuda.current_stream().cuda_stream)
    got = tc.cpu().numpy().astype(np.float64)
    exact = a.astype(np.float64) @ b.astype(np.float64).T
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T
    err = np.abs(got - exact)
    assert np.isfinite(got).all()
    worst = float((err / scale).max())

    def f16(x):
        return x.astype(np.float16).astype(np.float64)

    plain = float((np.abs(f16(a) @ f16(b).T - exact) / scale).max())
    print(f"m={m} n={n} k={k}: split FP16 {worst:.3e}  single FP16 {plain:.3e}")
    assert worst <= 2.0 ** -18, worst
    assert worst * 8 <= plain, (worst, plain)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(7, 576, 1536), (64, 3072, 576)])
def test_tc_gemm_split_k_is_deterministic(built, m, n, k):
    """Split-K partials are summed in slice order by the CTA that owns the row:
    repeated launches give bit-identical results, and a row's result does not
    depend on the other rows of the batch (the first rows of a larger M match
    the same rows computed alone)."""
    import torch
    from tinyinfer_b200 import device

    rng = np.random.default_rng(k + n)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    runs = []
    for _ in range(4):
        tc = torch.empty((m, n), device=dev)
        device.gemm_f32(ta.data_ptr(), tb.data_ptr(), tc.data_ptr(), m, n, k, stream)
        runs.append(tc.cpu().numpy())
    for r in runs[1:]:
        assert np.array_equal(r.view(np.uint32), runs[0].view(np.uint32))
    one = torch.empty((1, n), device=dev)
    device.gemm_f32(ta[:1].contiguous().data_ptr(), tb.data_ptr(), one.data_ptr(), 1, n, k, stream)
    assert np.array_equal(one.cpu().numpy()[0].view(np.uint32), runs[0][0].view(np.uint32))


@pytest.mark.gpu
def test_tc_gemm_operand_beyond_fp16_range_is_loud(built):
    """The split stores every operand as FP16 halves; a value beyond FP16's range
    (65504) becomes infinite instead of losing accuracy silently, so the products
    of its row come out nonfinite (in the forward, nonfinite logits fail the step).
    Rows without such a value are unaffected."""
    import torch
    from tinyinfer_b200 import device

    m, n, k = 4, 64, 64
    rng = np.random.default_rng(5)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    a[1, 7] = 1.0e5
    dev = torch.device("cuda:0")
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tc = torch.zeros((m, n), device=dev)
    device.gemm_f32(ta.data_ptr(), tb.data_ptr(), tc.data_ptr(), m, n, k, torch.cuda.current_stream().cuda_stream)
    got = tc.cpu().numpy()
    assert not np.isfinite(got[1]).any()
    exact = a.astype(np.float64) @ b.astype(np.float64).T
    for r in (0, 2, 3):
        assert np.allclose(got[r], exact[r], rtol=1e-5, atol=1e-5)
