"""The 3xTF32 tcgen05 GEMM alone vs float64 numpy: C = A . B^T.

3xTF32 keeps FP32-level accuracy. Per product the dropped a_lo.b_lo term and the
TF32 truncation of the lo halves are below ~3 x 2^-20 relative and of random
sign, so per element |gpu - exact| stays far below 2^-20 * sum_k |a_k b_k|; plain
TF32 (2^-11 relative per product) lands around 2^-12 / sqrt(k) of that sum --
above the bound for every k tested here.
"""
import numpy as np
import pytest


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 64, 32), (7, 128, 576), (128, 960, 576), (130, 576, 576), (256, 1536, 576),
                                   (256, 576, 1536), (300, 64, 64), (1000, 192, 128), (256, 4096, 576)])
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
    print(f"m={m} n={n} k={k}: max |err| / sum|ab| = {worst:.3e}")
    assert worst <= 2.0 ** -20, worst
