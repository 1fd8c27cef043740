"""The gate/up GEMM with the SwiGLU epilogue (ddq_w8a16_gemm_swiglu).

The oracle runs the two projections and the reference's SwiGLU
(``engine.py:189-193``, ``SwiGLU_d.cu:12-26``): gate and up rounded to fp16,
then silu(g) * u, rounded to fp16.  The fused kernel must match it on decode
(M <= 64) and prefill shapes within the GEMM tests' tolerance."""
import numpy as np
import pytest
import torch

from oracle import w8a16 as o

TIGHT = 3e-3


def test_interleave_matches_oracle_layout():
    from ddq_b200 import gemm_fp8
    rng = np.random.default_rng(0)
    wq = rng.integers(0, 255, (128, 48), dtype=np.uint8)
    s = rng.random(128).astype(np.float32)
    b = rng.random(128).astype(np.float32)
    w2, s2, b2 = gemm_fp8.interleave_gate_up(torch.from_numpy(wq), torch.from_numpy(s),
                                             torch.from_numpy(b))
    np.testing.assert_array_equal(w2.numpy(), o.interleave_gate_up(wq))
    np.testing.assert_array_equal(s2.numpy(), o.interleave_gate_up(s))
    np.testing.assert_array_equal(b2.numpy(), o.interleave_gate_up(b))
    # block 0: gate rows 0..15, then up rows 0..15 (= stacked rows 64..79)
    np.testing.assert_array_equal(w2.numpy()[:16], wq[:16])
    np.testing.assert_array_equal(w2.numpy()[16:32], wq[64:80])


def test_swiglu_oracle_edges():
    g = np.array([0.0, 1.0, -1.0, 20.0, -20.0, -80.0, 65504.0], np.float16)
    u = np.array([1.0, 2.0, 2.0, 1.0, 1.0, 3.0, 0.0], np.float16)
    z = o.swiglu_f16(g, u).astype(np.float64)
    assert z[0] == 0.0 and abs(z[1] - 1.4621) < 1e-3 and abs(z[3] - 20.0) < 1e-2
    assert abs(z[4]) < 1e-6 and z[5] == 0.0 and z[6] == 0.0


def _case(M, inter, K, seed, bias=False):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    w = rng.normal(0, 0.05, (2 * inter, K)).astype(np.float32)
    wq, s = o.quantize(w)
    b = rng.normal(0, 0.1, 2 * inter).astype(np.float32) if bias else None
    return x, wq, s, b


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 5, 16, 33, 64, 100, 300, 1024])
@pytest.mark.parametrize("inter,K", [(4864, 896), (256, 4864), (48, 64)])
def test_fused_swiglu_matches_oracle(cuda_device, M, inter, K):
    from ddq_b200 import gemm_fp8
    x, wq, s, _ = _case(M, inter, K, seed=M + inter + K)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wil, sil, _ = gemm_fp8.interleave_gate_up(dev(wq), dev(s))
    z = gemm_fp8.f8_forward_swiglu(dev(x), wil, sil)
    assert z.shape == (M, inter) and z.dtype == torch.float16
    ref = o.f8_forward_swiglu(x, wq, s)
    err = o.normwise_rel_err(z.cpu().numpy(), ref)
    assert err <= TIGHT, err
    # and against the unfused GPU path (two-projection GEMM, then SwiGLU in torch)
    y = gemm_fp8.f8_forward(dev(x), dev(wq), dev(s)).float()
    z2 = (y[:, :inter] * torch.sigmoid(y[:, :inter]) * y[:, inter:]).half()
    assert o.normwise_rel_err(z.cpu().numpy(), z2.cpu().numpy()) <= TIGHT


@pytest.mark.gpu
@pytest.mark.parametrize("M", [8, 512])
def test_fused_swiglu_with_bias_and_leading_dims(cuda_device, M):
    from ddq_b200 import gemm_fp8
    x, wq, s, b = _case(M, 512, 896, seed=7, bias=True)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wil, sil, bil = gemm_fp8.interleave_gate_up(dev(wq), dev(s), dev(b))
    z = gemm_fp8.f8_forward_swiglu(dev(x).reshape(2, M // 2, 896), wil, sil, bil)
    assert z.shape == (2, M // 2, 512)
    ref = o.f8_forward_swiglu(x, wq, s, b)
    assert o.normwise_rel_err(z.reshape(M, 512).cpu().numpy(), ref) <= TIGHT


@pytest.mark.gpu
def test_fused_swiglu_rejects_bad_shapes(cuda_device):
    from ddq_b200 import gemm_fp8
    x = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    wq = torch.zeros(40, 64, dtype=torch.uint8, device="cuda")   # 2I = 40: I not a multiple of 16
    s = torch.ones(40, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError):
        gemm_fp8.f8_forward_swiglu(x, wq, s)
    wq = torch.zeros(64, 40, dtype=torch.uint8, device="cuda")   # K = 40 not a multiple of 16
    s = torch.ones(64, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError):
        gemm_fp8.f8_forward_swiglu(torch.zeros(4, 40, dtype=torch.float16, device="cuda"), wq, s)
