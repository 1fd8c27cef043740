"""Residual add + RMSNorm (ddq_add_rmsnorm) against the PyTorch fp32 reference
of the unfused steps: fp16 residual add, then ``RMSnorm_d.cu`` semantics
(fp32 sum of squares, rsqrt(mean + eps), x * r * w rounded to fp16)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from gpu_helpers import decode_kernel_gemm  # noqa: E402


def ref(x, w, eps, delta=None):
    s = x if delta is None else x + delta
    sf = s.float()
    r = torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + eps)
    return s, (sf * r * w).half()


@pytest.mark.parametrize("M,H", [(1, 896), (64, 896), (4096, 896), (3, 8), (5, 4864), (2, 8192)])
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm_matches_reference(cuda_device, M, H, with_delta):
    from ddq_b200 import norm
    g = torch.Generator(device="cuda").manual_seed(M + H)
    x = (torch.randn(M, H, generator=g, device="cuda") * 3).half()
    d = (torch.randn(M, H, generator=g, device="cuda") * 3).half() if with_delta else None
    w = torch.rand(H, generator=g, device="cuda") + 0.5
    s_ref, h_ref = ref(x, w, 1e-6, d)
    s, h = norm.add_rmsnorm(x.clone(), w, 1e-6, d)
    assert torch.equal(s, s_ref)                       # the fp16 residual add is exact
    diff = (h.float() - h_ref.float()).abs()
    ulp = h_ref.float().abs().clamp_min(2 ** -14) * 2 ** -10
    assert bool((diff <= ulp).all()), float((diff / ulp).max())   # within one fp16 ulp


def test_add_rmsnorm_in_place(cuda_device):
    from ddq_b200 import norm
    x = torch.randn(4, 4096, device="cuda").half()
    d = torch.randn(4, 4096, device="cuda").half()
    w = torch.ones(4096, device="cuda")
    s_ref, h_ref = ref(x.clone(), w, 1e-6, d)
    s, h = norm.add_rmsnorm(x, w, 1e-6, d, inplace=True)
    assert s.data_ptr() == x.data_ptr() and torch.equal(x, s_ref)
    assert (h.float() - h_ref.float()).abs().max().item() <= 2e-3


@pytest.mark.parametrize("M", [1, 7, 16, 64])
@pytest.mark.parametrize("with_delta", [False, True])
def test_norm_split_feeds_the_decode_gemm_exactly(cuda_device, M, with_delta):
    """RMSNorm + split, then the GEMM on the planes, gives bit for bit what the
    RMSNorm's fp16 output gives through the decode kernel (whose pre-pass
    splits it the same way); the same for the SwiGLU epilogue."""
    import numpy as np
    from ddq_b200 import gemm_fp8, norm
    from oracle import w8a16 as o
    H, N, I = 896, 1152, 512
    g = torch.Generator(device="cuda").manual_seed(M)
    x = (torch.randn(1, M, H, generator=g, device="cuda") * 2).half()
    d = (torch.randn(1, M, H, generator=g, device="cuda") * 2).half() if with_delta else None
    w = torch.rand(H, generator=g, device="cuda") + 0.5
    wq, s = gemm_fp8.quantize(torch.randn(N, H, generator=g, device="cuda") * 0.02)
    b = torch.randn(N, generator=g, device="cuda") * 0.02
    s_ref, h = norm.add_rmsnorm(x.clone(), w, 1e-6, d)
    s_new, act = norm.add_rmsnorm_split(x.clone(), w, 1e-6, d)
    assert torch.equal(s_new, s_ref)
    y_ref = decode_kernel_gemm(h.reshape(M, H), wq, s, b)
    y = gemm_fp8.f8_forward_planes(act, wq, s, b)
    assert torch.equal(y, y_ref)
    wgu, sgu = gemm_fp8.quantize(torch.randn(2 * I, H, generator=g, device="cuda") * 0.05)
    wil, sil, _ = gemm_fp8.interleave_gate_up(wgu, sgu)
    z_ref = gemm_fp8.f8_forward_swiglu(h.reshape(M, H), wil, sil)
    z = gemm_fp8.f8_forward_planes(act, wil, sil, swiglu=True)
    assert torch.equal(z, z_ref)
    # and the oracle agrees with both
    ref = o.f8_forward(h.reshape(M, H).cpu().numpy(), wq.cpu().numpy(), s.cpu().numpy(),
                       b.cpu().numpy())
    assert o.normwise_rel_err(y.cpu().numpy(), ref) <= 3e-3
