"""Residual add + RMSNorm (ddq_add_rmsnorm) against the PyTorch fp32 reference
of the unfused steps: fp16 residual add, then ``RMSnorm_d.cu`` semantics
(fp32 sum of squares, rsqrt(mean + eps), x * r * w rounded to fp16)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


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
