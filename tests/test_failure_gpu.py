"""Failure detection on the GPU without a fault: the tensor-core kernel's
bounded waits.  A test hook makes the MMA warp skip the accumulator-ready
signal (a flag that nothing then sets); the epilogue's wait runs out after
20 ms, the kernel records DDQ_ERR_TIMEOUT, drains its own copies and MMAs,
frees TMEM and returns - and the context stays usable."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import w8a16 as o

pytestmark = pytest.mark.gpu

DDQ_ERR_TIMEOUT = 7


def device_error(lib):
    code = ctypes.c_int(-1)
    assert lib.ddq_device_error(ctypes.byref(code), torch.cuda.current_stream().cuda_stream) == 0
    return code.value


def test_bounded_wait_reports_timeout_and_context_survives(cuda_device):
    from ddq_b200 import _lib, gemm_fp8
    lib = _lib.load()
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (16, 896)).astype(np.float16)
    wq, s = o.quantize(rng.normal(0, 0.02, (896, 896)).astype(np.float32))
    xd, wqd, sd = (torch.from_numpy(a).cuda() for a in (x, wq, s))
    assert device_error(lib) == 0
    try:
        assert lib.ddq_set_debug(1, 20_000_000) == 0
        gemm_fp8.f8_forward(xd, wqd, sd)
        torch.cuda.synchronize()
        assert device_error(lib) == DDQ_ERR_TIMEOUT
    finally:
        lib.ddq_set_debug(0, 0)
    # the context is still healthy and the next call is correct
    y = gemm_fp8.f8_forward(xd, wqd, sd)
    torch.cuda.synchronize()
    assert device_error(lib) == 0
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s)) <= 3e-3


@pytest.mark.parametrize("M,N,K", [(512, 9728, 896), (600, 896, 896), (1024, 2048, 256)])
def test_prefill_bounded_waits_report_timeout(cuda_device, M, N, K):
    """The same hook in the prefill GEMM, on CTA pairs (N >= 2048: the pair's
    rank 0 commits for both CTAs, and both epilogues wait) and on single
    CTAs: DDQ_ERR_TIMEOUT, every role winds down, the context stays usable."""
    from ddq_b200 import _lib, gemm_fp8
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(M + N)
    xd = torch.randn(M, K, generator=g, device="cuda").half()
    wqd, sd = gemm_fp8.quantize(torch.randn(N, K, generator=g, device="cuda") * 0.02)
    ref = gemm_fp8.f8_forward(xd, wqd, sd)
    torch.cuda.synchronize()
    assert device_error(lib) == 0
    try:
        assert lib.ddq_set_debug(1, 20_000_000) == 0
        gemm_fp8.f8_forward(xd, wqd, sd)
        torch.cuda.synchronize()
        assert device_error(lib) == DDQ_ERR_TIMEOUT
    finally:
        lib.ddq_set_debug(0, 0)
    y = gemm_fp8.f8_forward(xd, wqd, sd)
    torch.cuda.synchronize()
    assert device_error(lib) == 0
    assert torch.equal(y, ref)
