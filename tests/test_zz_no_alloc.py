"""The allocation-free decode GEMM entry point (ddq_w8a16_gemm_noalloc).

It serves callers that cannot allocate device memory where they run a
projection (a host owning a fixed memory plan, a runtime that bans cudaMalloc
on its request path, graph recording): its scratch is an array inside the
library rather than a caller workspace.  Called through the C ABI, it must
match the ordinary entry point (ddq_w8a16_gemm via gemm_fp8.f8_forward, which
takes its scratch from the caller) on two calls in a row - the second call
finds the array holding the first call's contents - and reject sizes beyond
the array.  This file sorts last so a stop-at-first-failure run has already
run every other test; no other test calls this entry point."""
import numpy as np
import pytest
import torch

from oracle import w8a16 as o

pytestmark = pytest.mark.gpu

TIGHT = 3e-3  # the GEMM tests' tolerance (normwise relative error)
DDQ_ERR_SHAPE, DDQ_ERR_WORKSPACE = 2, 4


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("M,N,K", [(16, 1152, 896), (64, 896, 4864), (1, 9728, 896), (37, 256, 48)])
def test_noalloc_matches_workspace_entry_point(cuda_device, M, N, K):
    from ddq_b200 import _lib, gemm_fp8
    lib = _lib.load()
    rng = np.random.default_rng(M + N + K)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    wq, s = o.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    b = rng.normal(0, 0.02, N).astype(np.float32)
    xd, wqd, sd, bd = dev(x), dev(wq), dev(s), dev(b)
    ref = gemm_fp8.f8_forward(xd, wqd, sd, bd)
    y_oracle = o.f8_forward(x, wq, s, b)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        st = lib.ddq_w8a16_gemm_noalloc(xd.data_ptr(), wqd.data_ptr(), sd.data_ptr(), bd.data_ptr(),
                                        _lib.DTYPE_F32, y.data_ptr(), M, N, K, stream)
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        assert o.normwise_rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= TIGHT
        assert o.normwise_rel_err(y.cpu().numpy(), y_oracle) <= TIGHT


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    from ddq_b200 import _lib
    lib = _lib.load()
    x = torch.zeros(65, 8192, dtype=torch.float16, device="cuda")
    wq = torch.zeros(128, 8192, dtype=torch.uint8, device="cuda")
    s = torch.ones(128, dtype=torch.float32, device="cuda")
    y = torch.empty(65, 128, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # 3 * 64 * 8192 plane bytes = 1.5 MiB > the 1 MiB array
    assert lib.ddq_w8a16_gemm_noalloc(x.data_ptr(), wq.data_ptr(), s.data_ptr(), None, 0,
                                      y.data_ptr(), 64, 128, 8192, stream) == DDQ_ERR_WORKSPACE
    # more than 64 tokens is not a decode shape
    assert lib.ddq_w8a16_gemm_noalloc(x.data_ptr(), wq.data_ptr(), s.data_ptr(), None, 0,
                                      y.data_ptr(), 65, 128, 896, stream) == DDQ_ERR_SHAPE
