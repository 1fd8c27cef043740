"""Prefill GEMMs on CTA pairs (tcgen05 .cta_group::2, 256-token tiles, the
default from 512 tokens for N >= 2048) against the same GEMMs on single CTAs
(128-token tiles; ``ddq_set_debug`` bit 7), bit for bit: plain store with and
without bias and the SwiGLU epilogue, on exact and ragged token counts; the
narrower shapes check that the switch leaves single-CTA shapes alone.  Both paths sum each output over K in the same
order; the oracle tests of ``test_gemm_gpu.py`` / ``test_swiglu.py`` check
the values themselves."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SINGLE = 128  # ddq_set_debug bit 7


@pytest.fixture(scope="module")
def lib(cuda_device):
    from ddq_b200 import _lib
    return _lib.load()


def both(lib, fn):
    """fn() on CTA pairs, then on single CTAs."""
    torch.cuda.synchronize()
    a = fn()
    torch.cuda.synchronize()
    assert lib.ddq_set_debug(SINGLE, 0) == 0
    try:
        b = fn()
        torch.cuda.synchronize()
    finally:
        lib.ddq_set_debug(0, 0)
    return a, b


def weights(N, K, seed):
    from ddq_b200 import gemm_fp8
    g = torch.Generator(device="cuda").manual_seed(seed)
    wq, s = gemm_fp8.quantize(torch.randn(N, K, generator=g, device="cuda") * 0.02)
    return wq, s, g


@pytest.mark.parametrize("M,N,K,bias", [
    (512, 9728, 896, None), (4096, 1152, 896, torch.float32), (1000, 896, 4864, None),
    (700, 896, 896, torch.float16), (777, 4096, 128, torch.float32), (2048, 4864, 896, None),
    (1300, 2080, 896, torch.float16),
    # K % 64 != 0: the last K stage is a partial box, zero-filled past K
    (600, 2048, 144, torch.float32), (300, 896, 208, None)])
def test_pair_equals_single_cta(lib, M, N, K, bias):
    from ddq_b200 import _lib, gemm_fp8
    wq, s, g = weights(N, K, M + N)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    b = None if bias is None else torch.randn(N, generator=g, device="cuda").to(bias)
    pair, single = both(lib, lambda: gemm_fp8.f8_forward(x, wq, s, b))
    assert torch.equal(pair, single)
    code = ctypes.c_int(0)
    assert lib.ddq_device_error(ctypes.byref(code), torch.cuda.current_stream().cuda_stream) == 0
    assert code.value == 0


@pytest.mark.parametrize("M,inter", [(512, 4864), (1024, 4864), (600, 1024)])
def test_pair_swiglu_equals_single_cta(lib, M, inter):
    from ddq_b200 import gemm_fp8
    wq, s, g = weights(2 * inter, 896, M)
    wq_il, s_il, _ = gemm_fp8.interleave_gate_up(wq, s, None)
    x = torch.randn(M, 896, generator=g, device="cuda").half()
    pair, single = both(lib, lambda: gemm_fp8.f8_forward_swiglu(x, wq_il, s_il))
    assert torch.equal(pair, single)


@pytest.mark.parametrize("B,S,start", [(8, 512, 0), (3, 300, 21)])
def test_qkv_rope_unaffected_by_the_switch(lib, B, S, start):
    from ddq_b200 import attention
    nh, nkv, hd, K = 14, 2, 64, 896
    wq, s, g = weights((nh + 2 * nkv) * hd, K, B * S)
    bias = torch.randn(wq.shape[0], generator=g, device="cuda")
    x = torch.randn(B, S, K, generator=g, device="cuda").half()
    cap = start + S + 8
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32, device="cuda") / hd))
    f = torch.arange(start, start + S, dtype=torch.float32, device="cuda")[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    cos, sin = emb.cos(), emb.sin()
    caches = []

    def run():
        kc = torch.zeros(B, nkv, cap, hd, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        caches.append((kc, vc))
        return attention.qkv_rope_kv(x, wq, s, bias, kc, vc, cos, sin, start, nh, nkv, hd,
                                     kv_out=True)
    pair, single = both(lib, run)
    for a, b in zip(pair, single):
        assert torch.equal(a, b)
    assert torch.equal(caches[0][0], caches[1][0]) and torch.equal(caches[0][1], caches[1][1])


@pytest.mark.parametrize("M,N,K", [(600, 2048, 144), (300, 896, 208), (520, 2080, 80)])
def test_partial_last_k_stage_matches_oracle(lib, M, N, K):
    """K a multiple of 16 but not of 64: the last K stage's box reaches past K
    and is zero-filled; pairs (N >= 2048) and single CTAs against the oracle."""
    import numpy as np
    from oracle import w8a16 as o
    from ddq_b200 import gemm_fp8
    rng = np.random.default_rng(M + K)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    wq, s = o.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    y = gemm_fp8.f8_forward(torch.from_numpy(x).cuda(), torch.from_numpy(wq).cuda(),
                            torch.from_numpy(s).cuda())
    torch.cuda.synchronize()
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s)) <= 3e-3
