"""The q/k/v projection with RoPE and the KV-cache write in the prefill GEMM's
epilogue (``ddq_w8a16_gemm_qkv_rope_kv``), against the two calls it replaces -
the W8A16 GEMM to an fp16 [B * S, (Hq + 2 Hkv) * D] projection, then
``ddq_prefill_rope_kv`` - bit for bit: q, the token-major k and v copies, the
cache rows written and the cache rows left alone (``engine.py:215-222``)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _tables(S, start, hd):
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32, device="cuda") / hd))
    f = torch.arange(start, start + S, dtype=torch.float32, device="cuda")[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos(), emb.sin()


def _case(B, S, nh, nkv, hd, K, cap, start, bias_dtype, seed):
    from ddq_b200 import gemm_fp8
    g = torch.Generator(device="cuda").manual_seed(seed)
    N = (nh + 2 * nkv) * hd
    x = torch.randn(B, S, K, generator=g, device="cuda").half()
    wq, sc = gemm_fp8.quantize(torch.randn(N, K, generator=g, device="cuda") * 0.05)
    bias = None
    if bias_dtype is not None:
        bias = (torch.randn(N, generator=g, device="cuda") * 0.5).to(bias_dtype)
    kc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    vc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    cos, sin = _tables(S, start, hd)
    return x, wq, sc, bias, kc, vc, cos, sin


@pytest.mark.parametrize("B,S,nh,nkv,K,cap,start,bias_dtype", [
    (8, 512, 14, 2, 896, 528, 0, torch.float16),
    (2, 300, 14, 2, 896, 400, 37, torch.float32),
    (3, 129, 14, 2, 896, 200, 5, torch.float16),
    (1, 128, 4, 1, 256, 128, 0, None),
    (2, 200, 16, 8, 1024, 256, 56, torch.float32),
    (4, 333, 12, 4, 512, 400, 67, torch.float16),
])
def test_fused_equals_gemm_then_rope(cuda_device, B, S, nh, nkv, K, cap, start, bias_dtype):
    from ddq_b200 import attention, gemm_fp8
    hd = 64
    x, wq, sc, bias, kc, vc, cos, sin = _case(B, S, nh, nkv, hd, K, cap, start, bias_dtype,
                                              B * 1000 + S)
    kc2, vc2 = kc.clone(), vc.clone()
    kc0, vc0 = kc.clone(), vc.clone()
    qkv = gemm_fp8.f8_forward(x, wq, sc, bias)
    q_ref, k_ref, v_ref = attention.prefill_rope_kv(qkv, kc2, vc2, cos, sin, start, nh, nkv, hd,
                                                    kv_out=True)
    q, k, v = attention.qkv_rope_kv(x, wq, sc, bias, kc, vc, cos, sin, start, nh, nkv, hd,
                                    kv_out=True)
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref)
    assert torch.equal(k, k_ref) and torch.equal(v, v_ref)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(kc[:, :, :start], kc0[:, :, :start])
    assert torch.equal(vc[:, :, start + S:], vc0[:, :, start + S:])
    # without the token-major copies: the same q and cache rows
    kc3, vc3 = kc0.clone(), vc0.clone()
    q2 = attention.qkv_rope_kv(x, wq, sc, bias, kc3, vc3, cos, sin, start, nh, nkv, hd)
    torch.cuda.synchronize()
    assert torch.equal(q2, q_ref) and torch.equal(kc3, kc2) and torch.equal(vc3, vc2)


def _status(x, wq, sc, kc, vc, cos, sin, start, nh, nkv, hd):
    from ddq_b200 import _lib, gemm_fp8
    L = _lib.load()
    B, S = kc.shape[0], x.numel() // x.shape[-1] // kc.shape[0]
    N, K = wq.shape
    q = torch.empty(B, S, nh, hd, dtype=torch.float16, device="cuda")
    nws = L.ddq_w8a16_gemm_workspace_size(B * S, N, K)
    ws = gemm_fp8.workspace(x.device, nws) if nws else None
    st = L.ddq_w8a16_gemm_qkv_rope_kv(
        x.data_ptr(), wq.data_ptr(), sc.data_ptr(), None, 0, B, S, K, nh, nkv, hd,
        kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.shape[2], cos.data_ptr(), sin.data_ptr(),
        start, q.data_ptr(), None, None, ws.data_ptr() if ws is not None else None,
        ws.numel() if ws is not None else 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return st


def test_entry_takes_prefill_shapes_and_declines_others(cuda_device):
    """The C entry launches for head_dim 64 at prefill sizes and returns
    DDQ_ERR_SHAPE, launching nothing, for head_dim 128, for decode-size chunks
    and for a chunk past the cache's end; the Python wrapper then runs the two
    unfused calls."""
    from ddq_b200 import _lib, attention, gemm_fp8
    x, wq, sc, _, kc, vc, cos, sin = _case(2, 100, 14, 2, 64, 896, 128, 0, None, 7)
    assert _status(x, wq, sc, kc, vc, cos, sin, 0, 14, 2, 64) == 0
    assert _status(x, wq, sc, kc, vc, cos, sin, 29, 14, 2, 64) == _lib.ERR_SHAPE
    x1, wq1, sc1, _, kc1, vc1, cos1, sin1 = _case(2, 20, 14, 2, 64, 896, 64, 0, None, 8)
    kc1_0 = kc1.clone()
    assert _status(x1, wq1, sc1, kc1, vc1, cos1, sin1, 0, 14, 2, 64) == _lib.ERR_SHAPE
    assert torch.equal(kc1, kc1_0)
    x2, wq2, sc2, b2, kc2, vc2, cos2, sin2 = _case(2, 100, 8, 2, 128, 512, 128, 3,
                                                   torch.float16, 9)
    assert _status(x2, wq2, sc2, kc2, vc2, cos2, sin2, 3, 8, 2, 128) == _lib.ERR_SHAPE
    for (x_, wq_, sc_, b_, kc_, vc_, cs_, sn_, st_, nh_, hd_) in (
            (x1, wq1, sc1, None, kc1, vc1, cos1, sin1, 0, 14, 64),
            (x2, wq2, sc2, b2, kc2, vc2, cos2, sin2, 3, 8, 128)):
        kr, vr = kc_.clone(), vc_.clone()
        q_ref = attention.prefill_rope_kv(gemm_fp8.f8_forward(x_, wq_, sc_, b_), kr, vr, cs_,
                                          sn_, st_, nh_, 2, hd_)
        q = attention.qkv_rope_kv(x_, wq_, sc_, b_, kc_, vc_, cs_, sn_, st_, nh_, 2, hd_)
        torch.cuda.synchronize()
        assert torch.equal(q, q_ref) and torch.equal(kc_, kr) and torch.equal(vc_, vr)
    # the cache overflow is reported by the wrapper, not swallowed
    with pytest.raises(RuntimeError):
        attention.qkv_rope_kv(x, wq, sc, None, kc, vc, cos, sin, 29, 14, 2, 64)


def test_engine_prefill_fused_equals_unfused(cuda_device):
    """Engine prefill chunks (from position 0, then from 160) with the fused q/k/v
    epilogue give the same hidden states and KV cache, bit for bit, as with the
    GEMM and the RoPE + cache kernel separate."""
    from ddq_b200.engine import Config, Engine
    cfg = Config(num_hidden_layers=2)
    eng = Engine.random(cfg, seed=3)
    ids = torch.randint(0, cfg.vocab_size, (4, 290), device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(1))
    outs = []
    for fused in (True, False):
        eng.fused_qkv_rope = fused
        cache = eng.new_cache(4, 320)
        h1 = eng.hidden(ids[:, :160], cache, 0, 0)
        h2 = eng.hidden(ids[:, 160:], cache, 0, 160)
        torch.cuda.synchronize()
        outs.append((h1, h2, cache.k.clone(), cache.v.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
