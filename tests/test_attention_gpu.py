"""Decode-step attention with RoPE and the cache write fused (ddq_decode_attention),
against a PyTorch fp32 reference of the unfused steps it replaces: rotate-half
RoPE in fp32 rounded to fp16 (``RoPe_d.cu``), the cache write, and softmax
attention over positions 0..pos in fp32 (``engine.py:225-251``)."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from gpu_helpers import decode_kernel_gemm  # noqa: E402


def reference(qkv, kc, vc, cos, sin, pos, nh, nkv, hd, scale):
    B = qkv.shape[0]
    q = qkv[:, : nh * hd].reshape(B, nh, hd).float()
    k = qkv[:, nh * hd:(nh + nkv) * hd].reshape(B, nkv, hd).float()
    v = qkv[:, (nh + nkv) * hd:].reshape(B, nkv, hd)

    def rope(x):
        half = hd // 2
        rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
        return (x * cos + rot * sin).half()
    q, k = rope(q), rope(k)
    kc, vc = kc.clone(), vc.clone()
    kc[:, :, pos] = k
    vc[:, :, pos] = v
    g = nh // nkv
    kk = kc[:, :, : pos + 1].float().repeat_interleave(g, dim=1)
    vv = vc[:, :, : pos + 1].float().repeat_interleave(g, dim=1)
    s = torch.einsum("bhd,bhjd->bhj", q.float(), kk) * scale
    o = torch.einsum("bhj,bhjd->bhd", torch.softmax(s, dim=-1), vv)
    return o.reshape(B, nh * hd).half(), kc, vc


@pytest.mark.parametrize("B,nh,nkv,hd,cap,pos", [
    (1, 14, 2, 64, 64, 0), (3, 14, 2, 64, 100, 37), (64, 14, 2, 64, 768, 600),
    (2, 8, 8, 64, 300, 299), (4, 16, 2, 128, 256, 130), (5, 4, 1, 64, 40, 31),
    # more chunks than the 64-wide kernel keeps in flight (ring refills), G = 8 and G = 3
    (2, 16, 2, 64, 1100, 1099), (3, 6, 2, 64, 2048, 1500), (2, 14, 2, 64, 800, 767)])
def test_decode_attention_matches_reference(cuda_device, B, nh, nkv, hd, cap, pos):
    from ddq_b200 import attention
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + pos)
    qkv = torch.randn(B, (nh + 2 * nkv) * hd, generator=g, device="cuda").half()
    kc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    vc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32, device="cuda") / hd))
    f = torch.tensor([float(pos)], device="cuda")[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    cos, sin = emb.cos(), emb.sin()
    scale = 1.0 / math.sqrt(hd)
    o_ref, kc_ref, vc_ref = reference(qkv, kc, vc, cos, sin, pos, nh, nkv, hd, scale)
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    o = attention.decode_attention(qkv, kc, vc, cos, sin, p, nh, nkv, hd, scale)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)   # cache rows bit-exact
    err = ((o.float() - o_ref.float()).abs().amax(dim=1) /
           o_ref.float().abs().amax(dim=1).clamp_min(1e-6)).max().item()
    assert err < 2e-3, err


def test_decode_attention_strided_batch_and_graph(cuda_device):
    """A batch slice of a larger [L, B, ...] cache, replayed in a CUDA graph with
    the position advanced on the device between replays."""
    from ddq_b200 import attention
    nh, nkv, hd, cap = 14, 2, 64, 96
    g = torch.Generator(device="cuda").manual_seed(5)
    big_k = torch.zeros(3, 8, nkv, cap, hd, dtype=torch.float16, device="cuda")
    big_v = torch.zeros_like(big_k)
    kc, vc = big_k[1, 2:6], big_v[1, 2:6]
    qkv = torch.randn(4, (nh + 2 * nkv) * hd, generator=g, device="cuda").half()
    cos = torch.ones(hd, device="cuda")
    sin = torch.zeros(hd, device="cuda")
    pos = torch.zeros(1, dtype=torch.int64, device="cuda")
    out = attention.decode_attention(qkv, kc, vc, cos, sin, pos, nh, nkv, hd, 0.125)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o2 = attention.decode_attention(qkv, kc, vc, cos, sin, pos, nh, nkv, hd, 0.125)
    for step in range(1, 5):
        pos.fill_(step)
        graph.replay()
    torch.cuda.synchronize()
    # every written row holds the same (unrotated: cos=1, sin=0) k/v, so the
    # attention output equals v for every position count
    v = qkv[:, (nh + nkv) * hd:].reshape(4, nkv, hd)
    for step in range(5):
        assert torch.equal(vc[:, :, step], v)
    exp = v.repeat_interleave(nh // nkv, dim=1).reshape(4, nh * hd)
    assert (o2.float() - exp.float()).abs().max().item() < 1e-2
    assert big_k[0].abs().sum().item() == 0 and big_k[1, :2].abs().sum().item() == 0


def test_decode_attention_ignores_garbage_past_the_position(cuda_device):
    """Cache rows after `pos` are not part of the step: NaN and Inf there must not
    reach the output (a zero weight times NaN would)."""
    from ddq_b200 import attention
    B, nh, nkv, hd, cap, pos = 3, 14, 2, 64, 200, 70
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, (nh + 2 * nkv) * hd, generator=g, device="cuda").half()
    kc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    vc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    kc[:, :, pos + 1:] = float("nan")
    vc[:, :, pos + 1:] = float("inf")
    vc[:, :, pos + 1::2] = float("nan")
    cos = torch.ones(hd, device="cuda")
    sin = torch.zeros(hd, device="cuda")
    o_ref, _, _ = reference(qkv, kc, vc, cos, sin, pos, nh, nkv, hd, 0.125)
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    o = attention.decode_attention(qkv, kc, vc, cos, sin, p, nh, nkv, hd, 0.125)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    err = ((o.float() - o_ref.float()).abs().amax(dim=1) /
           o_ref.float().abs().amax(dim=1).clamp_min(1e-6)).max().item()
    assert err < 2e-3, err


@pytest.mark.parametrize("B,S,nh,nkv,hd,cap,start", [
    (2, 40, 14, 2, 64, 64, 0), (3, 17, 14, 2, 64, 50, 5), (2, 9, 16, 2, 128, 32, 20),
    (8, 512, 14, 2, 64, 528, 0)])
def test_prefill_rope_kv_is_the_fp32_torch_rope(cuda_device, B, S, nh, nkv, hd, cap, start):
    """ddq_prefill_rope_kv against the unfused steps it replaces, bit for bit:
    fp32 rotate-half RoPE of q and k rounded to fp16, and the cache writes."""
    from ddq_b200 import attention
    g = torch.Generator(device="cuda").manual_seed(B * 100 + S)
    qkv = torch.randn(B, S, (nh + 2 * nkv) * hd, generator=g, device="cuda").half()
    kc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    vc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    kc0, vc0 = kc.clone(), vc.clone()
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32, device="cuda") / hd))
    f = torch.arange(start, start + S, dtype=torch.float32, device="cuda")[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    cos, sin = emb.cos(), emb.sin()

    def rope(x):  # [B, H, S, D] fp16 -> fp16, as the engine's fp32 path
        xf = x.float()
        half = hd // 2
        rot = torch.cat([-xf[..., half:], xf[..., :half]], dim=-1)
        return (xf * cos + rot * sin).half()
    q_ref = rope(qkv[..., : nh * hd].reshape(B, S, nh, hd).transpose(1, 2))
    k_ref = rope(qkv[..., nh * hd:(nh + nkv) * hd].reshape(B, S, nkv, hd).transpose(1, 2))
    v_ref = qkv[..., (nh + nkv) * hd:].reshape(B, S, nkv, hd).transpose(1, 2)
    q, k, v = attention.prefill_rope_kv(qkv, kc, vc, cos, sin, start, nh, nkv, hd, kv_out=True)
    torch.cuda.synchronize()
    assert q.shape == (B, S, nh, hd) and k.shape == v.shape == (B, S, nkv, hd)
    assert torch.equal(q.transpose(1, 2), q_ref)
    assert torch.equal(k.transpose(1, 2), k_ref) and torch.equal(v.transpose(1, 2), v_ref)
    assert torch.equal(attention.prefill_rope_kv(qkv, kc, vc, cos, sin, start, nh, nkv, hd), q)
    assert torch.equal(kc[:, :, start:start + S], k_ref)
    assert torch.equal(vc[:, :, start:start + S], v_ref)
    # rows outside the chunk are untouched
    assert torch.equal(kc[:, :, :start], kc0[:, :, :start])
    assert torch.equal(kc[:, :, start + S:], kc0[:, :, start + S:])
    assert torch.equal(vc[:, :, start + S:], vc0[:, :, start + S:])


@pytest.mark.parametrize("B,nh,nkv,cap,pos", [
    (64, 14, 2, 768, 600), (3, 16, 8, 100, 57), (5, 4, 1, 40, 31), (2, 6, 2, 1100, 1099)])
def test_decode_attention_split_feeds_the_o_projection_exactly(cuda_device, B, nh, nkv, cap, pos):
    """ddq_decode_attention_split: its fp16 o equals ddq_decode_attention's, and the
    o projection on its planes equals the decode kernel's o projection on fp16
    o bit for bit (the GEMM's own split pre-pass of o)."""
    from ddq_b200 import attention, gemm_fp8
    hd = 64
    g = torch.Generator(device="cuda").manual_seed(B * 7 + pos)
    qkv = torch.randn(B, (nh + 2 * nkv) * hd, generator=g, device="cuda").half()
    kc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    vc = torch.randn(B, nkv, cap, hd, generator=g, device="cuda").half()
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32, device="cuda") / hd))
    f = float(pos) * inv
    cos, sin = torch.cat([f, f]).cos(), torch.cat([f, f]).sin()
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    o = attention.decode_attention(qkv, kc, vc, cos, sin, p, nh, nkv, hd, 0.125)
    act, o2 = attention.decode_attention_split(qkv, kc, vc, cos, sin, p, nh, nkv, hd, 0.125,
                                               with_out=True)
    act_only, none = attention.decode_attention_split(qkv, kc, vc, cos, sin, p, nh, nkv, hd,
                                                      0.125)
    # the position and earlier cache rows are final here: loading them ahead
    # of the grid wait changes nothing
    act_early, o3 = attention.decode_attention_split(qkv, kc, vc, cos, sin, p, nh, nkv, hd,
                                                     0.125, with_out=True, kv_ready=True)
    torch.cuda.synchronize()
    assert none is None and torch.equal(o, o2) and torch.equal(o, o3)
    assert torch.equal(act.planes, act_only.planes) and torch.equal(act.xscale, act_only.xscale)
    assert torch.equal(act.planes, act_early.planes) and torch.equal(act.xscale, act_early.xscale)
    wq, s = gemm_fp8.quantize(torch.randn(896, nh * hd, generator=g, device="cuda") * 0.02)
    y_ref = decode_kernel_gemm(o, wq, s)
    y = gemm_fp8.f8_forward_planes(act, wq, s)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
