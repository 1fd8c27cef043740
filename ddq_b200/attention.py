"""Attention-side kernels: the decode step with RoPE and the KV-cache write
fused in, and the prefill RoPE + cache write.

``decode_attention`` replaces, for one decode step, the reference engine's
q/k rotary embedding (``RoPe_d.cu:12-68``), the cache write
(``engine.py:126-130``) and the attention call (``engine.py:225-251``) with one
kernel (``ddq_decode_attention``): the new key/value row is written into the
cache at the device-side position and the query heads attend over positions
0..pos of their key/value head (grouped-query attention).
"""
from __future__ import annotations

import torch

from typing import Optional

from . import _lib
from .norm import SplitActivations


def _check_decode(qkv, k_cache, v_cache, cos, sin, pos, num_heads, num_kv_heads, head_dim):
    def need(cond, msg):
        if not cond:
            raise RuntimeError(msg)
    B = qkv.shape[0]
    need(qkv.is_cuda and qkv.dtype == torch.float16 and qkv.dim() == 2 and
         qkv.stride(1) == 1 and qkv.shape[1] == (num_heads + 2 * num_kv_heads) * head_dim,
         "decode_attention: qkv must be fp16 CUDA [B, (Hq + 2 Hkv) * D] with unit inner stride")
    for c in (k_cache, v_cache):
        need(c.is_cuda and c.dtype == torch.float16 and c.dim() == 4 and
             tuple(c.shape[:2]) == (B, num_kv_heads) and c.shape[3] == head_dim and
             c.stride(3) == 1 and c.stride(2) == head_dim and
             c.stride(1) == c.shape[2] * head_dim,
             "decode_attention: caches must be fp16 CUDA [B, Hkv, capacity, D], dense per sequence")
    need(k_cache.stride(0) == v_cache.stride(0) and k_cache.shape == v_cache.shape,
         "decode_attention: k and v caches must have the same shape and strides")
    cos = cos.reshape(-1).contiguous()
    sin = sin.reshape(-1).contiguous()
    need(cos.dtype == torch.float32 and sin.dtype == torch.float32 and
         cos.numel() == head_dim and sin.numel() == head_dim, "decode_attention: fp32 cos/sin [D]")
    need(pos.is_cuda and pos.dtype == torch.int64 and pos.numel() == 1,
         "decode_attention: pos must be an int64 CUDA scalar")
    return B, cos, sin


def decode_attention(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor,
                     num_heads: int, num_kv_heads: int, head_dim: int,
                     scale: float) -> torch.Tensor:
    """qkv fp16 [B, (Hq + 2 Hkv) * D] (one token per sequence); k_cache/v_cache
    fp16 [B, Hkv, capacity, D] (batch dim may be strided); cos/sin fp32 [D] for
    this position; pos int64 [1] on the device.  Returns o fp16 [B, Hq * D] and
    updates the caches at ``pos``."""
    B, cos, sin = _check_decode(qkv, k_cache, v_cache, cos, sin, pos, num_heads, num_kv_heads,
                                head_dim)
    out = torch.empty((B, num_heads * head_dim), dtype=torch.float16, device=qkv.device)
    with torch.cuda.device(qkv.device):
        st = _lib.load().ddq_decode_attention(
            qkv.data_ptr(), qkv.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.stride(0), k_cache.shape[2], cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
            out.data_ptr(), out.stride(0), B, num_heads, num_kv_heads, head_dim, float(scale),
            torch.cuda.current_stream(qkv.device).cuda_stream)
    _lib.check(st, "decode_attention")
    return out


def decode_attention_split(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor,
                           num_heads: int, num_kv_heads: int, head_dim: int, scale: float,
                           act: Optional[SplitActivations] = None, with_out: bool = False,
                           kv_ready: bool = False):
    """``decode_attention`` whose output is the o projection's operand
    (``ddq_decode_attention_split``): o's three e4m3 planes and token scales,
    for ``gemm_fp8.f8_forward_planes``, bit for bit what the GEMM's own split
    of fp16 o gives.  ``act`` reuses buffers of the same shape; ``with_out``
    also returns fp16 o.  ``kv_ready`` promises that ``pos`` and the cache rows
    before it were final before the previous kernel on the stream started (a
    decode loop, where earlier steps wrote them): the kernel then loads them
    while that kernel still runs.  Returns (act, o or None)."""
    B, cos, sin = _check_decode(qkv, k_cache, v_cache, cos, sin, pos, num_heads, num_kv_heads,
                                head_dim)
    K = num_heads * head_dim
    if act is None or act.M != B or act.H != K:
        act = SplitActivations(torch.empty((3, B, K), dtype=torch.uint8, device=qkv.device),
                               torch.empty((B,), dtype=torch.float32, device=qkv.device), B, K)
    out = torch.empty((B, K), dtype=torch.float16, device=qkv.device) if with_out else None
    with torch.cuda.device(qkv.device):
        st = _lib.load().ddq_decode_attention_split(
            qkv.data_ptr(), qkv.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.stride(0), k_cache.shape[2], cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
            out.data_ptr() if out is not None else None, K, act.planes.data_ptr(),
            act.xscale.data_ptr(), B, num_heads, num_kv_heads, head_dim, float(scale),
            1 if kv_ready else 0, torch.cuda.current_stream(qkv.device).cuda_stream)
    _lib.check(st, "decode_attention_split")
    return act, out


def prefill_rope_kv(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    cos: torch.Tensor, sin: torch.Tensor, start: int, num_heads: int,
                    num_kv_heads: int, head_dim: int, kv_out: bool = False):
    """Prefill chunk (``ddq_prefill_rope_kv``): qkv fp16 [B, S, (Hq + 2 Hkv) * D]
    (or [B * S, ...] with B taken from the caches); cos/sin fp32 [S, D] for
    positions start .. start + S - 1.  Writes rope(k) and v into the caches at
    start .. start + S - 1 and returns rope(q) fp16 [B, S, Hq, D]; with ``kv_out``
    returns (q, k, v), k and v token-major [B, S, Hkv, D] copies of the new rows
    (attention inputs whose strides do not depend on the cache).  Replaces the
    reference's q/k RoPE (``RoPe_d.cu:12-68``, ``engine.py:219-220``) and cache
    write (``engine.py:126-130``)."""
    def need(cond, msg):
        if not cond:
            raise RuntimeError(msg)
    B = k_cache.shape[0]
    width = (num_heads + 2 * num_kv_heads) * head_dim
    need(qkv.is_cuda and qkv.dtype == torch.float16 and qkv.shape[-1] == width and
         qkv.stride(-1) == 1, "prefill_rope_kv: qkv must be fp16 CUDA [..., (Hq + 2 Hkv) * D]")
    rows = qkv.reshape(-1, width)
    need(rows.shape[0] % B == 0, "prefill_rope_kv: qkv rows must be B * S")
    S = rows.shape[0] // B
    for c in (k_cache, v_cache):
        need(c.is_cuda and c.dtype == torch.float16 and c.dim() == 4 and
             tuple(c.shape[:2]) == (B, num_kv_heads) and c.shape[3] == head_dim and
             c.stride(3) == 1 and c.stride(2) == head_dim and
             c.stride(1) == c.shape[2] * head_dim,
             "prefill_rope_kv: caches must be fp16 CUDA [B, Hkv, capacity, D], dense per sequence")
    need(k_cache.stride(0) == v_cache.stride(0) and k_cache.shape == v_cache.shape,
         "prefill_rope_kv: k and v caches must have the same shape and strides")
    cos = cos.reshape(S, head_dim).contiguous()
    sin = sin.reshape(S, head_dim).contiguous()
    need(cos.dtype == torch.float32 and sin.dtype == torch.float32,
         "prefill_rope_kv: fp32 cos/sin [S, D]")
    q = torch.empty((B, S, num_heads, head_dim), dtype=torch.float16, device=qkv.device)
    k = v = None
    if kv_out:
        k = torch.empty((B, S, num_kv_heads, head_dim), dtype=torch.float16, device=qkv.device)
        v = torch.empty_like(k)
    with torch.cuda.device(qkv.device):
        st = _lib.load().ddq_prefill_rope_kv(
            rows.data_ptr(), rows.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.stride(0), k_cache.shape[2], cos.data_ptr(), sin.data_ptr(), int(start),
            q.data_ptr(), k.data_ptr() if kv_out else None, v.data_ptr() if kv_out else None,
            B, S, num_heads, num_kv_heads, head_dim,
            torch.cuda.current_stream(qkv.device).cuda_stream)
    _lib.check(st, "prefill_rope_kv")
    return (q, k, v) if kv_out else q
