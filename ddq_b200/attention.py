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


def qkv_rope_kv(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                bias: Optional[torch.Tensor], k_cache: torch.Tensor, v_cache: torch.Tensor,
                cos: torch.Tensor, sin: torch.Tensor, start: int, num_heads: int,
                num_kv_heads: int, head_dim: int, kv_out: bool = False):
    """The q/k/v projection of a prefill chunk followed by ``prefill_rope_kv``:
    x fp16 [B, S, K] (or [B * S, K] with B taken from the caches), wq/scales/bias
    the fused [(Hq + 2 Hkv) * D, K] projection.  Same results, bit for bit, as
    ``gemm_fp8.f8_forward`` then ``prefill_rope_kv``.  Where the prefill kernel
    takes the shape (D == 64, B * S at prefill size) one launch pair (weight
    expansion + GEMM) does all of it, RoPE and the cache write in the GEMM's
    epilogue (``ddq_w8a16_gemm_qkv_rope_kv``), and the [B * S, (Hq + 2 Hkv) D]
    projection is never written; elsewhere the two calls run.  Replaces the
    reference's q/k/v projections (``engine.py:215-217``), q/k RoPE
    (``engine.py:219-220``) and cache write (``engine.py:222``)."""
    from . import gemm_fp8

    def need(cond, msg):
        if not cond:
            raise RuntimeError(msg)
    B = k_cache.shape[0]
    width = (num_heads + 2 * num_kv_heads) * head_dim
    need(x.is_cuda and x.dtype == torch.float16, "qkv_rope_kv: x must be fp16 CUDA")
    need(wq.is_cuda and wq.dtype == torch.uint8 and wq.dim() == 2 and wq.size(0) == width,
         "qkv_rope_kv: wq must be uint8 [(Hq + 2 Hkv) * D, K]")
    K = wq.size(1)
    need(x.size(-1) == K, "qkv_rope_kv: inner dim mismatch")
    rows = x.contiguous().reshape(-1, K)
    need(rows.size(0) % B == 0, "qkv_rope_kv: x rows must be B * S")
    S = rows.size(0) // B
    st = _lib.ERR_SHAPE
    if head_dim == 64 and S > 0 and k_cache.data_ptr() % 32 == 0 and \
            v_cache.data_ptr() % 32 == 0 and k_cache.stride(0) % 16 == 0:
        for c in (k_cache, v_cache):
            need(c.is_cuda and c.dtype == torch.float16 and c.dim() == 4 and
                 tuple(c.shape[:2]) == (B, num_kv_heads) and c.shape[3] == head_dim and
                 c.stride(3) == 1 and c.stride(2) == head_dim and
                 c.stride(1) == c.shape[2] * head_dim,
                 "qkv_rope_kv: caches must be fp16 CUDA [B, Hkv, capacity, D], dense per sequence")
        need(k_cache.stride(0) == v_cache.stride(0) and k_cache.shape == v_cache.shape,
             "qkv_rope_kv: k and v caches must have the same shape and strides")
        need(scales.is_cuda and scales.dtype == torch.float32 and scales.numel() == width,
             "qkv_rope_kv: scales must be fp32 CUDA [(Hq + 2 Hkv) * D]")
        cs = cos.reshape(S, head_dim).contiguous()
        sn = sin.reshape(S, head_dim).contiguous()
        need(cs.dtype == torch.float32 and sn.dtype == torch.float32,
             "qkv_rope_kv: fp32 cos/sin [S, D]")
        if cs.data_ptr() % 32:
            cs = cs.clone()
        if sn.data_ptr() % 32:
            sn = sn.clone()
        bptr, bcode = None, _lib.DTYPE_NONE
        if bias is not None and bias.numel() > 0:
            need(bias.numel() == width and bias.is_cuda and
                 bias.dtype in (torch.float16, torch.float32), "qkv_rope_kv: bias mismatch")
            bias = bias.contiguous()
            bptr = bias.data_ptr()
            bcode = _lib.DTYPE_F16 if bias.dtype == torch.float16 else _lib.DTYPE_F32
        q = torch.empty((B, S, num_heads, head_dim), dtype=torch.float16, device=x.device)
        k = v = None
        if kv_out:
            k = torch.empty((B, S, num_kv_heads, head_dim), dtype=torch.float16, device=x.device)
            v = torch.empty_like(k)
        wqc, sc = wq.contiguous(), scales.contiguous()
        L = _lib.load()
        with torch.cuda.device(x.device):
            nws = L.ddq_w8a16_gemm_workspace_size(B * S, width, K)
            ws = gemm_fp8.workspace(x.device, nws) if nws else None
            st = L.ddq_w8a16_gemm_qkv_rope_kv(
                rows.data_ptr(), wqc.data_ptr(), sc.data_ptr(), bptr, bcode, B, S, K,
                num_heads, num_kv_heads, head_dim, k_cache.data_ptr(), v_cache.data_ptr(),
                k_cache.stride(0), k_cache.shape[2], cs.data_ptr(), sn.data_ptr(), int(start),
                q.data_ptr(), k.data_ptr() if kv_out else None, v.data_ptr() if kv_out else None,
                ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                torch.cuda.current_stream(x.device).cuda_stream)
        if st != _lib.ERR_SHAPE:
            _lib.check(st, "qkv_rope_kv")
            return (q, k, v) if kv_out else q
    qkv = gemm_fp8.f8_forward(rows, wq, scales, bias)
    return prefill_rope_kv(qkv, k_cache, v_cache, cos, sin, start, num_heads, num_kv_heads,
                           head_dim, kv_out=kv_out)
