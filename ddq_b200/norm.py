"""Residual add + RMSNorm in one kernel (``ddq_add_rmsnorm``), replacing the
reference's ``qwen2_rmsnorm_kernel`` (``RMSnorm_d.cu:23-87``) and the residual
addition before it (``engine.py:254-256``)."""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib


def add_rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float,
                delta: Optional[torch.Tensor] = None,
                inplace: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """s = fp16(x + delta) (or x), h = fp16(s * rsqrt(mean(s^2) + eps) * w).
    Returns (s, h); with ``inplace`` s is written into x."""
    if not (x.is_cuda and x.dtype == torch.float16 and x.is_contiguous()):
        raise RuntimeError("add_rmsnorm: x must be a contiguous fp16 CUDA tensor")
    H = x.shape[-1]
    if not (w.is_cuda and w.dtype == torch.float32 and w.numel() == H and w.is_contiguous()):
        raise RuntimeError("add_rmsnorm: w must be a contiguous fp32 CUDA tensor [H]")
    if delta is not None and not (delta.is_cuda and delta.dtype == torch.float16 and
                                  delta.shape == x.shape and delta.is_contiguous()):
        raise RuntimeError("add_rmsnorm: delta must match x")
    M = x.numel() // H
    h = torch.empty_like(x)
    s = x if (inplace or delta is None) else torch.empty_like(x)
    out_ptr = s.data_ptr() if delta is not None else None
    with torch.cuda.device(x.device):
        st = _lib.load().ddq_add_rmsnorm(
            x.data_ptr(), delta.data_ptr() if delta is not None else None, w.data_ptr(),
            float(eps), out_ptr, h.data_ptr(), M, H,
            torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(st, "add_rmsnorm")
    return s, h


class SplitActivations:
    """RMSNorm output in the decode GEMM's operand form: three e4m3 planes
    [3, M, H] and per-row scales [M] (``ddq_add_rmsnorm_split``)."""

    def __init__(self, planes: torch.Tensor, xscale: torch.Tensor, M: int, H: int):
        self.planes, self.xscale, self.M, self.H = planes, xscale, M, H


def add_rmsnorm_split(x: torch.Tensor, w: torch.Tensor, eps: float,
                      delta: Optional[torch.Tensor] = None,
                      out: Optional[SplitActivations] = None):
    """s = fp16(x + delta) (or x), h = rmsnorm(s), returned as (s, split h) for
    ``gemm_fp8.f8_forward_planes``; ``out`` reuses buffers of the same shape."""
    if not (x.is_cuda and x.dtype == torch.float16 and x.is_contiguous()):
        raise RuntimeError("add_rmsnorm_split: x must be a contiguous fp16 CUDA tensor")
    H = x.shape[-1]
    M = x.numel() // H
    if not (w.is_cuda and w.dtype == torch.float32 and w.numel() == H and w.is_contiguous()):
        raise RuntimeError("add_rmsnorm_split: w must be a contiguous fp32 CUDA tensor [H]")
    if delta is not None and not (delta.is_cuda and delta.dtype == torch.float16 and
                                  delta.shape == x.shape and delta.is_contiguous()):
        raise RuntimeError("add_rmsnorm_split: delta must match x")
    if out is None or out.M != M or out.H != H:
        out = SplitActivations(torch.empty((3, M, H), dtype=torch.uint8, device=x.device),
                               torch.empty((M,), dtype=torch.float32, device=x.device), M, H)
    s = x if delta is None else torch.empty_like(x)
    with torch.cuda.device(x.device):
        st = _lib.load().ddq_add_rmsnorm_split(
            x.data_ptr(), delta.data_ptr() if delta is not None else None, w.data_ptr(),
            float(eps), s.data_ptr() if delta is not None else None, None,
            out.planes.data_ptr(), out.xscale.data_ptr(), M, H,
            torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(st, "add_rmsnorm_split")
    return s, out
