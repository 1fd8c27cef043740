"""Drop-in mirror of the reference operator module ``gemm_FP8_d.cu``.

Same names, argument names, defaults, output shapes/dtypes and error
behaviour as the pybind11 module of ``gemm_FP8_d.cu:221-228``:

* ``quantize(w) -> [wq uint8 [N,K], scales fp32 [N]]``   (``gemm_FP8_d.cu:150-167``)
* ``f8_forward(x, wq, scales, bias=None) -> y``          (``gemm_FP8_d.cu:171-210``)
* ``forward(x, w, bias=None) -> y``                      (``gemm_FP8_d.cu:214-217``)

so ``engine.py``'s ``_linear`` (``engine.py:85-86``) can call
``f8_forward(x, module.wq, module.scales, module.bias)`` in place of
``gemm_naive.forward(x, module.weight, module.bias)``.

Differences from the reference, all widening what is accepted:
``quantize`` also takes fp32 weights and ``f8_forward`` also takes an fp32
bias (the reference takes fp16 only, ``gemm_FP8_d.cu:151,191``).  Errors are
``RuntimeError`` with the reference's message text, as ``TORCH_CHECK`` raises.
All work runs on the caller's current CUDA stream, asynchronously, through the
C ABI of ``libddq_b200.so``; nothing falls back to the CPU.
"""
from __future__ import annotations

import contextlib
from typing import List, Optional

import torch

from . import _lib

_workspaces: dict = {}
_ws_sizes: dict = {}   # (entry, device index, shape) -> workspace bytes
# the current stream's raw handle without building a Stream object (a few us
# per call on the eager path); torch's public API where it is missing
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _on_device(device: torch.device):
    """Make `device` current for the library call (which sizes and launches
    on the current device), without the two device switches when it already
    is."""
    if torch.cuda.current_device() == device.index:
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream_ptr(device: torch.device) -> int:
    if _raw_stream is not None and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-filled scratch per (device, current stream), grown on demand and
    then reused.

    The kernels leave the counters in it at zero after each call, so one
    workspace serves every call ordered on a stream; calls running on
    different streams at the same time get different workspaces.
    """
    key = (device.type, device.index, _stream_ptr(device))
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def quantize(w: torch.Tensor) -> List[torch.Tensor]:
    """Quantize fp16/fp32 [N,K] weights to e4m3fn bytes + per-row fp32 scales."""
    _check(w.is_cuda and w.dtype in (torch.float16, torch.float32),
           "gemm_fp8: fp16 CUDA weight required")
    _check(w.dim() == 2, "gemm_fp8: weight must be [N,K]")
    wc = w.contiguous()
    N, K = wc.shape
    wq = torch.empty((N, K), dtype=torch.uint8, device=w.device)
    scales = torch.empty((N,), dtype=torch.float32, device=w.device)
    code = _lib.DTYPE_F16 if wc.dtype == torch.float16 else _lib.DTYPE_F32
    with torch.cuda.device(w.device):
        st = _lib.load().ddq_quantize_e4m3(wc.data_ptr(), code, N, K, wq.data_ptr(),
                                           scales.data_ptr(), _stream_ptr(w.device))
    _lib.check(st, "gemm_fp8.quantize")
    return [wq, scales]


def f8_forward(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
               bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FP8 GEMM on pre-quantized weights: y[...,N] = x[...,K] @ (e4m3(wq)*s)^T (+bias)."""
    _check(x.is_cuda and wq.is_cuda, "gemm_fp8: CUDA tensors required")
    _check(x.dtype == torch.float16, "gemm_fp8: fp16 x required")
    _check(wq.dtype == torch.uint8, "gemm_fp8: wq must be uint8 e4m3")
    _check(wq.dim() == 2 and wq.size(0) == scales.numel(), "gemm_fp8: shape mismatch")
    _check(scales.is_cuda and scales.dtype == torch.float32, "gemm_fp8: scales must be fp32 CUDA")
    N, K = wq.shape
    _check(x.dim() >= 1 and x.size(-1) == K, "gemm_fp8: inner dim mismatch")
    xc = x.contiguous()
    x2 = xc.reshape(-1, K)
    M = x2.size(0)
    y2 = torch.empty((M, N), dtype=torch.float16, device=x.device)
    bptr, bcode = None, _lib.DTYPE_NONE
    if bias is not None and bias.numel() > 0:
        _check(bias.numel() == N, "gemm_fp8: bias length mismatch")
        _check(bias.is_cuda and bias.dtype in (torch.float16, torch.float32),
               "gemm_fp8: bias must be fp16 or fp32 CUDA")
        bias = bias.contiguous()
        bptr = bias.data_ptr()
        bcode = _lib.DTYPE_F16 if bias.dtype == torch.float16 else _lib.DTYPE_F32
    wqc = wq.contiguous()
    sc = scales.contiguous()
    L = _lib.load()
    dev = x.device
    with _on_device(dev):
        key = (dev.index, M, N, K)
        nws = _ws_sizes.get(key)
        if nws is None:
            nws = _ws_sizes[key] = L.ddq_w8a16_gemm_workspace_size(M, N, K)
        ws = workspace(dev, nws) if nws else None
        st = L.ddq_w8a16_gemm(x2.data_ptr(), wqc.data_ptr(), sc.data_ptr(), bptr, bcode,
                              y2.data_ptr(), M, N, K,
                              ws.data_ptr() if ws is not None else None,
                              ws.numel() if ws is not None else 0, _stream_ptr(dev))
    _lib.check(st, "gemm_fp8.f8_forward")
    return y2.reshape(*x.shape[:-1], N)


SWIGLU_BLOCK = 16  # gate/up interleave granularity of the fused SwiGLU GEMM (rows)


def interleave_gate_up(wq_gu: torch.Tensor, scales_gu: torch.Tensor,
                       bias_gu: Optional[torch.Tensor] = None):
    """Reorder a stacked [gate; up] projection ([2I, K] rows: gate 0..I-1, then up)
    into the layout of ``f8_forward_swiglu``: blocks of 16 gate rows followed by
    the same 16 up rows.  Returns (wq, scales, bias) with the same row count."""
    _check(wq_gu.dim() == 2 and wq_gu.size(0) % (2 * SWIGLU_BLOCK) == 0,
           "gemm_fp8: gate/up rows must be 2 * I with I a multiple of 16")
    two_i, K = wq_gu.shape
    nb = two_i // (2 * SWIGLU_BLOCK)

    def il(t, tail):
        return t.reshape(2, nb, SWIGLU_BLOCK, *tail).transpose(0, 1).reshape(two_i, *tail).contiguous()
    b = None if bias_gu is None or bias_gu.numel() == 0 else il(bias_gu, ())
    return il(wq_gu, (K,)), il(scales_gu, ()), b


def f8_forward_swiglu(x: torch.Tensor, wq_il: torch.Tensor, scales_il: torch.Tensor,
                      bias_il: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gate/up GEMM with the SwiGLU epilogue: z[..., I] = silu(gate) * up, where
    gate/up are the fp16 outputs the two projections would give.  The weight
    comes from ``interleave_gate_up``.  No [M, 2I] intermediate is written."""
    _check(x.is_cuda and wq_il.is_cuda, "gemm_fp8: CUDA tensors required")
    _check(x.dtype == torch.float16, "gemm_fp8: fp16 x required")
    _check(wq_il.dtype == torch.uint8 and wq_il.dim() == 2, "gemm_fp8: wq must be uint8 [2I,K]")
    _check(scales_il.is_cuda and scales_il.dtype == torch.float32 and
           scales_il.numel() == wq_il.size(0), "gemm_fp8: scales must be fp32 CUDA [2I]")
    two_i, K = wq_il.shape
    _check(two_i % (2 * SWIGLU_BLOCK) == 0, "gemm_fp8: gate/up rows must be 2 * I, I % 16 == 0")
    _check(x.dim() >= 1 and x.size(-1) == K, "gemm_fp8: inner dim mismatch")
    inter = two_i // 2
    x2 = x.contiguous().reshape(-1, K)
    M = x2.size(0)
    z = torch.empty((M, inter), dtype=torch.float16, device=x.device)
    bptr, bcode = None, _lib.DTYPE_NONE
    if bias_il is not None and bias_il.numel() > 0:
        _check(bias_il.numel() == two_i and bias_il.is_cuda and
               bias_il.dtype in (torch.float16, torch.float32), "gemm_fp8: bias mismatch")
        bias_il = bias_il.contiguous()
        bptr = bias_il.data_ptr()
        bcode = _lib.DTYPE_F16 if bias_il.dtype == torch.float16 else _lib.DTYPE_F32
    wqc, sc = wq_il.contiguous(), scales_il.contiguous()
    L = _lib.load()
    dev = x.device
    with _on_device(dev):
        key = ("swiglu", dev.index, M, inter, K)
        nws = _ws_sizes.get(key)
        if nws is None:
            nws = _ws_sizes[key] = L.ddq_w8a16_gemm_swiglu_workspace_size(M, inter, K)
        ws = workspace(dev, nws) if nws else None
        st = L.ddq_w8a16_gemm_swiglu(x2.data_ptr(), wqc.data_ptr(), sc.data_ptr(), bptr, bcode,
                                     z.data_ptr(), M, inter, K,
                                     ws.data_ptr() if ws is not None else None,
                                     ws.numel() if ws is not None else 0, _stream_ptr(dev))
    _lib.check(st, "gemm_fp8.f8_forward_swiglu")
    return z.reshape(*x.shape[:-1], inter)


def f8_forward_planes(act, wq: torch.Tensor, scales: torch.Tensor,
                      bias: Optional[torch.Tensor] = None, swiglu: bool = False) -> torch.Tensor:
    """The decode GEMM (M <= 64) on activations split by ``norm.add_rmsnorm_split``
    (``act``): y [M, N] (or, with ``swiglu`` and an interleaved gate/up weight,
    z [M, N/2]) - the same values f8_forward / f8_forward_swiglu give on h."""
    N, K = wq.shape
    _check(act.H == K, "gemm_fp8: inner dim mismatch")
    M = act.M
    y = torch.empty((M, N // 2 if swiglu else N), dtype=torch.float16, device=wq.device)
    bptr, bcode = None, _lib.DTYPE_NONE
    if bias is not None and bias.numel() > 0:
        bias = bias.contiguous()
        bptr = bias.data_ptr()
        bcode = _lib.DTYPE_F16 if bias.dtype == torch.float16 else _lib.DTYPE_F32
    with torch.cuda.device(wq.device):
        st = _lib.load().ddq_w8a16_gemm_planes(act.planes.data_ptr(), act.xscale.data_ptr(),
                                               wq.data_ptr(), scales.data_ptr(), bptr, bcode,
                                               y.data_ptr(), M, N, K, 1 if swiglu else 0,
                                               _stream_ptr(wq.device))
    _lib.check(st, "gemm_fp8.f8_forward_planes")
    return y


def forward(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Drop-in for gemm_d.forward: quantize w (every call, as the reference does), then GEMM."""
    wq, scales = quantize(w)
    return f8_forward(x, wq, scales, bias)
