"""Drop-in mirror of the reference operator module ``sampler_d.cu``.

``forward(logits) -> idx``: greedy argmax over fp16 logits ``[B,1,V]`` ->
int64 ``[B,1]``, ties to the lowest index (``sampler_d.cu:51-70``, kernel
``sampler_d.cu:10-49``).  Runs the CUDA kernel of ``libddq_b200.so`` on the
current stream.
"""
from __future__ import annotations

import torch

from . import _lib


def forward(logits: torch.Tensor) -> torch.Tensor:
    if not (logits.is_cuda and logits.dtype == torch.float16):
        raise RuntimeError("sampler_d: fp16 CUDA tensor required")
    if not (logits.dim() == 3 and logits.size(1) == 1):
        raise RuntimeError("sampler_d: expected [B,1,V]")
    B, _, V = logits.shape
    lc = logits.contiguous()
    idx = torch.empty((B, 1), dtype=torch.int64, device=logits.device)
    with torch.cuda.device(logits.device):
        st = _lib.load().ddq_argmax_f16(lc.data_ptr(), B, V, idx.data_ptr(),
                                        torch.cuda.current_stream(logits.device).cuda_stream)
    _lib.check(st, "sampler_d.forward")
    return idx
