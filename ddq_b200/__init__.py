"""ddq_b200 - B200-native (sm_100a) W8A16 projection GEMMs for Qwen2.5-shaped decoders.

Public surface (mirrors the reference operator modules of hdahroug/ddq):

* ``ddq_b200.gemm_fp8`` - ``quantize``, ``f8_forward``, ``forward`` (gemm_FP8_d.cu)
* ``ddq_b200.sampler``  - ``forward`` greedy argmax (sampler_d.cu)
* ``ddq_b200.lm_head``  - fused lm_head GEMM + argmax, vocab sharding
* ``ddq_b200.engine``   - Qwen2 engine whose projections run on the W8A16 kernels

All compute goes through the C ABI of ``ddq_b200/lib/libddq_b200.so``
(``include/ddq_b200.h``); build it with ``python -m ddq_b200.build``.
"""
from . import gemm_fp8, sampler, lm_head  # noqa: F401
from . import engine  # noqa: F401

__all__ = ["gemm_fp8", "sampler", "lm_head", "engine"]
