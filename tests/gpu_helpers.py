"""Helpers shared by GPU tests (imported, not collected: no test_ prefix)."""
import torch


def decode_kernel_gemm(x, wq, s, b=None):
    """The activation-split pre-pass + e4m3 decode kernel on fp16 activations,
    whatever kernel ``f8_forward`` would pick for the shape: ``ddq_w8a16_gemm``
    with a caller workspace while ``ddq_set_debug`` bit 2 routes the thin
    kernel's shapes to the split + decode kernels.  Fused producers of the
    decode kernel's operand (the norm and attention kernels' plane outputs) are
    compared bit for bit against this path."""
    from ddq_b200 import _lib, gemm_fp8
    lib = _lib.load()
    x = x.contiguous()
    M, K = x.shape
    N = wq.shape[0]
    y = torch.empty(M, N, dtype=torch.float16, device=x.device)
    nws = lib.ddq_w8a16_gemm_workspace_size(M, N, K)
    ws = gemm_fp8.workspace(x.device, nws)
    assert lib.ddq_set_debug(4, 0) == 0
    try:
        st = lib.ddq_w8a16_gemm(x.data_ptr(), wq.data_ptr(), s.data_ptr(),
                                b.data_ptr() if b is not None else None,
                                _lib.DTYPE_F32 if b is not None else _lib.DTYPE_NONE,
                                y.data_ptr(), M, N, K, ws.data_ptr(), ws.numel(),
                                torch.cuda.current_stream().cuda_stream)
    finally:
        lib.ddq_set_debug(0, 0)
    assert st == 0, _lib.status_string(st)
    return y
