"""CPU tests of the C ABI surface: the library loads, exports every function
include/ddq_b200.h declares, and rejects bad arguments with status codes
before touching a GPU."""
import ctypes
import os
import re

import pytest

from ddq_b200 import _lib
from ddq_b200.build import LIB_PATH, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(REPO, "include", "ddq_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ddq_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_library_exports_every_declared_function(lib):
    declared = header_functions()
    assert len(declared) >= 10
    raw = ctypes.CDLL(LIB_PATH)
    for name in declared:
        assert hasattr(raw, name), f"{name} declared in ddq_b200.h but not exported"
    assert set(declared) == set(_lib.EXPORTED), "ctypes signatures out of sync with the header"


def test_status_strings(lib):
    assert _lib.status_string(0) == "ok"
    for code in range(1, 8):
        assert _lib.status_string(code) not in ("ok", "unknown ddq status")
    assert _lib.status_string(99) == "unknown ddq status"
    assert lib.ddq_version() >= 1


def test_argument_validation_without_gpu(lib):
    # every case returns before any CUDA call
    assert lib.ddq_w8a16_gemm(None, None, None, None, 0, None, -1, 1, 1, None, 0, None) == 2
    assert lib.ddq_w8a16_gemm(None, None, None, None, 0, None, 4, 8, 16, None, 0, None) == 1
    assert lib.ddq_w8a16_gemm(None, None, None, None, 7, None, 4, 8, 16, None, 0, None) == 1
    assert lib.ddq_w8a16_gemm(None, None, None, None, 1, None, 4, 8, 16, None, 0, None) == 1
    assert lib.ddq_w8a16_gemm(None, None, None, None, 0, None, 0, 8, 16, None, 0, None) == 0
    assert lib.ddq_quantize_e4m3(None, 1, 4, 16, None, None, None) == 1
    assert lib.ddq_quantize_e4m3(None, 3, 4, 16, None, None, None) == 1
    assert lib.ddq_quantize_e4m3(None, 1, -4, 16, None, None, None) == 2
    assert lib.ddq_quantize_e4m3(None, 1, 0, 16, None, None, None) == 0
    assert lib.ddq_argmax_f16(None, 2, 10, None, None) == 1
    assert lib.ddq_argmax_f16(None, -2, 10, None, None) == 2
    assert lib.ddq_lm_head_argmax(None, None, None, 2, 10, 16, 0, None, None, None, 0, None) == 1
    assert lib.ddq_lm_head_argmax(None, None, None, 2, 10, 16, -1, None, None, None, 0, None) == 2
    assert lib.ddq_unpack_argmax(None, 3, None, None) == 1
    assert lib.ddq_device_error(None, None) == 1


def test_workspace_queries_are_host_only(lib):
    for M in (1, 16, 64, 4096):
        for N, K in ((896, 896), (1152, 896), (9728, 896), (896, 4864), (151936, 896)):
            assert lib.ddq_w8a16_gemm_workspace_size(M, N, K) < (1 << 34)
            assert lib.ddq_lm_head_argmax_workspace_size(M, N, K) < (1 << 34)


def test_missing_library_raises_instead_of_falling_back(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("DDQ_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()


def test_argument_validation_of_the_fused_operators_without_gpu(lib):
    """The decode/prefill operators reject bad arguments with status codes before
    any CUDA call (pointers below are placeholders that are never dereferenced:
    16-byte aligned A, misaligned U)."""
    A, U = 256, 258
    OK, INVALID, SHAPE, ALIGN = 0, 1, 2, 3
    # ddq_prefill_rope_kv(qkv, qkv_stride, kc, vc, bstride, cap, cos, sin, start,
    #                     q_out, k_out, v_out, B, S, Hq, Hkv, D, stream)
    hq, hkv, d, cap = 14, 2, 64, 16
    w, bs = (hq + 2 * hkv) * d, hkv * cap * d

    def rope(qkv=A, start=0, S=8, B=2, D=d, q=A):
        return lib.ddq_prefill_rope_kv(qkv, w, A, A, bs, cap, A, A, start, q, None, None,
                                       B, S, hq, hkv, D, None)
    assert lib.ddq_prefill_rope_kv(None, w, None, None, bs, cap, None, None, 0, None, None, None,
                                   -1, 8, hq, hkv, d, None) == SHAPE
    assert lib.ddq_prefill_rope_kv(None, w, None, None, bs, cap, None, None, 0, None, None, None,
                                   0, 8, hq, hkv, d, None) == OK
    assert lib.ddq_prefill_rope_kv(None, w, None, None, bs, cap, None, None, 0, None, None, None,
                                   2, 8, hq, hkv, d, None) == INVALID
    assert rope(start=10) == SHAPE          # start + S beyond the capacity
    assert rope(D=96) == SHAPE              # 64- or 128-wide heads only
    assert rope(qkv=U) == ALIGN
    assert rope(q=U) == ALIGN
    # ddq_decode_attention_split(qkv, qkv_stride, kc, vc, bstride, cap, cos, sin, pos, out,
    #                            out_stride, planes, xscale, B, Hq, Hkv, D, scale, flags, stream)

    def attn(planes=A, Hq=hq, Hkv=hkv, D=d, B=2):
        wd = (Hq + 2 * Hkv) * D
        return lib.ddq_decode_attention_split(A, wd, A, A, Hkv * cap * D, cap, A, A, A, None,
                                              Hq * D, planes, A, B, Hq, Hkv, D, 0.125, 0, None)
    assert attn(B=-1) == SHAPE
    assert lib.ddq_decode_attention_split(None, w, None, None, bs, cap, None, None, None, None,
                                          hq * d, None, None, 0, hq, hkv, d, 0.125, 0, None) == OK
    assert attn(planes=None) == INVALID
    assert attn(D=128) == SHAPE             # the split output is for 64-wide heads
    assert attn(Hq=16, Hkv=16) == SHAPE     # one cluster of at most 8 KV heads per token
    assert attn(planes=U) == ALIGN
    # ddq_add_rmsnorm_split(x, delta, w, eps, x_out, h, planes, xscale, M, H, stream)
    assert lib.ddq_add_rmsnorm_split(A, None, A, 1e-6, None, None, A, A, -1, 896, None) == SHAPE
    assert lib.ddq_add_rmsnorm_split(None, None, None, 1e-6, None, None, None, None, 0, 896,
                                     None) == OK
    assert lib.ddq_add_rmsnorm_split(A, None, None, 1e-6, None, None, A, A, 4, 896, None) == INVALID
    assert lib.ddq_add_rmsnorm_split(A, None, A, 1e-6, None, None, A, A, 4, 904, None) == SHAPE
    assert lib.ddq_add_rmsnorm_split(U, None, A, 1e-6, None, None, A, A, 4, 896, None) == ALIGN
    # ddq_w8a16_gemm_planes(planes, xscale, wq, scales, bias, bias_dtype, y, M, N, K, swiglu, stream)
    assert lib.ddq_w8a16_gemm_planes(A, A, A, A, None, 0, A, 65, 896, 896, 0, None) == SHAPE
    assert lib.ddq_w8a16_gemm_planes(A, A, A, A, None, 9, A, 16, 896, 896, 0, None) == INVALID
    assert lib.ddq_w8a16_gemm_planes(A, A, U, A, None, 0, A, 16, 896, 896, 0, None) == ALIGN


def test_argument_validation_of_the_fused_qkv_rope_gemm_without_gpu(lib):
    """ddq_w8a16_gemm_qkv_rope_kv returns its status before any CUDA call for
    bad arguments, for the shapes its fused epilogue does not take
    (DDQ_ERR_SHAPE: the caller then runs the GEMM and ddq_prefill_rope_kv) and
    for pointers that are not 32-byte aligned (fake addresses, nothing is
    dereferenced)."""
    A, A16, U = 256, 272, 258     # 32-byte aligned, 16- but not 32-byte, misaligned
    OK, INVALID, SHAPE, ALIGN = 0, 1, 2, 3
    hq, hkv, d, K = 14, 2, 64, 896

    def fused(x=A, bias_dtype=0, B=8, S=64, D=d, cap=64, start=0, q=A, kc=A, cs=A,
              bstride=None, null_x=False):
        bstride = hkv * cap * d if bstride is None else bstride
        return lib.ddq_w8a16_gemm_qkv_rope_kv(
            None if null_x else x, A, A, None, bias_dtype, B, S, K, hq, hkv, D, kc, A, bstride,
            cap, cs, A, start, q, None, None, A, 1 << 20, None)
    assert fused(B=-1) == SHAPE
    assert fused(B=0) == OK
    assert fused(null_x=True) == INVALID
    assert fused(bias_dtype=5) == INVALID
    assert fused(D=128) == SHAPE            # the fused epilogue takes 64-wide heads
    assert fused(B=1, S=16) == SHAPE        # 16 tokens: below the prefill kernel
    assert fused(start=8) == SHAPE          # start + S beyond the capacity
    assert fused(bstride=hkv * 64 * d - 8) == SHAPE
    assert fused(x=U) == ALIGN
    assert fused(q=A16) == ALIGN            # whole-sector stores need 32 bytes
    assert fused(kc=A16) == ALIGN
    assert fused(cs=A16) == ALIGN
