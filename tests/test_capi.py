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
