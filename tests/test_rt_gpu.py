"""GPU parity tests of the opt-in tensor-core resident-slice GEMM (``rt.cu``,
switched on by ddq_set_debug bit 6 for every test here: 17..64
tokens on the tcgen05 A operand, each CTA's weight rows converted to fp16 in
shared memory before the grid dependency as the B operand, K split over a
thread-block cluster when it is long) against the CPU oracle: the Qwen2.5
projection shapes at token counts across 17..64, ragged row counts, split K
with even and uneven splits, the three bias types, the SwiGLU epilogue, a
non-finite activation, chains of dependent calls issued back to back, graph
replay, bitwise reproducibility, the dispatch rule and the bounded-wait
timeout."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import w8a16 as o

pytestmark = pytest.mark.gpu

TIGHT = 3e-3  # the GEMM tests' tolerance (normwise relative error vs the fp32 result)
DDQ_ERR_TIMEOUT = 7
QWEN = [(1152, 896), (896, 896), (9728, 896), (896, 4864), (4864, 896)]


def gen(M, N, K, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    b = rng.normal(0, 0.02, N).astype(np.float32)
    return x, w, b


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def g(cuda_device):
    from ddq_b200 import gemm_fp8
    return gemm_fp8


@pytest.fixture(scope="module")
def lib(cuda_device):
    from ddq_b200 import _lib
    return _lib.load()


RT = 64  # ddq_set_debug bit 6: the (opt-in) tensor-core resident-slice kernel


@pytest.fixture(autouse=True)
def _with_tensor_core_resident_slices(lib):
    assert lib.ddq_set_debug(RT, 0) == 0
    yield
    lib.ddq_set_debug(0, 0)


def check(g, M, N, K, seed, bias=True):
    x, w, b = gen(M, N, K, seed)
    wq, s = o.quantize(w)
    bb = b if bias else None
    y = g.f8_forward(dev(x), dev(wq), dev(s), None if bb is None else dev(bb))
    assert y.shape == (M, N) and y.dtype == torch.float16
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bb))
    assert err <= TIGHT, (M, N, K, err)


@pytest.mark.parametrize("M", [17, 18, 23, 24, 31, 32, 33, 40, 47, 48, 49, 56, 63, 64])
@pytest.mark.parametrize("N,K", QWEN)
def test_token_counts_on_projection_shapes(g, lib, M, N, K):
    """One kernel per call; 896 x 4864 (down) splits K four ways."""
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=600 + M + N)


@pytest.mark.parametrize("M,N,K", [(20, 7, 256), (37, 1000, 512), (64, 17, 1024), (50, 2049, 640),
                                   (17, 8, 64), (29, 264, 192), (64, 4872, 896), (41, 9730, 896)])
def test_ragged_shapes(g, lib, M, N, K):
    """Row counts that leave the last CTA a partial 8-row unit (rows past N
    convert whatever the slice buffer holds and reach only columns that are
    never stored)."""
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=M * 13 + N)


@pytest.mark.parametrize("M", [17, 33, 64])
@pytest.mark.parametrize("N,K", [(512, 1344), (264, 1344), (896, 2048), (640, 2560),
                                 (1024, 4096), (896, 4864), (300, 8192)])
def test_split_k(g, lib, M, N, K):
    """K over 20 atoms of 64 splits over a cluster (21 atoms: 10 + 11; 128
    atoms: 7 uneven splits); the partials are summed in split order through
    distributed shared memory."""
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=700 + M + K)


@pytest.mark.parametrize("bias", ["none", "f16", "f32"])
@pytest.mark.parametrize("N,K", [(1152, 896), (896, 4864)])
def test_bias_types(g, bias, N, K):
    M = 40
    x, w, b = gen(M, N, K, seed=81)
    wq, s = o.quantize(w)
    bb = None if bias == "none" else (b.astype(np.float16) if bias == "f16" else b)
    y = g.f8_forward(dev(x), dev(wq), dev(s), None if bb is None else dev(bb))
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bb)) <= TIGHT


def test_every_e4m3_code_decodes_exactly(g):
    """Weight row r holds code r in column 0 and zeros elsewhere; every token
    is one-hot on column 0: y[m, r] = e4m3(code r) * scale, exactly (NaN for
    the two NaN codes)."""
    M, K = 32, 256
    wq = np.zeros((256, K), np.uint8)
    wq[:, 0] = np.arange(256, dtype=np.uint8)
    s = np.full(256, 0.5, np.float32)
    x = np.zeros((M, K), np.float16)
    x[:, 0] = 1.0
    y = g.f8_forward(dev(x), dev(wq), dev(s)).cpu().numpy().astype(np.float32)
    ref = o.f8_forward(x, wq, s)
    finite = np.isfinite(ref)
    assert (~finite).sum() == 2 * M
    np.testing.assert_array_equal(y[finite], ref[finite].astype(np.float16).astype(np.float32))
    assert np.isnan(y[~finite]).all()


@pytest.mark.parametrize("M", [17, 32, 64])
@pytest.mark.parametrize("inter,K", [(4864, 896), (2432, 896), (48, 64)])
def test_swiglu_epilogue(g, lib, M, inter, K):
    """Gate/up with SwiGLU: 32-row units keep each gate row and its up row in
    one CTA; gate and up are rounded to fp16, then silu(g) * u."""
    rng = np.random.default_rng(M + inter)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    wq, s = o.quantize(rng.normal(0, 0.05, (2 * inter, K)).astype(np.float32))
    b = rng.normal(0, 0.1, 2 * inter).astype(np.float32)
    wil, sil, bil = g.interleave_gate_up(dev(wq), dev(s), dev(b))
    z = g.f8_forward_swiglu(dev(x), wil, sil, bil)
    assert z.shape == (M, inter)
    err = o.normwise_rel_err(z.cpu().numpy(), o.f8_forward_swiglu(x, wq, s, b))
    assert err <= TIGHT, err


@pytest.mark.parametrize("N,K", [(1152, 896), (896, 4864)])
def test_nonfinite_activation_stays_in_its_token(g, N, K):
    M = 40
    x, w, b = gen(M, N, K, seed=73)
    wq, s = o.quantize(w)
    ref = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    x2 = x.copy()
    x2[35, 10] = np.inf
    y = g.f8_forward(dev(x2), dev(wq), dev(s), dev(b))
    assert not torch.isfinite(y[35]).all()
    keep = [i for i in range(M) if i != 35]
    assert torch.equal(y[keep], ref[keep])


def test_chained_calls_read_the_previous_output(g):
    """Each call consumes the previous call's output, issued back to back (the
    next kernel converts its weights while this one runs and reads its
    activations only after it has completed): equal, bit for bit, to the
    same chain with a device synchronisation between calls."""
    torch.manual_seed(11)
    shapes = [(896, 896), (1152, 896), (9728, 1152), (896, 9728), (4864, 896), (896, 4864)]
    for M in (17, 24, 64):
        ws = [g.quantize((torch.randn(N, K, device="cuda") * 0.02).half()) for N, K in shapes]
        x = torch.randn(M, 896, device="cuda").half()
        ys = [x]
        for rep in range(3):
            for wq, s in ws:
                ys.append(g.f8_forward(ys[-1], wq, s))
        torch.cuda.synchronize()
        ref = [x]
        for rep in range(3):
            for wq, s in ws:
                ref.append(g.f8_forward(ref[-1], wq, s))
                torch.cuda.synchronize()
        for i, (a, r) in enumerate(zip(ys[1:], ref[1:])):
            assert torch.equal(a, r), (M, i)


def test_graph_replay_matches_eager(g):
    for M, N, K in [(48, 9728, 896), (64, 896, 4864)]:
        x, w, b = gen(M, N, K, seed=91)
        wq, s = o.quantize(w)
        xd, wqd, sd, bd = dev(x), dev(wq), dev(s), dev(b)
        eager = g.f8_forward(xd, wqd, sd, bd)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = g.f8_forward(xd, wqd, sd, bd)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


@pytest.mark.parametrize("M,N,K", [(64, 9728, 896), (33, 896, 4864)])
def test_deterministic_bitwise(g, M, N, K):
    x, w, b = gen(M, N, K, seed=59)
    wq, s = o.quantize(w)
    xd, wqd, sd = dev(x), dev(wq), dev(s)
    a = g.f8_forward(xd, wqd, sd)
    for _ in range(3):
        assert torch.equal(g.f8_forward(xd, wqd, sd), a)


def test_dispatch(lib):
    for N, K in QWEN:
        for M in (17, 32, 64):
            assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    assert lib.ddq_w8a16_gemm_kernel_count(32, 1152, 912) == 2     # K % 64 != 0
    assert lib.ddq_w8a16_gemm_kernel_count(65, 1152, 896) == 1     # 64 < M < 128: tc_gemm
    assert lib.ddq_w8a16_gemm_kernel_count(200, 1152, 896) == 2    # expansion + prefill GEMM
    # lm_head rows: more than 256 rows per CTA, the decode kernel
    assert lib.ddq_w8a16_gemm_kernel_count(32, 151936, 896) == 2
    # without bit 6, 17..64 tokens go to the older kernels
    assert lib.ddq_set_debug(0, 0) == 0
    assert lib.ddq_w8a16_gemm_kernel_count(64, 9728, 896) == 2      # split + decode
    assert lib.ddq_w8a16_gemm_kernel_count(64, 1152, 896) == 1      # mma.sync, warps over tokens
    # bit 6 with an injection bit: the older kernels
    assert lib.ddq_set_debug(RT | 4, 0) == 0
    assert lib.ddq_w8a16_gemm_kernel_count(64, 1152, 896) == 2


def device_error(lib):
    code = ctypes.c_int(-1)
    assert lib.ddq_device_error(ctypes.byref(code), torch.cuda.current_stream().cuda_stream) == 0
    return code.value


@pytest.mark.parametrize("M,N,K", [(64, 9728, 896), (40, 896, 4864)])
def test_bounded_wait_reports_timeout_and_context_survives(g, lib, M, N, K):
    """Debug bit 4 makes the MMA thread skip the accumulator-ready signal (a
    flag that nothing then sets): the epilogue's wait runs out after 20 ms,
    the kernel records DDQ_ERR_TIMEOUT, drains its copies and MMAs, still
    takes part in the cluster barriers (split K), writes nothing, frees TMEM
    and returns; the next call is correct."""
    x, w, _ = gen(M, N, K, seed=5)
    wq, s = o.quantize(w)
    xd, wqd, sd = dev(x), dev(wq), dev(s)
    assert device_error(lib) == 0
    y0 = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    try:
        assert lib.ddq_set_debug(RT | 16, 20_000_000) == 0
        assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
        from ddq_b200 import _lib
        st = lib.ddq_w8a16_gemm(xd.data_ptr(), wqd.data_ptr(), sd.data_ptr(), None,
                                _lib.DTYPE_NONE, y0.data_ptr(), M, N, K, None, 0,
                                torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        assert device_error(lib) == DDQ_ERR_TIMEOUT
        assert not y0.any()  # nothing written
    finally:
        lib.ddq_set_debug(RT, 0)
    y = g.f8_forward(xd, wqd, sd)
    torch.cuda.synchronize()
    assert device_error(lib) == 0
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s)) <= TIGHT
