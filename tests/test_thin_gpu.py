"""GPU parity tests of the 1..16-token GEMM kernel (``thin.cu``; run with
``ddq_set_debug`` bit 3, which gives it the shapes the resident-slice kernel
would otherwise take) against the
CPU oracle: the token counts it takes (and the decode kernel beyond them),
ragged row counts, the smallest K, every per-CTA tile-count variant up to the
limit of 16, every e4m3 code, the three bias types, chained calls under
programmatic dependent launch and a CUDA graph, and the dispatch boundaries
(the kernel count the library reports for a shape).  The kernel takes a
shape of up to 16 tokens when each CTA holds at most 96 (8-row tile, 64-wide
K block) units, or any number at 1-2 tokens, and shared memory holds its
weight slice and the activations."""
import numpy as np
import pytest
import torch

from oracle import w8a16 as o

pytestmark = pytest.mark.gpu

TIGHT = 3e-3  # the GEMM tests' tolerance (normwise relative error vs the fp32 result)


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


@pytest.fixture(autouse=True)
def thin_dispatch(cuda_device):
    """ddq_set_debug bit 3: the shapes of the resident-slice kernel (rs.cu),
    which ddq_w8a16_gemm tries first, go to this file's kernel instead."""
    from ddq_b200 import _lib
    L = _lib.load()
    assert L.ddq_set_debug(8, 0) == 0
    yield
    L.ddq_set_debug(0, 0)


def sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("M", range(1, 17))
def test_every_token_count(g, lib, M):
    N, K = 1152, 896
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    x, w, b = gen(M, N, K, seed=200 + M)
    wq, s = o.quantize(w)
    y = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b))
    assert err <= TIGHT, (M, err)


@pytest.mark.parametrize("M,N,K", [
    (1, 896, 4864),      # down at M = 1: 38.9 KB slice, 9.7 KB activations
    (16, 896, 4864),     # down at M = 16: 156 KB of activations in shared memory
    (1, 9728, 896),      # gate/up at M = 1: 126 units per CTA (taken at M <= 2)
    (2, 9728, 896),
    (16, 4864, 896),     # 70 units per CTA
    (5, 4864, 896),      # 5 tiles per CTA
    (2, 10656, 512),     # 9 tiles per CTA
    (2, 4000, 640),      # 4 tiles per CTA
    (2, 1190, 64),       # 149 tiles: one CTA holds two, the last tile 6 rows
    (3, 1003, 128),      # last tile 3 rows
    (5, 7, 64),          # one partial tile, K = one block
    (16, 1152, 256),     # 16 tokens: both MMA row halves
    (12, 896, 384),      # 12 tokens
])
def test_shapes(g, lib, M, N, K):
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    x, w, b = gen(M, N, K, seed=M * 7 + N + K)
    wq, s = o.quantize(w)
    bh = b.astype(np.float16)
    y = g.f8_forward(dev(x), dev(wq), dev(s), dev(bh))
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bh))
    assert err <= TIGHT, (M, N, K, err)


def test_tile_limit_per_cta(g, lib):
    """16 tiles per CTA is the most the kernel takes; one tile more goes to the
    decode kernel.  Both give the oracle's result."""
    M, K = 4, 64
    for N, want in ((16 * 8 * sms(), 1), (16 * 8 * sms() + 8, 2)):
        assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == want, N
        x, w, b = gen(M, N, K, seed=N)
        wq, s = o.quantize(w)
        y = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
        err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b))
        assert err <= TIGHT, (N, err)


def test_dispatch_boundaries(lib):
    assert lib.ddq_w8a16_gemm_kernel_count(17, 1152, 256) == 2    # more than 16 tokens
    assert lib.ddq_w8a16_gemm_kernel_count(4, 1152, 912) == 2     # K % 64 != 0
    assert lib.ddq_w8a16_gemm_kernel_count(2, 9728, 896) == 1     # 126 units, 2 tokens
    assert lib.ddq_w8a16_gemm_kernel_count(3, 9728, 896) == 2     # 126 units, 3 tokens
    assert lib.ddq_w8a16_gemm_kernel_count(16, 896, 8192) == 2    # activations exceed shared memory
    assert lib.ddq_w8a16_gemm_kernel_count(16, 1152, 40) == 1     # K % 16 != 0: CUDA-core kernel
    assert lib.ddq_w8a16_gemm_kernel_count(0, 1152, 896) == 0


@pytest.mark.parametrize("bias", ["none", "f16", "f32"])
def test_bias_types(g, bias):
    M, N, K = 4, 896, 896
    x, w, b = gen(M, N, K, seed=41)
    wq, s = o.quantize(w)
    bb = None if bias == "none" else (b.astype(np.float16) if bias == "f16" else b)
    y = g.f8_forward(dev(x), dev(wq), dev(s), None if bb is None else dev(bb))
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bb))
    assert err <= TIGHT, (bias, err)


def test_every_e4m3_code_decodes_exactly(g, lib):
    """Every finite e4m3 code (both signs, subnormals included) times a one-hot
    activation: the integer e4m3 -> fp16 conversion and the factor 256 in the
    row scale are exact."""
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)   # 254 codes
    N, K = len(codes), 64
    assert lib.ddq_w8a16_gemm_kernel_count(4, N, K) == 1
    wq = np.zeros((N, K), np.uint8)
    wq[:, 37] = codes
    s = np.ones(N, np.float32)
    x = np.zeros((4, K), np.float16)
    x[:, 37] = 1.0
    y = g.f8_forward(dev(x), dev(wq), dev(s)).cpu().numpy().astype(np.float32)
    want = o.e4m3fn_decode(codes).astype(np.float16).astype(np.float32)
    for r in range(4):
        np.testing.assert_array_equal(y[r], want)


def test_nonfinite_activation_stays_in_its_row(g):
    """An inf in one token's activations makes that token's outputs non-finite
    and leaves the other tokens' rows exact (the zero rows past M and the
    other tokens share MMAs with it)."""
    M, N, K = 5, 896, 896
    x, w, b = gen(M, N, K, seed=43)
    wq, s = o.quantize(w)
    ref = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    x2 = x.copy()
    x2[2, 100] = np.inf
    y = g.f8_forward(dev(x2), dev(wq), dev(s), dev(b))
    assert not torch.isfinite(y[2]).all()
    keep = [0, 1, 3, 4]
    assert torch.equal(y[keep], ref[keep])


def test_chained_calls_read_the_previous_output(g):
    """Each call consumes the previous call's output, issued back to back (the
    next kernel copies its weights while the previous one still runs); the
    results equal the same chain with a device synchronisation between calls,
    bit for bit.  3 and 16 tokens run the thin kernel, 17 the decode kernel."""
    torch.manual_seed(5)
    shapes = [(896, 896), (4864, 896), (896, 4864), (1152, 896)]
    for M in (3, 16, 17):
        ws = []
        for N, K in shapes:
            wq, s = g.quantize((torch.randn(N, K, device="cuda") * 0.02).half())
            ws.append((wq, s))
        x = torch.randn(M, 896, device="cuda").half()
        ys = [x]
        for (wq, s), (N, K) in zip(ws, shapes):
            ys.append(g.f8_forward(ys[-1], wq, s))
        torch.cuda.synchronize()
        ref = [x]
        for (wq, s), (N, K) in zip(ws, shapes):
            ref.append(g.f8_forward(ref[-1], wq, s))
            torch.cuda.synchronize()
        for a, r in zip(ys[1:], ref[1:]):
            assert torch.equal(a, r), M


def test_graph_replay_matches_eager(g):
    M, N, K = 4, 1152, 896
    x, w, b = gen(M, N, K, seed=47)
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
