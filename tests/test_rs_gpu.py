"""GPU parity tests of the resident-slice GEMM kernels (``rs.cu``: each CTA's
weight slice in shared memory, weights on the MMA rows; 1..16 tokens with
the warps over K blocks, 17..64 with the warps over 8-token blocks) against
the CPU oracle: every token count, ragged row counts and K values, every
per-CTA tile count up to the limit (6 sixteen-row tiles at 1..8 tokens, 5 at
9..16), every e4m3 code,
the three bias types, a non-finite activation, chains of dependent calls
issued back to back (the kernel lets the next one start at its own entry),
graph replay, bitwise reproducibility and the dispatch boundaries."""
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




def sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def check(g, M, N, K, seed, bias=True):
    x, w, b = gen(M, N, K, seed)
    wq, s = o.quantize(w)
    bb = b if bias else None
    y = g.f8_forward(dev(x), dev(wq), dev(s), None if bb is None else dev(bb))
    assert y.shape == (M, N) and y.dtype == torch.float16
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bb))
    assert err <= TIGHT, (M, N, K, err)


@pytest.mark.parametrize("M", range(1, 17))
@pytest.mark.parametrize("N,K", [(1152, 896), (9728, 896), (896, 4864), (4864, 896)])
def test_every_token_count(g, lib, M, N, K):
    """(896 x 4864 at 16 tokens exceeds this kernel's shared memory and runs
    the thin kernel; every case is one kernel either way.)"""
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=300 + M + N)


@pytest.mark.parametrize("M,N,K", [(1, 7, 256), (3, 1000, 512), (9, 4872, 896), (16, 17, 1024),
                                   (5, 2049, 640), (2, 128, 8192), (8, 33, 2048), (12, 896, 512)])
def test_ragged_shapes(g, lib, M, N, K):
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=M * 7 + N)


@pytest.mark.parametrize("per_cta", range(1, 7))
def test_every_tile_count_per_cta(g, lib, per_cta):
    """N chosen so the busiest CTA holds per_cta tiles of 16 rows (one row
    past a multiple of 16: the last tile is partial and its rows past N read
    as zero)."""
    M, K = 6, 256
    N = (per_cta - 1) * 16 * sms() + 1 if per_cta > 1 else 97
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=per_cta)


def test_tile_limit_per_cta(g, lib):
    """6 tiles per CTA at up to 8 tokens, 5 at 9..16; one tile more goes to
    another kernel (both give the oracle's result)."""
    K = 512
    assert lib.ddq_w8a16_gemm_kernel_count(4, 6 * 16 * sms(), K) == 1
    assert lib.ddq_w8a16_gemm_kernel_count(4, 6 * 16 * sms() + 1, K) == 2
    check(g, 12, 5 * 16 * sms(), K, seed=61)
    check(g, 12, 5 * 16 * sms() + 1, K, seed=62)


def test_dispatch_boundaries(lib):
    assert lib.ddq_w8a16_gemm_kernel_count(3, 9728, 896) == 1     # gate/up, 3 tokens
    assert lib.ddq_w8a16_gemm_kernel_count(16, 9728, 896) == 1    # gate/up, 16 tokens
    assert lib.ddq_w8a16_gemm_kernel_count(24, 4864, 896) == 1    # 17..64 tokens: warps over tokens
    assert lib.ddq_w8a16_gemm_kernel_count(64, 1152, 896) == 1
    assert lib.ddq_w8a16_gemm_kernel_count(17, 896, 4864) == 2    # x exceeds shared memory
    assert lib.ddq_w8a16_gemm_kernel_count(4, 1152, 912) == 2     # K % 64 != 0
    assert lib.ddq_w8a16_gemm_kernel_count(16, 896, 8192) == 2    # x + slice exceed shared memory


@pytest.mark.parametrize("bias", ["none", "f16", "f32"])
def test_bias_types(g, bias):
    M, N, K = 11, 1152, 896
    x, w, b = gen(M, N, K, seed=51)
    wq, s = o.quantize(w)
    bb = None if bias == "none" else (b.astype(np.float16) if bias == "f16" else b)
    y = g.f8_forward(dev(x), dev(wq), dev(s), None if bb is None else dev(bb))
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bb))
    assert err <= TIGHT, (bias, err)


@pytest.mark.parametrize("M", [1, 9])
def test_every_e4m3_code_decodes_exactly(g, lib, M):
    """Every finite e4m3 code (both signs, subnormals included) times a one-hot
    activation, on the A operand's rows g and g + 8: exact."""
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)   # 254 codes
    N, K = len(codes), 512
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    wq = np.zeros((N, K), np.uint8)
    wq[:, 429] = codes
    s = np.ones(N, np.float32)
    x = np.zeros((M, K), np.float16)
    x[:, 429] = 1.0
    y = g.f8_forward(dev(x), dev(wq), dev(s)).cpu().numpy().astype(np.float32)
    want = o.e4m3fn_decode(codes).astype(np.float16).astype(np.float32)
    for r in range(M):
        np.testing.assert_array_equal(y[r], want)


def test_nonfinite_activation_stays_in_its_token(g):
    """An inf in one token's activations makes that token's outputs non-finite
    and leaves the other tokens exact (they share every A fragment with it)."""
    M, N, K = 13, 1152, 896
    x, w, b = gen(M, N, K, seed=53)
    wq, s = o.quantize(w)
    ref = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    x2 = x.copy()
    x2[9, 100] = np.inf
    y = g.f8_forward(dev(x2), dev(wq), dev(s), dev(b))
    assert not torch.isfinite(y[9]).all()
    keep = [i for i in range(M) if i != 9]
    assert torch.equal(y[keep], ref[keep])


def test_chained_calls_read_the_previous_output(g):
    """Each call consumes the previous call's output, issued back to back: the
    next kernel starts and fetches its weights while the previous one still
    runs, and reads its activations only after that one has completed.  The
    results equal the same chain with a device synchronisation between calls,
    bit for bit (1, 8 and 16 tokens; 17 runs the decode kernel)."""
    torch.manual_seed(7)
    shapes = [(896, 896), (4864, 896), (896, 4864), (1152, 896), (9728, 1152), (896, 9728)]
    for M in (1, 8, 16, 17):
        ws = []
        for N, K in shapes:
            wq, s = g.quantize((torch.randn(N, K, device="cuda") * 0.02).half())
            ws.append((wq, s))
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
    M, N, K = 7, 9728, 896
    x, w, b = gen(M, N, K, seed=57)
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


@pytest.mark.parametrize("M", [1, 16])
def test_deterministic_bitwise(g, M):
    N, K = 4864, 896
    x, w, b = gen(M, N, K, seed=59)
    wq, s = o.quantize(w)
    xd, wqd, sd = dev(x), dev(wq), dev(s)
    a = g.f8_forward(xd, wqd, sd)
    for _ in range(3):
        assert torch.equal(g.f8_forward(xd, wqd, sd), a)



@pytest.mark.parametrize("M", [17, 24, 31, 32, 33, 40, 48, 57, 63, 64])
@pytest.mark.parametrize("N,K", [(1152, 896), (896, 896), (2048, 896)])
def test_warps_over_tokens(g, lib, M, N, K):
    """17..64 tokens: every warp owns an 8-token block (and, up to 32 tokens,
    half of the K blocks; the two halves are summed in order)."""
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=400 + M + N)


@pytest.mark.parametrize("M,N,K", [(32, 9728, 896), (64, 9728, 896), (64, 4864, 896)])
def test_big_shapes_above_16_tokens_go_to_the_tensor_core_kernel(g, lib, M, N, K):
    """More than ~768 legacy MMAs per CTA: the split + tcgen05 decode kernel."""
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 2
    check(g, M, N, K, seed=500 + M)


@pytest.mark.parametrize("M,N,K", [(20, 7, 256), (37, 1000, 512), (64, 17, 1024), (50, 2049, 640),
                                   (33, 896, 2048)])
def test_warps_over_tokens_ragged(g, lib, M, N, K):
    assert lib.ddq_w8a16_gemm_kernel_count(M, N, K) == 1
    check(g, M, N, K, seed=M * 11 + N)


def test_warps_over_tokens_chained_and_replayed(g):
    """Chained calls of 24 and 64 tokens issued back to back equal the same
    chain with synchronisations, and a replayed graph equals the eager call."""
    torch.manual_seed(9)
    shapes = [(896, 896), (1152, 896), (9728, 1152), (896, 9728)]
    for M in (24, 64):
        ws = [g.quantize((torch.randn(N, K, device="cuda") * 0.02).half()) for N, K in shapes]
        x = torch.randn(M, 896, device="cuda").half()
        ys = [x]
        for rep in range(2):
            for wq, s in ws:
                ys.append(g.f8_forward(ys[-1], wq, s))
        torch.cuda.synchronize()
        ref = [x]
        for rep in range(2):
            for wq, s in ws:
                ref.append(g.f8_forward(ref[-1], wq, s))
                torch.cuda.synchronize()
        for i, (a, r) in enumerate(zip(ys[1:], ref[1:])):
            assert torch.equal(a, r), (M, i)
    M, N, K = 48, 2048, 896
    x, w, b = gen(M, N, K, seed=71)
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


def test_warps_over_tokens_nonfinite_and_bias(g):
    M, N, K = 40, 1152, 896
    x, w, b = gen(M, N, K, seed=73)
    wq, s = o.quantize(w)
    for bb in (b.astype(np.float16), b):
        y = g.f8_forward(dev(x), dev(wq), dev(s), dev(bb))
        assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bb)) <= TIGHT
    ref = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    x2 = x.copy()
    x2[35, 10] = np.inf
    y = g.f8_forward(dev(x2), dev(wq), dev(s), dev(b))
    assert not torch.isfinite(y[35]).all()
    keep = [i for i in range(M) if i != 35]
    assert torch.equal(y[keep], ref[keep])
