"""GPU parity tests of the W8A16 operators against the CPU oracle.

Quantization is byte-exact; the GEMM is held to the north_star tolerance
(normwise relative error <= 1e-2 against the fp32 semantics; in practice the
fp16 output rounding, ~5e-4, dominates)."""
import numpy as np
import pytest
import torch

from oracle import w8a16 as o

pytestmark = pytest.mark.gpu

TOL = 1e-2          # north_star: max relative error vs the fp32 result
TIGHT = 3e-3        # what the kernels actually achieve (fp16 output rounding + fp32 sums)

PROJ_SHAPES = [(896, 896), (128, 896), (1152, 896), (896, 4864), (9728, 896), (4864, 896)]


def gen(M, N, K, seed=0, wdtype=np.float32):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    w = rng.normal(0, 0.02, (N, K)).astype(wdtype)
    b = rng.normal(0, 0.02, N).astype(np.float32)
    return x, w, b


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def g(cuda_device):
    from ddq_b200 import gemm_fp8
    return gemm_fp8


@pytest.mark.parametrize("N,K", PROJ_SHAPES + [(136, 48), (3, 40), (7, 1)])
@pytest.mark.parametrize("wdtype", [np.float32, np.float16])
def test_quantize_is_byte_exact(g, N, K, wdtype):
    _, w, _ = gen(1, N, K, seed=N + K, wdtype=wdtype)
    w[min(2, N - 1)] = 0  # an all-zero row
    wq, s = g.quantize(dev(w))
    wq_ref, s_ref = o.quantize(w)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(wq.cpu().numpy(), wq_ref)


def test_quantize_crafted_values(g):
    # ties, subnormal/normal boundary, signed zeros, saturation point
    base = np.array([1.0625, 0.0146, 0.0155, 2.0 ** -10, 1.5 * 2.0 ** -10, -0.0, 0.0,
                     3.0, -1.0625, 448.0 / 1.0001], np.float32)
    w = np.tile(np.concatenate([base, [448.0]]).astype(np.float32), (4, 2))
    wq, s = g.quantize(dev(w))
    wq_ref, s_ref = o.quantize(w)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(wq.cpu().numpy(), wq_ref)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 16, 17, 32, 64])
@pytest.mark.parametrize("N,K", PROJ_SHAPES)
def test_f8_forward_decode_shapes(g, M, N, K):
    x, w, b = gen(M, N, K, seed=M * 7 + N)
    wq, s = o.quantize(w)
    bias = b if N in (896, 128, 1152) and K == 896 else None
    y = g.f8_forward(dev(x), dev(wq), dev(s), dev(bias) if bias is not None else None)
    assert y.dtype == torch.float16 and tuple(y.shape) == (M, N)
    y_ref = o.f8_forward(x, wq, s, bias)
    err = o.normwise_rel_err(y.cpu().numpy(), y_ref)
    assert err <= TIGHT, err


@pytest.mark.parametrize("M", [100, 129, 512, 1000])
@pytest.mark.parametrize("N,K", [(896, 896), (1152, 896), (896, 4864), (9728, 896), (1000, 136)])
def test_f8_forward_larger_m(g, M, N, K):
    x, w, b = gen(M, N, K, seed=M + N + K)
    wq, s = o.quantize(w)
    y = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b))
    assert err <= TIGHT, err


@pytest.mark.parametrize("M,N,K", [(3, 136, 48), (5, 7, 40), (2, 33, 1), (9, 100, 24)])
def test_f8_forward_ragged_and_generic_path(g, M, N, K):
    x, w, b = gen(M, N, K, seed=11)
    wq, s = o.quantize(w)
    y = g.f8_forward(dev(x), dev(wq), dev(s), dev(b))
    err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b))
    assert err <= TIGHT, err


def test_unaligned_activation_pointer_uses_generic_path(g):
    x, w, b = gen(5, 256, 896, seed=12)
    wq, s = o.quantize(w)
    xbig = torch.zeros(5 * 896 + 1, dtype=torch.float16, device="cuda")
    xbig[1:] = dev(x).reshape(-1)
    xv = xbig[1:].view(5, 896)  # 2-byte offset: not 16-byte aligned
    y = g.f8_forward(xv, dev(wq), dev(s), dev(b))
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b)) <= TIGHT


@pytest.mark.parametrize("M", [8, 700])
@pytest.mark.parametrize("bias_kind", ["none", "empty", "f16", "f32"])
def test_bias_variants(g, bias_kind, M):
    x, w, b = gen(M, 896, 896, seed=13)
    wq, s = o.quantize(w)
    if bias_kind == "none":
        bt, bref = None, None
    elif bias_kind == "empty":
        bt, bref = torch.empty(0, device="cuda", dtype=torch.float16), None
    elif bias_kind == "f16":
        bt, bref = dev(b.astype(np.float16)), b.astype(np.float16)
    else:
        bt, bref = dev(b), b
    y = g.f8_forward(dev(x), dev(wq), dev(s), bt)
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, bref)) <= TIGHT


def test_leading_dims_and_empty_batch(g):
    x, w, b = gen(6, 128, 896, seed=14)
    wq, s = o.quantize(w)
    x3 = dev(x).reshape(2, 3, 896)
    y = g.f8_forward(x3, dev(wq), dev(s), dev(b))
    assert tuple(y.shape) == (2, 3, 128)
    assert o.normwise_rel_err(y.reshape(6, 128).cpu().numpy(), o.f8_forward(x, wq, s, b)) <= TIGHT
    y0 = g.f8_forward(torch.empty(0, 896, dtype=torch.float16, device="cuda"), dev(wq), dev(s))
    assert tuple(y0.shape) == (0, 128)


def test_forward_quantizes_then_multiplies(g):
    x, w, b = gen(4, 896, 896, seed=15)
    y = g.forward(dev(x), dev(w.astype(np.float16)), dev(b.astype(np.float16)))
    y_ref = o.forward(x, w.astype(np.float16), b.astype(np.float16))
    assert o.normwise_rel_err(y.cpu().numpy(), y_ref) <= TIGHT


def test_error_messages_match_reference(g):
    wq = torch.zeros(8, 16, dtype=torch.uint8, device="cuda")
    s = torch.ones(8, dtype=torch.float32, device="cuda")
    xh = torch.zeros(2, 16, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="fp16 x required"):
        g.f8_forward(xh.float(), wq, s)
    with pytest.raises(RuntimeError, match="wq must be uint8"):
        g.f8_forward(xh, wq.half(), s)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        g.f8_forward(xh, wq, s[:4])
    with pytest.raises(RuntimeError, match="inner dim mismatch"):
        g.f8_forward(torch.zeros(2, 8, dtype=torch.float16, device="cuda"), wq, s)
    with pytest.raises(RuntimeError, match="bias length mismatch"):
        g.f8_forward(xh, wq, s, torch.zeros(3, device="cuda", dtype=torch.float16))
    with pytest.raises(RuntimeError, match="CUDA tensors required"):
        g.f8_forward(xh.cpu(), wq, s)
    with pytest.raises(RuntimeError, match="weight must be"):
        g.quantize(torch.zeros(4, device="cuda", dtype=torch.float16))
    with pytest.raises(RuntimeError, match="fp16 CUDA weight required"):
        g.quantize(torch.zeros(4, 4, dtype=torch.float16))


@pytest.mark.parametrize("M", [1, 16, 64, 512])
def test_deterministic_bitwise(g, M):
    x, w, b = gen(M, 1152, 896, seed=16)
    wq, s = o.quantize(w)
    args = (dev(x), dev(wq), dev(s), dev(b))
    y1 = g.f8_forward(*args)
    y2 = g.f8_forward(*args)
    assert torch.equal(y1, y2)


def test_runs_on_callers_stream(g):
    x, w, b = gen(16, 896, 896, seed=17)
    wq, s = o.quantize(w)
    xs, wqs, ss, bs = dev(x), dev(wq), dev(s), dev(b)
    st = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        y = g.f8_forward(xs, wqs, ss, bs)
    st.synchronize()
    assert o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b)) <= TIGHT


@pytest.mark.parametrize("M", [1, 16, 64, 300])
def test_e4m3_subnormal_weights_contribute(g, M):
    """Rows whose values (but the row maximum) quantize to e4m3 subnormals: the
    whole output comes from subnormal codes (the tensor-core operand then holds
    fp16 subnormals), so a flushed subnormal would show as a zero output."""
    N, K = 256, 896
    rng = np.random.default_rng(21)
    w = (rng.uniform(0.5, 1.5, (N, K)) * 1e-5 * rng.choice([-1, 1], (N, K))).astype(np.float32)
    w[:, 0] = 1.0                                    # row max -> scale 1/448
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    x[:, 0] = 0                                      # the max column contributes nothing
    wq, s = o.quantize(w)
    assert ((wq[:, 1:] & 0x78) == 0).all()           # every other code is subnormal
    y = g.f8_forward(dev(x), dev(wq), dev(s))
    y_ref = o.f8_forward(x, wq, s)
    assert np.abs(y_ref.astype(np.float32)).max() > 1e-4
    assert o.normwise_rel_err(y.cpu().numpy(), y_ref) <= TIGHT


def test_e4m3_all_codes_decode_exactly(g):
    """Every finite e4m3 code (both signs) times a one-hot activation row."""
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)   # 254 codes
    N, K = len(codes), 16
    wq = np.zeros((N, K), np.uint8)
    wq[:, 3] = codes
    s = np.ones(N, np.float32)
    x = np.zeros((4, K), np.float16)
    x[:, 3] = 1.0
    y = g.f8_forward(dev(x), dev(wq), dev(s)).cpu().numpy().astype(np.float32)
    want = o.e4m3fn_decode(codes).astype(np.float16).astype(np.float32)
    for r in range(4):
        np.testing.assert_array_equal(y[r], want)


def test_decode_calls_of_many_shapes_share_one_workspace(g):
    """Decode-shape calls of different shapes, twice over, through one caller
    workspace sized for the largest: each matches the oracle."""
    from ddq_b200 import _lib
    lib = _lib.load()
    shapes = [(16, 1152, 896), (64, 896, 4864), (1, 9728, 896), (37, 256, 48), (64, 896, 896)]
    need = max(lib.ddq_w8a16_gemm_workspace_size(M, N, K) for M, N, K in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for i, (M, N, K) in enumerate(shapes * 2):
        x, w, b = gen(M, N, K, seed=100 + i)
        wq, s = o.quantize(w)
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        xd, wqd, sd, bd = dev(x), dev(wq), dev(s), dev(b)
        st = lib.ddq_w8a16_gemm(xd.data_ptr(), wqd.data_ptr(), sd.data_ptr(), bd.data_ptr(),
                                _lib.DTYPE_F32, y.data_ptr(), M, N, K, ws.data_ptr(), need, stream)
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        err = o.normwise_rel_err(y.cpu().numpy(), o.f8_forward(x, wq, s, b))
        assert err <= TIGHT, (M, N, K, err)


def test_concurrent_streams_get_their_own_workspace(cuda_device):
    """Decode GEMMs issued on two streams at once (each with its own activation
    planes in a workspace) must not share scratch: both results equal the
    single-stream ones."""
    from ddq_b200 import gemm_fp8
    g = torch.Generator(device="cuda").manual_seed(21)
    wq, s = gemm_fp8.quantize(torch.randn(4864, 896, generator=g, device="cuda") * 0.02)
    xs = [torch.randn(16, 896, generator=g, device="cuda").half() for _ in range(2)]
    ref = [gemm_fp8.f8_forward(x, wq, s) for x in xs]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [[], []]
    torch.cuda.synchronize()
    for _ in range(20):
        for i in range(2):
            with torch.cuda.stream(streams[i]):
                outs[i].append(gemm_fp8.f8_forward(xs[i], wq, s))
    torch.cuda.synchronize()
    for i in range(2):
        for y in outs[i]:
            assert torch.equal(y, ref[i])


def test_prefill_and_decode_calls_chained_on_one_workspace(cuda_device):
    """Prefill-shape calls alternate the two fp16 buffers of a shared workspace
    and expand their weight before the previous kernel has finished; decode-
    shape calls keep their planes at the start of the same workspace.  Issued
    back to back in a mixed order with no synchronisation between them, every
    result equals the same call made alone."""
    from ddq_b200 import _lib, gemm_fp8
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(31)
    shapes = [(512, 1152, 896), (256, 4864, 896), (16, 896, 896), (512, 896, 4864),
              (1024, 896, 896), (8, 1152, 896), (64, 896, 4864), (384, 9728, 896),
              (256, 1152, 896), (512, 896, 896)]
    calls = []
    for M, N, K in shapes:
        wq, s = gemm_fp8.quantize(torch.randn(N, K, generator=g, device="cuda") * 0.02)
        x = torch.randn(M, K, generator=g, device="cuda").half()
        calls.append((x, wq, s, M, N, K))
    stream = torch.cuda.current_stream().cuda_stream

    def run(x, wq, s, M, N, K, ws, nbytes):
        y = torch.empty(M, N, dtype=torch.float16, device="cuda")
        st = lib.ddq_w8a16_gemm(x.data_ptr(), wq.data_ptr(), s.data_ptr(), None, _lib.DTYPE_NONE,
                                y.data_ptr(), M, N, K, ws.data_ptr() if ws is not None else None,
                                nbytes, stream)
        assert st == 0, _lib.status_string(st)
        return y

    ref = []
    for c in calls:  # each alone, with its own workspace, synchronised
        n = lib.ddq_w8a16_gemm_workspace_size(c[3], c[4], c[5])
        ws = torch.zeros(max(n, 256), dtype=torch.uint8, device="cuda")
        ref.append(run(*c, ws, n))
        torch.cuda.synchronize()
    need = max(lib.ddq_w8a16_gemm_workspace_size(c[3], c[4], c[5]) for c in calls)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for rep in range(3):
        outs = [run(*c, ws, need) for c in calls]   # back to back, one stream
        torch.cuda.synchronize()
        for (M, N, K), y, r in zip(shapes, outs, ref):
            assert torch.equal(y, r), (rep, M, N, K)


def _pf_case(g, M, N, K):
    from ddq_b200 import gemm_fp8
    wq, s = gemm_fp8.quantize(torch.randn(N, K, generator=g, device="cuda") * 0.02)
    return torch.randn(M, K, generator=g, device="cuda").half(), wq, s, M, N, K


def _run_ws(c, ws, nbytes):
    from ddq_b200 import _lib
    lib = _lib.load()
    x, wq, s, M, N, K = c
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    st = lib.ddq_w8a16_gemm(x.data_ptr(), wq.data_ptr(), s.data_ptr(), None, _lib.DTYPE_NONE,
                            y.data_ptr(), M, N, K, ws.data_ptr(), nbytes,
                            torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.status_string(st)
    return y


def _alone(c):
    from ddq_b200 import _lib
    lib = _lib.load()
    n = lib.ddq_w8a16_gemm_workspace_size(c[3], c[4], c[5])
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device="cuda")
    y = _run_ws(c, ws, n)
    torch.cuda.synchronize()
    return y


def test_prefill_calls_replayed_in_a_graph_on_one_workspace(cuda_device):
    """Three prefill calls (an odd number) and a decode call on one workspace,
    captured in a CUDA graph and replayed three times back to back, with an
    eager prefill call on the same workspace between two replays: every
    result equals the same call made alone.  (A call recorded in a graph never
    expands its weight ahead of the previous kernel, and a workspace once used
    in a graph is never expanded into early by eager calls either: the host
    cannot see what a replay runs between them.)"""
    from ddq_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(41)
    cap = [_pf_case(g, 512, 1152, 896), _pf_case(g, 16, 896, 896), _pf_case(g, 512, 896, 4864),
           _pf_case(g, 384, 9728, 896)]
    eager = _pf_case(g, 512, 896, 896)
    refs = [_alone(c) for c in cap]
    ref_e = _alone(eager)
    need = max(lib.ddq_w8a16_gemm_workspace_size(c[3], c[4], c[5]) for c in cap + [eager])
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in cap:                       # warm-up outside the capture
            _run_ws(c, ws, need)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        outs = [_run_ws(c, ws, need) for c in cap]
    got = []
    for rep in range(3):
        graph.replay()
        got.append([o.clone() for o in outs])
        if rep == 1:
            got.append([_run_ws(eager, ws, need)])
    torch.cuda.synchronize()
    for rep, ys in enumerate(got):
        want = [ref_e] if len(ys) == 1 else refs
        for y, r in zip(ys, want):
            assert torch.equal(y, r), rep
    del graph


def test_prefill_workspace_freed_and_reallocated_at_same_address(cuda_device):
    """A workspace freed after a prefill call and re-allocated at the same
    address (the caching allocator's stream-ordered reuse) serves the next
    prefill calls correctly, though the host-side history of the address says
    the previous call on it was a prefill call."""
    from ddq_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(43)
    calls = [_pf_case(g, 512, 1152, 896), _pf_case(g, 512, 896, 4864), _pf_case(g, 256, 4864, 896)]
    refs = [_alone(c) for c in calls]
    need = max(lib.ddq_w8a16_gemm_workspace_size(c[3], c[4], c[5]) for c in calls)
    torch.cuda.synchronize()
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    addr = ws.data_ptr()
    outs = [_run_ws(calls[0], ws, need)]
    del ws
    ws2 = torch.empty(need, dtype=torch.uint8, device="cuda")
    if ws2.data_ptr() != addr:
        pytest.skip("the allocator did not reuse the address")
    outs += [_run_ws(calls[1], ws2, need), _run_ws(calls[2], ws2, need)]
    torch.cuda.synchronize()
    for y, r in zip(outs, refs):
        assert torch.equal(y, r)
