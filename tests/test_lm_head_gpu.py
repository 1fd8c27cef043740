"""GPU tests of the greedy pick: the sampler mirror and the fused lm_head
argmax (single shard, emulated vocab shards, full 151936-row vocabulary)."""
import numpy as np
import pytest
import torch

from oracle import w8a16 as o

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN = 151936, 896


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def mods(cuda_device):
    from ddq_b200 import gemm_fp8, lm_head, sampler
    return gemm_fp8, lm_head, sampler


def test_sampler_matches_oracle_with_ties_nan_inf(mods):
    _, _, sampler = mods
    rng = np.random.default_rng(0)
    B, V = 6, 151936
    lg = rng.normal(0, 3, (B, V)).astype(np.float16)
    lg[1, 100] = lg[1, 50] = lg[1, 70000] = 60000   # three-way tie -> 50
    lg[2, :] = 7.0                                  # all equal -> 0
    lg[3, :] = -np.inf
    lg[3, 123] = -65504
    lg[4, 5] = np.nan                               # NaN never wins
    lg[4, 9] = 65504
    lg[5, :] = np.nan                               # all NaN -> 0 (sampler_d.cu:17)
    got = sampler.forward(dev(lg).reshape(B, 1, V))
    assert tuple(got.shape) == (B, 1) and got.dtype == torch.int64
    want = [int(o.argmax_f16(lg[0])), 50, 0, 123, 9, 0]
    assert got.reshape(-1).tolist() == want


@pytest.mark.parametrize("V", [1, 7, 8, 1001, 151936])
def test_sampler_ragged_vocab(mods, V):
    _, _, sampler = mods
    lg = np.random.default_rng(V).normal(0, 1, (3, V)).astype(np.float16)
    got = sampler.forward(dev(lg).reshape(3, 1, V)).reshape(-1).cpu().numpy()
    np.testing.assert_array_equal(got, o.argmax_f16(lg))


@pytest.mark.parametrize("M", [1, 3, 16, 64])
def test_fused_argmax_equals_gemm_then_sampler(mods, M):
    g, lm, _ = mods
    rng = np.random.default_rng(M)
    N = 20000
    x = rng.normal(0, 1, (M, HIDDEN)).astype(np.float16)
    wq, s = o.quantize(rng.normal(0, 0.02, (N, HIDDEN)).astype(np.float32))
    ids, packed = lm.lm_head_argmax(dev(x), dev(wq), dev(s))
    logits = g.f8_forward(dev(x), dev(wq), dev(s)).float().cpu().numpy()
    # the fused pick is the sampler's pick over f8_forward's fp16 logits, except
    # where their top two are within 2 fp16 ulps (the fused kernel and the GEMM
    # may sum in different orders); there the pick's logit is within 2 ulps
    top = np.sort(logits, axis=1)[:, -2:]
    ulp = np.spacing(np.abs(top[:, 1]).astype(np.float16)).astype(np.float32)
    clear = (top[:, 1] - top[:, 0]) > 2 * ulp
    got = ids.cpu().numpy()
    np.testing.assert_array_equal(got[clear], o.argmax_f16(logits)[clear])
    chosen = logits[np.arange(M), got]
    assert ((top[:, 1] - chosen) <= 2 * ulp).all()
    # and the oracle's pick wherever the oracle's top-2 gap exceeds 2 fp16 ulps
    y_ref = o.f8_forward(x, wq, s).astype(np.float32)
    top = np.sort(y_ref, axis=1)[:, -2:]
    ulp = np.spacing(np.abs(top[:, 1]).astype(np.float16)).astype(np.float32)
    clear = (top[:, 1] - top[:, 0]) > 2 * ulp
    np.testing.assert_array_equal(ids.cpu().numpy()[clear], o.argmax_f16(y_ref)[clear])
    assert clear.mean() > 0.8


def test_fused_argmax_tie_breaks_to_lowest_index(mods):
    _, lm, _ = mods
    rng = np.random.default_rng(3)
    N = 5000
    w = rng.normal(0, 0.02, (N, HIDDEN)).astype(np.float32)
    hot = rng.normal(0, 1, HIDDEN).astype(np.float32)
    for r in (4321, 77, 2500):   # identical rows -> bit-identical logits
        w[r] = hot
    x = (hot / np.abs(hot).max() * 4).astype(np.float16)[None, :]
    wq, s = o.quantize(w)
    ids, _ = lm.lm_head_argmax(dev(x), dev(wq), dev(s))
    assert ids.item() == 77


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_vocab_shards_combine_to_the_unsharded_pick(mods, shards):
    _, lm, _ = mods
    rng = np.random.default_rng(shards)
    M, N = 16, 30000
    x = dev(rng.normal(0, 1, (M, HIDDEN)).astype(np.float16))
    wq, s = o.quantize(rng.normal(0, 0.02, (N, HIDDEN)).astype(np.float32))
    wq, s = dev(wq), dev(s)
    ids_full, packed_full = lm.lm_head_argmax(x, wq, s)
    parts = []
    for r in range(shards):
        lo, hi = lm.shard_range(N, r, shards)
        parts.append(lm.lm_head_argmax(x, wq[lo:hi], s[lo:hi], vocab_offset=lo)[1])
    combined = torch.stack(parts).max(dim=0).values
    assert torch.equal(combined, packed_full)
    assert torch.equal(lm.unpack(combined), ids_full)


@pytest.mark.parametrize("M", [1, 16, 64])
def test_full_vocab_lm_head(mods, M):
    """Config 4 at full size: 896 -> 151936, against the fp32 semantics on the GPU
    (dequantised weights in torch fp32; checked against the numpy oracle on a row slice)."""
    _, lm, _ = mods
    gen = torch.Generator().manual_seed(100 + M)
    x = torch.randn(M, HIDDEN, generator=gen).half()
    w = (torch.randn(VOCAB, HIDDEN, generator=gen) * 0.02)
    wq_np, s_np = o.quantize(w[:2048].numpy())
    from ddq_b200 import gemm_fp8
    wq, s = gemm_fp8.quantize(w.cuda())
    np.testing.assert_array_equal(wq[:2048].cpu().numpy(), wq_np)
    ids, _ = lm.lm_head_argmax(x.cuda(), wq, s)
    lut = torch.from_numpy(o.E4M3_DECODE).cuda()
    wd = lut[wq.long()] * s[:, None]
    ref = (x.cuda().float() @ wd.T).half().float()
    top2 = ref.topk(2, dim=1).values
    ulp = torch.from_numpy(np.spacing(np.abs(top2[:, 0].cpu().numpy()).astype(np.float16)).astype(
        np.float32)).cuda()
    clear = (top2[:, 0] - top2[:, 1]) > 2 * ulp
    ref_ids = ref.argmax(dim=1)
    assert torch.equal(ids[clear], ref_ids[clear])
    # wherever the pick differs, the chosen logit is within 2 ulps of the max
    chosen = ref.gather(1, ids[:, None]).squeeze(1)
    assert ((top2[:, 0] - chosen) <= 2 * ulp).all()


@pytest.mark.parametrize("M,N", [(20, 1000), (64, 18992), (100, 20000), (130, 5000)])
def test_decode_path_zeroes_packed_and_writes_ids(mods, M, N):
    """Beyond the streaming kernel's token counts the lm_head runs the split
    pre-pass, which zeroes packed, and the decode GEMM, whose last CTA writes
    ids from packed and clears its arrival counter.  A packed buffer full of
    stale maxima must not leak into the result; ids decode packed; and a call
    repeated after one on other activations gives the same words (the counter
    was left at zero).  Shapes: split-K clusters (N = 1000), one 64-token
    chunk, two chunks (100, 130 tokens)."""
    import ctypes
    from ddq_b200 import _lib
    g, lm, _ = mods
    L = _lib.load()
    rng = np.random.default_rng(M + N)
    x1 = dev(rng.normal(0, 1, (M, HIDDEN)).astype(np.float16))
    x2 = dev((rng.normal(0, 1, (M, HIDDEN)) * 3).astype(np.float16))
    wq, s = o.quantize(rng.normal(0, 0.02, (N, HIDDEN)).astype(np.float32))
    wq, s = dev(wq), dev(s)

    def call(x):
        packed = torch.full((M,), -1, dtype=torch.int64, device="cuda")  # all bits set
        ids = torch.full((M,), -7, dtype=torch.int64, device="cuda")
        nws = L.ddq_lm_head_argmax_workspace_size(M, N, HIDDEN)
        ws = lm.lm_workspace(x.device, nws)
        st = L.ddq_lm_head_argmax(x.data_ptr(), wq.data_ptr(), s.data_ptr(), M, N, HIDDEN, 0,
                                  packed.data_ptr(), ids.data_ptr(), ws.data_ptr(), ws.numel(),
                                  torch.cuda.current_stream().cuda_stream)
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        return ids, packed

    ids1, p1 = call(x1)
    ids2, p2 = call(x2)
    ids1b, p1b = call(x1)
    code = ctypes.c_int(-1)
    assert L.ddq_device_error(ctypes.byref(code), torch.cuda.current_stream().cuda_stream) == 0
    assert code.value == 0
    assert torch.equal(p1, p1b) and torch.equal(ids1, ids1b)
    for ids, p in ((ids1, p1), (ids2, p2)):
        assert torch.equal(ids, lm.unpack(p))
        assert (p != -1).all()
    # the picks: the sampler's over f8_forward's logits where the top two are clear
    for x, ids in ((x1, ids1), (x2, ids2)):
        logits = g.f8_forward(x, wq, s).float().cpu().numpy()
        top = np.sort(logits, axis=1)[:, -2:]
        ulp = np.spacing(np.abs(top[:, 1]).astype(np.float16)).astype(np.float32)
        clear = (top[:, 1] - top[:, 0]) > 2 * ulp
        np.testing.assert_array_equal(ids.cpu().numpy()[clear], o.argmax_f16(logits)[clear])
        assert clear.mean() > 0.8
