"""CPU tests: the oracle pinned against torch's float8_e4m3fn cast (the byte
spec the reference names, gemm_FP8_d.cu:20-23) and against the reference's
own encoder where they are meant to agree."""
import numpy as np
import pytest
import torch

from oracle import w8a16 as o


def torch_cast(v: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(torch.float8_e4m3fn).view(
        torch.uint8).numpy()


def test_encode_matches_torch_cast_on_every_fp16_value():
    h = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    np.testing.assert_array_equal(o.e4m3fn_encode(h), torch_cast(h))


def test_encode_matches_torch_cast_on_every_rounding_boundary():
    # every positive e4m3 code value, the midpoints between neighbours, and
    # one fp32 ulp either side of each midpoint (ties and near-ties)
    vals = np.sort(o.E4M3_DECODE[:0x7F].astype(np.float64))
    mids = (vals[:-1] + vals[1:]) / 2
    pts = np.concatenate([vals, mids, [464.0, 480.0, 448.0 * 1.0001]]).astype(np.float32)
    up = np.nextafter(pts, np.float32(np.inf))
    dn = np.nextafter(pts, np.float32(-np.inf))
    allv = np.concatenate([pts, up, dn])
    allv = np.concatenate([allv, -allv])
    np.testing.assert_array_equal(o.e4m3fn_encode(allv), torch_cast(allv))


def test_encode_matches_torch_cast_on_random_fp32():
    rng = np.random.default_rng(1)
    v = np.concatenate([rng.normal(0, s, 200_000) for s in (1e-3, 0.02, 1.0, 50.0, 300.0)])
    v = v.astype(np.float32)
    np.testing.assert_array_equal(o.e4m3fn_encode(v), torch_cast(v))


def test_special_values():
    v = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 448.0, 449.0, 464.0, 465.0, 2.0 ** -9,
                  2.0 ** -10, 1.5 * 2.0 ** -10], np.float32)
    got = o.e4m3fn_encode(v)
    np.testing.assert_array_equal(got, torch_cast(v))
    assert got[0] == 0x00 and got[1] == 0x80
    assert got[5] == 0x7E and got[7] == 0x7E and got[8] == 0x7F


def test_decode_table_matches_torch():
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e4m3fn).float().numpy()
    got = o.E4M3_DECODE
    nan = np.isnan(ref)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan], ref[~nan])
    # bias 7, max 0x7E = 448, subnormal step 2^-9 (gemm_FP8_d.cu:20-23)
    assert got[0x7E] == 448.0 and got[0x01] == 2.0 ** -9 and got[0x38] == 1.0


def test_reference_encoder_divergences_are_the_documented_ones():
    # (1) ties round half-up in the reference (gemm_FP8_d.cu:56), to even in torch
    assert o.ref_fp32_to_e4m3(np.float32(1.0625)) == 0x39
    assert o.e4m3fn_encode(np.float32(1.0625)) == 0x38
    # (2) values in [~0.01465, 2^-6) clamp to 0x07 instead of reaching 0x08 (:50-53)
    assert o.ref_fp32_to_e4m3(np.float32(0.0155)) == 0x07
    assert o.e4m3fn_encode(np.float32(0.0155)) == 0x08
    # (3) saturation to 448 instead of NaN for |v| >= 464 (:43, :59-60)
    assert o.ref_fp32_to_e4m3(np.float32(500.0)) == 0x7E
    assert o.e4m3fn_encode(np.float32(500.0)) == 0x7F
    # elsewhere they agree: every non-tie value in the normal range
    rng = np.random.default_rng(2)
    v = rng.uniform(2.0 ** -6, 440.0, 20000).astype(np.float32)
    np.testing.assert_array_equal(o.ref_fp32_to_e4m3(v), o.e4m3fn_encode(v))


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_quantize_matches_baseline_formula(dtype):
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (64, 896)).astype(dtype)
    w[5] = 0  # all-zero row -> scale 1 (gemm_FP8_d.cu:78)
    wq, s = o.quantize(w)
    wt = torch.from_numpy(w.astype(np.float32))
    amax = wt.abs().amax(1)
    st = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    qt = (wt / st[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(s, st.numpy())
    np.testing.assert_array_equal(wq, qt)
    assert s[5] == 1.0 and not wq[5].any()
    # the row maximum lands exactly on 448
    assert (np.abs(o.e4m3fn_decode(wq)).max(axis=1)[np.arange(64) != 5] == 448.0).all()


def test_f8_forward_matches_torch_fp32_semantics():
    rng = np.random.default_rng(4)
    x = rng.normal(0, 1, (16, 896)).astype(np.float16)
    w = rng.normal(0, 0.02, (256, 896)).astype(np.float32)
    b = rng.normal(0, 0.02, 256).astype(np.float32)
    wq, s = o.quantize(w)
    y = o.f8_forward(x, wq, s, b)
    assert y.dtype == np.float16 and y.shape == (16, 256)
    wd = torch.from_numpy(wq).view(torch.float8_e4m3fn).float() * torch.from_numpy(s)[:, None]
    yt = (torch.from_numpy(x).float() @ wd.T + torch.from_numpy(b)).half().numpy()
    assert o.normwise_rel_err(y, yt) < 1e-3
    # the quantised GEMM is within the north_star tolerance of the unquantised one
    y32 = (x.astype(np.float64) @ w.astype(np.float64).T + b).astype(np.float16)
    assert o.normwise_rel_err(y, y32) < 1e-1


def test_f8_forward_leading_dims_and_empty():
    rng = np.random.default_rng(5)
    wq, s = o.quantize(rng.normal(0, 0.02, (32, 64)).astype(np.float32))
    x = rng.normal(0, 1, (2, 3, 64)).astype(np.float16)
    assert o.f8_forward(x, wq, s).shape == (2, 3, 32)
    assert o.f8_forward(np.zeros((0, 64), np.float16), wq, s).shape == (0, 32)


def test_argmax_ties_go_to_lowest_index():
    lg = np.array([[1, 3, 3, 2], [5, 5, 5, 5], [-np.inf, -1, -1, -np.inf],
                   [np.nan, -np.inf, -np.inf, -np.inf], [np.nan, 2, np.nan, 2]], np.float16)
    # NaN and -inf never win; nothing above -FLT_MAX -> 0 (sampler_d.cu:16-24)
    np.testing.assert_array_equal(o.argmax_f16(lg), [1, 0, 1, 0, 1])


def test_lm_head_argmax_equals_gemm_then_sampler():
    rng = np.random.default_rng(6)
    x = rng.normal(0, 1, (4, 128)).astype(np.float16)
    wq, s = o.quantize(rng.normal(0, 0.02, (1000, 128)).astype(np.float32))
    ids, vals = o.lm_head_argmax(x, wq, s)
    y = o.f8_forward(x, wq, s)
    np.testing.assert_array_equal(ids, o.argmax_f16(y))
    np.testing.assert_array_equal(vals, y[np.arange(4), ids])
