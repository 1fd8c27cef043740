"""CPU oracle for the W8A16 projection-GEMM path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker or as the timed
CPU baseline.  The product path (``ddq_b200``) never calls it: when the CUDA
library is missing, the product raises instead of falling back here.

What it restates (file:line refer to the reference project, hdahroug/ddq):

* ``quantize``     - ``gemm_FP8_d.cu:66-86`` (per-row absmax, scale = absmax/448,
  scale = 1 for an all-zero row, encode every element of the row) with the
  rounding of torch's ``float8_e4m3fn`` cast, which the reference names as its
  byte-level spec (``gemm_FP8_d.cu:20-23``, ``README.md:119-131``).
* ``e4m3fn_encode`` / ``e4m3fn_decode`` - the e4m3fn format of
  ``gemm_FP8_d.cu:28-62`` (bias 7, 3 mantissa bits, max 0x7E = 448, subnormal
  step 2^-9), round-to-nearest-even as torch does.
* ``ref_fp32_to_e4m3`` - the reference's own encoder, bit for bit
  (``gemm_FP8_d.cu:39-62``), kept to measure where it departs from the torch
  cast (ties round half-up, the [0.01465, 2^-6) boundary clamp, saturation).
* ``f8_forward``   - ``gemm_FP8_d.cu:171-210`` with the BASELINE semantics:
  fp32 (here: float64, then rounded) matmul of the dequantised weight, plus
  bias, cast to fp16.  Unlike ``fp8_gemm_kernel`` (``gemm_FP8_d.cu:127-129``)
  the dequantised weight is not rounded to fp16 first.
* ``forward``      - ``gemm_FP8_d.cu:214-217``: quantize, then f8_forward.
* ``argmax_f16``   - ``sampler_d.cu:10-49``: greedy argmax over fp16 logits,
  ties to the lowest index.

Parity pins: the encoder is checked against torch's ``float8_e4m3fn`` cast over
every fp16 value and over every rounding boundary of the e4m3 grid
(``tests/test_oracle.py``); the whole oracle is checked against outputs of the
reference's own CUDA operators recorded in ``tests/golden/``.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
E4M3_NAN = 0x7F


# --------------------------------------------------------------------------- e4m3fn
def e4m3fn_encode(v) -> np.ndarray:
    """fp32 -> e4m3fn byte, round-to-nearest-even, torch's overflow rule.

    Follows the cast that ``gemm_FP8_d.cu:20-23`` names as its spec: values
    whose rounded magnitude exceeds 448 (|v| > 464) and NaN/Inf become the NaN
    code 0x7F (with the sign bit of v).
    """
    v = np.asarray(v, dtype=np.float32)
    sign = (np.signbit(v).astype(np.uint16) << 7)
    with np.errstate(invalid="ignore"):
        a = np.abs(v.astype(np.float64))
    finite = np.isfinite(a)
    a_f = np.where(finite, a, 0.0)
    # subnormal range |v| < 2^-6: code = RNE(|v| * 2^9), 0..8 (8 is the first normal)
    sub_code = np.rint(a_f * 512.0)
    # normal range: a = mant * 2^(e-1), mant in [1,2)
    m, e = np.frexp(np.where(a_f > 0, a_f, 1.0))
    E = e.astype(np.int64) - 1
    frac = (2.0 * m - 1.0) * 8.0           # exact for fp32 inputs
    q = np.rint(frac)                       # RNE; q == 8 carries into the exponent
    norm_code = (E + 7) * 8 + q
    code = np.where(a_f < 2.0 ** -6, sub_code, norm_code)
    code = np.where(finite & (code <= 0x7E), code, E4M3_NAN)
    return (code.astype(np.uint16) | sign).astype(np.uint8)


def _decode_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if (b & 0x7F) == 0x7F:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * m * 2.0 ** -9
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_DECODE = _decode_table()


def e4m3fn_decode(b) -> np.ndarray:
    """e4m3fn byte -> fp32 (``gemm_FP8_d.cu:30-37``; 0x7F/0xFF decode to NaN)."""
    return E4M3_DECODE[np.asarray(b, dtype=np.uint8)]


def ref_fp32_to_e4m3(v) -> np.ndarray:
    """The reference encoder ``fp32_to_e4m3`` (``gemm_FP8_d.cu:39-62``), bit for bit.

    Kept only to count where it departs from the torch cast; the build follows
    the torch cast.
    """
    v = np.asarray(v, dtype=np.float32).ravel()
    out = np.empty(v.shape, dtype=np.uint8)
    for i, x in enumerate(v.tolist()):
        xf = np.float32(x)
        av = np.float32(abs(xf))
        sign = 0x80 if xf < 0 else 0                                  # :41
        if av == 0:                                                   # :42
            out[i] = sign
            continue
        if av >= 448.0:                                               # :43
            out[i] = sign | 0x7E
            continue
        bits = int(np.array(av, dtype=np.float32).view(np.uint32))
        e8 = ((bits >> 23) & 0xFF) - 127                              # :46
        m23 = bits & 0x7FFFFF                                         # :47
        if e8 < -10:                                                  # :49
            out[i] = sign
            continue
        if e8 < -6:                                                   # :50-54
            sub = int(np.rint(np.float32(av * np.float32(512.0))))
            out[i] = sign | min(sub, 7)
            continue
        m3 = (m23 + 0x80000) >> 20                                    # :56 half-up
        if m3 == 8:                                                   # :57
            m3 = 0
            e8 += 1
        e = e8 + 7                                                    # :58
        if e > 15:                                                    # :59
            out[i] = sign | 0x7E
            continue
        if m3 > 6 and e == 15:                                        # :60
            m3 = 6
        out[i] = sign | m3 | (e << 3)                                 # :61
    return out.reshape(np.shape(np.asarray(v)))


# --------------------------------------------------------------------------- ops
def quantize(w) -> tuple[np.ndarray, np.ndarray]:
    """[N,K] fp16/fp32 weight -> (wq uint8 [N,K], scales fp32 [N]).

    Row structure of ``gemm_FP8_d.cu:66-86``: ``scale = absmax/448`` (1.0 for an
    all-zero row, :78), every element encoded as ``e4m3(w / scale)``.  The
    division is IEEE fp32 ``w / scale`` as in torch's ``(W / s).to(e4m3fn)``.
    """
    wf = np.asarray(w).astype(np.float32)
    if wf.ndim != 2:
        raise ValueError("weight must be [N,K]")
    amax = np.abs(wf).max(axis=1) if wf.shape[1] else np.zeros(wf.shape[0], np.float32)
    scales = np.where(amax > 0, amax / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)
    wq = e4m3fn_encode(wf / scales[:, None])
    return wq, scales


def dequantize(wq, scales) -> np.ndarray:
    """fp32 [N,K] = e4m3 value * per-row scale (exact in fp64, then rounded)."""
    return (e4m3fn_decode(wq).astype(np.float64) * np.asarray(scales, np.float64)[:, None])


def f8_forward(x, wq, scales, bias=None) -> np.ndarray:
    """y[..., N] = fp16(x[..., K] @ (dec(wq) * s)^T + bias)  (``gemm_FP8_d.cu:171-210``).

    x is fp16 (any leading dims), wq uint8 [N,K], scales fp32 [N], bias fp16 or
    fp32 [N] or None.  Accumulation is float64 (an upper bound on fp32
    accuracy); the result is rounded to fp32 and then to fp16.
    """
    x = np.asarray(x)
    wq = np.asarray(wq)
    N, K = wq.shape
    if x.shape[-1] != K:
        raise ValueError("inner dim mismatch")
    x2 = x.reshape(-1, K).astype(np.float64)
    acc = x2 @ dequantize(wq, scales).T
    if bias is not None:
        acc = acc + np.asarray(bias).astype(np.float64)[None, :]
    y = acc.astype(np.float32).astype(np.float16)
    return y.reshape(x.shape[:-1] + (N,))


def forward(x, w, bias=None) -> np.ndarray:
    """``gemm_FP8_d.cu:214-217``: quantize w, then f8_forward."""
    wq, s = quantize(w)
    return f8_forward(x, wq, s, bias)


def swiglu_f16(gate, up) -> np.ndarray:
    """``SwiGLU_d.cu:12-26``: z = fp16( g / (1 + exp(-g)) * u ) with g, u the fp16
    inputs taken to float (evaluated here in float64, then rounded)."""
    g = np.asarray(gate, np.float16).astype(np.float64)
    u = np.asarray(up, np.float16).astype(np.float64)
    with np.errstate(over="ignore"):
        z = g / (1.0 + np.exp(-g)) * u
    return z.astype(np.float32).astype(np.float16)


def f8_forward_swiglu(x, wq_gu, scales_gu, bias_gu=None) -> np.ndarray:
    """The gate/up projections then SwiGLU (``engine.py:189-193``): wq_gu is the
    stacked [gate; up] weight [2I, K] (gate rows first), as the engine's two
    projections would be run; returns z [..., I]."""
    wq_gu = np.asarray(wq_gu)
    inter = wq_gu.shape[0] // 2
    y = f8_forward(x, wq_gu, scales_gu, bias_gu)
    return swiglu_f16(y[..., :inter], y[..., inter:])


def interleave_gate_up(a, block=16) -> np.ndarray:
    """Rows of a stacked [gate; up] array in the fused SwiGLU kernel's order:
    blocks of `block` gate rows followed by the same `block` up rows."""
    a = np.asarray(a)
    nb = a.shape[0] // (2 * block)
    tail = a.shape[1:]
    return a.reshape((2, nb, block) + tail).swapaxes(0, 1).reshape(a.shape)


def argmax_f16(logits) -> np.ndarray:
    """Greedy argmax over the last dim of fp16 logits, ties -> lowest index.

    ``sampler_d.cu:16-24`` starts from ``best = -FLT_MAX, idx = 0`` and keeps
    the first strict maximum per thread; ``sampler_d.cu:37-38`` breaks ties to
    the lower index.  So NaN and -inf are never picked, the first index of the
    maximum wins, and a row with no value above -FLT_MAX returns 0.
    """
    lg = np.asarray(logits, dtype=np.float16).astype(np.float32)
    with np.errstate(invalid="ignore"):
        ok = lg > -np.finfo(np.float32).max
    masked = np.where(ok, lg, -np.inf)
    idx = np.argmax(masked, axis=-1).astype(np.int64)
    return np.where(ok.any(axis=-1), idx, 0)


def lm_head_argmax(x, wq, scales) -> tuple[np.ndarray, np.ndarray]:
    """Fused lm_head + greedy pick: argmax of fp16(x @ dequant(W)^T) per row.

    Equals ``sampler_d.forward(gemm(x, W))`` of ``engine.py:338,345``.
    Returns (token ids int64 [M], fp16 max logits [M]).
    """
    y = f8_forward(x, wq, scales).reshape(-1, np.asarray(wq).shape[0])
    idx = argmax_f16(y)
    return idx, y[np.arange(y.shape[0]), idx]


def normwise_rel_err(y, y_ref) -> float:
    """max over rows of  max_n |y - y_ref| / max_n |y_ref|  (the parity metric)."""
    y = np.asarray(y, np.float64).reshape(-1, np.shape(y)[-1])
    r = np.asarray(y_ref, np.float64).reshape(-1, np.shape(y_ref)[-1])
    den = np.maximum(np.abs(r).max(axis=1), 1e-30)
    return float((np.abs(y - r).max(axis=1) / den).max()) if y.size else 0.0


# --------------------------------------------------------------------------- torch-CPU baseline
def f8_forward_torch_cpu(x, wq, scales, bias=None):
    """The reference semantics in PyTorch on the host cores (the CPU baseline).

    ``y = (x.float() @ (dec(wq) * s[:,None]).T + b).half()`` with the dequant
    done per call, as BASELINE states the path; x, wq, scales, bias are CPU
    torch tensors.
    """
    import torch
    lut = torch.from_numpy(E4M3_DECODE)
    w = lut[wq.long()] * scales[:, None]
    y = x.reshape(-1, x.shape[-1]).float() @ w.T
    if bias is not None:
        y = y + bias.float()
    return y.half().reshape(*x.shape[:-1], wq.shape[0])
