// attention.cu - one decode step of grouped-query attention with the rotary
// embedding and the KV-cache write fused in (replaces the reference's RoPE
// kernel, the cache copy and the attention call of a decode step:
// RoPe_d.cu:12-68, engine.py:126-130 and 225-251).
//
// For each sequence b and key/value head g (one CTA, 256 threads):
//   q_h  = fp16(rope(q_h, pos))   for the G query heads h of group g
//   k    = fp16(rope(k_g, pos)),  v = v_g        -> cache[b, g, pos, :]
//   o_h  = softmax_j( q_h . K[b, g, j, :] * scale ) V[b, g, j, :],  j = 0..pos
// Rotate-half RoPE in fp32 with the caller's cos/sin row for this position,
// rounded to fp16 as the unfused path rounds it; scores, softmax and the
// weighted sum in fp32; o rounded to fp16.  The position is read on the
// device, so a captured CUDA graph replays it for every step.
//
// Work split: the 8 warps take 32-position tiles in turn (lane = position for
// the scores, lane = two head dimensions for the weighted sum of V) with an
// online softmax per query head; the CTA merges the 8 partial results in
// shared memory.  K rows are read once per CTA, by one lane each (128
// contiguous bytes); V rows once, coalesced across the warp.  The step reads
// the cache at HBM rate; the arithmetic runs on the CUDA cores.
#include <cfloat>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int AT_WARPS = 8;
constexpr int AT_GMAX = 8;  // query heads per key/value head, at most

struct AtArgs {
  const __half* qkv;     // [B, (Hq + 2 Hkv) * D] row stride qkv_stride
  int64_t qkv_stride;
  __half* kc;            // [B, Hkv, cap, D] with batch stride cache_bstride
  __half* vc;
  int64_t cache_bstride;
  int cap;
  const float* cos;      // [D]
  const float* sin;      // [D]
  const int64_t* pos;    // device scalar
  __half* out;           // [B, Hq * D] row stride out_stride
  int64_t out_stride;
  int Hq, Hkv;
  float scale;
};

template <int D>
__global__ void __launch_bounds__(AT_WARPS * 32) decode_attention_kernel(const AtArgs a) {
  constexpr int DH = D / 2;
  constexpr int DPL = D / 32;  // head dimensions per lane in the weighted sum
  const int b = blockIdx.x / a.Hkv, g = blockIdx.x % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float q_s[AT_GMAX][D];
  __shared__ float m_s[AT_WARPS][AT_GMAX], l_s[AT_WARPS][AT_GMAX];
  __shared__ float acc_s[AT_WARPS][AT_GMAX][D];

  ptx::pdl_wait();  // qkv comes from the previous kernel
  const int64_t p = *a.pos;
  if (p < 0 || p >= a.cap) return;  // the host checks the range; nothing to do otherwise
  const int L = (int)p + 1;
  const __half* row = a.qkv + (size_t)b * a.qkv_stride;
  const size_t head = (size_t)a.cap * D;
  __half* kc = a.kc + (size_t)b * a.cache_bstride + (size_t)g * head;
  __half* vc = a.vc + (size_t)b * a.cache_bstride + (size_t)g * head;

  // ---- rotary embedding of the G query heads and the new key; cache write
  for (int i = threadIdx.x; i < (G + 1) * DH; i += blockDim.x) {
    const int h = i / DH, d = i % DH;
    const __half* src = h < G ? row + (size_t)(g * G + h) * D
                              : row + (size_t)(a.Hq + g) * D;
    const float x1 = __half2float(src[d]), x2 = __half2float(src[d + DH]);
    // x * cos + rotate_half(x) * sin, each product rounded as torch rounds it
    const float y1 = __half2float(
        __float2half_rn(__fadd_rn(__fmul_rn(x1, a.cos[d]), __fmul_rn(-x2, a.sin[d]))));
    const float y2 = __half2float(
        __float2half_rn(__fadd_rn(__fmul_rn(x2, a.cos[d + DH]), __fmul_rn(x1, a.sin[d + DH]))));
    if (h < G) {
      q_s[h][d] = y1;
      q_s[h][d + DH] = y2;
    } else {
      kc[(size_t)p * D + d] = __float2half_rn(y1);
      kc[(size_t)p * D + d + DH] = __float2half_rn(y2);
    }
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    vc[(size_t)p * D + d] = row[(size_t)(a.Hq + a.Hkv + g) * D + d];
  __syncthreads();  // the cache row and q_s are visible to the whole CTA
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  // ---- scores and the weighted sum over this warp's 32-position tiles
  float m[AT_GMAX], l[AT_GMAX], acc[AT_GMAX][DPL];
#pragma unroll
  for (int h = 0; h < AT_GMAX; ++h) {
    m[h] = -FLT_MAX;
    l[h] = 0.f;
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc[h][t] = 0.f;
  }
  for (int t0 = warp * 32; t0 < L; t0 += AT_WARPS * 32) {
    const int j = t0 + lane;
    const bool ok = j < L;
    float s[AT_GMAX];
#pragma unroll
    for (int h = 0; h < AT_GMAX; ++h) s[h] = 0.f;
    if (ok) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 u = kr[c];
        const __half2* hv = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kf = __half22float2(hv[e]);
          const int d = c * 8 + 2 * e;
#pragma unroll
          for (int h = 0; h < AT_GMAX; ++h)
            if (h < G) s[h] = fmaf(q_s[h][d], kf.x, fmaf(q_s[h][d + 1], kf.y, s[h]));
        }
      }
    }
    float pr[AT_GMAX];
#pragma unroll
    for (int h = 0; h < AT_GMAX; ++h) {
      if (h >= G) continue;
      const float sv = ok ? s[h] * a.scale : -FLT_MAX;
      float tm = sv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
      const float mn = fmaxf(m[h], tm);
      const float corr = __expf(m[h] - mn);
      pr[h] = ok ? __expf(sv - mn) : 0.f;
      float ps = pr[h];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[h] = l[h] * corr + ps;
      m[h] = mn;
#pragma unroll
      for (int t = 0; t < DPL; ++t) acc[h][t] *= corr;
    }
    const int jn = min(32, L - t0);
    for (int jj = 0; jj < jn; ++jj) {
      const __half* vr = vc + (size_t)(t0 + jj) * D + lane * DPL;
      float vf[DPL];
      if constexpr (DPL == 2) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vr));
        vf[0] = f.x;
        vf[1] = f.y;
      } else {
#pragma unroll
        for (int t = 0; t < DPL; ++t) vf[t] = __half2float(vr[t]);
      }
#pragma unroll
      for (int h = 0; h < AT_GMAX; ++h) {
        if (h >= G) continue;
        const float pj = __shfl_sync(0xffffffffu, pr[h], jj);
#pragma unroll
        for (int t = 0; t < DPL; ++t) acc[h][t] = fmaf(pj, vf[t], acc[h][t]);
      }
    }
  }

  // ---- merge the warps' partial softmax sums
#pragma unroll
  for (int h = 0; h < AT_GMAX; ++h) {
    if (h >= G) continue;
    if (lane == 0) {
      m_s[warp][h] = m[h];
      l_s[warp][h] = l[h];
    }
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc_s[warp][h][lane * DPL + t] = acc[h][t];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float mx = -FLT_MAX;
    for (int w = 0; w < AT_WARPS; ++w) mx = fmaxf(mx, m_s[w][h]);
    float den = 0.f, num = 0.f;
    for (int w = 0; w < AT_WARPS; ++w) {
      const float c = l_s[w][h] > 0.f ? __expf(m_s[w][h] - mx) : 0.f;
      den = fmaf(l_s[w][h], c, den);
      num = fmaf(acc_s[w][h][d], c, num);
    }
    a.out[(size_t)b * a.out_stride + (size_t)(g * G + h) * D + d] = __float2half_rn(num / den);
  }
}

int launch_decode_attention(const __half* qkv, int64_t qkv_stride, __half* kc, __half* vc,
                            int64_t cache_bstride, int cap, const float* cos, const float* sin,
                            const int64_t* pos, __half* out, int64_t out_stride, int B, int Hq,
                            int Hkv, int D, float scale, cudaStream_t s) {
  if (B < 1 || Hkv < 1 || Hq < Hkv || Hq % Hkv != 0 || Hq / Hkv > AT_GMAX || cap < 1)
    return DDQ_ERR_SHAPE;
  if (D != 64 && D != 128) return DDQ_ERR_SHAPE;
  if (!aligned16(kc) || !aligned16(vc) || (cache_bstride % 8) != 0) return DDQ_ERR_ALIGNMENT;
  AtArgs a{qkv, qkv_stride, kc, vc, cache_bstride, cap, cos, sin, pos, out, out_stride, Hq, Hkv,
           scale};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * Hkv));
  cfg.blockDim = dim3(AT_WARPS * 32);
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e = D == 64 ? cudaLaunchKernelEx(&cfg, decode_attention_kernel<64>, a)
                                : cudaLaunchKernelEx(&cfg, decode_attention_kernel<128>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace ddq
