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
// Work split: the warps (16 for 64-wide heads) take 32-position tiles in
// turn (lane = position for the scores, lane = D / 32 head dimensions for the
// weighted sum of V) with an online softmax per query head; the CTA merges
// the warps' partial results in shared memory.  Every K row and every group
// of 16 V rows is requested before it is used, so a warp waits on memory once
// per step instead of once per row.  K rows are read once per CTA, by one lane each (128
// contiguous bytes); V rows once, coalesced across the warp.  The step reads
// the cache at HBM rate; the arithmetic runs on the CUDA cores.
#include <cfloat>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int AT_GMAX = 8;  // query heads per key/value head, at most
// warps per CTA: 16 for 64-wide heads (one 32-position tile per warp for
// contexts up to 512), 8 for 128-wide heads (register budget)
__host__ __device__ constexpr int at_warps(int d) { return d == 64 ? 16 : 8; }

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
__global__ void __launch_bounds__(at_warps(D) * 32, 1) decode_attention_kernel(const AtArgs a) {
  constexpr int NW = at_warps(D);
  constexpr int DH = D / 2;
  constexpr int DPL = D / 32;  // head dimensions per lane in the weighted sum
  const int b = blockIdx.x / a.Hkv, g = blockIdx.x % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ __align__(16) float q_s[AT_GMAX][D];
  __shared__ float m_s[NW][AT_GMAX], l_s[NW][AT_GMAX];
  __shared__ float acc_s[NW][AT_GMAX][D];

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
  for (int t0 = warp * 32; t0 < L; t0 += NW * 32) {
    const int j = t0 + lane;
    const bool ok = j < L;
    float s[AT_GMAX];
#pragma unroll
    for (int h = 0; h < AT_GMAX; ++h) s[h] = 0.f;
    if (ok) {
      // the whole K row in flight at once, then G dot products against q
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * D);
      uint4 kv[D / 8];
#pragma unroll
      for (int c = 0; c < D / 8; ++c) kv[c] = kr[c];
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const __half2* hv = reinterpret_cast<const __half2*>(&kv[c]);
        float kf[8];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 f = __half22float2(hv[t]);
          kf[2 * t] = f.x;
          kf[2 * t + 1] = f.y;
        }
#pragma unroll
        for (int h = 0; h < AT_GMAX; ++h) {
          if (h < G) {
            const float4 qa = *reinterpret_cast<const float4*>(&q_s[h][c * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&q_s[h][c * 8 + 4]);
            float acc_s8 = s[h];
            acc_s8 = fmaf(qa.x, kf[0], acc_s8);
            acc_s8 = fmaf(qa.y, kf[1], acc_s8);
            acc_s8 = fmaf(qa.z, kf[2], acc_s8);
            acc_s8 = fmaf(qa.w, kf[3], acc_s8);
            acc_s8 = fmaf(qb.x, kf[4], acc_s8);
            acc_s8 = fmaf(qb.y, kf[5], acc_s8);
            acc_s8 = fmaf(qb.z, kf[6], acc_s8);
            acc_s8 = fmaf(qb.w, kf[7], acc_s8);
            s[h] = acc_s8;
          }
        }
      }
    }
    float pr[AT_GMAX];
#pragma unroll
    for (int h = 0; h < AT_GMAX; ++h) {
      pr[h] = 0.f;
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
    // weighted sum of V: 16 rows at a time, all their loads in flight first;
    // rows past the last position read as zero (their weights are zero too)
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += 16) {
      if (t0 + j0 >= L) break;
      float vf[16][DPL];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int pj = t0 + j0 + jj;
        const __half* vr = vc + (size_t)pj * D + lane * DPL;
        if (pj < L) {
          if constexpr (DPL == 2) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vr));
            vf[jj][0] = f.x;
            vf[jj][1] = f.y;
          } else {
            const uint2 u = *reinterpret_cast<const uint2*>(vr);
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            vf[jj][0] = f0.x;
            vf[jj][1] = f0.y;
            vf[jj][2] = f1.x;
            vf[jj][3] = f1.y;
          }
        } else {
#pragma unroll
          for (int t = 0; t < DPL; ++t) vf[jj][t] = 0.f;
        }
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
#pragma unroll
        for (int h = 0; h < AT_GMAX; ++h) {
          if (h >= G) continue;
          const float pj = __shfl_sync(0xffffffffu, pr[h], j0 + jj);
#pragma unroll
          for (int t = 0; t < DPL; ++t) acc[h][t] = fmaf(pj, vf[jj][t], acc[h][t]);
        }
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
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, m_s[w][h]);
    float den = 0.f, num = 0.f;
    for (int w = 0; w < NW; ++w) {
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
  cfg.blockDim = dim3(at_warps(D) * 32);
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
