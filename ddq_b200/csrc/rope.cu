// rope.cu - the prefill half of the rotary embedding and the KV-cache write
// (replaces, for a prefill chunk, the reference's RoPE kernel on q and k,
// RoPe_d.cu:12-68, called from engine.py:219-220, and the cache write,
// engine.py:126-130 and 222).
//
// For every token (b, s) of a chunk that starts at cache position `start`:
//   q_h  = fp16(rope(q_h, start + s))  -> q_out[b, s, h, :]   (token-major, the
//                                          layout attention reads without a copy)
//   k_g  = fp16(rope(k_g, start + s))  -> k_cache[b, g, start + s, :]  (and k_out[b, s, g, :])
//   v_g                                -> v_cache[b, g, start + s, :]  (and v_out[b, s, g, :])
// The optional token-major k_out / v_out give attention inputs whose strides do
// not depend on the cache capacity.
// rope(x)[d] = x[d] cos[d] + rotate_half(x)[d] sin[d] with rotate_half(x) =
// (-x[D/2:], x[:D/2]); each product and the sum rounded in fp32 as the
// unfused fp32 path rounds them, then to fp16.  cos/sin are the caller's fp32
// rows for the chunk's positions.
//
// One thread per 16-byte piece: 8 dimensions of the first half of a head
// together with the matching 8 of the second half (the two halves of every
// rotation pair), or 8 dimensions of a value row.  Memory bound: the chunk's
// qkv is read once and q, k, v written once.
#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

struct RkArgs {
  const __half* qkv;  // [B * S, (Hq + 2 Hkv) * D], row stride qkv_stride
  int64_t qkv_stride;
  __half* kc;         // [B, Hkv, cap, D], batch stride cache_bstride
  __half* vc;
  int64_t cache_bstride;
  int cap;
  const float* cos;   // [S, D]
  const float* sin;
  int start;
  __half* q_out;      // [B, S, Hq, D]
  __half* k_out;      // [B, S, Hkv, D] or null
  __half* v_out;
  int B, S, Hq, Hkv;
};

template <int D>
__global__ void __launch_bounds__(256) prefill_rope_kv_kernel(const RkArgs a) {
  constexpr int DH = D / 2;
  constexpr int PH = DH / 8;  // pieces per half head
  constexpr int VP = D / 8;   // pieces per value row
  ptx::pdl_wait();            // qkv comes from the projection just before
  ptx::pdl_launch_dependents();
  const int rot = (a.Hq + a.Hkv) * PH;
  const int per_tok = rot + a.Hkv * VP;
  const int64_t total = (int64_t)a.B * a.S * per_tok;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_tok;  // token b * S + s
    const int j = (int)(i - t * per_tok);
    const int b = (int)(t / a.S), s = (int)(t - (int64_t)b * a.S);
    const __half* row = a.qkv + t * a.qkv_stride;
    if (j < rot) {
      const int h = j / PH, d0 = 8 * (j % PH);  // q heads, then k heads
      const uint4 u1 = *reinterpret_cast<const uint4*>(row + (size_t)h * D + d0);
      const uint4 u2 = *reinterpret_cast<const uint4*>(row + (size_t)h * D + DH + d0);
      const float* cr = a.cos + (size_t)s * D;
      const float* sr = a.sin + (size_t)s * D;
      float c1[8], s1[8], c2[8], s2[8];
      *reinterpret_cast<float4*>(c1) = *reinterpret_cast<const float4*>(cr + d0);
      *reinterpret_cast<float4*>(c1 + 4) = *reinterpret_cast<const float4*>(cr + d0 + 4);
      *reinterpret_cast<float4*>(s1) = *reinterpret_cast<const float4*>(sr + d0);
      *reinterpret_cast<float4*>(s1 + 4) = *reinterpret_cast<const float4*>(sr + d0 + 4);
      *reinterpret_cast<float4*>(c2) = *reinterpret_cast<const float4*>(cr + DH + d0);
      *reinterpret_cast<float4*>(c2 + 4) = *reinterpret_cast<const float4*>(cr + DH + d0 + 4);
      *reinterpret_cast<float4*>(s2) = *reinterpret_cast<const float4*>(sr + DH + d0);
      *reinterpret_cast<float4*>(s2 + 4) = *reinterpret_cast<const float4*>(sr + DH + d0 + 4);
      const __half* x1 = reinterpret_cast<const __half*>(&u1);
      const __half* x2 = reinterpret_cast<const __half*>(&u2);
      uint4 o1, o2;
      __half* y1 = reinterpret_cast<__half*>(&o1);
      __half* y2 = reinterpret_cast<__half*>(&o2);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float a1 = __half2float(x1[e]), a2 = __half2float(x2[e]);
        y1[e] = __float2half_rn(__fadd_rn(__fmul_rn(a1, c1[e]), __fmul_rn(-a2, s1[e])));
        y2[e] = __float2half_rn(__fadd_rn(__fmul_rn(a2, c2[e]), __fmul_rn(a1, s2[e])));
      }
      __half* dst = h < a.Hq ? a.q_out + ((size_t)t * a.Hq + h) * D
                             : a.kc + (size_t)b * a.cache_bstride +
                                   ((size_t)(h - a.Hq) * a.cap + a.start + s) * D;
      *reinterpret_cast<uint4*>(dst + d0) = o1;
      *reinterpret_cast<uint4*>(dst + DH + d0) = o2;
      if (h >= a.Hq && a.k_out) {
        __half* ko = a.k_out + ((size_t)t * a.Hkv + (h - a.Hq)) * D;
        *reinterpret_cast<uint4*>(ko + d0) = o1;
        *reinterpret_cast<uint4*>(ko + DH + d0) = o2;
      }
    } else {
      const int jv = j - rot, g = jv / VP, d0 = 8 * (jv % VP);
      const uint4 u = *reinterpret_cast<const uint4*>(row + (size_t)(a.Hq + a.Hkv + g) * D + d0);
      *reinterpret_cast<uint4*>(a.vc + (size_t)b * a.cache_bstride +
                                ((size_t)g * a.cap + a.start + s) * D + d0) = u;
      if (a.v_out) *reinterpret_cast<uint4*>(a.v_out + ((size_t)t * a.Hkv + g) * D + d0) = u;
    }
  }
}

int launch_prefill_rope_kv(const __half* qkv, int64_t qkv_stride, __half* kc, __half* vc,
                           int64_t cache_bstride, int cap, const float* cos, const float* sin,
                           int start, __half* q_out, __half* k_out, __half* v_out, int B,
                           int S, int Hq, int Hkv, int D, cudaStream_t s) {
  if (B < 0 || S < 0 || Hq < 1 || Hkv < 1 || cap < 1 || start < 0) return DDQ_ERR_SHAPE;
  if (D != 64 && D != 128) return DDQ_ERR_SHAPE;
  if ((int64_t)start + S > cap) return DDQ_ERR_SHAPE;
  if (B == 0 || S == 0) return DDQ_OK;
  if (!aligned16(qkv) || qkv_stride % 8 != 0 || !aligned16(kc) || !aligned16(vc) ||
      cache_bstride % 8 != 0 || !aligned16(cos) || !aligned16(sin) || !aligned16(q_out) ||
      (k_out && !aligned16(k_out)) || (v_out && !aligned16(v_out)))
    return DDQ_ERR_ALIGNMENT;
  RkArgs a{qkv,   qkv_stride, kc,    vc, cache_bstride, cap, cos, sin,
           start, q_out,      k_out, v_out, B, S, Hq, Hkv};
  const int per_tok = (Hq + Hkv) * (D / 16) + Hkv * (D / 8);
  const int64_t total = (int64_t)B * S * per_tok;
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e = D == 64 ? cudaLaunchKernelEx(&cfg, prefill_rope_kv_kernel<64>, a)
                                : cudaLaunchKernelEx(&cfg, prefill_rope_kv_kernel<128>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace ddq
