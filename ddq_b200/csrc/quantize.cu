// quantize.cu - per-row e4m3fn weight quantization (load-time op).
//
// Replaces quantize_kernel (gemm_FP8_d.cu:66-86): there one thread walked a
// whole row serially with stride-K neighbours (uncoalesced, 7-38 CTAs).  Here
// one warp owns a row and reads it with 16-byte coalesced loads, so every
// weight byte crosses HBM once per pass; the second pass re-reads the row
// from L1/L2.
#include "common.cuh"

namespace ddq {

__device__ __forceinline__ void load8(const __half* p, float* f) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void load8(const float* p, float* f) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

// One warp per weight row; 8 rows per 256-thread CTA.
// scale = absmax / 448 with IEEE division (1.0 for an all-zero row, as
// gemm_FP8_d.cu:78), element = e4m3(w / scale) with IEEE division and
// round-to-nearest-even: the bytes equal torch's (W / s).to(float8_e4m3fn).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ w,
                                                            uint8_t* __restrict__ wq,
                                                            float* __restrict__ scales,
                                                            int64_t N, int64_t K) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= N) return;
  const T* wr = w + row * K;
  uint8_t* qr = wq + row * K;

  float amax = 0.f;
  if (VEC) {
    for (int64_t c = lane; c < K / 8; c += 32) {
      float f[8];
      load8(wr + c * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
    }
  } else {
    for (int64_t k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(to_f32(wr[k])));
  }
  amax = warp_max(amax);
  const float scale = amax > 0.f ? __fdiv_rn(amax, 448.f) : 1.f;

  if (VEC) {
    for (int64_t c = lane; c < K / 8; c += 32) {
      float f[8];
      load8(wr + c * 8, f);
      uint32_t lo = (uint32_t)float2_to_e4m3x2(__fdiv_rn(f[0], scale), __fdiv_rn(f[1], scale)) |
                    ((uint32_t)float2_to_e4m3x2(__fdiv_rn(f[2], scale), __fdiv_rn(f[3], scale)) << 16);
      uint32_t hi = (uint32_t)float2_to_e4m3x2(__fdiv_rn(f[4], scale), __fdiv_rn(f[5], scale)) |
                    ((uint32_t)float2_to_e4m3x2(__fdiv_rn(f[6], scale), __fdiv_rn(f[7], scale)) << 16);
      *reinterpret_cast<uint2*>(qr + c * 8) = make_uint2(lo, hi);
    }
  } else {
    for (int64_t k = lane; k < K; k += 32) {
      qr[k] = (uint8_t)(float2_to_e4m3x2(__fdiv_rn(to_f32(wr[k]), scale), 0.f) & 0xFF);
    }
  }
  if (lane == 0) scales[row] = scale;
}

}  // namespace ddq

using namespace ddq;

extern "C" int ddq_quantize_e4m3(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* wq,
                                 float* scales, void* stream) {
  if (N < 0 || K < 0) return DDQ_ERR_SHAPE;
  if (N == 0) return DDQ_OK;
  if (!w || !wq || !scales) return DDQ_ERR_INVALID_ARGUMENT;
  if (w_dtype != DDQ_DTYPE_F16 && w_dtype != DDQ_DTYPE_F32) return DDQ_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = (K % 8 == 0) && aligned16(w) && ((reinterpret_cast<uintptr_t>(wq) & 7u) == 0);
  const int rows_per_cta = 8;
  const int64_t grid = (N + rows_per_cta - 1) / rows_per_cta;
  if (grid > 0x7fffffff) return DDQ_ERR_SHAPE;
  if (w_dtype == DDQ_DTYPE_F16) {
    const __half* wp = reinterpret_cast<const __half*>(w);
    if (vec)
      quantize_rows_kernel<__half, true><<<(unsigned)grid, 256, 0, s>>>(wp, wq, scales, N, K);
    else
      quantize_rows_kernel<__half, false><<<(unsigned)grid, 256, 0, s>>>(wp, wq, scales, N, K);
  } else {
    const float* wp = reinterpret_cast<const float*>(w);
    if (vec)
      quantize_rows_kernel<float, true><<<(unsigned)grid, 256, 0, s>>>(wp, wq, scales, N, K);
    else
      quantize_rows_kernel<float, false><<<(unsigned)grid, 256, 0, s>>>(wp, wq, scales, N, K);
  }
  return check_launch();
}
