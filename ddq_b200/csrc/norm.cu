// norm.cu - RMSNorm with the residual add fused in front (replaces the
// reference's qwen2_rmsnorm_kernel, RMSnorm_d.cu:23-87, and the residual
// addition before it, engine.py:254-256).
//
//   s = fp16(x + delta)          (delta optional; the new residual stream)
//   h = fp16( (s * rsqrt(mean(s^2) + eps)) * w )      fp32 math
//
// One warp per row; rows of up to 2048 elements stay in registers (a 16-byte
// chunk of 8 values per lane and step), longer rows are read a second time.
#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

__device__ __forceinline__ uint4 nm_add8(const uint4& a, const uint4& b) {
  uint4 r;
  const __half2* x = reinterpret_cast<const __half2*>(&a);
  const __half2* y = reinterpret_cast<const __half2*>(&b);
  __half2* o = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __hadd2(x[i], y[i]);
  return r;
}

__device__ __forceinline__ float nm_sumsq8(const uint4& a) {
  const __half2* x = reinterpret_cast<const __half2*>(&a);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(x[i]);
    s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
  }
  return s;
}

__device__ __forceinline__ uint4 nm_scale8(const uint4& a, float r, const float* w) {
  uint4 out;
  const __half2* x = reinterpret_cast<const __half2*>(&a);
  __half2* o = reinterpret_cast<__half2*>(&out);
  const float4 w0 = reinterpret_cast<const float4*>(w)[0];
  const float4 w1 = reinterpret_cast<const float4*>(w)[1];
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(x[i]);
    o[i] = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, r), wv[2 * i]),
                             __fmul_rn(__fmul_rn(f.y, r), wv[2 * i + 1]));
  }
  return out;
}

__device__ __forceinline__ uint4 nm_scale8w(const uint4& a, float r, const float4& w0,
                                            const float4& w1) {
  uint4 out;
  const __half2* x = reinterpret_cast<const __half2*>(&a);
  __half2* o = reinterpret_cast<__half2*>(&out);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(x[i]);
    o[i] = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, r), wv[2 * i]),
                             __fmul_rn(__fmul_rn(f.y, r), wv[2 * i + 1]));
  }
  return out;
}

constexpr int NM_REG_CHUNKS = 8;  // 16-byte chunks per lane kept in registers

// RC: chunks per lane kept in registers (4 for rows of up to 1024: half the
// registers, twice the CTAs per SM).  Every RC sums a lane's chunks in the same
// order, so the result does not depend on it.
template <int RC>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const __half* x,
                                                          const __half* __restrict__ delta,
                                                          const float* __restrict__ w, float eps,
                                                          __half* x_out, __half* __restrict__ h,
                                                          int M, int H) {
  ptx::pdl_wait();  // x / delta come from the previous kernels
  ptx::pdl_launch_dependents();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const int nch = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + (size_t)row * H) : nullptr;
  uint4* xo = x_out ? reinterpret_cast<uint4*>(x_out + (size_t)row * H) : nullptr;
  uint4* hr = reinterpret_cast<uint4*>(h + (size_t)row * H);
  const bool in_regs = nch <= 32 * RC;
  uint4 v[RC];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < RC; ++j) {
    const int c = lane + 32 * j;
    if (in_regs && c < nch) {
      v[j] = dr ? nm_add8(xr[c], dr[c]) : xr[c];
      if (xo) xo[c] = v[j];
      ss += nm_sumsq8(v[j]);
    }
  }
  if (!in_regs) {
    for (int c = lane; c < nch; c += 32) {
      const uint4 s = dr ? nm_add8(xr[c], dr[c]) : xr[c];
      if (xo) xo[c] = s;
      ss += nm_sumsq8(s);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)H + eps);
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < RC; ++j) {
      const int c = lane + 32 * j;
      if (c < nch) hr[c] = nm_scale8(v[j], r, w + 8 * c);
    }
  } else {
    for (int c = lane; c < nch; c += 32) {  // x_out may alias x: re-read the stored sum
      const uint4 s = xo ? xo[c] : (dr ? nm_add8(xr[c], dr[c]) : xr[c]);
      hr[c] = nm_scale8(s, r, w + 8 * c);
    }
  }
}

// The same, followed by the three-plane e4m3 split of h that the decode GEMM
// takes as its B operand (as xsplit_kernel would produce it from h): planes
// [3][M][H], token scales 2^-e [M].  h itself is stored only if asked for.
// Rows of up to 2048 elements (one warp, in registers).
__global__ void __launch_bounds__(256) add_rmsnorm_split_kernel(
    const __half* x, const __half* __restrict__ delta, const float* __restrict__ w, float eps,
    __half* x_out, __half* __restrict__ h, uint8_t* __restrict__ planes,
    float* __restrict__ xscale, int M, int H) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int nch = H / 8;
  // the norm weight is not produced by the previous kernel: load it while that
  // kernel finishes
  float4 wr[NM_REG_CHUNKS][2];
#pragma unroll
  for (int j = 0; j < NM_REG_CHUNKS; ++j) {
    const int c = lane + 32 * j;
    if (c < nch) {
      wr[j][0] = __ldg(reinterpret_cast<const float4*>(w + 8 * c));
      wr[j][1] = __ldg(reinterpret_cast<const float4*>(w + 8 * c) + 1);
    }
  }
  ptx::pdl_wait();
  ptx::pdl_launch_dependents();
  if (row >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + (size_t)row * H) : nullptr;
  uint4* xo = x_out ? reinterpret_cast<uint4*>(x_out + (size_t)row * H) : nullptr;
  uint4 v[NM_REG_CHUNKS];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NM_REG_CHUNKS; ++j) {
    const int c = lane + 32 * j;
    if (c < nch) {
      v[j] = dr ? nm_add8(xr[c], dr[c]) : xr[c];
      if (xo) xo[c] = v[j];
      ss += nm_sumsq8(v[j]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)H + eps);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < NM_REG_CHUNKS; ++j) {
    const int c = lane + 32 * j;
    if (c < nch) {
      v[j] = nm_scale8w(v[j], r, wr[j][0], wr[j][1]);
      if (h) reinterpret_cast<uint4*>(h + (size_t)row * H)[c] = v[j];
      const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hv[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const int e = split_shift(amax);
  const float up = ldexpf(1.f, e);
  if (lane == 0) xscale[row] = ldexpf(1.f, -e);
  const size_t plane = (size_t)M * H;
  uint8_t* p1 = planes + (size_t)row * H;
#pragma unroll
  for (int j = 0; j < NM_REG_CHUNKS; ++j) {
    const int c = lane + 32 * j;
    if (c < nch) {
      const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
      float z[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hv[i]);
        z[2 * i] = f.x * up;  // exact: power-of-two scale
        z[2 * i + 1] = f.y * up;
      }
      uint2 a, b, cc;
      split8(z, a, b, cc);
      *reinterpret_cast<uint2*>(p1 + (size_t)c * 8) = a;
      *reinterpret_cast<uint2*>(p1 + plane + (size_t)c * 8) = b;
      *reinterpret_cast<uint2*>(p1 + 2 * plane + (size_t)c * 8) = cc;
    }
  }
}

// The same with one row per CTA of 128 threads (H <= 2048: at most two
// 16-byte chunks per thread), for the few rows of a decode step: four times
// the threads on each row.  The sum of squares is reduced in the one-warp
// kernels' order (chunk partials; lane L adds chunks L, L + 32, ... in turn,
// then the same butterfly), so h is bit-identical to add_rmsnorm's.
// SPLIT = false: h only (the add_rmsnorm of a decode step).
constexpr int NR_THREADS = 128;
template <bool SPLIT>
__global__ void __launch_bounds__(NR_THREADS) add_rmsnorm_split_row_kernel(
    const __half* x, const __half* __restrict__ delta, const float* __restrict__ w, float eps,
    __half* x_out, __half* __restrict__ h, uint8_t* __restrict__ planes,
    float* __restrict__ xscale, int M, int H) {
  constexpr int CPT = 2;
  const int row = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nch = H / 8;
  __shared__ float part[32 * NM_REG_CHUNKS];  // per-chunk sums of squares
  __shared__ float red[2][NR_THREADS / 32];
  float4 wr[CPT][2];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = t + NR_THREADS * j;
    if (c < nch) {  // the norm weight does not come from the previous kernel
      wr[j][0] = __ldg(reinterpret_cast<const float4*>(w + 8 * c));
      wr[j][1] = __ldg(reinterpret_cast<const float4*>(w + 8 * c) + 1);
    }
  }
  ptx::pdl_wait();
  ptx::pdl_launch_dependents();
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + (size_t)row * H) : nullptr;
  uint4* xo = x_out ? reinterpret_cast<uint4*>(x_out + (size_t)row * H) : nullptr;
  uint4 v[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = t + NR_THREADS * j;
    if (c < nch) {
      v[j] = dr ? nm_add8(xr[c], dr[c]) : xr[c];
      if (xo) xo[c] = v[j];
      part[c] = nm_sumsq8(v[j]);
    }
  }
  __syncthreads();
  if (warp == 0) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NM_REG_CHUNKS; ++j)
      if (lane + 32 * j < nch) ss += part[lane + 32 * j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[0][0] = ss;
  }
  __syncthreads();
  const float r = rsqrtf(red[0][0] / (float)H + eps);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = t + NR_THREADS * j;
    if (c < nch) {
      v[j] = nm_scale8w(v[j], r, wr[j][0], wr[j][1]);
      if (h) reinterpret_cast<uint4*>(h + (size_t)row * H)[c] = v[j];
      const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hv[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  if (!SPLIT) return;
  amax = warp_max(amax);
  if (lane == 0) red[1][warp] = amax;
  __syncthreads();
  amax = 0.f;
#pragma unroll
  for (int i = 0; i < NR_THREADS / 32; ++i) amax = fmaxf(amax, red[1][i]);
  const int e = split_shift(amax);
  const float up = ldexpf(1.f, e);
  if (t == 0) xscale[row] = ldexpf(1.f, -e);
  const size_t plane = (size_t)M * H;
  uint8_t* p1 = planes + (size_t)row * H;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = t + NR_THREADS * j;
    if (c < nch) {
      const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
      float z[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hv[i]);
        z[2 * i] = f.x * up;  // exact: power-of-two scale
        z[2 * i + 1] = f.y * up;
      }
      uint2 a, b, cc;
      split8(z, a, b, cc);
      *reinterpret_cast<uint2*>(p1 + (size_t)c * 8) = a;
      *reinterpret_cast<uint2*>(p1 + plane + (size_t)c * 8) = b;
      *reinterpret_cast<uint2*>(p1 + 2 * plane + (size_t)c * 8) = cc;
    }
  }
}

int launch_add_rmsnorm_split(const __half* x, const __half* delta, const float* w, float eps,
                             __half* x_out, __half* h, uint8_t* planes, float* xscale, int M,
                             int H, cudaStream_t s) {
  if (M < 0 || H < 16 || H % 16 != 0 || H > 32 * NM_REG_CHUNKS * 8) return DDQ_ERR_SHAPE;
  if (M == 0) return DDQ_OK;
  if (!aligned16(x) || (delta && !aligned16(delta)) || !aligned16(w) ||
      (x_out && !aligned16(x_out)) || (h && !aligned16(h)) || !aligned16(planes))
    return DDQ_ERR_ALIGNMENT;
  cudaLaunchConfig_t cfg = {};
  // few rows (a decode step): one row per CTA; many rows: one row per warp
  const bool per_cta = M <= 256;
  cfg.gridDim = dim3(per_cta ? (unsigned)M : (unsigned)((M + 7) / 8));
  cfg.blockDim = dim3(per_cta ? NR_THREADS : 256);
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg,
                         per_cta ? add_rmsnorm_split_row_kernel<true> : add_rmsnorm_split_kernel,
                         x, delta, w, eps, x_out, h, planes, xscale, M, H) != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

int launch_add_rmsnorm(const __half* x, const __half* delta, const float* w, float eps,
                       __half* x_out, __half* h, int M, int H, cudaStream_t s) {
  if (M < 0 || H < 8 || H % 8 != 0) return DDQ_ERR_SHAPE;
  if (M == 0) return DDQ_OK;
  if (!aligned16(x) || (delta && !aligned16(delta)) || !aligned16(w) ||
      (x_out && !aligned16(x_out)) || !aligned16(h))
    return DDQ_ERR_ALIGNMENT;
  cudaLaunchConfig_t cfg = {};
  // few rows of at most 2048 (a decode step): one row per CTA; else one per warp
  const bool per_cta = M <= 256 && H <= 32 * NM_REG_CHUNKS * 8 && H % 16 == 0;
  cfg.gridDim = dim3(per_cta ? (unsigned)M : (unsigned)((M + 7) / 8));
  cfg.blockDim = dim3(per_cta ? NR_THREADS : 256);
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e =
      per_cta ? cudaLaunchKernelEx(&cfg, add_rmsnorm_split_row_kernel<false>, x, delta, w, eps,
                                   x_out, h, (uint8_t*)nullptr, (float*)nullptr, M, H)
          : H / 8 <= 128
              ? cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<4>, x, delta, w, eps, x_out, h, M, H)
              : cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<NM_REG_CHUNKS>, x, delta, w, eps,
                                   x_out, h, M, H);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace ddq
