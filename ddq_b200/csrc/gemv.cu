// gemv.cu - CUDA-core W8A16 kernels: the skinny GEMV for very small M, the
// generic any-shape kernel, and the greedy-argmax kernels.
//
// The skinny kernel streams the e4m3 weight once with 16-byte coalesced,
// L1-bypassing loads (8 loads in flight per lane), decodes with the hardware
// e4m3x2 -> f16x2 converter, and accumulates in fp32 against activations
// staged once per CTA in shared memory (as fp32).  Scale, bias and the fp16
// cast are applied in one pass; the lm_head variant instead keeps a running
// (fp16 logit, index) maximum and never writes logits.
#include "common.cuh"
#include "launch.cuh"

#include <cfloat>

namespace ddq {

__device__ int g_device_error = 0;
__device__ unsigned long long g_trace[kTraceCtas * kTraceSlots];

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float load_bias(const void* bias, int bias_dtype, int n) {
  if (bias_dtype == DDQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (bias_dtype == DDQ_DTYPE_F32) return reinterpret_cast<const float*>(bias)[n];
  return 0.f;
}

__device__ __forceinline__ void decode16(const uint4& w, float* f) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 a = e4m3x2_to_float2((uint16_t)(u[i] & 0xFFFF));
    float2 b = e4m3x2_to_float2((uint16_t)(u[i] >> 16));
    f[4 * i + 0] = a.x;
    f[4 * i + 1] = a.y;
    f[4 * i + 2] = b.x;
    f[4 * i + 3] = b.y;
  }
}

// Packed greedy key: (ordered fp16 << 32) | (0xFFFFFFFF - index).  MAX over
// packed words = largest logit, ties to the lowest index (sampler_d.cu:37-38).
__device__ __forceinline__ unsigned long long pack_key(__half v, int64_t idx) {
  return ((unsigned long long)f16_order_key(v) << 32) |
         (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

// ----------------------------------------------------------------------------
// Skinny kernel.  An 8-lane team owns one weight row at a time (a warp works
// on 4 rows, a 256-thread CTA on 32); lane `sub` of the team takes the
// 16-byte chunks sub, sub+8, ... of the row.  MT token rows per CTA
// (blockIdx.y selects the token block).
// ----------------------------------------------------------------------------
template <int MT, bool ARGMAX>
__global__ void __launch_bounds__(256) gemv_skinny_kernel(
    const __half* __restrict__ x, const uint8_t* __restrict__ wq, const float* __restrict__ scales,
    const void* __restrict__ bias, int bias_dtype, __half* __restrict__ y,
    unsigned long long* __restrict__ packed, int64_t vocab_offset, int M, int N, int K) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);  // [MT][K] fp32
  const int m0 = blockIdx.y * MT;
  const int mt = min(MT, M - m0);

  for (int i = threadIdx.x; i < MT * (K / 8); i += blockDim.x) {
    const int m = i / (K / 8), c = i % (K / 8);
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (m < mt) {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(m0 + m) * K) + c);
      const __half2* h = reinterpret_cast<const __half2*>(&v);
      float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
      float2 cc = __half22float2(h[2]), d = __half22float2(h[3]);
      lo = make_float4(a.x, a.y, b.x, b.y);
      hi = make_float4(cc.x, cc.y, d.x, d.y);
    }
    float4* dst = reinterpret_cast<float4*>(xs + (size_t)m * K + (size_t)c * 8);
    dst[0] = lo;
    dst[1] = hi;
  }
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int team = lane >> 3, sub = lane & 7;
  const int nchunks = K / 16;
  constexpr int U = 8;

  unsigned long long best[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) best[m] = 0ull;

  for (int row_base = blockIdx.x * 32; row_base < N; row_base += gridDim.x * 32) {
    const int n = row_base + warp * 4 + team;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    if (n < N) {
      const uint4* wrow = reinterpret_cast<const uint4*>(wq + (size_t)n * K);
      for (int c0 = sub; c0 < nchunks; c0 += 8 * U) {
        uint4 wv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + u * 8;
          wv[u] = (c < nchunks) ? ld_stream(wrow + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + u * 8;
          if (c < nchunks) {
            float wf[16];
            decode16(wv[u], wf);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              const float4* xr = reinterpret_cast<const float4*>(xs + (size_t)m * K + (size_t)c * 16);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 xv = xr[q];
                acc[m] = fmaf(xv.x, wf[4 * q + 0], acc[m]);
                acc[m] = fmaf(xv.y, wf[4 * q + 1], acc[m]);
                acc[m] = fmaf(xv.z, wf[4 * q + 2], acc[m]);
                acc[m] = fmaf(xv.w, wf[4 * q + 3], acc[m]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 4);
      acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 2);
      acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 1);
    }
    if (sub == 0 && n < N) {
      const float s = scales[n];
      if (ARGMAX) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const __half v = __float2half_rn(acc[m] * s);
          if (m < mt && __half2float(v) > -FLT_MAX) {
            const unsigned long long k = pack_key(v, (int64_t)n + vocab_offset);
            best[m] = k > best[m] ? k : best[m];
          }
        }
      } else {
        const float b = load_bias(bias, bias_dtype, n);
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (m < mt) y[(size_t)(m0 + m) * N + n] = __float2half_rn(fmaf(acc[m], s, b));
      }
    }
  }

  if (ARGMAX) {
    // CTA-wide max of the packed keys, then one atomicMax per token row.
    __syncthreads();  // xs no longer needed: reuse it for the reduction
    unsigned long long* red = reinterpret_cast<unsigned long long*>(smem_raw);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      unsigned long long v = best[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
      }
      if (lane == 0) red[m * 8 + warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < MT) {
      const int m = threadIdx.x;
      unsigned long long v = 0ull;
      for (int w = 0; w < 8; ++w) v = red[m * 8 + w] > v ? red[m * 8 + w] : v;
      if (m < mt && v != 0ull) atomicMax(packed + m0 + m, v);
    }
  }
}

// ----------------------------------------------------------------------------
// Generic kernel for any K / alignment: one warp per (weight row, 4 tokens).
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemm_generic_kernel(
    const __half* __restrict__ x, const uint8_t* __restrict__ wq, const float* __restrict__ scales,
    const void* __restrict__ bias, int bias_dtype, __half* __restrict__ y, int64_t M, int64_t N,
    int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t mblocks = (M + 3) / 4;
  if (gw >= N * mblocks) return;
  const int64_t n = gw / mblocks;
  const int64_t m0 = (gw % mblocks) * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t k = lane; k < K; k += 32) {
    const float2 wf = e4m3x2_to_float2((uint16_t)wq[n * K + k]);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (m0 + j < M) acc[j] = fmaf(__half2float(x[(m0 + j) * K + k]), wf.x, acc[j]);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  }
  if (lane == 0) {
    const float s = scales[n];
    const float b = load_bias(bias, bias_dtype, (int)n);
    for (int j = 0; j < 4; ++j)
      if (m0 + j < M) y[(m0 + j) * N + n] = __float2half_rn(fmaf(acc[j], s, b));
  }
}

// ----------------------------------------------------------------------------
// Greedy argmax over fp16 rows (sampler_d.cu:10-49 semantics: NaN never
// wins, ties to the lowest index, an all-NaN row returns 0).
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(512) argmax_f16_kernel(const __half* __restrict__ logits,
                                                         int64_t V, int64_t* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const __half* base = logits + row * V;
  unsigned long long best = 0ull;
  const bool vec = ((reinterpret_cast<uintptr_t>(base) & 15u) == 0);
  int64_t i0 = 0;
  if (vec) {
    const int64_t nv = V / 8;
    for (int64_t c = threadIdx.x; c < nv; c += blockDim.x) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(base) + c);
      const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (__half2float(h[j]) > -FLT_MAX) {
          const unsigned long long k = pack_key(h[j], c * 8 + j);
          best = k > best ? k : best;
        }
      }
    }
    i0 = nv * 8;
  }
  for (int64_t i = i0 + threadIdx.x; i < V; i += blockDim.x) {
    const __half h = base[i];
    if (__half2float(h) > -FLT_MAX) {
      const unsigned long long k = pack_key(h, i);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  __shared__ unsigned long long red[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long v = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = red[w] > v ? red[w] : v;
    out[row] = v ? (int64_t)(0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull)) : 0;
  }
}

__global__ void unpack_argmax_kernel(const unsigned long long* __restrict__ packed, int64_t M,
                                     int64_t* __restrict__ ids) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M) return;
  const unsigned long long v = packed[i];
  ids[i] = v ? (int64_t)(0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull)) : 0;
}

// ----------------------------------------------------------------------------
// Launchers
// ----------------------------------------------------------------------------
template <int MT, bool ARGMAX>
static int launch_skinny_t(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                           int bias_dtype, __half* y, unsigned long long* packed,
                           int64_t vocab_offset, int M, int N, int K, cudaStream_t s) {
  const size_t smem = (size_t)MT * K * sizeof(float);
  if (smem > 200 * 1024) return DDQ_ERR_SHAPE;
  auto kern = gemv_skinny_kernel<MT, ARGMAX>;
  const int dev = current_device();
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, dev, kern, 200 * 1024);
  if (ast) return ast;
  const int sms = device_sm_count(dev);
  if (sms <= 0) return DDQ_ERR_DEVICE;
  const int per_sm = smem <= 48 * 1024 ? 4 : (smem <= 100 * 1024 ? 2 : 1);
  const int row_blocks = (N + 31) / 32;
  const int gx = row_blocks < sms * per_sm ? row_blocks : sms * per_sm;
  const int gy = (M + MT - 1) / MT;
  if (gy > 65535) return DDQ_ERR_SHAPE;
  kern<<<dim3(gx, gy), 256, smem, s>>>(x, wq, scales, bias, bias_dtype, y, packed, vocab_offset,
                                       M, N, K);
  return check_launch();
}

int launch_skinny(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                  int bias_dtype, __half* y, int M, int N, int K, cudaStream_t s) {
  if (M <= 1) return launch_skinny_t<1, false>(x, wq, scales, bias, bias_dtype, y, nullptr, 0, M, N, K, s);
  if (M <= 2) return launch_skinny_t<2, false>(x, wq, scales, bias, bias_dtype, y, nullptr, 0, M, N, K, s);
  return launch_skinny_t<4, false>(x, wq, scales, bias, bias_dtype, y, nullptr, 0, M, N, K, s);
}

int launch_skinny_argmax(const __half* x, const uint8_t* wq, const float* scales,
                         unsigned long long* packed, int64_t vocab_offset, int M, int N, int K,
                         cudaStream_t s) {
  if (M <= 1)
    return launch_skinny_t<1, true>(x, wq, scales, nullptr, 0, nullptr, packed, vocab_offset, M, N, K, s);
  if (M <= 2)
    return launch_skinny_t<2, true>(x, wq, scales, nullptr, 0, nullptr, packed, vocab_offset, M, N, K, s);
  return launch_skinny_t<4, true>(x, wq, scales, nullptr, 0, nullptr, packed, vocab_offset, M, N, K, s);
}

int launch_generic(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                   int bias_dtype, __half* y, int64_t M, int64_t N, int64_t K, cudaStream_t s) {
  const int64_t warps = N * ((M + 3) / 4);
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return DDQ_ERR_SHAPE;
  gemm_generic_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, wq, scales, bias, bias_dtype, y, M, N, K);
  return check_launch();
}

int launch_argmax_f16(const __half* logits, int64_t B, int64_t V, int64_t* out, cudaStream_t s) {
  if (B > 0x7fffffff) return DDQ_ERR_SHAPE;
  argmax_f16_kernel<<<(unsigned)B, 512, 0, s>>>(logits, V, out);
  return check_launch();
}

int launch_unpack_argmax(const unsigned long long* packed, int64_t M, int64_t* ids, cudaStream_t s) {
  const int64_t blocks = (M + 255) / 256;
  unpack_argmax_kernel<<<(unsigned)blocks, 256, 0, s>>>(packed, M, ids);
  return check_launch();
}

}  // namespace ddq
