// thin.cu - W8A16 GEMM for 1..16 tokens: every SM holds a slice of the
// weight in shared memory before the grid dependency resolves, then runs the
// whole K on the legacy tensor path (mma.sync m16n8k16, fp16 operands, fp32
// accumulation).
//
// Semantics are those of the reference's f8_forward (gemm_FP8_d.cu:171-210,
// the decode-shape calls of engine.py's projections), like every other path
// of ddq_w8a16_gemm:
//   y[m, n] = fp16( (sum_k x[m, k] * e4m3(W[n, k])) * scale[n] + bias[n] )
// with the sum in fp32.
//
// Why a kernel of its own: at a handful of tokens the weight stream is the
// whole job, and the e4m3 tensor-core decode kernel (tc_decode.cu) tiles the
// weight in 128-row blocks, which for the Qwen2.5-0.5B gate/up (9728 rows)
// busies 76 of 148 SMs and can start only a ring's depth of the stream
// before the dependency resolves.  Here:
//   * the weight is cut into 8-row tiles spread evenly over one CTA per SM
//     (up to 16 tiles each); a CTA copies its whole slice (rows x K bytes,
//     at most 40 KB) into shared memory with cp.async before
//     griddepcontrol.wait, which leaves room for the next kernel's CTA on the
//     same SM, so that it starts its own copy while this one computes;
//   * after the wait: the M x K fp16 activations (L2, at most 10 KB) into
//     shared memory, then per (tile, 64-wide K block) one 16-byte weight
//     load, 16 exact e4m3 -> fp16 conversions and 4 MMAs, tokens on the MMA
//     rows (zero rows past M), the tile's 8 weight rows on the MMA columns;
//   * no activation split pre-pass (fp16 activations are used as they are),
//     no spin-wait of any kind (cp.async.wait_all and griddepcontrol.wait
//     always complete), no workspace.
//
// K order inside a 64-wide block: lane quad position t holds the 16
// consecutive k at 16t .. 16t+15 of its token row (A operand) and of its
// weight row (B operand); MMA j takes k 16t+4j .. 16t+4j+3 as the logical
// k {2t, 2t+1, 2t+8, 2t+9} of the m16n8k16 fragments.  A and B follow the
// same map, so each MMA adds the same products as in natural order, and one
// 16-byte load per operand feeds four MMAs.
//
// Conversion: e4m3x2_to_half2_bits_x2m8 (integer ALU ops) gives each weight
// times 2^-8 exactly, subnormals included; the factor 256 is folded into the
// row scale (exact).  The eight warps split the (tile, K block) units
// round-robin, write their partial sums to shared memory and the epilogue
// adds them in warp order, so results are bitwise reproducible.
#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {
namespace {

constexpr int TH_WARPS = 8;
constexpr int TH_THREADS = TH_WARPS * 32;
constexpr int TH_MAX_TILES = 16;     // 8-row tiles per CTA (accumulator registers)
constexpr int TH_SMEM_MAX = 232448;  // 227 KB opt-in limit per CTA
// Shapes taken: per CTA at most this much weight slice and activations.
// Staged by per-thread cp.async (16 B each), larger slices and activation
// blocks were measured slower than the e4m3 decode kernel (M = 1 gate/up,
// 64.5 KB slice: 7.2 vs 6.9 us; M = 8: 9.8 vs 6.6 us; M = 8 down, 78 KB of
// activations: 11.1 vs 6.9 us), smaller ones faster (M = 1 qkv, 7 KB + 1.8 KB:
// 3.8 vs 5.7 us; M = 1 down, 38.9 KB + 9.7 KB: 4.9 vs 6.6 us).
constexpr int64_t TH_W_MAX = 40 * 1024;
constexpr int64_t TH_X_MAX = 10 * 1024;

struct ThinArgs {
  const __half* x;
  const uint8_t* wq;
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  int M, N, K;
  int tiles;        // ceil(N / 8)
  int off_x, off_sc, off_bi, off_red;  // shared-memory offsets (bytes)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128_zero(uint32_t a) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
}

// d += A (16 x 16, row-major fragment a0..a3) * B (16 x 8, column fragment b0, b1)
__device__ __forceinline__ void th_mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared memory (bytes from the dynamic base):
//   [0, ...)   weight slice: unit (tile tl, K block kb) = 512 B at
//              (tl * KB + kb) * 512; lane g * 4 + t holds row tl * 8 + g,
//              k = kb * 64 + 16 t .. + 15
//   off_x      activations: 16 B at (((kb * 2 + h) * M + m) * 4 + t) * 16
//              = x[m, kb * 64 + 16 t + 8 h .. + 7]
//   off_sc     per-row scale * 256 (fp32), off_bi per-row bias (fp32)
//   off_red    partial sums [warp][m][tile][8 rows] (fp32); aliases the
//              weight and activation area, which is dead by then, when it fits
template <int NT>
__global__ void __launch_bounds__(TH_THREADS) w8a16_thin_kernel(const ThinArgs a) {
  extern __shared__ __align__(16) uint8_t th_smem[];
  const uint32_t sbase = ptx::smem_u32(th_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  const int tile0 = (int)(((int64_t)b * a.tiles) / G);
  const int tile1 = (int)(((int64_t)(b + 1) * a.tiles) / G);
  const int ntl = tile1 - tile0;  // 1..NT (the launcher guarantees it)
  const int row0 = tile0 * 8, rows = ntl * 8;
  const int M = a.M, N = a.N, K = a.K;
  const int KB = K >> 6, kc16 = K >> 4, kc8 = K >> 3;

  // 1) the weight slice, before the dependency (weights are not written by
  //    the kernel this one depends on)
  for (int rl = warp; rl < rows; rl += TH_WARPS) {
    const int n = row0 + rl;
    const uint8_t* src = a.wq + (size_t)n * K;
    const uint32_t rbase = sbase + (uint32_t)(((rl >> 3) * KB * 32 + (rl & 7) * 4) * 16);
    for (int c = lane; c < kc16; c += 32) {
      const uint32_t dst = rbase + (uint32_t)((((c >> 2) * 32) + (c & 3)) * 16);
      if (n < N) cp_async16(dst, src + (size_t)c * 16);
      else sts128_zero(dst);
    }
  }
  cp_async_commit();

  ptx::pdl_wait();  // x comes from the previous kernel
  ptx::pdl_launch_dependents();

  // 2) activations (L2), row scales and biases
  const uint32_t sx = sbase + (uint32_t)a.off_x;
  for (int m = warp; m < M; m += TH_WARPS) {
    const __half* src = a.x + (size_t)m * K;
    for (int c = lane; c < kc8; c += 32) {
      const int kb = c >> 3, t = (c & 7) >> 1, h = c & 1;
      cp_async16(sx + (uint32_t)(((((kb * 2 + h) * M + m) * 4) + t) * 16), src + (size_t)c * 8);
    }
  }
  cp_async_commit();
  float* sc = reinterpret_cast<float*>(th_smem + a.off_sc);
  float* bi = reinterpret_cast<float*>(th_smem + a.off_bi);
  if (tid < rows) {
    const int n = row0 + tid;
    float s = 0.f, bv = 0.f;
    if (n < N) {
      s = a.scales[n] * 256.f;
      if (a.bias_dtype == DDQ_DTYPE_F16) bv = __half2float(reinterpret_cast<const __half*>(a.bias)[n]);
      else if (a.bias_dtype == DDQ_DTYPE_F32) bv = reinterpret_cast<const float*>(a.bias)[n];
    }
    sc[tid] = s;
    bi[tid] = bv;
  }
  cp_async_wait_all();
  __syncthreads();

  // 3) MMAs: warp w takes the units u = tl * KB + kb with u = w (mod 8)
  const int g = lane >> 2, t = lane & 3;
  const bool lo_ok = g < M, hi_ok = g + 8 < M;
  const uint32_t xlo = sx + (uint32_t)((g * 4 + t) * 16);
  const uint32_t xhi = sx + (uint32_t)(((g + 8) * 4 + t) * 16);
  const uint32_t xstep = (uint32_t)(M * 64);  // bytes per (kb, h)
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
  for (int tl = 0; tl < NT; ++tl) {
    if (tl < ntl) {
      int kb = (warp - (tl * KB) % TH_WARPS + TH_WARPS) % TH_WARPS;
      for (; kb < KB; kb += TH_WARPS) {
        const uint4 wv = lds128(sbase + (uint32_t)(((tl * KB + kb) * 32 + lane) * 16));
        uint4 l0 = make_uint4(0u, 0u, 0u, 0u), l1 = l0, h0 = l0, h1 = l0;
        if (lo_ok) {
          l0 = lds128(xlo + (uint32_t)(kb * 2) * xstep);
          l1 = lds128(xlo + (uint32_t)(kb * 2 + 1) * xstep);
        }
        if (hi_ok) {
          h0 = lds128(xhi + (uint32_t)(kb * 2) * xstep);
          h1 = lds128(xhi + (uint32_t)(kb * 2 + 1) * xstep);
        }
        th_mma(acc[tl], l0.x, h0.x, l0.y, h0.y, e4m3x2_to_half2_bits_x2m8(wv.x, 0x4140u),
               e4m3x2_to_half2_bits_x2m8(wv.x, 0x4342u));
        th_mma(acc[tl], l0.z, h0.z, l0.w, h0.w, e4m3x2_to_half2_bits_x2m8(wv.y, 0x4140u),
               e4m3x2_to_half2_bits_x2m8(wv.y, 0x4342u));
        th_mma(acc[tl], l1.x, h1.x, l1.y, h1.y, e4m3x2_to_half2_bits_x2m8(wv.z, 0x4140u),
               e4m3x2_to_half2_bits_x2m8(wv.z, 0x4342u));
        th_mma(acc[tl], l1.z, h1.z, l1.w, h1.w, e4m3x2_to_half2_bits_x2m8(wv.w, 0x4140u),
               e4m3x2_to_half2_bits_x2m8(wv.w, 0x4342u));
      }
    }
  }
  __syncthreads();  // weights and activations are dead: the partial sums may alias them

  // 4) partial sums [warp][m][tile][row], then the warp-ordered sum
  float* red = reinterpret_cast<float*>(th_smem + a.off_red);
#pragma unroll
  for (int tl = 0; tl < NT; ++tl) {
    if (tl < ntl) {
      if (lo_ok)
        *reinterpret_cast<float2*>(red + (((size_t)warp * M + g) * ntl + tl) * 8 + 2 * t) =
            make_float2(acc[tl][0], acc[tl][1]);
      if (hi_ok)
        *reinterpret_cast<float2*>(red + (((size_t)warp * M + g + 8) * ntl + tl) * 8 + 2 * t) =
            make_float2(acc[tl][2], acc[tl][3]);
    }
  }
  __syncthreads();
  const int per_w = M * rows;  // floats per warp
  for (int i = tid; i < per_w; i += TH_THREADS) {
    const int m = i / rows, rl = i - m * rows;
    const int n = row0 + rl;
    if (n < N) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < TH_WARPS; ++w) s += red[(size_t)w * per_w + i];
      a.y[(size_t)m * N + n] = __float2half_rn(fmaf(s, sc[rl], bi[rl]));
    }
  }
}

struct ThinPlan {
  bool ok;
  int grid, nt, smem;
  int off_x, off_sc, off_bi, off_red;
};

ThinPlan thin_plan(int64_t M, int64_t N, int64_t K, int sms) {
  ThinPlan p{};
  if (M < 1 || M > 16 || N < 1 || K < 64 || K % 64 != 0 || sms <= 0) return p;
  if (N > 0x7fffffff - 8 || K > (1 << 20)) return p;
  const int64_t tiles = (N + 7) / 8;
  const int64_t grid = tiles < sms ? tiles : sms;
  const int64_t ntl = (tiles + grid - 1) / grid;  // largest per-CTA tile count
  if (ntl > TH_MAX_TILES) return p;
  const int64_t w_bytes = ntl * 8 * K;
  const int64_t x_bytes = M * K * 2;
  if (w_bytes > TH_W_MAX || x_bytes > TH_X_MAX) return p;
  const int64_t off_sc = w_bytes + x_bytes;                    // multiple of 16
  const int64_t off_bi = off_sc + ntl * 8 * 4;
  const int64_t end = off_bi + ntl * 8 * 4;
  const int64_t red_bytes = (int64_t)TH_WARPS * M * ntl * 8 * 4;
  const int64_t off_red = red_bytes <= w_bytes + x_bytes ? 0 : end;
  const int64_t total = off_red ? off_red + red_bytes : end;
  if (total > TH_SMEM_MAX) return p;
  p.ok = true;
  p.grid = (int)grid;
  p.nt = ntl <= 1 ? 1 : ntl <= 2 ? 2 : ntl <= 4 ? 4 : ntl <= 8 ? 8 : ntl <= 12 ? 12 : 16;
  p.smem = (int)total;
  p.off_x = (int)w_bytes;
  p.off_sc = (int)off_sc;
  p.off_bi = (int)off_bi;
  p.off_red = (int)off_red;
  return p;
}

template <int NT>
int launch_thin_t(const ThinPlan& p, const ThinArgs& a, cudaStream_t s) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return DDQ_ERR_DEVICE;
  // Raise the dynamic shared-memory limit once per device (not a stream
  // operation; the launch's own size still sets the occupancy).
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(w8a16_thin_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TH_SMEM_MAX) != cudaSuccess) {
      cudaGetLastError();
      return DDQ_ERR_LAUNCH;
    }
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(TH_THREADS);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_thin_kernel<NT>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace

bool thin_eligible(int64_t M, int64_t N, int64_t K, int sms) {
  return thin_plan(M, N, K, sms).ok;
}

int launch_thin(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                int bias_dtype, __half* y, int M, int N, int K, cudaStream_t s) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  const ThinPlan p = thin_plan(M, N, K, sms);
  if (!p.ok) return DDQ_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(wq)) return DDQ_ERR_ALIGNMENT;
  ThinArgs a{};
  a.x = x;
  a.wq = wq;
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles = (int)((N + 7) / 8);
  a.off_x = p.off_x;
  a.off_sc = p.off_sc;
  a.off_bi = p.off_bi;
  a.off_red = p.off_red;
  switch (p.nt) {
    case 1: return launch_thin_t<1>(p, a, s);
    case 2: return launch_thin_t<2>(p, a, s);
    case 4: return launch_thin_t<4>(p, a, s);
    case 8: return launch_thin_t<8>(p, a, s);
    case 12: return launch_thin_t<12>(p, a, s);
    default: return launch_thin_t<16>(p, a, s);
  }
}

}  // namespace ddq
