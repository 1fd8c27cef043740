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
//     (up to 16 tiles each); a CTA copies its whole slice (rows x K bytes)
//     into shared memory before griddepcontrol.wait, one bulk copy (TMA
//     engine, no multicast) per row counted on an mbarrier; where the slice
//     and activations leave room, the next kernel's CTA shares the SM and
//     starts its own copy while this one computes;
//   * after the wait: the M x K fp16 activations (L2), one bulk copy per
//     token row, then per (tile, 64-wide K block) one 16-byte weight load,
//     8 exact e4m3 -> fp16x2 conversions and 4 MMAs, tokens on the MMA rows
//     (zero rows past M), the tile's 8 weight rows on the MMA columns;
//   * no activation split pre-pass (fp16 activations are used as they are),
//     no workspace; both mbarrier waits are bounded (DDQ_ERR_TIMEOUT in the
//     device error word, no output, on expiry).
//
// K order inside a 64-wide block: lane quad position t holds the 16
// consecutive k at 16t .. 16t+15 of its token row (A operand) and of its
// weight row (B operand); MMA j takes k 16t+4j .. 16t+4j+3 as the logical
// k {2t, 2t+1, 2t+8, 2t+9} of the m16n8k16 fragments.  A and B follow the
// same map, so each MMA adds the same products as in natural order, and one
// 16-byte load per operand feeds four MMAs.
//
// Conversion: the hardware converter (cvt.rn.f16x2.e4m3x2, one instruction per
// pair of weights; exact, subnormals included - it measured faster than the
// four-instruction integer form in the resident-slice kernel).  The eight warps split the (tile, K block) units
// round-robin, write their partial sums to shared memory and the epilogue
// adds them in warp order, so results are bitwise reproducible.
#include <cstdlib>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {
namespace {

constexpr int TH_WARPS = 8;
constexpr int TH_THREADS = TH_WARPS * 32;
constexpr int TH_MAX_TILES = 16;     // 8-row tiles per CTA (accumulator registers)
constexpr int TH_SMEM_MAX = 232448;  // 227 KB opt-in limit per CTA
// Shapes taken: at most this many (8-row tile, 64-wide K block) units per
// CTA, or any unit count at M <= 2, as long as shared memory holds the slice
// and the activations.  Per call in a replayed chain, against the split +
// e4m3 decode kernel: the Qwen2.5 q/k/v, o and down projections win at every
// M from 1 to 16 (14-76 units; e.g. M = 16 down 3.95 vs 6.02 us, M = 16
// 4864 x 896 4.16 vs 5.33 us); gate/up (126 units) wins at M = 1 (5.05 vs
// 5.43 us) and loses from M = 8 on (5.52 vs 5.39 us; M = 16 6.24 vs 5.44 us),
// where the per-CTA conversion and MMA work is on the critical path.
constexpr int64_t TH_MAX_UNITS = 96;

struct ThinArgs {
  const __half* x;
  const uint8_t* wq;
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  int M, N, K;
  int tiles;                 // ceil(N / 8)
  int sw, sx;                // shared-memory row strides (bytes) of weights and activations
  int off_x, off_sc, off_bi, off_red, off_bar;  // shared-memory offsets (bytes)
  unsigned long long timeout_ns;
  int trace;                 // debug flag bit 1: per-CTA phase stamps (trace_stamp)
};

// One bulk (TMA engine) copy global -> this CTA's shared memory, counted on
// an mbarrier (no multicast).  16-byte aligned addresses, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
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
//   [0, ...)   weight slice, row-major, row stride sw = K (+64 when K % 128
//              == 0, so that rows g and g + 1 fall on different banks)
//   off_x      activations, row-major fp16, row stride sx = 2K + 16 (rows
//              g and g + 1 on different banks)
//   off_sc     per-row scale (fp32), off_bi per-row bias (fp32)
//   off_red    partial sums [warp][m][tile][8 rows] (fp32); aliases the
//              weight and activation area, which is dead by then, when it fits
//   off_bar    weight barrier, activation barrier, abort flag
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
  const int KB = K >> 6;
  const int valid = min(rows, N - row0);  // rows past N are never stored
  const uint32_t bar_w = sbase + (uint32_t)a.off_bar, bar_x = bar_w + 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(th_smem + a.off_bar + 16);
  volatile int* drain_flag = reinterpret_cast<volatile int*>(th_smem + a.off_bar + 20);
  const bool tr = a.trace != 0;
  if (tid == 0) trace_stamp(tr, 0);
  if (tid == 0) {
    ptx::mbar_init(bar_w, 1);
    ptx::mbar_init(bar_x, 1);
    *abort_flag = 0;
    *drain_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  // 1) the weight slice, one bulk copy per row, before the dependency
  //    (weights are not written by the kernel this one depends on)
  if (tid == 0) ptx::mbar_arrive_expect_tx(bar_w, (uint32_t)(valid * K));
  if (tid < valid)
    bulk_g2s(sbase + (uint32_t)(tid * a.sw), a.wq + (size_t)(row0 + tid) * K, (uint32_t)K, bar_w);
  if (tid == 0) trace_stamp(tr, 2);

  ptx::pdl_wait();  // x comes from the previous kernel
  ptx::pdl_launch_dependents();
  if (tid == 0) trace_stamp(tr, 3);

  // 2) activations (L2), one bulk copy per token row; row scales and biases
  const uint32_t sx = sbase + (uint32_t)a.off_x;
  if (tid == 0) ptx::mbar_arrive_expect_tx(bar_x, (uint32_t)(M * K * 2));
  if (tid < M)
    bulk_g2s(sx + (uint32_t)(tid * a.sx), a.x + (size_t)tid * K, (uint32_t)(K * 2), bar_x);
  float* sc = reinterpret_cast<float*>(th_smem + a.off_sc);
  float* bi = reinterpret_cast<float*>(th_smem + a.off_bi);
  if (tid < rows) {
    const int n = row0 + tid;
    float s = 0.f, bv = 0.f;
    if (n < N) {
      s = a.scales[n] * kE4m3ToF16Scale<true>;
      if (a.bias_dtype == DDQ_DTYPE_F16) bv = __half2float(reinterpret_cast<const __half*>(a.bias)[n]);
      else if (a.bias_dtype == DDQ_DTYPE_F32) bv = reinterpret_cast<const float*>(a.bias)[n];
    }
    sc[tid] = s;
    bi[tid] = bv;
  }
  // bounded waits: on a timeout the CTA records DDQ_ERR_TIMEOUT, waits once
  // more (bounded) for its copies and leaves without writing y
  if (ptx::mbar_wait(bar_w, 0u, a.timeout_ns, abort_flag))
    ptx::mbar_wait(bar_x, 0u, a.timeout_ns, abort_flag);
  __syncthreads();
  if (tid == 0) trace_stamp(tr, 5);
  if (*abort_flag) {
    if (tid == 0) {
      record_device_error(DDQ_ERR_TIMEOUT);
      ptx::mbar_wait(bar_w, 0u, a.timeout_ns, drain_flag);
      ptx::mbar_wait(bar_x, 0u, a.timeout_ns, drain_flag);
    }
    return;
  }

  // 3) MMAs: warp w takes the units u = tl * KB + kb with u = w (mod 8)
  const int g = lane >> 2, t = lane & 3;
  const bool lo_ok = g < M, hi_ok = g + 8 < M;
  const uint32_t wrow = sbase + (uint32_t)(g * a.sw + t * 16);
  const uint32_t wtile = (uint32_t)(8 * a.sw);
  const uint32_t xlo = sx + (uint32_t)(g * a.sx + t * 32);
  const uint32_t xhi = sx + (uint32_t)((g + 8) * a.sx + t * 32);
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
  for (int tl = 0; tl < NT; ++tl) {
    if (tl < ntl) {
      int kb = (warp - (tl * KB) % TH_WARPS + TH_WARPS) % TH_WARPS;
      for (; kb < KB; kb += TH_WARPS) {
        const uint4 wv = lds128(wrow + (uint32_t)tl * wtile + (uint32_t)(kb * 64));
        uint4 l0 = make_uint4(0u, 0u, 0u, 0u), l1 = l0, h0 = l0, h1 = l0;
        if (lo_ok) {
          l0 = lds128(xlo + (uint32_t)(kb * 128));
          l1 = lds128(xlo + (uint32_t)(kb * 128 + 16));
        }
        if (hi_ok) {
          h0 = lds128(xhi + (uint32_t)(kb * 128));
          h1 = lds128(xhi + (uint32_t)(kb * 128 + 16));
        }
        uint32_t b[8];
        e4m3x4_to_half2x2<true>(wv.x, b[0], b[1]);
        e4m3x4_to_half2x2<true>(wv.y, b[2], b[3]);
        e4m3x4_to_half2x2<true>(wv.z, b[4], b[5]);
        e4m3x4_to_half2x2<true>(wv.w, b[6], b[7]);
        th_mma(acc[tl], l0.x, h0.x, l0.y, h0.y, b[0], b[1]);
        th_mma(acc[tl], l0.z, h0.z, l0.w, h0.w, b[2], b[3]);
        th_mma(acc[tl], l1.x, h1.x, l1.y, h1.y, b[4], b[5]);
        th_mma(acc[tl], l1.z, h1.z, l1.w, h1.w, b[6], b[7]);
      }
    }
  }
  __syncthreads();  // weights and activations are dead: the partial sums may alias them
  if (tid == 0) trace_stamp(tr, 4);

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
  if (tr) {
    __syncthreads();
    if (tid == 0) {
      trace_stamp(tr, 6);
      trace_stamp(tr, 7);
    }
  }
}

// Unit limit of the shapes taken at M > 2 (DDQ_THIN_MAX_UNITS overrides it
// for measurements).
int64_t thin_max_units() {
  static const int64_t v = [] {
    const char* e = std::getenv("DDQ_THIN_MAX_UNITS");
    return e ? (int64_t)std::atoll(e) : TH_MAX_UNITS;
  }();
  return v;
}

struct ThinPlan {
  bool ok;
  int grid, nt, smem;
  int sw, sx;
  int off_x, off_sc, off_bi, off_red, off_bar;
};

ThinPlan thin_plan(int64_t M, int64_t N, int64_t K, int sms) {
  ThinPlan p{};
  if (M < 1 || M > 16 || N < 1 || K < 64 || K % 64 != 0 || sms <= 0) return p;
  if (N > 0x7fffffff - 8 || K > (1 << 20)) return p;
  const int64_t tiles = (N + 7) / 8;
  const int64_t grid = tiles < sms ? tiles : sms;
  const int64_t ntl = (tiles + grid - 1) / grid;  // largest per-CTA tile count
  if (ntl > TH_MAX_TILES) return p;
  if (M > 2 && ntl * (K / 64) > thin_max_units()) return p;
  const int64_t sw = K % 128 == 0 ? K + 64 : K;
  const int64_t sx = 2 * K + 16;
  const int64_t w_bytes = ntl * 8 * sw;
  const int64_t x_bytes = M * sx;
  const int64_t off_sc = w_bytes + x_bytes;                    // multiple of 16
  const int64_t off_bi = off_sc + ntl * 8 * 4;
  const int64_t end = off_bi + ntl * 8 * 4;
  const int64_t red_bytes = (int64_t)TH_WARPS * M * ntl * 8 * 4;
  const int64_t off_red = red_bytes <= w_bytes + x_bytes ? 0 : end;
  const int64_t off_bar = off_red ? off_red + red_bytes : end;  // multiple of 16
  const int64_t total = off_bar + 32;
  if (total > TH_SMEM_MAX) return p;
  p.ok = true;
  p.grid = (int)grid;
  p.nt = ntl <= 1 ? 1 : ntl <= 2 ? 2 : ntl <= 4 ? 4 : ntl <= 8 ? 8 : ntl <= 12 ? 12 : 16;
  p.smem = (int)total;
  p.sw = (int)sw;
  p.sx = (int)sx;
  p.off_x = (int)w_bytes;
  p.off_sc = (int)off_sc;
  p.off_bi = (int)off_bi;
  p.off_red = (int)off_red;
  p.off_bar = (int)off_bar;
  return p;
}

template <int NT>
int launch_thin_t(const ThinPlan& p, const ThinArgs& a, cudaStream_t s) {
  // the launch's own size still sets the occupancy
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), w8a16_thin_kernel<NT>, TH_SMEM_MAX);
  if (ast) return ast;
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
                int bias_dtype, __half* y, int M, int N, int K, unsigned long long timeout_ns,
                cudaStream_t s, int debug_flags) {
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
  a.sw = p.sw;
  a.sx = p.sx;
  a.off_x = p.off_x;
  a.off_sc = p.off_sc;
  a.off_bi = p.off_bi;
  a.off_red = p.off_red;
  a.off_bar = p.off_bar;
  a.timeout_ns = timeout_ns;
  a.trace = (debug_flags & 2) != 0;
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
