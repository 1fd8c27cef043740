// rs.cu - W8A16 GEMM for 1..16 tokens with every CTA's slice of the weight
// resident in shared memory before the grid dependency resolves, the weight
// rows on the MMA's 16-row A operand and the tokens on its 8-column B
// operand (mma.sync m16n8k16, fp16 operands, fp32 accumulation).
//
// Semantics are those of the reference's f8_forward (gemm_FP8_d.cu:171-210):
//   y[m, n] = fp16( (sum_k x[m, k] * e4m3(W[n, k])) * scale[n] + bias[n] )
// with the sum in fp32.
//
// What bounds a chain of dependent small GEMMs is the work left after the
// grid dependency resolves, not the weight bytes; this kernel keeps that
// work short and lets the next GEMM stream its weights during it:
//   * each CTA owns a contiguous run of 16-row tiles; its weight slice is one
//     contiguous range of global memory, fetched with ONE bulk copy (the TMA
//     engine at full rate: a copy per 896-byte row streams at about half the
//     speed of one large copy when one CTA per SM issues them);
//   * the CTA signals griddepcontrol.launch_dependents at entry, so the next
//     kernel's CTAs are scheduled as soon as every CTA of this one runs and,
//     where shared memory leaves room, stream their own slices meanwhile;
//   * after the dependency: one bulk copy of all of x (M x K fp16,
//     contiguous), then warp w runs the 64-wide K blocks kb = w, w + 8, ...
//     of all its tiles (tile by tile; ordering the MMAs so that consecutive
//     ones never share an accumulator measured slower), then a
//     warp-ordered sum of the 8 partials per output, scale, bias, fp16.
// Weights on the A operand: one MMA covers 16 weight rows x 8 tokens, so at
// up to 8 tokens it takes half the MMAs (and the same e4m3 conversions) of
// tokens-on-rows; 9..16 tokens use two 8-token blocks per A fragment.
//
// K order inside a 64-wide block: lane quad position t holds the 16
// consecutive k at 16t .. 16t+15 of its weight rows (A) and of its token's
// activations (B); MMA j takes k 16t+4j .. 16t+4j+3 as the fragment's logical
// k {2t, 2t+1, 2t+8, 2t+9}.  A and B follow the same map, so each MMA adds
// the same products as in natural order, and one 16-byte weight load per
// row feeds four MMAs.  The e4m3 -> fp16 conversion is the hardware
// converter (one instruction per pair, exact, subnormals included; it
// measured faster than the integer-ALU form, which DDQ_E4M3_CVT=int selects
// and whose factor 2^-8 the row scale then undoes).  Results are bitwise
// reproducible (fixed warp-ordered sum).
#include <cstdlib>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {
namespace {

constexpr int RS_WARPS = 8;
constexpr int RS_THREADS = RS_WARPS * 32;
constexpr int RS_TILE = 16;          // weight rows per MMA tile
// tiles per CTA: the accumulators and the K block's raw weight words of every
// tile stay in registers (no spills up to 6 tiles at 1..8 tokens, 5 at 9..16)
constexpr int RS_MAX_TILES = 6;
constexpr int RS_SMEM_MAX = 232448;  // 227 KB opt-in limit per CTA

struct RsArgs {
  const __half* x;
  const uint8_t* wq;
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  int M, N, K;
  int tiles;                                 // ceil(N / 16)
  int off_x, off_sc, off_bi, off_bar;        // shared-memory offsets (bytes)
  unsigned long long timeout_ns;
  int trace;                                 // debug flag bit 1: phase stamps
};

__device__ __forceinline__ void rs_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint4 rs_lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
// d += A (16 x 16 fragment a0..a3) * B (16 x 8 fragment b0, b1)
__device__ __forceinline__ void rs_mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared memory (bytes from the dynamic base):
//   [0, rows * K)   the weight slice, row-major (rows past N zero-filled);
//                   after the MMAs, the partial sums [warp][NB * 8][rows]
//                   fp32 reuse it
//   off_x           x, row-major fp16 [M][K] (one bulk copy)
//   off_sc, off_bi  per-row scale (times 256 with the integer conversion) and
//                   bias (fp32)
//   off_bar         weight barrier, activation barrier, abort and drain flags
template <int NT, int NB, bool HW>
__global__ void __launch_bounds__(RS_THREADS, 2) w8a16_rs_kernel(const RsArgs a) {
  extern __shared__ __align__(128) uint8_t rs_smem[];
  const uint32_t sbase = ptx::smem_u32(rs_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  const int tile0 = (int)(((int64_t)b * a.tiles) / G);
  const int ntl = (int)(((int64_t)(b + 1) * a.tiles) / G) - tile0;  // 1..NT
  const int row0 = tile0 * RS_TILE, rows = ntl * RS_TILE;
  const int M = a.M, N = a.N, K = a.K, KB = K >> 6;
  const int valid = min(rows, N - row0);
  const uint32_t bar_w = sbase + (uint32_t)a.off_bar, bar_x = bar_w + 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(rs_smem + a.off_bar + 16);
  volatile int* drain_flag = reinterpret_cast<volatile int*>(rs_smem + a.off_bar + 20);
  const bool tr = a.trace != 0;
  if (tid == 0) {
    trace_stamp(tr, 0);
    ptx::mbar_init(bar_w, 1);
    ptx::mbar_init(bar_x, 1);
    *abort_flag = 0;
    *drain_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  // 1) the weight slice: one bulk copy of its contiguous bytes (weights are
  //    never written by the kernel this one depends on), then let the next
  //    kernel be scheduled
  if (tid == 0) {
    ptx::mbar_arrive_expect_tx(bar_w, (uint32_t)(valid * K));
    rs_bulk_g2s(sbase, a.wq + (size_t)row0 * K, (uint32_t)(valid * K), bar_w);
    trace_stamp(tr, 2);
  }
  ptx::pdl_launch_dependents();
  // rows past N (the last CTA's partial tile) read as zero; the bulk copy
  // does not touch them
  for (int i = valid * K / 16 + tid; i < rows * K / 16; i += RS_THREADS)
    reinterpret_cast<uint4*>(rs_smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  float* sc = reinterpret_cast<float*>(rs_smem + a.off_sc);
  float* bi = reinterpret_cast<float*>(rs_smem + a.off_bi);
  if (tid < rows) {
    const int n = row0 + tid;
    float s = 0.f, bv = 0.f;
    if (n < N) {
      s = a.scales[n] * kE4m3ToF16Scale<HW>;
      if (a.bias_dtype == DDQ_DTYPE_F16) bv = __half2float(reinterpret_cast<const __half*>(a.bias)[n]);
      else if (a.bias_dtype == DDQ_DTYPE_F32) bv = reinterpret_cast<const float*>(a.bias)[n];
    }
    sc[tid] = s;
    bi[tid] = bv;
  }

  // 2) x comes from the previous kernel: one bulk copy once it has finished
  ptx::pdl_wait();
  if (tid == 0) {
    trace_stamp(tr, 3);
    ptx::mbar_arrive_expect_tx(bar_x, (uint32_t)(M * K * 2));
    rs_bulk_g2s(sbase + (uint32_t)a.off_x, a.x, (uint32_t)(M * K * 2), bar_x);
  }
  // bounded waits: on a timeout the CTA records DDQ_ERR_TIMEOUT, waits once
  // more (bounded) for its copies and leaves without writing y
  if (ptx::mbar_wait(bar_w, 0u, a.timeout_ns, abort_flag))
    ptx::mbar_wait(bar_x, 0u, a.timeout_ns, abort_flag);
  __syncthreads();
  if (*abort_flag) {
    if (tid == 0) {
      record_device_error(DDQ_ERR_TIMEOUT);
      ptx::mbar_wait(bar_w, 0u, a.timeout_ns, drain_flag);
      ptx::mbar_wait(bar_x, 0u, a.timeout_ns, drain_flag);
    }
    return;
  }
  if (tid == 0) trace_stamp(tr, 5);

  // 3) MMAs: warp w takes the K blocks kb = w, w + 8, ... of every tile
  const int g = lane >> 2, t = lane & 3;
  const uint32_t wlo = sbase + (uint32_t)(g * K + t * 16);
  const uint32_t whi = wlo + (uint32_t)(8 * K);
  const uint32_t tstride = (uint32_t)(RS_TILE * K);
  uint32_t xrow[NB];
  bool xok[NB];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const int tok = nb * 8 + g;
    xok[nb] = tok < M;
    xrow[nb] = sbase + (uint32_t)a.off_x + (uint32_t)((xok[nb] ? tok : 0) * K * 2 + t * 32);
  }
  float acc[NT][NB][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) acc[i][nb][0] = acc[i][nb][1] = acc[i][nb][2] = acc[i][nb][3] = 0.f;
  for (int kb = warp; kb < KB; kb += RS_WARPS) {
    uint4 x0[NB], x1[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      x0[nb] = make_uint4(0u, 0u, 0u, 0u);
      x1[nb] = x0[nb];
      if (xok[nb]) {
        x0[nb] = rs_lds128(xrow[nb] + (uint32_t)(kb * 128));
        x1[nb] = rs_lds128(xrow[nb] + (uint32_t)(kb * 128 + 16));
      }
    }
#pragma unroll
    for (int tl = 0; tl < NT; ++tl) {
      if (tl < ntl) {
        const uint4 lo = rs_lds128(wlo + (uint32_t)tl * tstride + (uint32_t)(kb * 64));
        const uint4 hi = rs_lds128(whi + (uint32_t)tl * tstride + (uint32_t)(kb * 64));
        const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
        const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_half2x2<HW>(lw[j], a0, a2);
          e4m3x4_to_half2x2<HW>(hw[j], a1, a3);
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint32_t xs[8] = {x0[nb].x, x0[nb].y, x0[nb].z, x0[nb].w,
                                    x1[nb].x, x1[nb].y, x1[nb].z, x1[nb].w};
            rs_mma(acc[tl][nb], a0, a1, a2, a3, xs[2 * j], xs[2 * j + 1]);
          }
        }
      }
    }
  }
  __syncthreads();  // the weight slice is dead: the partial sums reuse it
  if (tid == 0) trace_stamp(tr, 4);

  // 4) partial sums [warp][token NB*8][row] (row-contiguous, so the final
  //    sum's consecutive threads read consecutive words), then the
  //    warp-ordered sum
  constexpr int TOK = NB * 8;
  float* red = reinterpret_cast<float*>(rs_smem);
#pragma unroll
  for (int tl = 0; tl < NT; ++tl) {
    if (tl < ntl) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        float* p = red + ((size_t)warp * TOK + nb * 8 + 2 * t) * rows + tl * RS_TILE + g;
        p[0] = acc[tl][nb][0];
        p[rows] = acc[tl][nb][1];
        p[8] = acc[tl][nb][2];
        p[rows + 8] = acc[tl][nb][3];
      }
    }
  }
  __syncthreads();
  const int per_w = rows * TOK;  // floats per warp
  for (int i = tid; i < rows * M; i += RS_THREADS) {
    const int m = i / rows, rl = i - m * rows;  // consecutive threads: consecutive rows
    const int n = row0 + rl;
    if (n < N) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < RS_WARPS; ++w) s += red[(size_t)w * per_w + (size_t)m * rows + rl];
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

// ----------------------------------------------------------------------------
// 17..64 tokens: warps over token blocks
// ----------------------------------------------------------------------------
// Same resident weight slice and bulk-copied activations, but the 8 warps
// form a grid of NBW token blocks of 8 tokens x KSW = 8 / NBW K slices:
// warp w takes token block w mod NBW and the 64-wide K blocks kb = w / NBW
// (mod KSW) of every tile.  Each warp then owns its tokens' outputs (no
// cross-warp sum at all at 64 tokens, a sum of two slices at 17..32), at the
// price of converting every weight once per token block - cheap with the
// hardware converter - instead of holding 8 token blocks of accumulators.
template <int NT, int NBW, bool HW>
__global__ void __launch_bounds__(RS_THREADS, 1) w8a16_rsw_kernel(const RsArgs a) {
  constexpr int KSW = RS_WARPS / NBW;
  extern __shared__ __align__(128) uint8_t rs_smem[];
  const uint32_t sbase = ptx::smem_u32(rs_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  const int tile0 = (int)(((int64_t)b * a.tiles) / G);
  const int ntl = (int)(((int64_t)(b + 1) * a.tiles) / G) - tile0;  // 1..NT
  const int row0 = tile0 * RS_TILE, rows = ntl * RS_TILE;
  const int M = a.M, N = a.N, K = a.K, KB = K >> 6;
  const int valid = min(rows, N - row0);
  const uint32_t bar_w = sbase + (uint32_t)a.off_bar, bar_x = bar_w + 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(rs_smem + a.off_bar + 16);
  volatile int* drain_flag = reinterpret_cast<volatile int*>(rs_smem + a.off_bar + 20);
  const bool tr = a.trace != 0;
  if (tid == 0) {
    trace_stamp(tr, 0);
    ptx::mbar_init(bar_w, 1);
    ptx::mbar_init(bar_x, 1);
    *abort_flag = 0;
    *drain_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    ptx::mbar_arrive_expect_tx(bar_w, (uint32_t)(valid * K));
    rs_bulk_g2s(sbase, a.wq + (size_t)row0 * K, (uint32_t)(valid * K), bar_w);
    trace_stamp(tr, 2);
  }
  ptx::pdl_launch_dependents();
  for (int i = valid * K / 16 + tid; i < rows * K / 16; i += RS_THREADS)
    reinterpret_cast<uint4*>(rs_smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  float* sc = reinterpret_cast<float*>(rs_smem + a.off_sc);
  float* bi = reinterpret_cast<float*>(rs_smem + a.off_bi);
  if (tid < rows) {
    const int n = row0 + tid;
    float s = 0.f, bv = 0.f;
    if (n < N) {
      s = a.scales[n] * kE4m3ToF16Scale<HW>;
      if (a.bias_dtype == DDQ_DTYPE_F16) bv = __half2float(reinterpret_cast<const __half*>(a.bias)[n]);
      else if (a.bias_dtype == DDQ_DTYPE_F32) bv = reinterpret_cast<const float*>(a.bias)[n];
    }
    sc[tid] = s;
    bi[tid] = bv;
  }
  ptx::pdl_wait();
  if (tid == 0) {
    trace_stamp(tr, 3);
    ptx::mbar_arrive_expect_tx(bar_x, (uint32_t)(M * K * 2));
    rs_bulk_g2s(sbase + (uint32_t)a.off_x, a.x, (uint32_t)(M * K * 2), bar_x);
  }
  if (ptx::mbar_wait(bar_w, 0u, a.timeout_ns, abort_flag))
    ptx::mbar_wait(bar_x, 0u, a.timeout_ns, abort_flag);
  __syncthreads();
  if (*abort_flag) {
    if (tid == 0) {
      record_device_error(DDQ_ERR_TIMEOUT);
      ptx::mbar_wait(bar_w, 0u, a.timeout_ns, drain_flag);
      ptx::mbar_wait(bar_x, 0u, a.timeout_ns, drain_flag);
    }
    return;
  }
  if (tid == 0) trace_stamp(tr, 5);

  const int g = lane >> 2, t = lane & 3;
  const int nb = warp % NBW, ks = warp / NBW;
  const int tok = nb * 8 + g;
  const bool xok = tok < M;
  const uint32_t xrow = sbase + (uint32_t)a.off_x + (uint32_t)((xok ? tok : 0) * K * 2 + t * 32);
  const uint32_t wlo = sbase + (uint32_t)(g * K + t * 16);
  const uint32_t whi = wlo + (uint32_t)(8 * K);
  const uint32_t tstride = (uint32_t)(RS_TILE * K);
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  for (int kb = ks; kb < KB; kb += KSW) {
    uint4 x0 = make_uint4(0u, 0u, 0u, 0u), x1 = x0;
    if (xok) {
      x0 = rs_lds128(xrow + (uint32_t)(kb * 128));
      x1 = rs_lds128(xrow + (uint32_t)(kb * 128 + 16));
    }
    const uint32_t xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int tl = 0; tl < NT; ++tl) {
      if (tl < ntl) {
        const uint4 lo = rs_lds128(wlo + (uint32_t)tl * tstride + (uint32_t)(kb * 64));
        const uint4 hi = rs_lds128(whi + (uint32_t)tl * tstride + (uint32_t)(kb * 64));
        const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
        const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_half2x2<HW>(lw[j], a0, a2);
          e4m3x4_to_half2x2<HW>(hw[j], a1, a3);
          rs_mma(acc[tl], a0, a1, a2, a3, xs[2 * j], xs[2 * j + 1]);
        }
      }
    }
  }
  __syncthreads();  // the weight slice is dead: the K slices' partials reuse it
  if (tid == 0) trace_stamp(tr, 4);
  // partials [K slice][token][row] (row-contiguous), then the slice-ordered sum
  const int mpad = NBW * 8;
  float* red = reinterpret_cast<float*>(rs_smem);
#pragma unroll
  for (int tl = 0; tl < NT; ++tl) {
    if (tl < ntl) {
      float* p = red + ((size_t)ks * mpad + nb * 8 + 2 * t) * rows + tl * RS_TILE + g;
      p[0] = acc[tl][0];
      p[rows] = acc[tl][1];
      p[8] = acc[tl][2];
      p[rows + 8] = acc[tl][3];
    }
  }
  __syncthreads();
  for (int i = tid; i < rows * M; i += RS_THREADS) {
    const int m = i / rows, rl = i - m * rows;  // consecutive threads: consecutive rows
    const int n = row0 + rl;
    if (n < N) {
      float s = 0.f;
#pragma unroll
      for (int k2 = 0; k2 < KSW; ++k2) s += red[((size_t)k2 * mpad + m) * rows + rl];
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

// DDQ_RS_MAX_M overrides the largest token count the kernel takes (0
// switches it off) for measurements.
int64_t rs_max_m() {
  static const int64_t v = [] {
    const char* e = std::getenv("DDQ_RS_MAX_M");
    return e ? (int64_t)std::atoll(e) : (int64_t)16;
  }();
  return v;
}

struct RsPlan {
  bool ok;
  int grid, nt, nb, smem;
  int off_x, off_sc, off_bi, off_bar;
};

RsPlan rs_plan(int64_t M, int64_t N, int64_t K, int sms) {
  RsPlan p{};
  if (M < 1 || M > 16 || M > rs_max_m() || N < 1 || K < 64 || K % 64 != 0 || sms <= 0) return p;
  if (N > 0x7fffffff - RS_TILE || K > (1 << 20)) return p;
  const int64_t tiles = (N + RS_TILE - 1) / RS_TILE;
  const int64_t grid = tiles < sms ? tiles : sms;
  const int64_t ntl = (tiles + grid - 1) / grid;  // largest per-CTA tile count
  const int64_t nb = M <= 8 ? 1 : 2;
  if (ntl > (nb == 1 ? RS_MAX_TILES : RS_MAX_TILES - 1)) return p;
  // one tile per CTA with a long K (the Qwen2.5 down projection, 56 CTAs):
  // the thin kernel's 8-row tiles on twice the SMs measured faster
  if (ntl == 1 && K >= 2048) return p;
  // 9..16 tokens with one tile per CTA (q/k/v, o, up to ~2300 rows): two
  // 8-token MMAs per weight fragment on at most one SM per 16 rows; the thin
  // kernel's 8-row tiles with all 16 tokens on the MMA rows measured 0.2-0.55
  // us faster per chained call (e.g. 1152 x 896 at 16 tokens: 2.91 vs 3.44)
  if (ntl == 1 && nb == 2 && thin_eligible(M, N, K, sms)) return p;
  const int64_t w_bytes = ntl * RS_TILE * K;
  const int64_t red_bytes = (int64_t)RS_WARPS * ntl * RS_TILE * nb * 8 * 4;
  if (red_bytes > w_bytes) return p;  // the partial sums reuse the weight slice
  const int64_t x_bytes = M * K * 2;
  if (w_bytes + x_bytes > (int64_t)0xFFFFF) return p;  // mbarrier transaction count
  const int64_t off_x = w_bytes;                   // multiple of 16 (K % 64 == 0)
  const int64_t off_sc = off_x + ((x_bytes + 15) & ~15ll);
  const int64_t off_bi = off_sc + ntl * RS_TILE * 4;
  const int64_t off_bar = off_bi + ntl * RS_TILE * 4;  // multiple of 16
  const int64_t total = off_bar + 32;
  if (total > RS_SMEM_MAX) return p;
  p.ok = true;
  p.grid = (int)grid;
  p.nt = (int)ntl;
  p.nb = (int)nb;
  p.smem = (int)total;
  p.off_x = (int)off_x;
  p.off_sc = (int)off_sc;
  p.off_bi = (int)off_bi;
  p.off_bar = (int)off_bar;
  return p;
}

// DDQ_E4M3_CVT=int selects the integer-ALU weight conversion, hw (default)
// the hardware converter (for measurements).
bool hw_cvt() {
  static const bool v = [] {
    const char* e = std::getenv("DDQ_E4M3_CVT");
    return !(e && e[0] == 'i');
  }();
  return v;
}

template <int NT, int NB, bool HW>
int launch_rs_t(const RsPlan& p, const RsArgs& a, cudaStream_t s) {
  // the launch's own size still sets the occupancy
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), w8a16_rs_kernel<NT, NB, HW>, RS_SMEM_MAX);
  if (ast) return ast;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(RS_THREADS);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_rs_kernel<NT, NB, HW>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

template <int NB, bool HW>
int launch_rs_nb(const RsPlan& p, const RsArgs& a, cudaStream_t s) {
  switch (p.nt) {
    case 1: return launch_rs_t<1, NB, HW>(p, a, s);
    case 2: return launch_rs_t<2, NB, HW>(p, a, s);
    case 3: return launch_rs_t<3, NB, HW>(p, a, s);
    case 4: return launch_rs_t<4, NB, HW>(p, a, s);
    case 5: return launch_rs_t<5, NB, HW>(p, a, s);
    default:
      if constexpr (NB == 1) return launch_rs_t<6, NB, HW>(p, a, s);
      else return DDQ_ERR_SHAPE;  // 9..16 tokens take at most 5 tiles per CTA
  }
}

// 17..64 tokens (warps over token blocks).  DDQ_RSW_MAX_M overrides the
// largest token count it takes (0 switches it off) for measurements.
int64_t rsw_max_m() {
  static const int64_t v = [] {
    const char* e = std::getenv("DDQ_RSW_MAX_M");
    return e ? (int64_t)std::atoll(e) : (int64_t)64;
  }();
  return v;
}

RsPlan rsw_plan(int64_t M, int64_t N, int64_t K, int sms) {
  RsPlan p{};
  if (M <= 16 || M > 64 || M > rsw_max_m() || N < 1 || K < 64 || K % 64 != 0 || sms <= 0)
    return p;
  if (N > 0x7fffffff - RS_TILE || K > (1 << 20)) return p;
  const int64_t tiles = (N + RS_TILE - 1) / RS_TILE;
  const int64_t grid = tiles < sms ? tiles : sms;
  const int64_t ntl = (tiles + grid - 1) / grid;
  if (ntl > RS_MAX_TILES) return p;
  const int64_t nbw = M <= 32 ? 4 : 8;
  // The legacy mma.sync path runs at about one m16n8k16 per 8 SM cycles on
  // B200 (gate/up 9728 x 896 at 64 tokens: 272K MMAs took 7.7 us on 148 SMs),
  // so beyond ~768 MMAs per CTA (~3 us) the tcgen05 decode kernel is faster
  // (measured: q/k/v and o at 32-64 tokens 4.3-5.1 us here against 6.1-7.9;
  // gate/up at 32 tokens 7.7 against 6.9).
  if (ntl * (K / 16) * ((M + 7) / 8) > 768) return p;
  const int64_t w_bytes = ntl * RS_TILE * K;
  const int64_t red_bytes = (int64_t)(RS_WARPS / nbw) * nbw * 8 * ntl * RS_TILE * 4;
  if (red_bytes > w_bytes) return p;  // the partials reuse the weight slice
  const int64_t x_bytes = M * K * 2;
  if (w_bytes > (int64_t)0xFFFFF || x_bytes > (int64_t)0xFFFFF) return p;
  const int64_t off_x = w_bytes;
  const int64_t off_sc = off_x + ((x_bytes + 15) & ~15ll);
  const int64_t off_bi = off_sc + ntl * RS_TILE * 4;
  const int64_t off_bar = off_bi + ntl * RS_TILE * 4;
  const int64_t total = off_bar + 32;
  if (total > RS_SMEM_MAX) return p;
  p.ok = true;
  p.grid = (int)grid;
  p.nt = (int)ntl;
  p.nb = (int)nbw;
  p.smem = (int)total;
  p.off_x = (int)off_x;
  p.off_sc = (int)off_sc;
  p.off_bi = (int)off_bi;
  p.off_bar = (int)off_bar;
  return p;
}

template <int NT, int NBW, bool HW>
int launch_rsw_t(const RsPlan& p, const RsArgs& a, cudaStream_t s) {
  static SmemAttrOnce attr;
  const int ast =
      ensure_smem_attr(attr, current_device(), w8a16_rsw_kernel<NT, NBW, HW>, RS_SMEM_MAX);
  if (ast) return ast;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(RS_THREADS);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_rsw_kernel<NT, NBW, HW>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

template <int NBW>
int launch_rsw_nb(const RsPlan& p, const RsArgs& a, cudaStream_t s) {
  switch (p.nt) {
    case 1: return launch_rsw_t<1, NBW, true>(p, a, s);
    case 2: return launch_rsw_t<2, NBW, true>(p, a, s);
    case 3: return launch_rsw_t<3, NBW, true>(p, a, s);
    case 4: return launch_rsw_t<4, NBW, true>(p, a, s);
    case 5: return launch_rsw_t<5, NBW, true>(p, a, s);
    default: return launch_rsw_t<6, NBW, true>(p, a, s);
  }
}

}  // namespace

bool rs_eligible(int64_t M, int64_t N, int64_t K, int sms) {
  return rs_plan(M, N, K, sms).ok || rsw_plan(M, N, K, sms).ok;
}

int launch_rs(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, unsigned long long timeout_ns,
              cudaStream_t s, int debug_flags) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  if (!aligned16(x) || !aligned16(wq)) return DDQ_ERR_ALIGNMENT;
  const RsPlan pw = rsw_plan(M, N, K, sms);
  const RsPlan p = pw.ok ? pw : rs_plan(M, N, K, sms);
  if (!p.ok) return DDQ_ERR_SHAPE;
  RsArgs a{};
  a.x = x;
  a.wq = wq;
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles = (N + RS_TILE - 1) / RS_TILE;
  a.off_x = p.off_x;
  a.off_sc = p.off_sc;
  a.off_bi = p.off_bi;
  a.off_bar = p.off_bar;
  a.timeout_ns = timeout_ns;
  a.trace = (debug_flags & 2) != 0;
  if (pw.ok) return p.nb == 4 ? launch_rsw_nb<4>(p, a, s) : launch_rsw_nb<8>(p, a, s);
  if (hw_cvt()) return p.nb == 1 ? launch_rs_nb<1, true>(p, a, s) : launch_rs_nb<2, true>(p, a, s);
  return p.nb == 1 ? launch_rs_nb<1, false>(p, a, s) : launch_rs_nb<2, false>(p, a, s);
}

}  // namespace ddq
