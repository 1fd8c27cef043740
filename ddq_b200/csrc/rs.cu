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
//     of all its tiles with the tiles' MMAs interleaved (independent
//     accumulators, no long dependency chains), then a warp-ordered sum of
//     the 8 partials per output, scale * 256, bias, fp16.
// Weights on the A operand: one MMA covers 16 weight rows x 8 tokens, so at
// up to 8 tokens it takes half the MMAs (and the same e4m3 conversions) of
// tokens-on-rows; 9..16 tokens use two 8-token blocks per A fragment.
//
// K order inside a 64-wide block: lane quad position t holds the 16
// consecutive k at 16t .. 16t+15 of its weight rows (A) and of its token's
// activations (B); MMA j takes k 16t+4j .. 16t+4j+3 as the fragment's logical
// k {2t, 2t+1, 2t+8, 2t+9}.  A and B follow the same map, so each MMA adds
// the same products as in natural order, and one 16-byte weight load per
// row feeds four MMAs.  The e4m3 -> fp16 conversion is integer-only and
// exact (value * 2^-8, subnormals included); the factor 256 is folded into
// the row scale.  Results are bitwise reproducible (fixed warp-ordered sum).
#include <cfloat>
#include <cstdlib>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {
namespace {

constexpr int RS_WARPS = 8;
constexpr int RS_THREADS = RS_WARPS * 32;
constexpr int RS_TILE = 16;          // weight rows per MMA tile
constexpr int RS_MAX_TILES = 8;      // tiles per CTA (accumulator registers)
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
//   off_sc, off_bi  per-row scale * 256 and bias (fp32)
//   off_bar         weight barrier, activation barrier, abort and drain flags
template <int NT, int NB>
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
      s = a.scales[n] * 256.f;
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
          const uint32_t a0 = e4m3x2_to_half2_bits_x2m8(lw[j], 0x4140u);
          const uint32_t a2 = e4m3x2_to_half2_bits_x2m8(lw[j], 0x4342u);
          const uint32_t a1 = e4m3x2_to_half2_bits_x2m8(hw[j], 0x4140u);
          const uint32_t a3 = e4m3x2_to_half2_bits_x2m8(hw[j], 0x4342u);
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
// e4m3 variant: no weight conversion at all.
// ----------------------------------------------------------------------------
// The weight bytes feed mma.sync m16n8k32 .e4m3 directly (A operand, 16
// weight rows x 32 k); the activations are split once per CTA, after the
// dependency, into three e4m3 planes under a per-token power-of-two scale
//     z = x[m,:] * 2^e_m (exact; max |z| in [128, 256)),
//     h1 = e4m3(z), h2 = e4m3(z - h1), h3 = e4m3(z - h1 - h2)   (RNE)
// (the decode kernel's split, tc_decode.cu), and the B operand's 8 columns
// are (token, plane) pairs j = 3 m + p, so one A fragment serves
// ceil(3 M / 8) MMAs: y[m, n] = scale[n] * 2^-e_m * sum_p sum_k W[n,k] h_p[m,k]
// + bias[n].  The three planes carry x to 2^-12 relative (finer than fp16's
// own rounding of x).
// Work units are (tile, column block, K slice): the K slices are chosen per
// CTA so that every warp has a unit even when the CTA holds a single tile;
// each unit accumulates in two alternating sets (half-length MMA chains) and
// writes its partial to [slice][column][row] (row-contiguous, so the final
// warp-ordered sum reads conflict-free); the epilogue sums slices and planes
// in a fixed order (bitwise reproducible).
//
// Fragments of m16n8k32 with 8-bit operands (thread = 4 g + t): a0 = A[g][4t
// .. 4t+3], a1 = A[g+8][4t ..], a2 = A[g][4t+16 ..], a3 = A[g+8][4t+16 ..];
// b0 = B[4t .. 4t+3][g], b1 = B[4t+16 ..][g]; d as for m16n8k16.  Inside a
// 64-wide K block thread t holds k 16t .. 16t+15 of its weight rows and of
// its column's plane in one 16-byte load each; MMA 0 takes bytes 0-7 of both
// (logical k 4t.. and 4t+16..), MMA 1 bytes 8-15, the same map in A and B.
struct Rs8Args {
  const __half* x;
  const uint8_t* wq;
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  int M, N, K;
  int tiles;          // ceil(N / 16)
  int cb;             // column blocks: ceil(3 M / 8)
  int pk;             // plane row stride (bytes)
  int off_p, off_red, off_sc, off_bi, off_xs, off_rmax, off_bar;
  unsigned long long timeout_ns;
  int trace;
};

__device__ __forceinline__ void rs_mma8(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// K slices of a CTA holding ntl tiles: the smallest power of two giving at
// least one unit per warp (at most the number of 64-wide K blocks).
__host__ __device__ inline int rs8_kslices(int ntl, int cb, int kb) {
  int ks = 1;
  while (ntl * cb * ks < RS_WARPS && ks * 2 <= kb) ks *= 2;
  return ks;
}

// Shared memory: [0, rows * K) the weight slice (rows past N zero-filled);
// off_p the planes [3 M][pk] (row j = 3 m + p); off_red the units' partials
// [slice][column][row] fp32; off_sc / off_bi per-row scale and bias;
// off_xs 2^-e per token; off_rmax the token rows' max |x| (as uint bits);
// off_bar weight barrier, abort and drain flags.
template <int CPT>
__global__ void __launch_bounds__(RS_THREADS, 2) w8a16_rs8_kernel(const Rs8Args a) {
  extern __shared__ __align__(128) uint8_t rs_smem[];
  const uint32_t sbase = ptx::smem_u32(rs_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  const int tile0 = (int)(((int64_t)b * a.tiles) / G);
  const int ntl = (int)(((int64_t)(b + 1) * a.tiles) / G) - tile0;
  const int row0 = tile0 * RS_TILE, rows = ntl * RS_TILE;
  const int M = a.M, N = a.N, K = a.K, KB = K >> 6, CB = a.cb, COLS = CB * 8;
  const int valid = min(rows, N - row0);
  const uint32_t bar_w = sbase + (uint32_t)a.off_bar;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(rs_smem + a.off_bar + 16);
  volatile int* drain_flag = reinterpret_cast<volatile int*>(rs_smem + a.off_bar + 20);
  float* sc = reinterpret_cast<float*>(rs_smem + a.off_sc);
  float* bi = reinterpret_cast<float*>(rs_smem + a.off_bi);
  float* xs = reinterpret_cast<float*>(rs_smem + a.off_xs);
  unsigned int* rmax = reinterpret_cast<unsigned int*>(rs_smem + a.off_rmax);
  uint8_t* planes = rs_smem + a.off_p;
  const bool tr = a.trace != 0;
  if (tid == 0) {
    trace_stamp(tr, 0);
    ptx::mbar_init(bar_w, 1);
    *abort_flag = 0;
    *drain_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  // 1) the weight slice: one bulk copy (weights are never written by the
  //    kernel this one depends on); then the next kernel may be scheduled
  if (tid == 0) {
    ptx::mbar_arrive_expect_tx(bar_w, (uint32_t)(valid * K));
    rs_bulk_g2s(sbase, a.wq + (size_t)row0 * K, (uint32_t)(valid * K), bar_w);
    trace_stamp(tr, 2);
  }
  ptx::pdl_launch_dependents();
  for (int i = valid * K / 16 + tid; i < rows * K / 16; i += RS_THREADS)
    reinterpret_cast<uint4*>(rs_smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid < rows) {
    const int n = row0 + tid;
    float s = 0.f, bv = 0.f;
    if (n < N) {
      s = a.scales[n];
      if (a.bias_dtype == DDQ_DTYPE_F16) bv = __half2float(reinterpret_cast<const __half*>(a.bias)[n]);
      else if (a.bias_dtype == DDQ_DTYPE_F32) bv = reinterpret_cast<const float*>(a.bias)[n];
    }
    sc[tid] = s;
    bi[tid] = bv;
  }
  if (tid < M) rmax[tid] = 0u;
  __syncthreads();

  // 2) x (written by the previous kernel): chunks of 8 into registers
  //    (bypassing L1), per-token max |x|, then the three planes
  ptx::pdl_wait();
  if (tid == 0) trace_stamp(tr, 3);
  const int cpr = K >> 3;  // 8-element chunks per token row
  const int nch = M * cpr;
  uint4 xv[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = tid + j * RS_THREADS;
    xv[j] = c < nch ? __ldcg(reinterpret_cast<const uint4*>(a.x) + c) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = tid + j * RS_THREADS;
    if (c < nch) {
      const __half2* h = reinterpret_cast<const __half2*>(&xv[j]);
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
      atomicMax(&rmax[c / cpr], __float_as_uint(m));  // |x| >= 0: bit order = value order
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = tid + j * RS_THREADS;
    if (c < nch) {
      const int m = c / cpr, kc = c - m * cpr;
      const float up = ldexpf(1.f, split_shift(__uint_as_float(rmax[m])));
      const __half2* h = reinterpret_cast<const __half2*>(&xv[j]);
      float z[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        z[2 * i] = f.x * up;  // exact: power-of-two scale
        z[2 * i + 1] = f.y * up;
      }
      uint2 p1, p2, p3;
      split8(z, p1, p2, p3);
      uint8_t* dst = planes + (size_t)(3 * m) * a.pk + kc * 8;
      *reinterpret_cast<uint2*>(dst) = p1;
      *reinterpret_cast<uint2*>(dst + a.pk) = p2;
      *reinterpret_cast<uint2*>(dst + 2 * a.pk) = p3;
    }
  }
  // a token row holding inf (or a NaN that fmaxf skipped and the split turns
  // into NaN codes) gives non-finite outputs: the split saturates inf, so its
  // scale is made NaN instead of 2^-e
  if (tid < M) {
    const float am = __uint_as_float(rmax[tid]);
    xs[tid] = am <= FLT_MAX ? ldexpf(1.f, -split_shift(am)) : __int_as_float(0x7fc00000);
  }
  // the weight slice (bounded wait: on a timeout the CTA records
  // DDQ_ERR_TIMEOUT, waits once more for its copy and leaves without output)
  ptx::mbar_wait(bar_w, 0u, a.timeout_ns, abort_flag);
  __syncthreads();
  if (*abort_flag) {
    if (tid == 0) {
      record_device_error(DDQ_ERR_TIMEOUT);
      ptx::mbar_wait(bar_w, 0u, a.timeout_ns, drain_flag);
    }
    return;
  }
  if (tid == 0) trace_stamp(tr, 5);

  // 3) MMA units (tile, column block, K slice)
  const int g = lane >> 2, t = lane & 3;
  const int KS = rs8_kslices(ntl, CB, KB);
  const int kper = (KB + KS - 1) / KS;
  const int units = ntl * CB * KS;
  float* red = reinterpret_cast<float*>(rs_smem + a.off_red);
  for (int u = warp; u < units; u += RS_WARPS) {
    const int ks = u % KS, cbi = (u / KS) % CB, tl = u / (KS * CB);
    const int kb0 = ks * kper, kb1 = min(KB, kb0 + kper);
    const uint32_t wlo = sbase + (uint32_t)(tl * RS_TILE * K + g * K + t * 16);
    const uint32_t whi = wlo + (uint32_t)(8 * K);
    const int j = cbi * 8 + g;
    const bool pok = j < 3 * M;
    const uint32_t prow = sbase + (uint32_t)(a.off_p + (pok ? j : 0) * a.pk + t * 16);
    // two accumulator sets (even / odd K blocks): half-length MMA chains
    float e0[4] = {0.f, 0.f, 0.f, 0.f}, e1[4] = {0.f, 0.f, 0.f, 0.f};
    auto step = [&](int kb, float* d) {
      const uint4 wl = rs_lds128(wlo + (uint32_t)(kb * 64));
      const uint4 wh = rs_lds128(whi + (uint32_t)(kb * 64));
      const uint4 pv = pok ? rs_lds128(prow + (uint32_t)(kb * 64)) : make_uint4(0u, 0u, 0u, 0u);
      rs_mma8(d, wl.x, wh.x, wl.y, wh.y, pv.x, pv.y);
      rs_mma8(d, wl.z, wh.z, wl.w, wh.w, pv.z, pv.w);
    };
    int kb = kb0;
    for (; kb + 1 < kb1; kb += 2) {
      step(kb, e0);
      step(kb + 1, e1);
    }
    if (kb < kb1) step(kb, e0);
    float* p = red + (size_t)ks * COLS * rows + tl * RS_TILE + g;
    const int c0 = cbi * 8 + 2 * t;
    p[(size_t)c0 * rows] = e0[0] + e1[0];
    p[(size_t)(c0 + 1) * rows] = e0[1] + e1[1];
    p[(size_t)c0 * rows + 8] = e0[2] + e1[2];
    p[(size_t)(c0 + 1) * rows + 8] = e0[3] + e1[3];
  }
  __syncthreads();
  if (tid == 0) trace_stamp(tr, 4);
  // 4) y = scale * 2^-e * (sum over slices, planes in order) + bias
  for (int i = tid; i < rows * M; i += RS_THREADS) {
    const int m = i / rows, rl = i - m * rows;  // consecutive threads: consecutive rows
    const int n = row0 + rl;
    if (n < N) {
      float s = 0.f;
      for (int ks = 0; ks < KS; ++ks) {
        const float* q = red + ((size_t)ks * COLS + 3 * m) * rows + rl;
        s += (q[0] + q[rows]) + q[2 * rows];
      }
      a.y[(size_t)m * N + n] = __float2half_rn(fmaf(s * sc[rl], xs[m], bi[rl]));
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
  if (ntl > RS_MAX_TILES) return p;
  const int64_t nb = M <= 8 ? 1 : 2;
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
  p.nt = ntl <= 1 ? 1 : ntl <= 2 ? 2 : ntl <= 3 ? 3 : ntl <= 4 ? 4 : ntl <= 5 ? 5 : ntl <= 6 ? 6 : 8;
  p.nb = (int)nb;
  p.smem = (int)total;
  p.off_x = (int)off_x;
  p.off_sc = (int)off_sc;
  p.off_bi = (int)off_bi;
  p.off_bar = (int)off_bar;
  return p;
}

template <int NT, int NB>
int launch_rs_t(const RsPlan& p, const RsArgs& a, cudaStream_t s) {
  // the launch's own size still sets the occupancy
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), w8a16_rs_kernel<NT, NB>, RS_SMEM_MAX);
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_rs_kernel<NT, NB>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

template <int NB>
int launch_rs_nb(const RsPlan& p, const RsArgs& a, cudaStream_t s) {
  switch (p.nt) {
    case 1: return launch_rs_t<1, NB>(p, a, s);
    case 2: return launch_rs_t<2, NB>(p, a, s);
    case 3: return launch_rs_t<3, NB>(p, a, s);
    case 4: return launch_rs_t<4, NB>(p, a, s);
    case 5: return launch_rs_t<5, NB>(p, a, s);
    case 6: return launch_rs_t<6, NB>(p, a, s);
    default: return launch_rs_t<8, NB>(p, a, s);
  }
}

// DDQ_RS8=0 keeps the fp16 variant for every shape (for measurements).
bool rs8_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("DDQ_RS8");
    return !(e && e[0] == '0');
  }();
  return v;
}

struct Rs8Plan {
  bool ok;
  int grid, cpt, cb, pk, smem;
  int off_p, off_red, off_sc, off_bi, off_xs, off_rmax, off_bar;
};

Rs8Plan rs8_plan(int64_t M, int64_t N, int64_t K, int sms) {
  Rs8Plan p{};
  if (!rs8_enabled()) return p;
  if (M < 1 || M > 16 || M > rs_max_m() || N < 1 || K < 64 || K % 64 != 0 || sms <= 0) return p;
  if (N > 0x7fffffff - RS_TILE || K > (1 << 20)) return p;
  const int64_t chunks = M * K / 8;                 // x in registers: at most 8 chunks a thread
  const int64_t cpt = (chunks + RS_THREADS - 1) / RS_THREADS;
  if (cpt > 8) return p;
  const int64_t tiles = (N + RS_TILE - 1) / RS_TILE;
  const int64_t grid = tiles < sms ? tiles : sms;
  const int64_t ntl_max = (tiles + grid - 1) / grid, ntl_min = tiles / grid;
  if (ntl_max > RS_MAX_TILES) return p;
  const int64_t cb = (3 * M + 7) / 8;
  const int64_t kb = K / 64;
  int64_t red = 0;  // partials of the largest CTA layout: slices x columns x rows
  for (int64_t ntl : {ntl_min < 1 ? ntl_max : ntl_min, ntl_max}) {
    const int64_t r = (int64_t)rs8_kslices((int)ntl, (int)cb, (int)kb) * cb * 8 * ntl * RS_TILE * 4;
    red = r > red ? r : red;
  }
  const int64_t pk = (K % 128 == 0) ? K + 64 : K;   // plane rows j, j + 1 on different banks
  const int64_t w_bytes = ntl_max * RS_TILE * K;
  if (w_bytes > (int64_t)0xFFFFF) return p;         // mbarrier transaction count
  const int64_t off_p = w_bytes;
  const int64_t off_red = off_p + ((3 * M * pk + 15) & ~15ll);
  const int64_t off_sc = off_red + red;
  const int64_t off_bi = off_sc + ntl_max * RS_TILE * 4;
  const int64_t off_xs = off_bi + ntl_max * RS_TILE * 4;
  const int64_t off_rmax = off_xs + 64;
  const int64_t off_bar = off_rmax + 64;
  const int64_t total = off_bar + 32;
  if (total > RS_SMEM_MAX) return p;
  p.ok = true;
  p.grid = (int)grid;
  p.cpt = cpt <= 1 ? 1 : cpt <= 2 ? 2 : cpt <= 4 ? 4 : 8;
  p.cb = (int)cb;
  p.pk = (int)pk;
  p.smem = (int)total;
  p.off_p = (int)off_p;
  p.off_red = (int)off_red;
  p.off_sc = (int)off_sc;
  p.off_bi = (int)off_bi;
  p.off_xs = (int)off_xs;
  p.off_rmax = (int)off_rmax;
  p.off_bar = (int)off_bar;
  return p;
}

template <int CPT>
int launch_rs8_t(const Rs8Plan& p, const Rs8Args& a, cudaStream_t s) {
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), w8a16_rs8_kernel<CPT>, RS_SMEM_MAX);
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_rs8_kernel<CPT>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

int launch_rs8(const Rs8Plan& p, const __half* x, const uint8_t* wq, const float* scales,
               const void* bias, int bias_dtype, __half* y, int M, int N, int K,
               unsigned long long timeout_ns, cudaStream_t s, int debug_flags) {
  Rs8Args a{};
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
  a.cb = p.cb;
  a.pk = p.pk;
  a.off_p = p.off_p;
  a.off_red = p.off_red;
  a.off_sc = p.off_sc;
  a.off_bi = p.off_bi;
  a.off_xs = p.off_xs;
  a.off_rmax = p.off_rmax;
  a.off_bar = p.off_bar;
  a.timeout_ns = timeout_ns;
  a.trace = (debug_flags & 2) != 0;
  switch (p.cpt) {
    case 1: return launch_rs8_t<1>(p, a, s);
    case 2: return launch_rs8_t<2>(p, a, s);
    case 4: return launch_rs8_t<4>(p, a, s);
    default: return launch_rs8_t<8>(p, a, s);
  }
}

}  // namespace

bool rs_eligible(int64_t M, int64_t N, int64_t K, int sms) {
  return rs8_plan(M, N, K, sms).ok || rs_plan(M, N, K, sms).ok;
}

int launch_rs(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, unsigned long long timeout_ns,
              cudaStream_t s, int debug_flags) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  if (!aligned16(x) || !aligned16(wq)) return DDQ_ERR_ALIGNMENT;
  const Rs8Plan p8 = rs8_plan(M, N, K, sms);
  if (p8.ok)
    return launch_rs8(p8, x, wq, scales, bias, bias_dtype, y, M, N, K, timeout_ns, s, debug_flags);
  const RsPlan p = rs_plan(M, N, K, sms);
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
  return p.nb == 1 ? launch_rs_nb<1>(p, a, s) : launch_rs_nb<2>(p, a, s);
}

}  // namespace ddq
