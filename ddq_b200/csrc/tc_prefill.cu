// tc_prefill.cu - the prefill-shape (large M) W8A16 GEMM: an exact e4m3 -> fp16
// expansion of the weight matrix, then an fp16 tcgen05 GEMM at tensor rate.
//
// With hundreds of tokens per weight tile the GEMM is tensor-bound, and
// converting the e4m3 weight tile in shared memory for every token block
// (the in-kernel conversion of tc_gemm.cu) costs more SM issue slots than the
// MMAs themselves.  Here the conversion runs once per call instead:
//   e4m3_to_f16_kernel   w16[n, k] = fp16(e4m3(wq[n, k]))  (exact: every e4m3
//                        value is an fp16 value), HBM-bound, 1 byte in -> 2 out
//   w8a16_pf_kernel      D[m, n] = sum_k x[m, k] * w16[n, k]   (fp32 in TMEM)
//                        y[m, n] = fp16( D[m, n] * scale[n] + bias[n] )
// so the per-row weight scale is applied to the fp32 sum, as in the
// reference's dequantize-then-multiply semantics (gemm_FP8_d.cu:94-146).
//
// w8a16_pf_kernel: persistent, one CTA per SM, 384 threads; output tile =
// 128 tokens (the MMA M, TMEM lanes) x 256 weight rows (the MMA N, TMEM
// columns), K in stages of 64 (one 128-byte swizzle atom of fp16):
//   warp 0      TMA producer: the x tile (128 x 64) and the w16 tile (BN x 64,
//               BN <= 256 chosen per shape) of each stage on one full barrier
//   warp 1      MMA issuer: 4 x tcgen05.mma kind::f16 (K = 16) per stage into
//               one of two 256-column TMEM accumulators (double buffered, so a
//               tile's epilogue overlaps the next tile's MMAs)
//   warps 4-11  epilogue, two groups of four over alternate 32-column chunks:
//               tcgen05.ld -> scale, bias -> fp16 -> 64-byte-swizzled staging ->
//               one TMA store per warp and chunk (32 tokens x 32 columns)
// Tiles run token-tile-major across the grid (consecutive CTAs share an x
// tile; the 2-byte weights of a 9728 x 896 projection, 17 MB, stay in L2).
// Every mbarrier wait is bounded; on timeout the CTA records DDQ_ERR_TIMEOUT,
// drains its copies and MMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <mutex>
#include <iterator>
#include <unordered_map>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int PF_BM = 128;       // tokens per tile (MMA M, TMEM lanes)
constexpr int PF_BN = 256;       // weight rows per tile (MMA N, TMEM columns)
constexpr int PF_BK = 64;        // K elements per stage (128 B of fp16)
constexpr int PF_ST = 4;         // ring stages, one CTA per tile
constexpr int PF_ST2 = 5;        // ring stages, CTA pairs (half the weight rows per CTA)
constexpr int PF_THREADS = 384;  // 12 warps
constexpr int PF_CH = 32;        // epilogue column chunk

template <int ST, int BROWS, int NSTG>
struct PfLayoutT {
  static constexpr int STAGES = ST;
  static constexpr int NSTAGING = NSTG;             // staging buffers per epilogue warp
  static constexpr int A_BYTES = PF_BM * PF_BK * 2;   // 16 KB x tile
  static constexpr int B_BYTES = BROWS * PF_BK * 2;   // this CTA's w16 rows (32 or 16 KB)
  static constexpr int S_BYTES = A_BYTES + B_BYTES;
  static constexpr int OW_BYTES = 32 * PF_CH * 2;     // one warp's staging (32 x 32 fp16)
  static constexpr int OFF_O = ST * S_BYTES;          // 8 warps x NSTG staging buffers
  static constexpr int OFF_SB = OFF_O + 8 * NSTG * OW_BYTES;  // [2 tiles][scale | bias] fp32
  static constexpr int OFF_BAR = OFF_SB + 2 * 2 * PF_BN * 4;
  static constexpr int NBAR = 2 * ST + 4 + 1;         // full, empty; acc x2 x2; drain
  static constexpr int OFF_MISC = (OFF_BAR + NBAR * 8 + 15) & ~15;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(S_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "1024-B aligned operand tiles");
  static_assert(ALLOC <= 232448, "shared memory budget");
};
using PfLayout = PfLayoutT<PF_ST, PF_BN, 1>;        // 4 stages x 48 KB
using PfLayout2 = PfLayoutT<PF_ST2, PF_BN / 2, 2>;  // 5 stages x 32 KB, 2 staging buffers

constexpr int PF_EPI_STORE = 0, PF_EPI_SWIGLU = 1, PF_EPI_ROPE = 2;

struct PfArgs {
  const float* scales;
  const void* bias;
  int bias_dtype;
  int M, N, K;
  int bn;               // weight rows per tile: a multiple of 32, at most PF_BN
  int tiles_m, tiles_n;
  unsigned long long timeout_ns;
  int debug_flags;
  PfRope rope;          // PF_EPI_ROPE only
};

__device__ __forceinline__ float pf_load_bias(const void* bias, int bias_dtype, int n) {
  if (bias_dtype == DDQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (bias_dtype == DDQ_DTYPE_F32) return reinterpret_cast<const float*>(bias)[n];
  return 0.f;
}

__device__ __forceinline__ bool pf_wait_drain(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  const long long t0 = clock64();
  const long long limit = (long long)(timeout_ns * 2ull);
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

__device__ __forceinline__ void pf_reg_fence8(uint32_t (&r)[8]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7])::"memory");
}

// 32-byte global accesses (one whole L2 sector; the address must be 32-byte
// aligned): 8 fp32 read-only loads, 8 words stored
__device__ __forceinline__ void pf_ld32(const float* p, float* v) {
  asm volatile("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
                 "=f"(v[6]), "=f"(v[7])
               : "l"(p));
}

__device__ __forceinline__ void pf_st32(__half* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void pf_reg_fence(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])::"memory");
  asm volatile(""
               : "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]),
                 "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])::"memory");
}

// Exact expansion e4m3 -> fp16: each thread keeps four 16-byte loads in
// flight (64 bytes in, 128 out per step) so that the pass runs at HBM rate.
__device__ __forceinline__ void pf_expand16(const uint4& v, uint4* dst) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t h[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    h[2 * j] = e4m3x2_to_half2_bits((uint16_t)(w[j] & 0xFFFFu));
    h[2 * j + 1] = e4m3x2_to_half2_bits((uint16_t)(w[j] >> 16));
  }
  dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
  dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
}

// early: w16 is a buffer the previous GEMM does not read (consecutive calls
// alternate two), so the expansion runs before the grid dependency resolves
// and only waits before it exits (its completion then still implies the
// previous kernel's).  Otherwise w16 may still be read by the previous GEMM:
// wait first.
__global__ void __launch_bounds__(256) e4m3_to_f16_kernel(const uint8_t* __restrict__ wq,
                                                          __half* __restrict__ w16, size_t n16,
                                                          int early) {
  ptx::pdl_launch_dependents();
  if (!early) ptx::pdl_wait();
  const uint4* src = reinterpret_cast<const uint4*>(wq);
  uint4* dst = reinterpret_cast<uint4*>(w16);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) pf_expand16(v[u], dst + 2 * (i + u * stride));
  }
  for (; i < n16; i += stride) pf_expand16(__ldcs(src + i), dst + 2 * i);
  if (early) ptx::pdl_wait();
}

// PF_EPI_SWIGLU: the weight is a 16-row interleave of gate and up (rows 32 b
// + i = gate row 16 b + i, rows 32 b + 16 + i = up row 16 b + i) and the
// kernel stores silu(gate) * up, N / 2 columns.  PF_EPI_ROPE: the QKV
// projection of a prefill chunk; tiles hold whole 64-row heads (both halves
// of every rotation pair), each epilogue warp group takes a quarter of every
// head's dims, rounds the projection to fp16 as the plain store does, then
// applies RoPE to q and k heads in fp32 with the rounding of the separate
// kernel (rope.cu) and writes q token-major and k, v into the cache (and
// token-major copies): bit for bit the result of the GEMM followed by
// ddq_prefill_rope_kv, without the qkv round trip.
//
// PAIR: clusters of two CTAs run 256-token tiles with tcgen05 .cta_group::2
// MMAs (M = 256, issued by rank 0): each CTA loads its own 128 tokens of x
// and half of the tile's weight rows (32 KB a stage instead of 48 KB, so six
// stages fit), rank 0's full barrier counts both CTAs' bytes, rank 0
// commits to both CTAs' empty and accumulator barriers, and both
// CTAs' epilogues release rank 0's accumulator barrier.  Each CTA's TMEM
// holds its 128 tokens x all the tile's columns, so the epilogues are those
// of the single-CTA kernel.
template <int EPI, bool PAIR>
__global__ void __launch_bounds__(PF_THREADS, 1)
    w8a16_pf_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_y, const PfArgs args) {
  constexpr bool SWIGLU = EPI == PF_EPI_SWIGLU;
  constexpr bool ROPE = EPI == PF_EPI_ROPE;
  using L = typename std::conditional<PAIR, PfLayout2, PfLayout>::type;
  constexpr int ST = L::STAGES;
  constexpr int TBM = PAIR ? 2 * PF_BM : PF_BM;  // tokens per tile
  constexpr uint32_t ACC_COLS = PF_BN;
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = (args.K + PF_BK - 1) / PF_BK;
  const int units = args.tiles_m * args.tiles_n;
  const int rank = PAIR ? (int)ptx::cluster_ctarank() : 0;  // 0 issues the pair's MMAs
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const uint64_t tmo = args.timeout_ns;
  const bool tr = (args.debug_flags & 2) != 0;

  const uint32_t bar_full = sbase + L::OFF_BAR;
  const uint32_t bar_empty = bar_full + 8 * ST;
  const uint32_t bar_accfull = bar_empty + 8 * ST;     // [2]
  const uint32_t bar_accempty = bar_accfull + 16;      // [2]
  const uint32_t bar_drain = bar_accempty + 16;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) trace_stamp(tr, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar_accfull + 8 * b, 1);
      ptx::mbar_init(bar_accempty + 8 * b, PAIR ? 16 : 8);  // epilogue warps (of both CTAs)
    }
    ptx::mbar_init(bar_drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_x);
    ptx::prefetch_tmap(&tm_w);
    ptx::prefetch_tmap(&tm_y);
  }
  if (warp == 0) {
    if constexpr (PAIR) {
      ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), TMEM_COLS);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(ptx::smem_u32(tmem_holder), TMEM_COLS);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  // pairs: both CTAs' barriers are initialised before either signals the other's
  if constexpr (PAIR) ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // rank 0's full and accumulator-empty barriers as cluster addresses
  const uint32_t full0 = PAIR ? ptx::mapa_shared(bar_full, 0) : bar_full;
  const uint32_t accempty0 = PAIR ? ptx::mapa_shared(bar_accempty, 0) : bar_accempty;
  // rank 1's empty and accumulator-full barriers, which rank 0's commits signal too
  const uint32_t empty1 = PAIR ? ptx::mapa_shared(bar_empty, 1) : bar_empty;
  const uint32_t accfull1 = PAIR ? ptx::mapa_shared(bar_accfull, 1) : bar_accfull;
  if (threadIdx.x == 0) trace_stamp(tr, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::pdl_wait();  // x and w16 come from earlier kernels
      // dependents launch only now: a following expansion may then write the
      // other workspace buffer, whose last reader (the GEMM before this one)
      // has finished once this grid's dependency has resolved
      ptx::pdl_launch_dependents();
      int g = 0;
      bool ok = true;
      // this CTA's weight rows of a tile: all of them, or its half of a pair's
      const int brows = PAIR ? args.bn >> 1 : args.bn;
      for (int u = unit0; u < units && ok; u += ustride) {
        const int m0 = (u / args.tiles_n) * TBM + rank * PF_BM;
        const int n0 = (u % args.tiles_n) * args.bn + rank * brows;
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int s = g % ST;
          if (!ptx::mbar_wait(bar_empty + 8 * s, ((uint32_t)(g / ST) & 1u) ^ 1u, tmo,
                              abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t dst = sbase + s * L::S_BYTES;
          if constexpr (PAIR) {
            // rank 0's barrier counts the bytes of both CTAs
            if (rank == 0)
              ptx::mbar_arrive_expect_tx(bar_full + 8 * s,
                                         (uint32_t)(2 * (L::A_BYTES + brows * PF_BK * 2)));
            ptx::tma_load_2d_pair(dst, &tm_x, ks * PF_BK, m0, full0 + 8 * s);
            ptx::tma_load_2d_pair(dst + L::A_BYTES, &tm_w, ks * PF_BK, n0, full0 + 8 * s);
          } else {
            const uint32_t full = bar_full + 8 * s;
            ptx::mbar_arrive_expect_tx(full, (uint32_t)(L::A_BYTES + brows * PF_BK * 2));
            ptx::tma_load_2d(dst, &tm_x, ks * PF_BK, m0, full);
            ptx::tma_load_2d(dst + L::A_BYTES, &tm_w, ks * PF_BK, n0, full);
          }
        }
      }
      if (*abort_flag) {
        if (!PAIR || rank == 0) {
          for (int i = g > ST ? g - ST : 0; i < g; ++i)
            pf_wait_drain(bar_full + 8 * (i % ST), (uint32_t)(i / ST) & 1u, tmo);
        }
        // a pair's rank 1 has no barrier of its own for its copies: they
        // land within microseconds; the teardown waits before exiting
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = ptx::idesc_f16_f32(TBM, args.bn);
      const uint64_t desc0 = ptx::smem_desc_sw128(sbase);
      // test hook (ddq_set_debug bit 0): no accumulator-ready signal, so the
      // epilogues' bounded waits run out and every role winds down
      const bool skip_accfull = (args.debug_flags & 1) != 0;
      ptx::pdl_wait();
      bool ok = true;
      int g = 0, it = 0;
      for (int u = unit0; u < units && ok; u += ustride, ++it) {
        const int b = it & 1;
        const uint32_t tmem_d = tmem_base + (uint32_t)(b * ACC_COLS);
        const uint32_t par = ((uint32_t)(it >> 1) & 1u) ^ 1u;
        if (it == 2) trace_stamp(tr, 13);  // the third tile wants the first buffer back
        ok = PAIR ? ptx::mbar_wait_cluster(bar_accempty + 8 * b, par, tmo, abort_flag)
                  : ptx::mbar_wait(bar_accempty + 8 * b, par, tmo, abort_flag);
        if (!ok) break;
        if (it == 2) trace_stamp(tr, 14);
        ptx::tc_fence_after();
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int s = g % ST;
          ok = ptx::mbar_wait(bar_full + 8 * s, (uint32_t)(g / ST) & 1u, tmo, abort_flag);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint64_t da = desc0 + (uint64_t)((s * L::S_BYTES) >> 4);
          const uint64_t db = da + (uint64_t)(L::A_BYTES >> 4);
#pragma unroll
          for (int kk = 0; kk < PF_BK / 16; ++kk) {  // 32 bytes of K per MMA
            if constexpr (PAIR)
              ptx::mma_f16_ss_pair(tmem_d, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk),
                                   idesc, (ks | kk) != 0 ? 1u : 0u);
            else
              ptx::mma_f16_ss(tmem_d, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk), idesc,
                              (ks | kk) != 0 ? 1u : 0u);
          }
          if constexpr (PAIR) {  // the stage is free in both CTAs
            ptx::mma_commit_pair(bar_empty + 8 * s);
            ptx::mma_commit_pair(empty1 + 8 * s);
          } else {
            ptx::mma_commit(bar_empty + 8 * s);
          }
        }
        if (!ok) break;
        if (!skip_accfull) {
          if constexpr (PAIR) {
            ptx::mma_commit_pair(bar_accfull + 8 * b);
            ptx::mma_commit_pair(accfull1 + 8 * b);
          } else {
            ptx::mma_commit(bar_accfull + 8 * b);
          }
        }
        // the tile's last MMA issued (its last stage landed)
        if (it < 2) trace_stamp(tr, 2 + it);
        else if (it == 2) trace_stamp(tr, 12);
      }
      trace_stamp(tr, 4);
      if constexpr (PAIR)
        ptx::mma_commit_pair(bar_drain);
      else
        ptx::mma_commit(bar_drain);
      pf_wait_drain(bar_drain, 0, tmo);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;              // TMEM lanes 32 q .. 32 q + 31 = tokens
    const int grp = (warp - 4) >> 2;     // column chunks grp, grp + 2, ...
    const uint32_t stg0 = sbase + L::OFF_O + (uint32_t)((warp - 4) * L::NSTAGING * L::OW_BYTES);
    int nchunk = 0;  // this warp's chunks so far: staging buffer nchunk % NSTAGING
    const int e = threadIdx.x - 128;     // 0..255: one column's scale and bias per tile
    ptx::pdl_wait();
    int it = 0;
    for (int u = unit0; u < units; u += ustride, ++it) {
      // this CTA's 128 tokens of the tile, all of the tile's columns
      const int m0 = (u / args.tiles_n) * TBM + rank * PF_BM, n0 = (u % args.tiles_n) * args.bn;
      const int b = it & 1;
      // the tile's weight scales and biases, once, into shared memory (two
      // buffers by tile parity: the barrier below keeps every warp within one
      // tile of the others)
      float* sb = reinterpret_cast<float*>(smem + L::OFF_SB) + b * 2 * PF_BN;
      {
        const int n = n0 + e;
        const bool in = e < args.bn && n < args.N;
        sb[e] = in ? __ldg(args.scales + n) : 0.f;
        sb[PF_BN + e] = in ? pf_load_bias(args.bias, args.bias_dtype, n) : 0.f;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      // RoPE: this thread's token row and its cos/sin values, loaded while
      // the tile's MMAs run
      int rm = 0, rb = 0, rs = 0;
      bool rtok = false;
      float rc1[16], rs1[16], rc2[16], rs2[16];
      if constexpr (ROPE) {
        rm = m0 + q * 32 + lane;
        rtok = rm < args.M;
        if (rtok) {
          rb = rm / args.rope.S;
          rs = rm - rb * args.rope.S;
          const float* cr = args.rope.cos + (size_t)rs * 64 + 16 * grp;
          const float* sr = args.rope.sin + (size_t)rs * 64 + 16 * grp;
          pf_ld32(cr, rc1);
          pf_ld32(cr + 8, rc1 + 8);
          pf_ld32(cr + 32, rc2);
          pf_ld32(cr + 40, rc2 + 8);
          pf_ld32(sr, rs1);
          pf_ld32(sr + 8, rs1 + 8);
          pf_ld32(sr + 32, rs2);
          pf_ld32(sr + 40, rs2 + 8);
        }
      }
      if (!ptx::mbar_wait(bar_accfull + 8 * b, (uint32_t)(it >> 1) & 1u, tmo, abort_flag)) break;
      if (warp == 4 && lane == 0 && it == 0) trace_stamp(tr, 5);
      if (warp == 4 && lane == 0 && it == 1) trace_stamp(tr, 10);
      ptx::tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t)(b * ACC_COLS) + ((uint32_t)(q * 32) << 16);
      if constexpr (ROPE) {
        // this thread's token row of the tile; group grp takes dims 16 grp ..
        // 16 grp + 15 of both halves of every head in the tile (32-byte
        // stores: whole L2 sectors).  The row's cos/sin values for those dims
        // were loaded before the accumulator wait and serve all the heads.
        const PfRope& rp = args.rope;
        const int heads = min(args.bn, args.N - n0) >> 6;  // N and n0 are multiples of 64
        const int gh0 = n0 >> 6;                            // q heads, then k, then v heads
        const int d0 = 16 * grp;
#pragma unroll 1
        for (int hh = 0; hh < heads; ++hh) {
          const int col0 = hh * 64;
          uint32_t o1[8], o2[8];  // dims d0 .. d0 + 15 and 32 + d0 .. 32 + d0 + 15, fp16 pairs
          const int gh = gh0 + hh;
          const bool rot = gh < rp.Hq + rp.Hkv;
          const float* scl = sb + col0;
          const float* bia = sb + PF_BN + col0;
#pragma unroll
          for (int c8 = 0; c8 < 2; ++c8) {
            uint32_t r[8], r2[8];  // dims d0 + 8 c8 .. and 32 + d0 + 8 c8 .. of head hh
            __syncwarp();          // tcgen05.ld is warp-collective
            ptx::tmem_ld_32x32b_x8(taddr + (uint32_t)(col0 + d0 + 8 * c8), r);
            ptx::tmem_ld_32x32b_x8(taddr + (uint32_t)(col0 + 32 + d0 + 8 * c8), r2);
            ptx::tmem_ld_wait();
            pf_reg_fence8(r);
            pf_reg_fence8(r2);
#pragma unroll
            for (int e2 = 0; e2 < 4; ++e2) {
              float y1[2], y2[2];
#pragma unroll
              for (int t2 = 0; t2 < 2; ++t2) {
                const int j = 8 * c8 + 2 * e2 + t2, d = d0 + j;
                // the projection's fp16 output, as the plain store rounds it
                const float a1 = __half2float(
                    __float2half_rn(fmaf(__uint_as_float(r[2 * e2 + t2]), scl[d], bia[d])));
                const float a2 = __half2float(__float2half_rn(
                    fmaf(__uint_as_float(r2[2 * e2 + t2]), scl[32 + d], bia[32 + d])));
                if (rot) {
                  y1[t2] = __fadd_rn(__fmul_rn(a1, rc1[j]), __fmul_rn(-a2, rs1[j]));
                  y2[t2] = __fadd_rn(__fmul_rn(a2, rc2[j]), __fmul_rn(a1, rs2[j]));
                } else {
                  y1[t2] = a1;
                  y2[t2] = a2;
                }
              }
              const __half2 h1 = __floats2half2_rn(y1[0], y1[1]);
              const __half2 h2 = __floats2half2_rn(y2[0], y2[1]);
              o1[4 * c8 + e2] = *reinterpret_cast<const uint32_t*>(&h1);
              o2[4 * c8 + e2] = *reinterpret_cast<const uint32_t*>(&h2);
            }
          }
          if (!rtok) continue;
          __half* dst;
          __half* dst2 = nullptr;
          if (gh < rp.Hq) {
            dst = rp.q_out + ((size_t)rm * rp.Hq + gh) * 64;
          } else {
            const bool isk = rot;
            const int g = isk ? gh - rp.Hq : gh - rp.Hq - rp.Hkv;
            dst = (isk ? rp.kc : rp.vc) + (size_t)rb * rp.cache_bstride +
                  ((size_t)g * rp.cap + rp.start + rs) * 64;
            __half* tm_out = isk ? rp.k_out : rp.v_out;
            if (tm_out) dst2 = tm_out + ((size_t)rm * rp.Hkv + g) * 64;
          }
          pf_st32(dst + d0, o1);
          pf_st32(dst + 32 + d0, o2);
          if (dst2) {
            pf_st32(dst2 + d0, o1);
            pf_st32(dst2 + 32 + d0, o2);
          }
        }
      }
#pragma unroll 1
      for (int c = grp; !ROPE && c < args.bn / PF_CH; c += 2) {
        const int col0 = c * PF_CH;
        if (n0 + col0 >= args.N) break;
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(taddr + (uint32_t)col0, r);
        // this chunk's 32 weight scales and biases (shared-memory broadcasts)
        float sc[PF_CH], bb[PF_CH];
#pragma unroll
        for (int j4 = 0; j4 < PF_CH / 4; ++j4) {
          const float4 s4 = reinterpret_cast<const float4*>(sb + col0)[j4];
          const float4 b4 = reinterpret_cast<const float4*>(sb + PF_BN + col0)[j4];
          sc[4 * j4] = s4.x; sc[4 * j4 + 1] = s4.y; sc[4 * j4 + 2] = s4.z; sc[4 * j4 + 3] = s4.w;
          bb[4 * j4] = b4.x; bb[4 * j4 + 1] = b4.y; bb[4 * j4 + 2] = b4.z; bb[4 * j4 + 3] = b4.w;
        }
        ptx::tmem_ld_wait();
        pf_reg_fence(r);
        // the staging buffer is free again once at most NSTAGING - 1 of this
        // warp's stores are still reading
        if (lane == 0) {
          if constexpr (L::NSTAGING == 2)
            ptx::bulk_wait_group_read1();
          else
            ptx::bulk_wait_group_read0();
        }
        __syncwarp();
        const uint32_t stg = stg0 + (uint32_t)((nchunk++ % L::NSTAGING) * L::OW_BYTES);
        if constexpr (SWIGLU) {
          // a 32-column chunk is one interleave block: columns 0-15 are gate
          // rows 16 b .. 16 b + 15, columns 16-31 the matching up rows.  gate
          // and up are rounded to fp16 as the two-GEMM path rounds them, then
          // silu(g) * u in fp32 (SwiGLU_d.cu:22-24); 16 outputs per token row.
          uint32_t hz[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float o[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int c = 2 * j + t;
              const float g = __half2float(__float2half_rn(fmaf(__uint_as_float(r[c]), sc[c], bb[c])));
              const float u = __half2float(
                  __float2half_rn(fmaf(__uint_as_float(r[16 + c]), sc[16 + c], bb[16 + c])));
              o[t] = __fdividef(g, 1.0f + __expf(-g)) * u;
            }
            const __half2 hv = __floats2half2_rn(o[0], o[1]);
            hz[j] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          // staging: 32 rows (tokens) x 32 B, unswizzled
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint32_t a = stg + (uint32_t)(lane * 32 + j * 16);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(hz[4 * j]),
                         "r"(hz[4 * j + 1]), "r"(hz[4 * j + 2]), "r"(hz[4 * j + 3])
                         : "memory");
          }
        } else {
          uint32_t h[PF_CH / 2];
#pragma unroll
          for (int j = 0; j < PF_CH / 2; ++j) {
            const float v0 = fmaf(__uint_as_float(r[2 * j]), sc[2 * j], bb[2 * j]);
            const float v1 = fmaf(__uint_as_float(r[2 * j + 1]), sc[2 * j + 1], bb[2 * j + 1]);
            const __half2 hv = __floats2half2_rn(v0, v1);
            h[j] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          // staging: 32 rows (tokens) x 64 B, 64-byte swizzle (16-byte chunk
          // j of row r at chunk j ^ ((r >> 1) & 3)), matching the store map
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a = stg + (uint32_t)(lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4));
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(h[4 * j]),
                         "r"(h[4 * j + 1]), "r"(h[4 * j + 2]), "r"(h[4 * j + 3])
                         : "memory");
          }
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && m0 + q * 32 < args.M) {
          ptx::tma_store_2d(&tm_y, stg, SWIGLU ? (n0 + col0) >> 1 : n0 + col0, m0 + q * 32);
          ptx::bulk_commit_group();
        }
      }
      // release the accumulator once this warp's TMEM loads are done (a
      // pair's MMAs wait on rank 0's barrier for the warps of both CTAs)
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          ptx::mbar_arrive_cluster(accempty0 + 8 * b);
        else
          ptx::mbar_arrive(bar_accempty + 8 * b);
        if (warp == 4 && it < 2) trace_stamp(tr, 9 + 2 * it);  // tile 0 / 1 released
      }
    }
    if (lane == 0) ptx::bulk_wait_group0();
    __syncwarp();
  }

  if (threadIdx.x == 128) trace_stamp(tr, 6);
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {
    // neither CTA exits (or frees TMEM) while the other may still signal its
    // barriers or run MMAs on its shared memory; after a timeout, rank 1's
    // copies in flight (counted on rank 0's barriers) get 20 us to land
    ptx::cluster_sync();
    if (*abort_flag) {
      const uint64_t t0 = ptx::globaltimer_ns();
      while (ptx::globaltimer_ns() - t0 < 20000ull) __nanosleep(1000);
    }
    __syncthreads();
  }
  if (warp == 0) {
    ptx::tc_fence_after();
    if constexpr (PAIR)
      ptx::tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
  if (threadIdx.x == 0) trace_stamp(tr, 7);
}

// ============================================================================
// Host side
// ============================================================================
namespace {

PFN_cuTensorMapEncodeTiled_v12000 pf_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int pf_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
            uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto enc = pf_encoder();
  if (!enc) return DDQ_ERR_DEVICE;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDQ_OK : DDQ_ERR_ALIGNMENT;
}

cudaLaunchAttribute pdl_attr() {
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  return at;
}

// Tile width over the weight rows: the time of a tile grows with its width,
// and the CTAs (or CTA pairs) run ceil(tiles / slots) tiles each; pick the
// width that minimises waves x (width + a fixed per-tile cost).  The cost,
// ~300 columns' worth, is fitted to gate/up at 4096 tokens on pairs: 60.5,
// 62.4, 68.4 and 78.0 us at widths 256, 224, 192 and 160 (9, 10, 12 and 14
// waves), i.e. ~3.65 us a wave plus ~0.012 us a column.
// Weight rows from which pairs are used; DDQ_PF_PAIR_MIN_N overrides it for
// measurements.
int64_t pf_pair_min_n() {
  static const int64_t v = [] {
    const char* e = std::getenv("DDQ_PF_PAIR_MIN_N");
    return e ? (int64_t)std::atoll(e) : (int64_t)2048;
  }();
  return v;
}

int pf_env_bn() {
  static const int v = [] {
    const char* e = std::getenv("DDQ_PF_BN");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

// Token count from which prefill GEMMs run on CTA pairs; DDQ_PF_PAIR_MIN_M
// overrides it for measurements (0: never).
int64_t pf_pair_min_m() {
  static const int64_t v = [] {
    const char* e = std::getenv("DDQ_PF_PAIR_MIN_M");
    const int64_t n = e ? (int64_t)std::atoll(e) : (int64_t)512;
    return n <= 0 ? (int64_t)1 << 62 : n;
  }();
  return v;
}

int pf_pick_bn(int M, int N, int sms, int step, bool pair) {
  const int tbm = pair ? 2 * PF_BM : PF_BM;
  const int tm = (M + tbm - 1) / tbm;
  const int slots = pair ? sms / 2 : sms;
  int best = PF_BN;
  long best_cost = -1;
  for (int bn = PF_BN; bn >= 128; bn -= step) {
    const long tiles = (long)tm * ((N + bn - 1) / bn);
    const long waves = (tiles + slots - 1) / slots;
    const long cost = waves * (bn + 300);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace

size_t pf_workspace_bytes(int64_t N, int64_t K) { return (size_t)N * (size_t)K * 2; }

namespace {
// Per workspace: which of its two fp16 buffers the next prefill call uses,
// and whether that call's expansion may write before the previous kernel has
// finished.  That is safe only when the kernel just before it on the stream
// is this library's prefill GEMM reading the other buffer (that GEMM lets its
// dependents launch only after its own dependency, so the GEMM before it -
// the other buffer's last reader - has finished).  The host can know that
// only for calls made eagerly, in stream order, on a workspace whose calls
// were never recorded into a CUDA graph: a replayed graph runs its kernels
// between eager calls without the host seeing them.  Hence:
//   * a call made while its stream is capturing never expands early, and
//     marks the workspace "captured" for good (later eager calls on it never
//     expand early either);
//   * an eager call expands early only if the previous call on the workspace
//     was an eager prefill call on a never-captured workspace.
// A decode-shape call keeps its activation planes at the start of the same
// workspace and resets the history (ws_note_other_use).  Forgetting an entry
// is always safe (the next call waits), so the table is cleared if a caller
// cycles through very many workspaces; a captured mark lost that way is
// re-established only by the next capture, so the table is cleared only of
// never-captured entries.
struct PfWs {
  int half = 0;
  bool last_pf = false;   // unknown history: wait, as with a single buffer
  bool captured = false;  // used inside a stream capture at least once
};
std::mutex g_pf_ws_mu;
std::unordered_map<const void*, PfWs> g_pf_ws;
constexpr size_t kPfWsMax = 4096;
PfWs& pf_ws_entry(const void* ws) {
  if (g_pf_ws.size() >= kPfWsMax && g_pf_ws.find(ws) == g_pf_ws.end()) {
    for (auto it = g_pf_ws.begin(); it != g_pf_ws.end();)
      it = it->second.captured ? std::next(it) : g_pf_ws.erase(it);
  }
  return g_pf_ws[ws];
}

bool stream_capturing(cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
    cudaGetLastError();
    return true;  // unknown: treat as captured (never early)
  }
  return cs != cudaStreamCaptureStatusNone;
}
}  // namespace

void ws_note_other_use(const void* ws, cudaStream_t s) {
  if (!ws) return;
  const bool cap = stream_capturing(s);
  std::lock_guard<std::mutex> lock(g_pf_ws_mu);
  PfWs& st = pf_ws_entry(ws);
  st.last_pf = false;
  st.captured = st.captured || cap;
}

// The buffer (0 or 1) for this prefill call, and whether its expansion may
// run ahead of the previous kernel.
static int pf_take_buffer(const void* ws, cudaStream_t s, bool* early) {
  const bool cap = stream_capturing(s);
  std::lock_guard<std::mutex> lock(g_pf_ws_mu);
  PfWs& st = pf_ws_entry(ws);
  st.captured = st.captured || cap;
  *early = st.last_pf && !st.captured;
  st.last_pf = !st.captured;
  st.half ^= 1;
  return st.half;
}

int launch_pf(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, void* ws, size_t ws_bytes,
              unsigned long long timeout_ns, int debug_flags, cudaStream_t s, bool swiglu,
              const PfRope* rope) {
  const int dev = current_device();
  const int sms = device_sm_count(dev);
  if (sms <= 0 || dev < 0 || dev >= 64) return DDQ_ERR_DEVICE;
  if (M < 1 || N < 1 || K < 16 || K % 16 != 0) return DDQ_ERR_SHAPE;
  if (!ws || ws_bytes < pf_workspace_bytes(N, K)) return DDQ_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) || !aligned16(x) || (!rope && !aligned16(y)) ||
      (N % 8) != 0)
    return DDQ_ERR_ALIGNMENT;
  if (swiglu && N % 32 != 0) return DDQ_ERR_SHAPE;
  if (rope && (swiglu || N != (rope->Hq + 2 * rope->Hkv) * 64 || rope->S < 1 || M % rope->S != 0))
    return DDQ_ERR_SHAPE;
  // a workspace of two buffers at fixed offsets (0 and half the workspace,
  // whatever the shape, so that calls of different shapes never overlap):
  // consecutive calls alternate them, so this call's expansion need not wait
  // for the previous GEMM
  const size_t need = pf_workspace_bytes(N, K);
  const size_t half = (ws_bytes / 2) & ~static_cast<size_t>(255);
  bool early = false;
  size_t off = 0;
  if (need <= half) {
    off = (size_t)pf_take_buffer(ws, s, &early) * half;
  } else {
    ws_note_other_use(ws, s);  // the single buffer: always wait for the previous kernel
  }
  __half* w16 = reinterpret_cast<__half*>(static_cast<uint8_t*>(ws) + off);
  // 1) exact e4m3 -> fp16 expansion of the weights
  {
    const size_t n16 = (size_t)N * (size_t)K / 16;
    cudaLaunchConfig_t cfg = {};
    const size_t want = (n16 + 255) / 256;
    const size_t cap = (size_t)sms * 4;
    cfg.gridDim = dim3((unsigned)(want < cap ? want : cap));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at = pdl_attr();
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, e4m3_to_f16_kernel, wq, w16, n16, early ? 1 : 0) !=
        cudaSuccess) {
      cudaGetLastError();
      return DDQ_ERR_LAUNCH;
    }
  }
  // 2) the fp16 GEMM, on CTA pairs from pf_pair_min_m() tokens for wide
  //    weights (gate/up at 4096 tokens: 62.3 against 64.1 us; the 896- and
  //    1152-row projections measured 1-11 % slower on pairs)
  const bool pair =
      (debug_flags & 128) == 0 && M >= pf_pair_min_m() && N >= pf_pair_min_n() && sms >= 2;
  const int epi = rope ? PF_EPI_ROPE : swiglu ? PF_EPI_SWIGLU : PF_EPI_STORE;
  using PfKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, PfArgs);
  static const PfKernel kernels[2][3] = {
      {w8a16_pf_kernel<PF_EPI_STORE, false>, w8a16_pf_kernel<PF_EPI_SWIGLU, false>,
       w8a16_pf_kernel<PF_EPI_ROPE, false>},
      {w8a16_pf_kernel<PF_EPI_STORE, true>, w8a16_pf_kernel<PF_EPI_SWIGLU, true>,
       w8a16_pf_kernel<PF_EPI_ROPE, true>}};
  const PfKernel kern = kernels[pair ? 1 : 0][epi];
  const int alloc = pair ? PfLayout2::ALLOC : PfLayout::ALLOC;
  static SmemAttrOnce attr[2][3];
  const int ast = ensure_smem_attr(attr[pair ? 1 : 0][epi], dev, kern, alloc);
  if (ast) return ast;
  CUtensorMap tm_x, tm_w, tm_y;
  int st = pf_tmap(&tm_x, x, (uint64_t)K, (uint64_t)M, PF_BK, PF_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  // the RoPE epilogue takes whole 64-row heads: head-aligned tile widths
  // (DDQ_PF_BN fixes the width, for measurements)
  const int bn_env = pf_env_bn();
  const int bn = bn_env >= 128 && bn_env <= PF_BN && bn_env % (rope ? 64 : 32) == 0
                     ? bn_env
                     : pf_pick_bn(M, N, sms, rope ? 64 : 32, pair);
  // a pair's CTAs load half of the tile's weight rows each
  st = pf_tmap(&tm_w, w16, (uint64_t)K, (uint64_t)N, PF_BK, (uint32_t)(pair ? bn / 2 : bn),
               CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  if (rope)
    tm_y = tm_x;  // not stored through: the RoPE epilogue writes q, k, v directly
  else if (swiglu)
    st = pf_tmap(&tm_y, y, (uint64_t)(N / 2), (uint64_t)M, PF_CH / 2, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    st = pf_tmap(&tm_y, y, (uint64_t)N, (uint64_t)M, PF_CH, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (st) return st;
  PfArgs a{};
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.M = M;
  a.N = N;
  a.K = K;
  a.bn = bn;
  const int tbm = pair ? 2 * PF_BM : PF_BM;
  a.tiles_m = (M + tbm - 1) / tbm;
  a.tiles_n = (N + bn - 1) / bn;
  a.timeout_ns = timeout_ns;
  a.debug_flags = debug_flags;
  if (rope) a.rope = *rope;
  const int units = a.tiles_m * a.tiles_n;
  const int slots = pair ? sms / 2 : sms;
  const int grid = (units < slots ? units : slots) * (pair ? 2 : 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(PF_THREADS);
  cfg.dynamicSmemBytes = alloc;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0] = pdl_attr();
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = pair ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, tm_x, tm_w, tm_y, a) != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace ddq
