// tc_decode.cu - the decode-shape (M <= 64) W8A16 GEMM on the e4m3 tensor
// cores: no per-weight-byte conversion at all.
//
// Converting every weight byte to fp16 costs a few ALU instructions per byte;
// at decode rates (tens of bytes per SM clock) that is more issue bandwidth
// than an SM has.  Instead the activations - M x K, tiny - are split once,
// per token row m, into three e4m3 planes under a power-of-two scale:
//     z = x[m,:] * 2^e_m        (exact; e_m puts max|z| in [128, 256))
//     h1 = e4m3(z), h2 = e4m3(z - h1), h3 = e4m3(z - h1 - h2)   (RNE)
// h1 + h2 + h3 equals z to within 2^-12 |z| (or 2^-10 absolute for the
// smallest elements), finer than fp16's own 2^-11 rounding of x.  Then
//     y[m, n] = scale[n] * 2^-e_m * sum_k Wq[n,k] * (h1 + h2 + h3)[m,k] + bias[n]
// is one tcgen05.mma kind::f8f6f4 (e4m3 x e4m3, fp32 accumulate in TMEM)
// per 32-wide K step with the weight tile as the 128-row A operand straight
// from TMA and the three planes stacked as the B operand (N = 3 * BT); the
// epilogue adds the three accumulator column blocks.
//
// Kernels:
//   xsplit_kernel   one CTA per token row: row max, e_m, the three planes
//                   (written to the workspace) and 2^-e_m.
//   w8a16_dec_kernel  persistent (or, for few tiles, split-K over a cluster
//                   with a distributed-shared-memory reduction, as in
//                   tc_gemm.cu), 256 threads:
//     warp 0     TMA producer of the e4m3 weight stages (128 rows x 128 B,
//                128-byte swizzle); issues its first stages and an L2
//                prefetch of the rest of its first tile before the grid
//                dependency (the split pre-pass) resolves
//     warp 1     MMA issuer (4 MMAs of K = 32 per stage, double-buffered TMEM
//                accumulator)
//     warp 2     TMA producer of the activation planes (after the grid wait)
//     warps 4-7  epilogue: tcgen05.ld of the three blocks (the next chunk's
//                loads in flight while this one is stored) -> sum -> weight
//                and token scales, bias, fp16 -> a TMA store of each warp's
//                32 x 16 tile; or the fused lm_head's running greedy key.
// Every mbarrier wait is bounded (see sm100_ptx.cuh); on timeout the CTA
// records DDQ_ERR_TIMEOUT, drains its copies and MMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cfloat>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int DC_BN = 128;       // weight rows per tile (MMA M)
constexpr int DC_AK = 128;       // K bytes per 128-byte swizzle atom (one TMA box)
constexpr int DC_THREADS = 384;  // 12 warps

// K bytes per pipeline stage: two swizzle atoms (8 MMAs per barrier round
// trip) where the ring still holds enough stages, one for the 64-token tile.
__host__ __device__ constexpr int dc_stage_k(int bt) { return bt <= 32 ? 256 : 128; }

// ----------------------------------------------------------------------------
// Activation split pre-pass
// ----------------------------------------------------------------------------
// One CTA (256 threads) per token row; the row's 16-byte chunks stay in
// registers (CPT per thread), so x is read once: load, row max, scale, split,
// store.  Rows longer than 256 * CPT * 8 elements use the CPT = 0 variant,
// which reads the row twice.
template <int CPT>
__global__ void __launch_bounds__(256) xsplit_kernel(const __half* __restrict__ x,
                                                     uint8_t* __restrict__ planes,
                                                     float* __restrict__ xscale, int M, int K,
                                                     unsigned long long* __restrict__ zero_packed) {
  // Let the GEMM that follows launch now (it prefetches its weights while
  // this grid and the one before it finish), then wait for x, which may be
  // the previous kernel's output (both no-ops without PDL).
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int m = blockIdx.x;
  const int nch = K / 8;
  // the greedy GEMM after this pass takes its per-token maxima with atomicMax
  // (after its own grid dependency on this pass): start them at zero here
  if (zero_packed != nullptr && threadIdx.x == 0) zero_packed[m] = 0ull;
  const __half* xr = x + (size_t)m * K;
  constexpr int R = CPT > 0 ? CPT : 1;
  uint4 v[R];
  float amax = 0.f;
  if (CPT > 0) {
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int c = threadIdx.x + j * 256;
      v[j] = c < nch ? __ldg(reinterpret_cast<const uint4*>(xr) + c) : make_uint4(0u, 0u, 0u, 0u);
      const __half2* h = reinterpret_cast<const __half2*>(&v[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  } else {
    for (int c = threadIdx.x; c < nch; c += 256) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr) + c);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  __shared__ float red[8];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const int e = split_shift(amax);      // max |z| in [128, 256)
  const float up = ldexpf(1.f, e);
  if (threadIdx.x == 0) xscale[m] = ldexpf(1.f, -e);
  const size_t plane = (size_t)M * K;
  uint8_t* p1 = planes + (size_t)m * K;
  auto emit = [&](int c, const uint4& u) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    float z[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      z[2 * i] = f.x * up;                // exact: power-of-two scale
      z[2 * i + 1] = f.y * up;
    }
    uint2 a, b, cc;
    split8(z, a, b, cc);
    *reinterpret_cast<uint2*>(p1 + (size_t)c * 8) = a;
    *reinterpret_cast<uint2*>(p1 + plane + (size_t)c * 8) = b;
    *reinterpret_cast<uint2*>(p1 + 2 * plane + (size_t)c * 8) = cc;
  };
  if (CPT > 0) {
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int c = threadIdx.x + j * 256;
      if (c < nch) emit(c, v[j]);
    }
  } else {
    for (int c = threadIdx.x; c < nch; c += 256)
      emit(c, __ldg(reinterpret_cast<const uint4*>(xr) + c));
  }
}

// ----------------------------------------------------------------------------
// Decode GEMM
// ----------------------------------------------------------------------------
// Split-K ownership: rank r of a cluster of n owns the 4-token groups of
// tokens [r tpo, (r + 1) tpo), tpo = ceil(M / n) rounded up to 4.
__host__ __device__ constexpr int dc_tpo(int m, int n) { return ((m + n - 1) / n + 3) & ~3; }
// bytes of one rank's own groups (128 rows x 16 B per group), worst case over n
__host__ __device__ constexpr int dc_own_bytes_max(int bt) { return dc_tpo(bt, 2) * DC_BN * 4; }
// bytes a rank receives: n - 1 senders x its groups, worst case over 2 <= n <= 8
static_assert(kMaxSplits <= 8, "split-K bounds below assume at most 8 ranks");
__host__ __device__ constexpr int dc_recv_bytes_max(int bt) {
  int w = 0;
  for (int n = 2; n <= 8; ++n) {
    const int b = (n - 1) * dc_tpo(bt, n) * DC_BN * 4;
    w = b > w ? b : w;
  }
  return w;
}

// A stage holds KB bytes of K (NA = KB / 128 swizzle atoms) of the weight
// tile and of the three activation planes.
template <int BT, int ST, int KB>
struct DcLayout {
  static constexpr int CH = 16;                          // epilogue token chunk
  static constexpr int NA = KB / DC_AK;                  // atoms per stage
  static constexpr int WA_BYTES = DC_BN * DC_AK;         // 16 KB: one weight atom
  static constexpr int XA_BYTES = 3 * BT * DC_AK;        // one atom of the three planes
  static constexpr int W_BYTES = NA * WA_BYTES;
  static constexpr int X_BYTES = NA * XA_BYTES;          // B operand rows: plane p, token m -> p BT + m
  static constexpr int S_BYTES = W_BYTES + X_BYTES;
  static constexpr int OFF_S = 0;
  static constexpr int P_BYTES = DC_BN * BT * 4;         // split-K partial (ring reused)
  static constexpr int OW_BYTES = CH * 32 * 2;          // one warp's output staging chunk
  static constexpr int OFF_O = ST * S_BYTES;             // 8 warps x 2 staging buffers
  static constexpr int OFF_BAR = OFF_O + 16 * OW_BYTES;
  static constexpr int NBAR = 2 * ST + 4 + 2;            // full, empty; acc x2 x2; drain; recv
  static constexpr int OFF_MISC = (OFF_BAR + NBAR * 8 + 15) & ~15;
  static constexpr int OFF_RED = OFF_MISC + 16;
  static constexpr int RED_BYTES = 4 * BT * 8;
  static constexpr int OFF_XS = OFF_RED + RED_BYTES;  // token scales 2^-e [BT]
  static constexpr int CORE_BYTES = OFF_XS + BT * 4;
  // split-K: this CTA's own 4-token groups at the start of the ring (free
  // once its MMAs are done); the groups the other ranks send, which may
  // arrive while this CTA still streams, behind everything else when that
  // fits, else in the last ring stage (ring depth ST - 1 in split mode)
  static constexpr int OFF_OWN = 0;
  static constexpr bool RECV_IN_RING = CORE_BYTES + 16 + dc_recv_bytes_max(BT) + 1024 > 232448;
  static constexpr int OFF_RECV = RECV_IN_RING ? (ST - 1) * S_BYTES : (CORE_BYTES + 15) & ~15;
  static constexpr int BYTES = RECV_IN_RING ? CORE_BYTES : OFF_RECV + dc_recv_bytes_max(BT);
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr int ACC_COLS = 3 * BT <= 64 ? 64 : 3 * BT <= 128 ? 128 : 256;  // per buffer
  static_assert(S_BYTES % 1024 == 0 && XA_BYTES % 1024 == 0, "atoms keep 1024-B alignment");
  static_assert(KB == 128 || KB == 256, "stage K bytes");
  static_assert(OFF_XS % 16 == 0, "token scales are read as float4");
  static_assert(ST >= 2, "split-K keeps ST - 1 ring stages");
  static_assert(dc_own_bytes_max(BT) <= (ST - 1) * S_BYTES, "own split-K groups fit the ring");
  static_assert(!RECV_IN_RING || dc_recv_bytes_max(BT) <= S_BYTES,
                "received split-K groups fit one stage");
  static_assert(ALLOC <= 232448, "shared memory budget");
  static_assert(3 * BT <= 256, "N = 3 BT must fit one MMA");
};

struct DcArgs {
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  unsigned long long* packed;
  int64_t vocab_offset;
  const float* xscale;  // 2^-e per token row
  int M, N, K, kps;     // kps in stages of KB bytes of K
  int n_tiles;
  int out_n;            // output row length: N, or N / 2 for the SwiGLU epilogue
  int y_tma;
  unsigned long long timeout_ns;
  int debug_flags;
  long long* ids;          // greedy epilogue: token ids, written by the last CTA (or NULL)
  unsigned int* counter;   // its arrival counter, zero between calls (NULL: no ids here)
};

__device__ __forceinline__ float dc_load_bias(const void* bias, int bias_dtype, int n) {
  if (bias_dtype == DDQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (bias_dtype == DDQ_DTYPE_F32) return reinterpret_cast<const float*>(bias)[n];
  return 0.f;
}

__device__ __forceinline__ unsigned long long dc_warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}

// The three plane blocks (columns c, BT + c, 2 BT + c) of CH = 16 token columns.
template <int BT>
__device__ __forceinline__ void dc_ld_chunk_t(uint32_t taddr, int c, uint32_t (&r)[3][16]) {
  ptx::tmem_ld_32x32b_x16(taddr + (uint32_t)c, r[0]);
  ptx::tmem_ld_32x32b_x16(taddr + (uint32_t)(BT + c), r[1]);
  ptx::tmem_ld_32x32b_x16(taddr + (uint32_t)(2 * BT + c), r[2]);
}
#define dc_ld_chunk(taddr, c, r) dc_ld_chunk_t<BT>(taddr, c, r)

// Ties the loaded registers to the preceding tcgen05.wait::ld: no use of them
// can be scheduled above the wait.
__device__ __forceinline__ void dc_reg_fence(uint32_t (&r)[3][16]) {
#pragma unroll
  for (int p = 0; p < 3; ++p)
    asm volatile(""
                 : "+r"(r[p][0]), "+r"(r[p][1]), "+r"(r[p][2]), "+r"(r[p][3]), "+r"(r[p][4]),
                   "+r"(r[p][5]), "+r"(r[p][6]), "+r"(r[p][7]), "+r"(r[p][8]), "+r"(r[p][9]),
                   "+r"(r[p][10]), "+r"(r[p][11]), "+r"(r[p][12]), "+r"(r[p][13]),
                   "+r"(r[p][14]), "+r"(r[p][15])::"memory");
}

__device__ __forceinline__ void dc_epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ bool dc_wait_drain(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  const long long t0 = clock64();
  const long long limit = (long long)(timeout_ns * 2ull);
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

// Instruction descriptor, kind::f8f6f4: D fp32, A/B e4m3 (format 0), K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Epilogue kinds: plain fp16 store, the fused lm_head's greedy argmax, and
// SwiGLU over a 16-row interleaved gate/up weight (silu(gate) * up stored).
constexpr int DC_EPI_STORE = 0, DC_EPI_ARGMAX = 1, DC_EPI_SWIGLU = 2;

template <int BT, int ST, int KB, int EPI>
__global__ void __launch_bounds__(DC_THREADS, 1)
    w8a16_dec_kernel(const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_y, const DcArgs args) {
  using L = DcLayout<BT, ST, KB>;
  constexpr bool ARGMAX = EPI == DC_EPI_ARGMAX;
  constexpr bool SWIGLU = EPI == DC_EPI_SWIGLU;
  constexpr int CH = L::CH;
  constexpr uint32_t ACC_COLS = L::ACC_COLS;
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsplit = gridDim.z;
  const int KS = (args.K + KB - 1) / KB;
  const uint64_t tmo = args.timeout_ns;
  const bool tr = (args.debug_flags & 2) != 0;
  const int units = args.n_tiles;  // one token tile (M <= BT)
  const int unit0 = (int)blockIdx.x;
  const int ustride = (nsplit > 1) ? units : (int)gridDim.x;
  const int mvalid = min(BT, args.M);
  // split-K partials: up to 32 tokens each rank pushes the owners their
  // groups; 64-token tiles (4x the bytes, where pushing measured slower) park
  // them for the owners to read
  constexpr bool PUSH = BT <= 32;
  // ring depth: in split-K mode the last stage may receive the other ranks' partials
  const int NS = nsplit > 1 && PUSH && L::RECV_IN_RING ? ST - 1 : ST;
  const int tpo = dc_tpo(mvalid, nsplit);  // split-K tokens per rank (multiple of 4)
  const int m4 = (mvalid + 3) & ~3;
  auto unit_k = [&](int& kb, int& nk) {
    kb = (nsplit > 1 ? (int)blockIdx.z : 0) * args.kps;
    nk = max(0, min(args.kps, KS - kb));
  };

  // full[s]: both producers arrive (expect_tx) and their TMA bytes land
  const uint32_t bar_full = sbase + L::OFF_BAR;
  const uint32_t bar_empty = bar_full + 8 * ST;
  const uint32_t bar_accfull = bar_empty + 8 * ST;   // [2]
  const uint32_t bar_accempty = bar_accfull + 16;    // [2]
  const uint32_t bar_drain = bar_accempty + 16;
  const uint32_t bar_recv = bar_drain + 8;           // split-K partials from the other ranks
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) trace_stamp(tr, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 2);
      ptx::mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar_accfull + 8 * b, 1);
      ptx::mbar_init(bar_accempty + 8 * b, 8);
    }
    ptx::mbar_init(bar_drain, 1);
    if (PUSH && nsplit > 1) ptx::mbar_init(bar_recv, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    if (PUSH && nsplit > 1) {
      // this rank's groups, 16 bytes per row from each of the other ranks
      const int r = (int)ptx::cluster_ctarank();
      const int ng = max(0, min(tpo, m4 - r * tpo)) >> 2;
      ptx::mbar_arrive_expect_tx(bar_recv, (uint32_t)((nsplit - 1) * ng * DC_BN * 16));
    }
    ptx::prefetch_tmap(&tm_w);
    ptx::prefetch_tmap(&tm_x);
    if (args.y_tma) ptx::prefetch_tmap(&tm_y);
  }
  if (warp == 0) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // split-K: every rank's receive barrier is initialised before any rank sends
  // (the matching wait comes just before the first send, or at the end)
  if (PUSH && nsplit > 1) ptx::cluster_arrive_relaxed();
  if (threadIdx.x == 0) trace_stamp(tr, 1);
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  // K atoms of stage index ks that hold data (the last stage may be short)
  auto stage_atoms = [&](int ks) {
    const int rem = args.K - ks * KB;
    return rem >= KB ? L::NA : (rem + DC_AK - 1) / DC_AK;
  };

  bool have_acc = false;
  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      auto issue_w = [&](int s, int ks, int n0) {
        const int na = stage_atoms(ks);
        const uint32_t full = bar_full + 8 * s;
        ptx::mbar_arrive_expect_tx(full, (uint32_t)(na * L::WA_BYTES));
        for (int a = 0; a < na; ++a)
          ptx::tma_load_2d(sbase + L::OFF_S + s * L::S_BYTES + a * L::WA_BYTES, &tm_w,
                           ks * KB + a * DC_AK, n0, full);
      };
      int g = 0, rs = 0;  // stage count; its ring slot g % NS and phase (g / NS) & 1
      uint32_t rph = 0u;
      auto adv = [&] {
        ++g;
        if (++rs == NS) {
          rs = 0;
          rph ^= 1u;
        }
      };
      bool ok = true, waited = false;
      for (int u = unit0; u < units && ok; u += ustride) {
        int kb, nk;
        unit_k(kb, nk);
        const int n0 = u * DC_BN;
        int i = 0;
        if (!waited) {
          const int pre = nk < NS ? nk : NS;
          for (; i < pre; ++i, adv()) issue_w(rs, kb + i, n0);  // fresh stages: no wait
          for (int i2 = NS; i2 < nk; ++i2)
            for (int a = 0; a < stage_atoms(kb + i2); ++a)
              ptx::tma_prefetch_l2_2d(&tm_w, (kb + i2) * KB + a * DC_AK, n0);
          trace_stamp(tr, 2);
          ptx::pdl_wait();
          waited = true;
        }
        for (; i < nk; ++i, adv()) {
          if (!ptx::mbar_wait(bar_empty + 8 * rs, rph ^ 1u, tmo, abort_flag)) {
            ok = false;
            break;
          }
          issue_w(rs, kb + i, n0);
        }
      }
      if (!waited) ptx::pdl_wait();
      if (*abort_flag) {
        for (int i = g > NS ? g - NS : 0; i < g; ++i)
          dc_wait_drain(bar_full + 8 * (i % NS), (uint32_t)(i / NS) & 1u, tmo);
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ activation-plane producer
    // one 3-D box {128 B of K, BT tokens, 3 planes} per atom: the B operand
    // rows p BT + m, tokens m >= M zero-filled
    if (lane == 0) {
      ptx::pdl_wait();  // the planes come from the split pre-pass
      trace_stamp(tr, 3);
      int g = 0, rs = 0;
      uint32_t rph = 0u;
      bool ok = true;
      for (int u = unit0; u < units && ok; u += ustride) {
        int kb, nk;
        unit_k(kb, nk);
        for (int i = 0; i < nk; ++i) {
          if (!ptx::mbar_wait(bar_empty + 8 * rs, rph ^ 1u, tmo, abort_flag)) {
            ok = false;
            break;
          }
          const int na = stage_atoms(kb + i);
          const uint32_t full = bar_full + 8 * rs;
          ptx::mbar_arrive_expect_tx(full, (uint32_t)(na * L::XA_BYTES));
          const uint32_t dst = sbase + L::OFF_S + rs * L::S_BYTES + L::W_BYTES;
          for (int a = 0; a < na; ++a)
            ptx::tma_load_3d(dst + a * L::XA_BYTES, &tm_x, (kb + i) * KB + a * DC_AK, 0, 0, full);
          ++g;
          if (++rs == NS) {
            rs = 0;
            rph ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        for (int i = g > NS ? g - NS : 0; i < g; ++i)
          dc_wait_drain(bar_full + 8 * (i % NS), (uint32_t)(i / NS) & 1u, tmo);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(DC_BN, 3 * BT);
      // descriptor of stage 0's weight atom 0; other atoms and K steps are
      // offsets in the 16-byte address field
      const uint64_t desc0 = ptx::smem_desc_sw128(sbase + L::OFF_S);
      ptx::pdl_wait();
      bool ok = true;
      int it = 0, rs = 0;
      uint32_t rph = 0u;
      for (int u = unit0; u < units && ok; u += ustride, ++it) {
        int kb, nk;
        unit_k(kb, nk);
        const int b = it & 1;
        const uint32_t tmem_d = tmem_base + (uint32_t)(b * ACC_COLS);
        ok = ptx::mbar_wait(bar_accempty + 8 * b, ((uint32_t)(it >> 1) & 1u) ^ 1u, tmo, abort_flag);
        if (!ok) break;
        ptx::tc_fence_after();
        for (int i = 0; i < nk; ++i) {
          const int s = rs;  // ring slot and phase of this stage
          const uint32_t ph = rph;
          if (++rs == NS) {
            rs = 0;
            rph ^= 1u;
          }
          ok = ptx::mbar_wait(bar_full + 8 * s, ph, tmo, abort_flag);
          if (!ok) break;
          ptx::tc_fence_after();
          const int rem = args.K - (kb + i) * KB;
          const int nkk = rem >= KB ? KB / 32 : (rem + 31) / 32;  // 32-byte K steps with data
          const uint64_t dw = desc0 + (uint64_t)((s * L::S_BYTES) >> 4);
          const uint64_t dx = dw + (uint64_t)(L::W_BYTES >> 4);
#pragma unroll
          for (int a = 0; a < L::NA; ++a)
#pragma unroll
            for (int kk = 0; kk < DC_AK / 32; ++kk)
              if (a * (DC_AK / 32) + kk < nkk)
                mma_f8_ss(tmem_d, dw + (uint64_t)((a * L::WA_BYTES + 32 * kk) >> 4),
                          dx + (uint64_t)((a * L::XA_BYTES + 32 * kk) >> 4), idesc,
                          (i | a | kk) != 0 ? 1u : 0u);
          ptx::mma_commit(bar_empty + 8 * s);
        }
        if (!ok) break;
        if (!(args.debug_flags & 1)) ptx::mma_commit(bar_accfull + 8 * b);
      }
      trace_stamp(tr, 4);
      ptx::mma_commit(bar_drain);
      dc_wait_drain(bar_drain, 0, tmo);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // Two groups of four warps (two warps per SM sub-partition, so one
    // group's TMEM loads and stores overlap the other's arithmetic); group g
    // takes the CH-token chunks ci with ci % 2 == g.  Warp w reads TMEM lanes
    // 32 (w % 4) .. 32 (w % 4) + 31, so both groups cover all 128 rows.
    const int e = threadIdx.x - 128;
    const int q = warp & 3;
    const int grp = (warp - 4) >> 2;
    const int row = q * 32 + lane;
    ptx::pdl_wait();
    // token scales once into shared memory (written by the split pre-pass)
    float* xs_s = reinterpret_cast<float*>(smem + L::OFF_XS);
    if (e < BT) xs_s[e] = e < args.M ? __ldg(args.xscale + e) : 0.f;
    dc_epi_bar();
    // split-K: the other ranks' receive barriers are ready (arrived at set-up)
    const uint32_t rank = nsplit > 1 ? ptx::cluster_ctarank() : 0u;
    if (PUSH && nsplit > 1) ptx::cluster_wait();
    constexpr int NCH = BT / CH;                // chunks per tile
    constexpr int NCG = (NCH + 1) / 2;          // chunks per group (at most)
    constexpr int NB = ARGMAX ? NCG * CH : 1;   // running best per owned token
    uint32_t best[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) best[j] = 0u;
    int it = 0, ostage = 0;
    for (int u = unit0; u < units; u += ustride, ++it) {
      int kb, nk;
      unit_k(kb, nk);
      const int n0 = u * DC_BN;
      const int b = it & 1;
      // per-row weight scale and bias do not depend on the accumulator: load first
      const int n = n0 + row;
      const bool nok = n < args.N;
      const float sc = nok ? args.scales[n] : 0.f;
      const float bb = nok ? dc_load_bias(args.bias, args.bias_dtype, n) : 0.f;
      const bool got = nk > 0 && ptx::mbar_wait(bar_accfull + 8 * b, (uint32_t)(it >> 1) & 1u, tmo,
                                                abort_flag);
      if (e == 0 && it == 0) trace_stamp(tr, 5);
      if (!got) break;
      ptx::tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t)(b * ACC_COLS) + ((uint32_t)(q * 32) << 16);
      const int nch = (mvalid + CH - 1) / CH;
#pragma unroll
      for (int cl = 0; cl < NCG; ++cl) {
        const int ci = 2 * cl + grp;
        if (ci < nch) {
          const int c0 = ci * CH;
          // token scales 2^-e of these columns, into registers before the
          // stores (read between them they would be ordered behind each one)
          float xsr[CH];
#pragma unroll
          for (int j4 = 0; j4 < CH / 4; ++j4) {
            const float4 v = reinterpret_cast<const float4*>(xs_s + c0)[j4];
            xsr[4 * j4] = v.x;
            xsr[4 * j4 + 1] = v.y;
            xsr[4 * j4 + 2] = v.z;
            xsr[4 * j4 + 3] = v.w;
          }
          uint32_t rr[3][16];
          dc_ld_chunk(taddr, c0, rr);
          ptx::tmem_ld_wait();
          dc_reg_fence(rr);
          // the three plane blocks summed in plane order
          float acc[CH];
#pragma unroll
          for (int jj = 0; jj < CH; ++jj)
            acc[jj] = (__uint_as_float(rr[0][jj]) + __uint_as_float(rr[1][jj])) +
                      __uint_as_float(rr[2][jj]);
          if (nsplit > 1 && !PUSH) {
            // 64-token split-K: park the partial [token][row] in the ring
            float* part = reinterpret_cast<float*>(smem);
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) part[(c0 + jj) * DC_BN + row] = acc[jj];
          } else if (nsplit > 1) {
            // split-K: each 4-token group of this row goes to the rank that
            // owns it (16 bytes straight from registers into its shared
            // memory, counted on its receive barrier); this rank's own
            // groups stay in the start of its ring
#pragma unroll
            for (int gq = 0; gq < CH / 4; ++gq) {
              const int t0 = c0 + 4 * gq;
              if (t0 < m4) {
                const int o = t0 / tpo;
                const int gl = (t0 - o * tpo) >> 2;
                const float4 v = make_float4(acc[4 * gq], acc[4 * gq + 1], acc[4 * gq + 2],
                                             acc[4 * gq + 3]);
                if (o == (int)rank) {
                  *reinterpret_cast<float4*>(smem + L::OFF_OWN + (gl * DC_BN + row) * 16) = v;
                } else {
                  const int slot = (int)rank < o ? (int)rank : (int)rank - 1;
                  const uint32_t off =
                      sbase + (uint32_t)(L::OFF_RECV + ((slot * (tpo >> 2) + gl) * DC_BN + row) * 16);
                  ptx::st_async_v4(ptx::mapa_shared(off, (uint32_t)o), v,
                                   ptx::mapa_shared(bar_recv, (uint32_t)o));
                }
              }
            }
          } else if constexpr (ARGMAX) {
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) {
              const __half v = __float2half_rn(acc[jj] * sc * xsr[jj]);
              const uint32_t cand = (nok && c0 + jj < mvalid && __half2float(v) > -FLT_MAX)
                                        ? ((f16_order_key(v) << 16) | (0xFFFFu - (uint32_t)it))
                                        : 0u;
              uint32_t& bj = best[cl * CH + jj];
              bj = cand > bj ? cand : bj;
            }
          } else if constexpr (SWIGLU) {
            // rows 32 b + i (i < 16) hold gate row 16 b + i and rows 32 b + 16 + i
            // the matching up row, so lane L < 16 takes its up value from lane
            // L + 16.  gate and up are rounded to fp16 as the two-GEMM path
            // rounds them, then silu(g) * u in fp32 (SwiGLU_d.cu:22-24).
            float o[CH];
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) {
              const float v = __half2float(__float2half_rn(fmaf(acc[jj] * sc, xsr[jj], bb)));
              const float u = __shfl_down_sync(0xffffffffu, v, 16);
              o[jj] = __fdividef(v, 1.0f + __expf(-v)) * u;
            }
            const int oc0 = (n0 >> 1) + q * 16;  // this warp's 16 output columns
            if (args.y_tma) {
              __half* stg = reinterpret_cast<__half*>(smem + L::OFF_O +
                                                      (2 * (warp - 4) + ostage) * L::OW_BYTES);
              if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
              __syncwarp();
              if (lane < 16) {
#pragma unroll
                for (int jj = 0; jj < CH; ++jj) stg[jj * 16 + lane] = __float2half_rn(o[jj]);
              }
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0 && oc0 < args.out_n) {
                ptx::tma_store_2d(&tm_y, ptx::smem_u32(stg), oc0, c0);
                ptx::bulk_commit_group();
              }
              ostage ^= 1;
            } else if (lane < 16 && oc0 + lane < args.out_n) {
#pragma unroll
              for (int jj = 0; jj < CH; ++jj)
                if (c0 + jj < mvalid)
                  args.y[(size_t)(c0 + jj) * args.out_n + oc0 + lane] = __float2half_rn(o[jj]);
            }
          } else if (args.y_tma) {
            // each warp stages its 32 rows x CH tokens and stores them with its
            // own TMA store: no barrier across the epilogue warps
            __half* stg = reinterpret_cast<__half*>(smem + L::OFF_O +
                                                    (2 * (warp - 4) + ostage) * L::OW_BYTES);
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            __syncwarp();
#pragma unroll
            for (int jj = 0; jj < CH; ++jj)
              stg[jj * 32 + lane] = __float2half_rn(fmaf(acc[jj] * sc, xsr[jj], bb));
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && n0 + q * 32 < args.N) {
              ptx::tma_store_2d(&tm_y, ptx::smem_u32(stg), n0 + q * 32, c0);
              ptx::bulk_commit_group();
            }
            ostage ^= 1;
          } else {
            __half* yp = args.y + (size_t)c0 * args.N + n;
#pragma unroll
            for (int jj = 0; jj < CH; ++jj)
              if (nok && c0 + jj < mvalid)
                yp[(size_t)jj * args.N] = __float2half_rn(fmaf(acc[jj] * sc, xsr[jj], bb));
          }
        }
      }
      if (nsplit > 1) {
        have_acc = true;
        break;  // one unit per CTA in split mode
      }
      // every epilogue warp releases the accumulator once its TMEM loads are done
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_accempty + 8 * b);
    }
    if (PUSH && nsplit > 1) {
      // ---------------------------------------------------------- split-K owner
      // sum the partials of this rank's groups in rank (= K) order, then the
      // same scale / bias / fp16 (or greedy key) as the unsplit epilogue.
      // The receive wait is never skipped: no CTA may leave while another
      // rank can still store into its shared memory (after an abort it is a
      // bounded drain).
      if (e == 0) trace_stamp(tr, 8);
      // per-row weight scale and bias: read while the partials arrive
      const int n = unit0 * DC_BN + row;
      const bool nok = n < args.N;
      const float sc = nok ? args.scales[n] : 0.f;
      const float bb = nok ? dc_load_bias(args.bias, args.bias_dtype, n) : 0.f;
      dc_epi_bar();  // own groups written by both thread groups
      const int ng = max(0, min(tpo, m4 - (int)rank * tpo)) >> 2;
      bool got = ng == 0 || ptx::mbar_wait_cluster(bar_recv, 0u, tmo, abort_flag);
      if (!got) {
        const long long t0 = clock64();
        while (!ptx::mbar_try_wait_cluster(bar_recv, 0u)) {
          if (clock64() - t0 > (long long)(tmo * 2ull)) break;
        }
      }
      if (e == 0) trace_stamp(tr, 9);
      if (got && have_acc) {
        for (int gl = grp; gl < ng; gl += 2) {
          float4 pv[kMaxSplits];
#pragma unroll
          for (int sp = 0; sp < kMaxSplits; ++sp) {
            if (sp < nsplit) {
              const int off = sp == (int)rank
                                  ? L::OFF_OWN + (gl * DC_BN + row) * 16
                                  : L::OFF_RECV +
                                        (((sp < (int)rank ? sp : sp - 1) * (tpo >> 2) + gl) *
                                             DC_BN + row) * 16;
              pv[sp] = *reinterpret_cast<const float4*>(smem + off);
            }
          }
          float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int sp = 0; sp < kMaxSplits; ++sp) {  // rank order
            if (sp < nsplit) {
              a4.x += pv[sp].x;
              a4.y += pv[sp].y;
              a4.z += pv[sp].z;
              a4.w += pv[sp].w;
            }
          }
          const int t0 = (int)rank * tpo + 4 * gl;
          const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int t = t0 + q4;
            if (ARGMAX) {
              unsigned long long k = 0ull;
              if (t < mvalid) {
                const __half v = __float2half_rn(av[q4] * sc * xs_s[t]);
                if (nok && __half2float(v) > -FLT_MAX)
                  k = ((unsigned long long)f16_order_key(v) << 32) |
                      (unsigned long long)(0xFFFFFFFFu - (uint32_t)((int64_t)n + args.vocab_offset));
              }
              k = dc_warp_max_u64(k);
              if (lane == 0 && k) atomicMax(args.packed + t, k);
            } else if (nok && t < mvalid) {
              args.y[(size_t)t * args.N + n] = __float2half_rn(fmaf(av[q4] * sc, xs_s[t], bb));
            }
          }
        }
      }
      if (e == 0) trace_stamp(tr, 10);
    }
    if (args.y_tma && lane == 0) ptx::bulk_wait_group_read0();
    if constexpr (ARGMAX) {
      if (nsplit == 1) {
        unsigned long long* red = reinterpret_cast<unsigned long long*>(smem + L::OFF_RED);
#pragma unroll
        for (int cl = 0; cl < NCG; ++cl) {
#pragma unroll
          for (int jj = 0; jj < CH; ++jj) {
            const int j = (2 * cl + grp) * CH + jj;
            if (j < mvalid) {
              const uint32_t bj = best[cl * CH + jj];
              unsigned long long k = 0ull;
              if (bj) {
                const int itb = 0xFFFF - (int)(bj & 0xFFFFu);
                const int nb = (unit0 + itb * ustride) * DC_BN + row;
                k = ((unsigned long long)(bj >> 16) << 32) |
                    (unsigned long long)(0xFFFFFFFFu - (uint32_t)((int64_t)nb + args.vocab_offset));
              }
              k = dc_warp_max_u64(k);
              if (lane == 0) red[q * BT + j] = k;
            }
          }
        }
        dc_epi_bar();
        for (int j = e; j < mvalid; j += 256) {
          unsigned long long v = red[j];
          for (int w = 1; w < 4; ++w) v = red[w * BT + j] > v ? red[w * BT + j] : v;
          if (v) atomicMax(args.packed + j, v);
        }
      }
    }
    __syncwarp();
  }

  // split-K: the other warps pass the cluster barrier they arrived at during set-up
  if (PUSH && nsplit > 1 && warp < 4) ptx::cluster_wait();

  if (!PUSH && nsplit > 1) {
    // ------------------------------------------------------------ 64-token split-K
    // after a cluster barrier the owner of token jb (rank jb mod n, one warp
    // per token) reads that token's 128-row partial from every rank - all
    // the remote loads in flight together - and sums them in rank (= K)
    // order; a second barrier keeps every CTA alive while others read it
    const int n0 = unit0 * DC_BN;
    const int r0 = 4 * lane;
    float sc4[4] = {0.f, 0.f, 0.f, 0.f}, bb4[4] = {0.f, 0.f, 0.f, 0.f};
    if (warp >= 4) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int ne = n0 + r0 + q;
        sc4[q] = ne < args.N ? args.scales[ne] : 0.f;
        bb4[q] = ne < args.N ? dc_load_bias(args.bias, args.bias_dtype, ne) : 0.f;
      }
    }
    __syncwarp();
    if (threadIdx.x == 128) trace_stamp(tr, 8);
    ptx::cluster_sync();
    if (threadIdx.x == 128) trace_stamp(tr, 9);
    if (warp >= 4 && have_acc) {
      const uint32_t rank = ptx::cluster_ctarank();
      const int w8 = warp - 4;
      for (int jb = (int)rank + w8 * nsplit; jb < mvalid; jb += 8 * nsplit) {
        const uint32_t loc = sbase + (uint32_t)((jb * DC_BN + r0) * 4);
        float4 pv[kMaxSplits];
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp)
          if (sp < nsplit) pv[sp] = ptx::ld_dsmem_f4(ptx::mapa_shared(loc, (uint32_t)sp));
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp) {  // rank order: deterministic
          if (sp < nsplit) {
            acc.x += pv[sp].x;
            acc.y += pv[sp].y;
            acc.z += pv[sp].z;
            acc.w += pv[sp].w;
          }
        }
        const float xs = reinterpret_cast<const float*>(smem + L::OFF_XS)[jb];
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
        if (ARGMAX) {
          unsigned long long k = 0ull;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int nq = n0 + r0 + q;
            const __half v = __float2half_rn(a4[q] * sc4[q] * xs);
            if (nq < args.N && __half2float(v) > -FLT_MAX) {
              const unsigned long long kq =
                  ((unsigned long long)f16_order_key(v) << 32) |
                  (unsigned long long)(0xFFFFFFFFu - (uint32_t)((int64_t)nq + args.vocab_offset));
              k = kq > k ? kq : k;
            }
          }
          k = dc_warp_max_u64(k);
          if (lane == 0 && k) atomicMax(args.packed + jb, k);
        } else {
          __half* yrow = args.y + (size_t)jb * args.N;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + r0 + q < args.N)
              yrow[n0 + r0 + q] = __float2half_rn(fmaf(a4[q] * sc4[q], xs, bb4[q]));
        }
      }
    }
    __syncwarp();
    if (threadIdx.x == 128) trace_stamp(tr, 10);
    ptx::cluster_sync();
  }

  // greedy epilogue with ids: this thread's atomicMax words are visible
  // device-wide before the CTA's arrival below
  if (ARGMAX && args.counter != nullptr) __threadfence();
  if (threadIdx.x == 128) trace_stamp(tr, 6);
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (ARGMAX) {
    if (args.counter != nullptr) {
      // the last CTA to arrive (timed-out CTAs arrive too) turns every
      // token's packed word into its id - the unpack kernel's work - and
      // clears the counter for the next call
      volatile int* last = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 8);
      if (threadIdx.x == 0) {
        const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
        *last = atomicAdd(args.counter, 1u) == total - 1u ? 1 : 0;
      }
      __syncthreads();
      if (*last) {
        __threadfence();
        for (int m = threadIdx.x; m < args.M; m += blockDim.x) {
          const unsigned long long v = __ldcg(args.packed + m);
          args.ids[m] = v ? (long long)(0xFFFFFFFFull - (v & 0xFFFFFFFFull)) : 0ll;
        }
        if (threadIdx.x == 0) *args.counter = 0u;
      }
    }
  }
  if (threadIdx.x == 0 && *abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
  if (threadIdx.x == 0) trace_stamp(tr, 7);
}

// ============================================================================
// Host side
// ============================================================================
namespace {

PFN_cuTensorMapEncodeTiled_v12000 dc_encoder() {
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

int dc_tmap(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
            uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
            CUtensorMapSwizzle sw) {
  auto enc = dc_encoder();
  if (!enc) return DDQ_ERR_DEVICE;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDQ_OK : DDQ_ERR_ALIGNMENT;
}

// The activation planes [3][M][K] e4m3 as a 3-D tensor {K, M, 3}; a box
// {128, BT, 3} lands as the B operand rows p BT + m, tokens m >= M zero.
int dc_tmap_planes(CUtensorMap* m, const void* base, uint64_t K, uint64_t M, uint32_t bt) {
  auto enc = dc_encoder();
  if (!enc) return DDQ_ERR_DEVICE;
  cuuint64_t dims[3] = {K, M, 3};
  cuuint64_t strides[2] = {K, K * M};
  cuuint32_t box[3] = {(cuuint32_t)DC_AK, bt, 3};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDQ_OK : DDQ_ERR_ALIGNMENT;
}

template <int BT, int ST, int KB, int EPI>
int launch_dec_t(const DecPlan& p, const uint8_t* wq, const uint8_t* planes, DcArgs a,
                 cudaStream_t s) {
  using Lay = DcLayout<BT, ST, KB>;
  auto kern = w8a16_dec_kernel<BT, ST, KB, EPI>;
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), kern, Lay::ALLOC);
  if (ast) return ast;
  CUtensorMap tm_w, tm_x, tm_y;
  int st = dc_tmap(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)a.K, (uint64_t)a.N,
                   (uint64_t)a.K, DC_AK, DC_BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = dc_tmap_planes(&tm_x, planes, (uint64_t)a.K, (uint64_t)a.M, (uint32_t)BT);
  if (st) return st;
  a.y_tma = 0;
  std::memset(&tm_y, 0, sizeof(tm_y));
  if (EPI != DC_EPI_ARGMAX && p.splits == 1 && a.out_n % 8 == 0 && aligned16(a.y)) {
    st = dc_tmap(&tm_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.y, (uint64_t)a.out_n, (uint64_t)a.M,
                 (uint64_t)a.out_n * 2, EPI == DC_EPI_SWIGLU ? 16 : 32, Lay::CH,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    a.y_tma = 1;
  }
  a.n_tiles = (a.N + DC_BN - 1) / DC_BN;
  cudaLaunchConfig_t cfg = {};
  if (p.splits > 1)
    cfg.gridDim = dim3((unsigned)a.n_tiles, 1, (unsigned)p.splits);
  else
    cfg.gridDim = dim3((unsigned)(a.n_tiles < p.sms ? a.n_tiles : p.sms), 1, 1);
  cfg.blockDim = dim3(DC_THREADS);
  cfg.dynamicSmemBytes = Lay::ALLOC;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[na].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++na;
  if (p.splits > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = (unsigned)p.splits;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, kern, tm_w, tm_x, tm_y, a) != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace

DecPlan dec_plan(int64_t M, int64_t N, int64_t K, int sms, bool no_split) {
  DecPlan p{};
  p.sms = sms;
  p.bt = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  const int64_t KS = (K + dc_stage_k(p.bt) - 1) / dc_stage_k(p.bt);
  const int64_t tiles = (N + DC_BN - 1) / DC_BN;
  int64_t splits = 1, kps = KS;
  if (sms > 0 && tiles * 2 <= sms && !no_split) {
    splits = sms / tiles;
    if (splits > kMaxSplits) splits = kMaxSplits;
    if (splits > KS) splits = KS;
    if (splits < 1) splits = 1;
    kps = (KS + splits - 1) / splits;
    splits = (KS + kps - 1) / kps;
  }
  p.splits = (int)splits;
  p.kps = (int)kps;
  p.plane_bytes = (size_t)3 * M * K;
  p.ws_bytes = ((p.plane_bytes + 255) & ~(size_t)255) + (size_t)M * sizeof(float);
  return p;
}

int launch_dec(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
               int bias_dtype, __half* y, unsigned long long* packed, int64_t vocab_offset, int M,
               int N, int K, void* ws, size_t ws_bytes, unsigned long long timeout_ns,
               int debug_flags, cudaStream_t s, bool swiglu, const uint8_t* ext_planes,
               const float* ext_xscale, int64_t* ids, unsigned int* counter) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  if (M < 1 || M > 64) return DDQ_ERR_SHAPE;
  if (swiglu && (packed || N % 32 != 0)) return DDQ_ERR_SHAPE;
  const DecPlan p = dec_plan(M, N, K, sms, swiglu);
  if (!ext_planes) ws_note_other_use(ws, s);
  uint8_t* planes;
  float* xscale;
  if (ext_planes) {  // the caller split the activations already
    if (!ext_xscale) return DDQ_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(ext_planes) & 15u) return DDQ_ERR_ALIGNMENT;
    planes = const_cast<uint8_t*>(ext_planes);
    xscale = const_cast<float*>(ext_xscale);
  } else {
    if (!ws || ws_bytes < p.ws_bytes) return DDQ_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(ws) & 255u) return DDQ_ERR_ALIGNMENT;
    planes = reinterpret_cast<uint8_t*>(ws);
    xscale = reinterpret_cast<float*>(planes + ((p.plane_bytes + 255) & ~(size_t)255));
  }
  // 1) split the activations into three e4m3 planes (PDL: waits for the
  //    producer of x, lets the GEMM launch early)
  if (!ext_planes) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)M);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    const int nch = K / 8;
    cudaError_t le;
    if (nch <= 256) le = cudaLaunchKernelEx(&cfg, xsplit_kernel<1>, x, planes, xscale, M, K, packed);
    else if (nch <= 512) le = cudaLaunchKernelEx(&cfg, xsplit_kernel<2>, x, planes, xscale, M, K, packed);
    else if (nch <= 768) le = cudaLaunchKernelEx(&cfg, xsplit_kernel<3>, x, planes, xscale, M, K, packed);
    else if (nch <= 1024) le = cudaLaunchKernelEx(&cfg, xsplit_kernel<4>, x, planes, xscale, M, K, packed);
    else le = cudaLaunchKernelEx(&cfg, xsplit_kernel<0>, x, planes, xscale, M, K, packed);
    if (le != cudaSuccess) {
      cudaGetLastError();
      return DDQ_ERR_LAUNCH;
    }
  }
  // 2) the GEMM on the e4m3 tensor cores
  DcArgs a{};
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.packed = packed;
  a.vocab_offset = vocab_offset;
  a.xscale = xscale;
  a.M = M;
  a.N = N;
  a.K = K;
  a.kps = p.kps;
  a.timeout_ns = timeout_ns;
  a.debug_flags = debug_flags;
  a.out_n = swiglu ? N / 2 : N;
  a.ids = packed && ids && counter ? reinterpret_cast<long long*>(ids) : nullptr;
  a.counter = a.ids ? counter : nullptr;
  const int epi = packed ? DC_EPI_ARGMAX : swiglu ? DC_EPI_SWIGLU : DC_EPI_STORE;
#define DDQ_DC_CASE(BT_, ST_)                                                                  \
  case BT_:                                                                                    \
    return epi == DC_EPI_ARGMAX                                                                \
               ? launch_dec_t<BT_, ST_, dc_stage_k(BT_), DC_EPI_ARGMAX>(p, wq, planes, a, s)   \
           : epi == DC_EPI_SWIGLU                                                              \
               ? launch_dec_t<BT_, ST_, dc_stage_k(BT_), DC_EPI_SWIGLU>(p, wq, planes, a, s)   \
               : launch_dec_t<BT_, ST_, dc_stage_k(BT_), DC_EPI_STORE>(p, wq, planes, a, s);
  switch (p.bt) {
    DDQ_DC_CASE(16, 4)
    DDQ_DC_CASE(32, 3)
    DDQ_DC_CASE(64, 5)
    default:
      return DDQ_ERR_SHAPE;
  }
#undef DDQ_DC_CASE
}

// ============================================================================
// Allocation-free entry point
// ============================================================================
// Some callers cannot allocate device memory at the point where they call a
// projection: a host that hands the library a fixed, pre-planned memory
// budget and owns every allocation itself, a serving runtime that forbids
// cudaMalloc on its request path (it synchronises the device and can fail
// under fragmentation), or code that records its launches into a CUDA graph
// and may not allocate while recording.  For them the decode-shape GEMM has a
// variant whose scratch - the three activation planes and the token scales -
// lives in this file-scope device array instead of a caller workspace.  Every
// GPU that loads the library holds these 1 MiB until the process exits.
constexpr size_t kNoAllocScratchBytes = (size_t)1 << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
// Device address of g_noalloc_scratch per device, with the context it was
// looked up in: after cudaDeviceReset (or a released and re-created primary
// context) the module is loaded again, possibly at another address, so a
// change of context triggers a new lookup.
struct NoallocAddr {
  void* ctx;
  void* addr;
};
NoallocAddr g_noalloc_addr[64];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// The array's name in host code is only a host-side stand-in; the device
// address comes from cudaGetSymbolAddress, asked once per device (and again
// after its context changed) with that device current.
int noalloc_scratch(int dev, void** out) {
  if (dev < 0 || dev >= 64) return DDQ_ERR_DEVICE;
  CtxGetCurrentFn get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (!get || get(&ctx) != CUDA_SUCCESS) return DDQ_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocAddr& e = g_noalloc_addr[dev];
  if (!e.addr || e.ctx != (void*)ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return DDQ_ERR_DEVICE;
    }
    e.addr = p;
    e.ctx = (void*)ctx;
  }
  *out = e.addr;
  return DDQ_OK;
}
}  // namespace

size_t noalloc_scratch_bytes() { return kNoAllocScratchBytes; }

}  // namespace ddq

using namespace ddq;

extern "C" int ddq_w8a16_gemm_noalloc(const void* x, const uint8_t* wq, const float* scales,
                                      const void* bias, int bias_dtype, void* y, int64_t M,
                                      int64_t N, int64_t K, void* stream) {
  if (M < 0 || N < 0 || K < 0) return DDQ_ERR_SHAPE;
  if (bias_dtype != DDQ_DTYPE_NONE && bias_dtype != DDQ_DTYPE_F16 && bias_dtype != DDQ_DTYPE_F32)
    return DDQ_ERR_INVALID_ARGUMENT;
  if (bias_dtype != DDQ_DTYPE_NONE && !bias) return DDQ_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return DDQ_OK;
  if (!x || !wq || !scales || !y) return DDQ_ERR_INVALID_ARGUMENT;
  // decode shapes only: 1 <= M <= 64 tokens, K a multiple of 16
  if (M > 64 || K == 0 || K % 16 != 0 || N > 0x7fffffff || K > 0x7fffffff) return DDQ_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(wq)) return DDQ_ERR_ALIGNMENT;
  const int dev = current_device();
  const int sms = device_sm_count(dev);
  if (sms <= 0) return DDQ_ERR_DEVICE;
  // 3*M*K plane bytes (rounded up to 256) + 4*M scale bytes must fit the array
  if (dec_plan(M, N, K, sms).ws_bytes > kNoAllocScratchBytes) return DDQ_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = noalloc_scratch(dev, &scratch);
  if (st != DDQ_OK) return st;
  return launch_dec(reinterpret_cast<const __half*>(x), wq, scales, bias, bias_dtype,
                    reinterpret_cast<__half*>(y), nullptr, 0, (int)M, (int)N, (int)K, scratch,
                    kNoAllocScratchBytes, wait_timeout_ns(), debug_flags(),
                    reinterpret_cast<cudaStream_t>(stream));
}
