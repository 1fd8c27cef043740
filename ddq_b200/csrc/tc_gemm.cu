// tc_gemm.cu - the sm_100a tensor-core W8A16 GEMM (tcgen05 + TMA + TMEM).
//
// Formulation ("swap AB"): the weight is the 128-row A operand, the
// activations the B operand, so the MMA N dimension is the token tile BT
// (16..256) and decode shapes (M <= 64) waste no tensor-core rows:
//     D[n, m] = sum_k  fp16(e4m3(Wq[n, k])) * x[m, k]        (fp32 in TMEM)
//     y[m, n] = fp16( D[n, m] * scale[n] + bias[n] )
// Every e4m3 value is exact in fp16, so converting the weight tile loses
// nothing before the fp32 accumulation.
//
// Work unit = one 128 x BT output tile over one K range.  A persistent CTA
// (at most one per SM) walks its units in a continuous pipeline, 384 threads:
//   warp 0      TMA producer of the e4m3 weight ring (WS stages of 128 rows x
//               256 B, i.e. four K steps).  Before the grid dependency on the previous
//               kernel resolves (programmatic dependent launch) it already
//               fills the ring and warms L2 with the rest of its first unit:
//               weights never depend on the previous kernel.
//   warp 1      MMA issuer: 4 x tcgen05.mma kind::f16 (K = 16) per 64-wide K
//               step into one of two TMEM accumulators (double buffered), so
//               the next tile's MMAs overlap this tile's epilogue.
//   warp 2      TMA producer of the activation ring (XS stages, its own depth).
//   warps 4-7   converters: e4m3 -> fp16 into the canonical 128-byte-swizzled
//               K-major A layout, two K steps at a time; the e4m3 stage is
//               released as soon as it is in registers.
//   warps 8-11  epilogue: tcgen05.ld -> scale, bias, fp16 -> shared memory ->
//               TMA tile stores in 32-token chunks (double-buffered); for the
//               fused lm_head a running per-token best over all of the CTA's
//               tiles, reduced across the CTA once.
// Split-K (few tiles, one unit per CTA): the K splits of a tile form one
// thread-block cluster; each CTA parks its fp32 partial in its own shared
// memory and, after a cluster barrier, every CTA sums a share of the tile's
// columns over all splits in split order through distributed shared memory -
// deterministic, no workspace, no atomics.
// Every mbarrier wait is bounded and starts after the grid dependency has
// resolved; on timeout the CTA records DDQ_ERR_TIMEOUT in the device error
// word, drains its own TMA copies and MMAs, still takes part in the cluster
// barriers, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cfloat>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int TC_BN = 128;       // weight rows per tile (MMA M)
constexpr int TC_BK = 64;        // K elements per MMA step (one fp16 A / activation slot)
constexpr int TC_WK = 256;       // K bytes per e4m3 weight stage (TMA box 256 B x 128 rows)
constexpr int TC_THREADS = 384;  // 12 warps

template <int BT, int WS, int AS, int XS>
struct TcLayout {
  static constexpr int CH = BT < 32 ? BT : 32;        // epilogue token chunk
  static constexpr int A_BYTES = TC_BN * TC_BK * 2;  // fp16 weight tile (one 64-wide K step)
  static constexpr int X_BYTES = BT * TC_BK * 2;     // activation tile
  static constexpr int W_BYTES = TC_BN * TC_WK;      // e4m3 weight stage (4 K steps)
  static constexpr int O_BYTES = CH * TC_BN * 2;     // output staging chunk [CH][128] fp16
  static constexpr int OFF_A = 0;
  static constexpr int OFF_X = OFF_A + AS * A_BYTES;
  static constexpr int OFF_W = OFF_X + XS * X_BYTES;
  static constexpr int OFF_O = OFF_W + WS * W_BYTES;
  static constexpr int RING_END = OFF_O;
  // split-K only (one unit per CTA): the ring area is reused for the fp32
  // partial [BT][128] once the unit's MMAs have completed
  static constexpr int P_BYTES = TC_BN * BT * 4;
  static constexpr int OFF_BAR = OFF_O + 2 * O_BYTES;
  static constexpr int NBAR = 2 * WS + 2 * AS + 2 * XS + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_RED = OFF_MISC + 16;  // lm_head: [4 warps][BT] packed keys
  static constexpr int RED_BYTES = BT <= 64 ? 4 * BT * 8 : 0;
  static constexpr int BYTES = OFF_RED + RED_BYTES;
  static constexpr int ALLOC = BYTES + 1024;     // slack to align the base to 1024 B
  static_assert(AS % 2 == 0, "converters fill fp16 weight slots in pairs");
  static_assert(X_BYTES % 1024 == 0, "activation slots must keep 1024-B alignment");
  static_assert(P_BYTES <= RING_END, "split-K partial must fit in the ring area");
  static_assert(ALLOC <= 232448, "shared memory budget");
};

__device__ __forceinline__ float tc_load_bias(const void* bias, int bias_dtype, int n) {
  if (bias_dtype == DDQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (bias_dtype == DDQ_DTYPE_F32) return reinterpret_cast<const float*>(bias)[n];
  return 0.f;
}

__device__ __forceinline__ unsigned long long tc_pack_key(float acc, float sc, int n, int N,
                                                          int64_t offset) {
  const __half v = __float2half_rn(acc * sc);
  if (n >= N || !(__half2float(v) > -FLT_MAX)) return 0ull;  // NaN / -inf never win
  return ((unsigned long long)f16_order_key(v) << 32) |
         (unsigned long long)(0xFFFFFFFFu - (uint32_t)((int64_t)n + offset));
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}

// named barrier among the 4 epilogue warps
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Wait ignoring the abort flag (used only while winding down); the same
// cycle-count limit as ptx::mbar_wait.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  const long long t0 = clock64();
  const long long limit = (long long)(timeout_ns * 2ull);
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

struct TcArgs {
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  unsigned long long* packed;  // lm_head: per-token packed greedy key (ARGMAX)
  int64_t vocab_offset;
  int M, N, K, kps;
  int n_tiles, units;          // output tiles (= work units without split-K)
  int y_tma;                   // 1: store the output tile with TMA
  unsigned long long timeout_ns;
  int debug_flags;             // bit 0: never signal the accumulator (timeout test); bit 1: trace
};

template <int BT, int WS, int AS, int XS, bool ARGMAX>
__global__ void __launch_bounds__(TC_THREADS, 1)
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_y, const TcArgs args) {
  using L = TcLayout<BT, WS, AS, XS>;
  constexpr int CH = L::CH;
  constexpr uint32_t ACC_COLS = BT < 32 ? 32 : BT;  // one accumulator
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;       // double buffered
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsplit = gridDim.z;  // > 1: one unit per CTA, the splits of a tile = one cluster
  const int KT = (args.K + TC_BK - 1) / TC_BK;
  const uint64_t tmo = args.timeout_ns;
  const bool tr = (args.debug_flags & 2) != 0;

  // Units are output tiles; a persistent CTA takes tiles blockIdx.x, +gridDim.x, ...
  // In split-K mode the grid is (tiles, 1, splits) and each CTA owns one
  // (tile, split) unit.
  const int unit0 = (int)blockIdx.x;
  const int ustride = (nsplit > 1) ? args.units : (int)gridDim.x;
  auto unit_coords = [&](int u, int& n0, int& m0, int& kb, int& nk) {
    n0 = (u % args.n_tiles) * TC_BN;
    m0 = (u / args.n_tiles) * BT;
    kb = (nsplit > 1 ? (int)blockIdx.z : 0) * args.kps;
    nk = max(0, min(args.kps, KT - kb));
  };

  const uint32_t bar_wfull = sbase + L::OFF_BAR;
  const uint32_t bar_wempty = bar_wfull + 8 * WS;
  const uint32_t bar_afull = bar_wempty + 8 * WS;
  const uint32_t bar_aempty = bar_afull + 8 * AS;
  const uint32_t bar_xfull = bar_aempty + 8 * AS;
  const uint32_t bar_xempty = bar_xfull + 8 * XS;
  const uint32_t bar_accfull = bar_xempty + 8 * XS;  // [2]
  const uint32_t bar_accempty = bar_accfull + 16;     // [2]
  const uint32_t bar_drain = bar_accempty + 16;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) trace_stamp(tr, 0);  // entry
  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      ptx::mbar_init(bar_wfull + 8 * s, 1);
      ptx::mbar_init(bar_wempty + 8 * s, 4);
    }
    for (int j = 0; j < AS; ++j) {
      ptx::mbar_init(bar_afull + 8 * j, 4);
      ptx::mbar_init(bar_aempty + 8 * j, 1);
    }
    for (int j = 0; j < XS; ++j) {
      ptx::mbar_init(bar_xfull + 8 * j, 1);
      ptx::mbar_init(bar_xempty + 8 * j, 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar_accfull + 8 * b, 1);
      ptx::mbar_init(bar_accempty + 8 * b, 4);
    }
    ptx::mbar_init(bar_drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
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
  if (threadIdx.x == 0) trace_stamp(tr, 1);  // set-up done
  // Let the next kernel on the stream start its own weight prefetch now.
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  bool have_acc = false;  // epilogue warps, split-K mode: this CTA's partial is valid
  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    // One stage = TMA box of 256 B (four 64-wide K steps) x 128 rows: 256-byte
    // row segments keep the TMA engine at full rate even when only a part of
    // the SMs stream (half the SMs at 64-byte rows reach ~40% of it).
    if (lane == 0) {
      int g = 0;  // stage counter over all (unit, stage) of this CTA
      bool ok = true;
      bool waited = false;
      for (int u = unit0; u < args.units && ok; u += ustride) {
        int n0, m0, kb, nk;
        unit_coords(u, n0, m0, kb, nk);
        const int nst = (nk + 3) / 4;  // weight stages of this unit
        int i = 0;
        if (!waited) {
          // Before the grid dependency resolves: fill the (fresh) ring and warm
          // L2 with the rest of the first unit's slice.
          const int pre = nst < WS ? nst : WS;
          for (; i < pre; ++i, ++g) {
            ptx::mbar_arrive_expect_tx(bar_wfull + 8 * g, L::W_BYTES);
            ptx::tma_load_2d(sbase + L::OFF_W + g * L::W_BYTES, &tm_w, (kb + 4 * i) * TC_BK, n0,
                             bar_wfull + 8 * g);
          }
          for (int i2 = WS; i2 < nst; ++i2)
            ptx::tma_prefetch_l2_2d(&tm_w, (kb + 4 * i2) * TC_BK, n0);
          trace_stamp(tr, 2);  // first ring of weight loads issued
          ptx::pdl_wait();
          waited = true;
        }
        for (; i < nst; ++i, ++g) {
          const int s = g % WS;
          if (!ptx::mbar_wait(bar_wempty + 8 * s, ((uint32_t)(g / WS) & 1u) ^ 1u, tmo,
                              abort_flag)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(bar_wfull + 8 * s, L::W_BYTES);
          ptx::tma_load_2d(sbase + L::OFF_W + s * L::W_BYTES, &tm_w, (kb + 4 * i) * TC_BK, n0,
                           bar_wfull + 8 * s);
        }
      }
      if (!waited) ptx::pdl_wait();
      if (*abort_flag) {  // let this thread's copies land before the CTA winds down
        for (int i = g > WS ? g - WS : 0; i < g; ++i)
          mbar_wait_drain(bar_wfull + 8 * (i % WS), (uint32_t)(i / WS) & 1u, tmo);
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ activation producer
    if (lane == 0) {
      ptx::pdl_wait();  // x may be the previous kernel's output
      int g = 0;
      bool ok = true;
      for (int u = unit0; u < args.units && ok; u += ustride) {
        int n0, m0, kb, nk;
        unit_coords(u, n0, m0, kb, nk);
        for (int i = 0; i < nk; ++i, ++g) {
          const int j = g % XS;
          if (!ptx::mbar_wait(bar_xempty + 8 * j, ((uint32_t)(g / XS) & 1u) ^ 1u, tmo,
                              abort_flag)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(bar_xfull + 8 * j, L::X_BYTES);
          ptx::tma_load_2d(sbase + L::OFF_X + j * L::X_BYTES, &tm_x, (kb + i) * TC_BK, m0,
                           bar_xfull + 8 * j);
        }
      }
      if (*abort_flag) {
        for (int i = g > XS ? g - XS : 0; i < g; ++i)
          mbar_wait_drain(bar_xfull + 8 * (i % XS), (uint32_t)(i / XS) & 1u, tmo);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_f16_f32(TC_BN, BT);
      ptx::pdl_wait();
      bool ok = true;
      int g = 0, it = 0;
      for (int u = unit0; u < args.units && ok; u += ustride, ++it) {
        int n0, m0, kb, nk;
        unit_coords(u, n0, m0, kb, nk);
        const int b = it & 1;
        const uint32_t tmem_d = tmem_base + (uint32_t)(b * ACC_COLS);
        // the epilogue must have drained this accumulator (two units ago)
        ok = ptx::mbar_wait(bar_accempty + 8 * b, ((uint32_t)(it >> 1) & 1u) ^ 1u, tmo, abort_flag);
        if (!ok) break;
        ptx::tc_fence_after();
        for (int i = 0; i < nk; ++i, ++g) {
          const int ja = g % AS, jx = g % XS;
          ok = ptx::mbar_wait(bar_afull + 8 * ja, (uint32_t)(g / AS) & 1u, tmo, abort_flag) &&
               ptx::mbar_wait(bar_xfull + 8 * jx, (uint32_t)(g / XS) & 1u, tmo, abort_flag);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t a0 = sbase + L::OFF_A + ja * L::A_BYTES;
          const uint32_t b0 = sbase + L::OFF_X + jx * L::X_BYTES;
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk) {
            ptx::mma_f16_ss(tmem_d, ptx::smem_desc_sw128(a0 + 32 * kk),
                            ptx::smem_desc_sw128(b0 + 32 * kk), idesc, (i | kk) != 0 ? 1u : 0u);
          }
          ptx::mma_commit(bar_aempty + 8 * ja);
          ptx::mma_commit(bar_xempty + 8 * jx);
        }
        if (!ok) break;
        if (!(args.debug_flags & 1)) ptx::mma_commit(bar_accfull + 8 * b);
      }
      trace_stamp(tr, 4);  // last MMA issued
      // wind down: wait for this thread's MMAs before TMEM is freed
      ptx::mma_commit(bar_drain);
      mbar_wait_drain(bar_drain, 0, tmo);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ converters
    // Thread t converts weight row t.  Per half stage (128 B = two K steps) it
    // reads the 8 16-byte chunks in a rotated order (chunk (c + t) & 7), so
    // the 8 threads of a shared-memory phase hit 8 different bank groups of
    // the unswizzled 256-byte rows, and writes two fp16 A slots.
    const int t = threadIdx.x - 128;
    const int sw_a = t & 7;  // 128-byte swizzle phase of row t (fp16 tile)
    ptx::pdl_wait();
    int gw = 0, ga = 0;      // weight stages / fp16 slots consumed so far
    bool ok = true;
    for (int u = unit0; u < args.units && ok; u += ustride) {
      int n0, m0, kb, nk;
      unit_coords(u, n0, m0, kb, nk);
      for (int i = 0; i < nk && ok; i += 4, ++gw) {
        const int s = gw % WS;
        if (!ptx::mbar_wait(bar_wfull + 8 * s, (uint32_t)(gw / WS) & 1u, tmo, abort_flag)) {
          ok = false;
          break;
        }
        if (t == 0 && gw == 0) trace_stamp(tr, 3);  // first weight stage landed
        const uint8_t* wrow = smem + L::OFF_W + s * L::W_BYTES + t * TC_WK;
        for (int h = 0; h < 2 && i + 2 * h < nk; ++h) {
          const int nsteps = min(2, nk - (i + 2 * h));  // 64-wide K steps in this half
          uint4 v[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int ch = (c + t) & 7;  // rotated chunk order
            v[c] = *reinterpret_cast<const uint4*>(wrow + h * 128 + ch * 16);
          }
          if (h == 1 || i + 2 >= nk) {
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar_wempty + 8 * s);  // e4m3 stage free again
          }
          // both fp16 slots of this half must be free (their MMAs done)
          bool free_ok = true;
          for (int q2 = 0; q2 < nsteps; ++q2) {
            const int ja = (ga + q2) % AS;
            free_ok = free_ok && ptx::mbar_wait(bar_aempty + 8 * ja,
                                                ((uint32_t)((ga + q2) / AS) & 1u) ^ 1u, tmo,
                                                abort_flag);
          }
          if (!free_ok) {
            ok = false;
            break;
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int ch = (c + t) & 7;      // 16 e4m3 = K [16ch, 16ch+16) of this half
            const int step = ch >> 2;        // which 64-wide K step (slot of the pair)
            if (step >= nsteps) continue;
            uint4 lo, hi;  // fp16 of e4m3 * 2^-8 (the epilogue multiplies by 256)
            lo.x = e4m3x2_to_half2_bits_x2m8(v[c].x, 0x4140u);
            lo.y = e4m3x2_to_half2_bits_x2m8(v[c].x, 0x4342u);
            lo.z = e4m3x2_to_half2_bits_x2m8(v[c].y, 0x4140u);
            lo.w = e4m3x2_to_half2_bits_x2m8(v[c].y, 0x4342u);
            hi.x = e4m3x2_to_half2_bits_x2m8(v[c].z, 0x4140u);
            hi.y = e4m3x2_to_half2_bits_x2m8(v[c].z, 0x4342u);
            hi.z = e4m3x2_to_half2_bits_x2m8(v[c].w, 0x4140u);
            hi.w = e4m3x2_to_half2_bits_x2m8(v[c].w, 0x4342u);
            const int cc = ch & 3;           // 16-element group within the 64-wide step
            uint8_t* arow = smem + L::OFF_A + ((ga + step) % AS) * L::A_BYTES + t * 128;
            *reinterpret_cast<uint4*>(arow + (((2 * cc) ^ sw_a) << 4)) = lo;
            *reinterpret_cast<uint4*>(arow + (((2 * cc + 1) ^ sw_a) << 4)) = hi;
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0)
            for (int q2 = 0; q2 < nsteps; ++q2) ptx::mbar_arrive(bar_afull + 8 * ((ga + q2) % AS));
          ga += nsteps;
        }
      }
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    const int e = threadIdx.x - 256;  // 0..127
    const int q = warp & 3;           // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;    // tile row == TMEM lane
    ptx::pdl_wait();                  // outputs may alias buffers the previous kernel reads
    // lm_head: running best per token column over every tile this thread saw,
    // (ordered fp16 key << 16) | (0xFFFF - unit iteration); reduced across the
    // CTA once at the end.  Equal keys keep the earlier iteration, i.e. the
    // lower vocabulary row (one token tile, so iteration order = row order).
    constexpr int NB = (ARGMAX && BT <= 64) ? BT : 1;
    uint32_t best[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) best[j] = 0u;
    int it = 0;
    int ostage = 0;  // output staging buffer toggle (TMA stores)
    for (int u = unit0; u < args.units; u += ustride, ++it) {
      int n0, m0, kb, nk;
      unit_coords(u, n0, m0, kb, nk);
      const int mvalid = min(BT, args.M - m0);
      const int b = it & 1;
      const bool got = nk > 0 && ptx::mbar_wait(bar_accfull + 8 * b, (uint32_t)(it >> 1) & 1u, tmo,
                                                abort_flag);
      if (e == 0 && it == 0) trace_stamp(tr, 5);  // first accumulator ready
      if (!got) break;
      ptx::tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t)(b * ACC_COLS) + ((uint32_t)(q * 32) << 16);
      const int n = n0 + row;
      const bool nok = n < args.N;
      const float sc = nok ? args.scales[n] * 256.f : 0.f;  // undo the 2^-8 of the A operand
      const float bb = nok ? tc_load_bias(args.bias, args.bias_dtype, n) : 0.f;

      if (nsplit > 1) {
        // park the partial; the cluster reduction below finishes the tile
        float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
        for (int c0 = 0; c0 < mvalid; c0 += CH) {
          uint32_t r[32];
          if (CH == 32) ptx::tmem_ld_32x32b_x32(taddr + c0, r);
          else ptx::tmem_ld_32x32b_x16(taddr + c0, r);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < CH; ++jj) part[(c0 + jj) * TC_BN + row] = __uint_as_float(r[jj]);
        }
        have_acc = true;
        break;  // exactly one unit per CTA in split mode
      }

      if constexpr (ARGMAX) {
        if constexpr (BT <= 64) {
#pragma unroll
          for (int c0 = 0; c0 < BT; c0 += CH) {
            if (c0 < mvalid) {
              uint32_t r[32];
              if (CH == 32) ptx::tmem_ld_32x32b_x32(taddr + c0, r);
              else ptx::tmem_ld_32x32b_x16(taddr + c0, r);
              ptx::tmem_ld_wait();
              if (c0 + CH >= mvalid) {
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(bar_accempty + 8 * b);
              }
#pragma unroll
              for (int jj = 0; jj < CH; ++jj) {
                const __half v = __float2half_rn(__uint_as_float(r[jj]) * sc);
                const uint32_t cand = (nok && __half2float(v) > -FLT_MAX)
                                          ? ((f16_order_key(v) << 16) | (0xFFFFu - (uint32_t)it))
                                          : 0u;
                best[c0 + jj] = cand > best[c0 + jj] ? cand : best[c0 + jj];
              }
            }
          }
        }
        continue;
      }

#pragma unroll 1
      for (int c0 = 0; c0 < mvalid; c0 += CH) {
        uint32_t r[32];
        if (CH == 32) ptx::tmem_ld_32x32b_x32(taddr + c0, r);
        else ptx::tmem_ld_32x32b_x16(taddr + c0, r);
        ptx::tmem_ld_wait();
        if (c0 + CH >= mvalid) {
          // last read of this accumulator: hand it back to the MMA warp
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar_accempty + 8 * b);
        }
        if (args.y_tma) {
          // chunk [CH tokens][128 rows] -> staging buffer -> TMA store
          __half* stg = reinterpret_cast<__half*>(smem + L::OFF_O + ostage * L::O_BYTES);
          if (e == 0) bulk_wait_group_read1();  // the store that used this buffer has read it
          epi_bar();
#pragma unroll
          for (int jj = 0; jj < CH; ++jj)
            stg[jj * TC_BN + row] = __float2half_rn(fmaf(__uint_as_float(r[jj]), sc, bb));
          ptx::fence_proxy_async_smem();
          epi_bar();
          if (e == 0) {
            ptx::tma_store_2d(&tm_y, ptx::smem_u32(stg), n0, m0 + c0);
            ptx::bulk_commit_group();
          }
          ostage ^= 1;
        } else {
#pragma unroll
          for (int jj = 0; jj < CH; ++jj)
            if (nok && c0 + jj < mvalid)
              args.y[(size_t)(m0 + c0 + jj) * args.N + n] =
                  __float2half_rn(fmaf(__uint_as_float(r[jj]), sc, bb));
        }
      }
    }
    if constexpr (ARGMAX && BT <= 64) {
      if (nsplit == 1) {
        // one cross-row reduction per CTA: rebuild the packed greedy words
        unsigned long long* red = reinterpret_cast<unsigned long long*>(smem + L::OFF_RED);
        const int mvalid = min(BT, args.M);  // one token tile (m0 = 0)
#pragma unroll
        for (int j = 0; j < BT; ++j) {
          if (j < mvalid) {
            unsigned long long k = 0ull;
            if (best[j]) {
              const int itb = 0xFFFF - (int)(best[j] & 0xFFFFu);
              const int ub = unit0 + itb * ustride;
              const int nb = (ub % args.n_tiles) * TC_BN + row;
              k = ((unsigned long long)(best[j] >> 16) << 32) |
                  (unsigned long long)(0xFFFFFFFFu - (uint32_t)((int64_t)nb + args.vocab_offset));
            }
            k = warp_max_u64(k);
            if (lane == 0) red[q * BT + j] = k;
          }
        }
        epi_bar();
        for (int j = e; j < mvalid; j += 128) {
          unsigned long long v = red[j];
          for (int w = 1; w < 4; ++w) v = red[w * BT + j] > v ? red[w * BT + j] : v;
          if (v) atomicMax(args.packed + j, v);
        }
      }
    }
    if (args.y_tma && e == 0) ptx::bulk_wait_group_read0();  // staging read before exit
    __syncwarp();
  }

  if (nsplit > 1) {
    // ------------------------------------------------------------ cluster split-K reduction
    __syncwarp();
    ptx::cluster_sync();  // every split's partial is parked in its CTA's shared memory
    if (warp >= 8 && have_acc) {
      int n0, m0, kb, nk;
      unit_coords(unit0, n0, m0, kb, nk);
      const int mvalid = min(BT, args.M - m0);
      const uint32_t rank = ptx::cluster_ctarank();
      const int w4 = warp - 8;
      const int r0 = 4 * lane;  // this lane's 4 consecutive tile rows
      float sc4[4], bb4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int ne = n0 + r0 + q;
        sc4[q] = ne < args.N ? args.scales[ne] * 256.f : 0.f;
        bb4[q] = ne < args.N ? tc_load_bias(args.bias, args.bias_dtype, ne) : 0.f;
      }
      for (int jb = (int)rank + w4 * nsplit; jb < mvalid; jb += 4 * nsplit) {
        const uint32_t loc = sbase + (uint32_t)((jb * TC_BN + r0) * 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp = 0; sp < nsplit; ++sp) {  // fixed order: deterministic
          const float4 p = ptx::ld_dsmem_f4(ptx::mapa_shared(loc, (uint32_t)sp));
          acc.x += p.x;
          acc.y += p.y;
          acc.z += p.z;
          acc.w += p.w;
        }
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
        if (ARGMAX) {
          unsigned long long k = 0ull;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const unsigned long long kq =
                tc_pack_key(a4[q], sc4[q], n0 + r0 + q, args.N, args.vocab_offset);
            k = kq > k ? kq : k;
          }
          k = warp_max_u64(k);
          if (lane == 0 && k) atomicMax(args.packed + m0 + jb, k);
        } else {
          __half* yrow = args.y + (size_t)(m0 + jb) * args.N;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + r0 + q < args.N) yrow[n0 + r0 + q] = __float2half_rn(fmaf(a4[q], sc4[q], bb4[q]));
        }
      }
    }
    __syncwarp();
    ptx::cluster_sync();  // no CTA leaves while another still reads its shared memory
  }

  // ------------------------------------------------------------ teardown
  if (threadIdx.x == 256) trace_stamp(tr, 6);  // epilogue done
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
  if (threadIdx.x == 0) trace_stamp(tr, 7);  // exit
}

// ============================================================================
// Host side
// ============================================================================
namespace {

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
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

int make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle sw) {
  auto enc = tmap_encoder();
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

template <int BT, int WS, int AS, int XS, bool ARGMAX>
int launch_tc_t(const TcPlan& p, const __half* x, const uint8_t* wq, TcArgs a, int sms,
                cudaStream_t s) {
  using Lay = TcLayout<BT, WS, AS, XS>;
  auto kern = w8a16_tc_kernel<BT, WS, AS, XS, ARGMAX>;
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), kern, Lay::ALLOC);
  if (ast) return ast;
  CUtensorMap tm_w, tm_x, tm_y;
  int st = make_tmap_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)a.K, (uint64_t)a.N,
                        (uint64_t)a.K, TC_WK, TC_BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st) return st;
  st = make_tmap_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)a.K, (uint64_t)a.M,
                    (uint64_t)a.K * 2, TC_BK, BT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  a.y_tma = 0;
  std::memset(&tm_y, 0, sizeof(tm_y));
  if (!ARGMAX && p.splits == 1 && a.N % 8 == 0 && aligned16(a.y)) {
    st = make_tmap_2d(&tm_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.y, (uint64_t)a.N, (uint64_t)a.M,
                      (uint64_t)a.N * 2, TC_BN, Lay::CH, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    a.y_tma = 1;
  }
  a.n_tiles = (a.N + TC_BN - 1) / TC_BN;
  const int64_t m_tiles = (a.M + BT - 1) / BT;
  const int64_t tiles = (int64_t)a.n_tiles * m_tiles;
  if (tiles > 0x7fffffff) return DDQ_ERR_SHAPE;
  a.units = (int)tiles;
  cudaLaunchConfig_t cfg = {};
  if (p.splits > 1)
    cfg.gridDim = dim3((unsigned)tiles, 1, (unsigned)p.splits);  // one unit per CTA
  else
    cfg.gridDim = dim3((unsigned)(tiles < sms ? tiles : sms), 1, 1);  // persistent
  cfg.blockDim = dim3(TC_THREADS);
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

TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int sms) {
  TcPlan p{};
  p.bt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const int64_t KT = (K + TC_BK - 1) / TC_BK;
  const int64_t tiles = ((N + TC_BN - 1) / TC_BN) * ((M + p.bt - 1) / p.bt);
  int64_t splits = 1, kps = KT;
  // Split K over a cluster (at most kMaxSplits CTAs, within the portable
  // cluster size) only when the tiles alone would leave most SMs idle.
  if (sms > 0 && tiles * 2 <= sms) {
    splits = sms / tiles;
    if (splits > kMaxSplits) splits = kMaxSplits;
    if (splits > KT) splits = KT;
    if (splits < 1) splits = 1;
    kps = (KT + splits - 1) / splits;
    kps = (kps + 3) & ~(int64_t)3;  // whole 256-wide weight stages per split
    splits = (KT + kps - 1) / kps;
  }
  p.splits = (int)splits;
  p.kps = (int)kps;
  p.tiles = tiles;
  p.ws_part_bytes = 0;
  p.ws_bytes = 0;
  return p;
}

int launch_tc(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, unsigned long long* packed, int64_t vocab_offset,
              int M, int N, int K, void* ws, size_t ws_bytes, unsigned long long timeout_ns,
              int debug_flags, cudaStream_t s) {
  (void)ws;
  (void)ws_bytes;
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  const TcPlan p = tc_plan(M, N, K, sms);
  TcArgs a{};
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.packed = packed;
  a.vocab_offset = vocab_offset;
  a.M = M;
  a.N = N;
  a.K = K;
  a.kps = p.kps;
  a.timeout_ns = timeout_ns;
  a.debug_flags = debug_flags;
  const bool am = packed != nullptr;
  // (token tile, e4m3 stages of 4 K steps, fp16 weight slots, activation slots)
#define DDQ_TC_CASE(BT_, WS_, AS_, XS_)                                                 \
  case BT_:                                                                             \
    return am ? launch_tc_t<BT_, WS_, AS_, XS_, true>(p, x, wq, a, sms, s)              \
              : launch_tc_t<BT_, WS_, AS_, XS_, false>(p, x, wq, a, sms, s);
  switch (p.bt) {
    DDQ_TC_CASE(16, 3, 4, 14)
    DDQ_TC_CASE(32, 3, 4, 8)
    DDQ_TC_CASE(64, 3, 4, 4)
    DDQ_TC_CASE(128, 2, 4, 4)
    DDQ_TC_CASE(256, 2, 2, 3)
    default:
      return DDQ_ERR_SHAPE;
  }
#undef DDQ_TC_CASE
}

}  // namespace ddq
