// lmh.cu - fused lm_head GEMM + greedy argmax for 1..8 tokens, streaming the
// weight through shared memory with large contiguous bulk copies.
//
// Semantics (engine.py:338 + sampler_d.cu:10-70 on the last position): for
// each token row m of x, the largest fp16 logit
//     logit[m, n] = fp16( (sum_k x[m, k] * e4m3(W[n, k])) * scale[n] )
// over this shard's rows n, ties to the lowest global index n + vocab_offset,
// NaN and -inf never winning, reported as the packed word
//     (ordered fp16 key << 32) | (0xFFFFFFFF - (n + vocab_offset))
// (0 when no row qualifies) and, optionally, as the decoded index.
//
// Layout of the work: the rows are cut into 16-row tiles (the mma.sync A
// operand, tokens on the 8-column B operand as in rs.cu) and every CTA takes a
// contiguous run of tiles - 151,936 rows are 9,496 tiles, 64 or 65 per CTA on
// 148 SMs, so the last CTAs finish within 1.5 % of the others.  A tile's
// 16 x K bytes are one contiguous range: one bulk copy (TMA engine) per tile,
// issued by a producer warp into a ring of two stages per consumer warp.
// Each consumer warp takes whole tiles (tile i goes to warp i mod the
// consumer count), so no partial sums cross warps; a thread keeps the best
// packed word of the rows it sees per token.  At the end the CTA reduces them and
// writes one word per token to a per-CTA slot of the workspace; the last CTA
// to finish (an arrival counter in the workspace) combines the slots in CTA
// order into packed[] and ids[] and clears the counter for the next call.
// One kernel per call: no memset of packed, no activation split, no separate
// unpack.
#include <cfloat>
#include <cstdlib>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {
namespace {

// Consumer warps and ring stages: tile i goes to warp i mod NC and to stage
// i mod 2 NC, so every stage belongs to one warp, which consumes its uses in
// order - a warp never waits on a phase two ahead of the last one completed
// (a parity wait cannot tell those apart) - and each warp's next tile loads
// while it computes the current one.  NC = 7: 14 stages of a 16 x 896-byte
// tile plus 16 tokens of activations fit in shared memory.
constexpr int LM_NC = 7;
constexpr int LM_MAX_CONSUMERS = LM_NC;
constexpr int LM_TILE = 16;
constexpr int LM_MAX_STAGES = 2 * 7;
constexpr int LM_SMEM_MAX = 232448;

struct LmArgs {
  const __half* x;
  const uint8_t* wq;
  const float* scales;
  unsigned long long* packed;   // [M]
  long long* ids;               // [M] or null
  unsigned long long* part;     // [grid][M] per-CTA best words (workspace)
  unsigned int* counter;        // arrival counter (workspace), zero between calls
  long long vocab_offset;
  int M, N, K;
  int tiles;                    // ceil(N / 16)
  int stages;
  int off_x, off_bar;
  unsigned long long timeout_ns;
  int trace;
};

__device__ __forceinline__ void lm_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint4 lm_lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ void lm_mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <int NC>
__device__ __forceinline__ void lm_consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
}
__device__ __forceinline__ unsigned long long lm_max(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

// Shared memory: [0, stages * 16 * K) the ring of weight tiles; off_x the
// activations [M][K] fp16; off_bar full[stages], empty[stages], the x
// barrier, the abort, drain and last-CTA flags, then (at + 32) the per-warp
// best words [NC][16 tokens] (u64).
template <int NB, int NC, bool HW>
__global__ void __launch_bounds__((NC + 1) * 32, 1) w8a16_lmh_kernel(const LmArgs a) {
  extern __shared__ __align__(128) uint8_t lm_smem[];
  const uint32_t sbase = ptx::smem_u32(lm_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  const int tile0 = (int)(((int64_t)b * a.tiles) / G);
  const int ntl = (int)(((int64_t)(b + 1) * a.tiles) / G) - tile0;
  const int M = a.M, N = a.N, K = a.K, KB = K >> 6, S = a.stages;
  const uint32_t tile_bytes = (uint32_t)(LM_TILE * K);
  const uint32_t bar_full = sbase + (uint32_t)a.off_bar;
  const uint32_t bar_empty = bar_full + 8 * S;
  const uint32_t bar_x = bar_empty + 8 * S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(lm_smem + a.off_bar + 16 * S + 8);
  volatile int* drain_flag = abort_flag + 1;
  volatile int* last_flag = abort_flag + 2;
  unsigned long long* wbest =
      reinterpret_cast<unsigned long long*>(lm_smem + a.off_bar + 16 * S + 32);
  const bool tr = a.trace != 0;
  if (tid == 0) {
    trace_stamp(tr, 0);
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);
    }
    ptx::mbar_init(bar_x, 1);
    *abort_flag = 0;
    *drain_flag = 0;
    *last_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  ptx::pdl_launch_dependents();

  if (warp == NC) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      auto issue = [&](int i) {
        const int s = i % S;
        const int row0 = (tile0 + i) * LM_TILE;
        const int valid = min(LM_TILE, N - row0);
        ptx::mbar_arrive_expect_tx(bar_full + 8 * s, (uint32_t)(valid * K));
        lm_bulk_g2s(sbase + (uint32_t)s * tile_bytes, a.wq + (size_t)row0 * K,
                    (uint32_t)(valid * K), bar_full + 8 * s);
      };
      const int pre = ntl < S ? ntl : S;
      for (int i = 0; i < pre; ++i) issue(i);  // weights: before the dependency
      trace_stamp(tr, 2);
      ptx::pdl_wait();
      trace_stamp(tr, 3);
      ptx::mbar_arrive_expect_tx(bar_x, (uint32_t)(M * K * 2));
      lm_bulk_g2s(sbase + (uint32_t)a.off_x, a.x, (uint32_t)(M * K * 2), bar_x);
      int i = pre;
      for (; i < ntl; ++i) {
        const int s = i % S;
        if (!ptx::mbar_wait(bar_empty + 8 * s, (uint32_t)((i / S - 1) & 1), a.timeout_ns,
                            abort_flag))
          break;
        issue(i);
      }
      // after an abort: wait (bounded) for every copy still in flight
      if (*abort_flag) {
        for (int j = (i > S ? i - S : 0); j < i; ++j)
          ptx::mbar_wait(bar_full + 8 * (j % S), (uint32_t)((j / S) & 1), a.timeout_ns, drain_flag);
        ptx::mbar_wait(bar_x, 0u, a.timeout_ns, drain_flag);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    uint32_t xrow[NB];
    bool xok[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int tok = nb * 8 + g;
      xok[nb] = tok < M;
      xrow[nb] = sbase + (uint32_t)a.off_x + (uint32_t)((xok[nb] ? tok : 0) * K * 2 + t * 32);
    }
    // running best word per (token block, token 2t / 2t + 1)
    unsigned long long best[NB][2];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) best[nb][0] = best[nb][1] = 0ull;
    bool ok = ptx::mbar_wait(bar_x, 0u, a.timeout_ns, abort_flag);
    if (ok && warp == 0 && lane == 0) trace_stamp(tr, 5);
    for (int i = warp; ok && i < ntl; i += NC) {
      const int s = i % S;
      const int row0 = (tile0 + i) * LM_TILE;
      // the two rows this thread scores, and their scales (issued early)
      const int nlo = row0 + g, nhi = row0 + g + 8;
      const float slo = nlo < N ? a.scales[nlo] * kE4m3ToF16Scale<HW> : 0.f;
      const float shi = nhi < N ? a.scales[nhi] * kE4m3ToF16Scale<HW> : 0.f;
      if (!ptx::mbar_wait(bar_full + 8 * s, (uint32_t)((i / S) & 1), a.timeout_ns, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t wlo = sbase + (uint32_t)s * tile_bytes + (uint32_t)(g * K + t * 16);
      const uint32_t whi = wlo + (uint32_t)(8 * K);
      // Two K blocks per step, each MMA j into set (block parity, j parity):
      // consecutive MMAs never feed each other (mma.sync issues in order), so
      // four independent accumulator chains per token block.
      float acc[4][NB][4];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) acc[h][nb][0] = acc[h][nb][1] = acc[h][nb][2] = acc[h][nb][3] = 0.f;
      for (int kb = 0; kb < KB; kb += 2) {
        const int nk = kb + 1 < KB ? 2 : 1;
        uint32_t lw[2][4], hw[2][4], xs[2][NB][8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h < nk) {
            const uint4 lo = lm_lds128(wlo + (uint32_t)((kb + h) * 64));
            const uint4 hi = lm_lds128(whi + (uint32_t)((kb + h) * 64));
            lw[h][0] = lo.x; lw[h][1] = lo.y; lw[h][2] = lo.z; lw[h][3] = lo.w;
            hw[h][0] = hi.x; hw[h][1] = hi.y; hw[h][2] = hi.z; hw[h][3] = hi.w;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              uint4 x0 = make_uint4(0u, 0u, 0u, 0u), x1 = x0;
              if (xok[nb]) {
                x0 = lm_lds128(xrow[nb] + (uint32_t)((kb + h) * 128));
                x1 = lm_lds128(xrow[nb] + (uint32_t)((kb + h) * 128 + 16));
              }
              xs[h][nb][0] = x0.x; xs[h][nb][1] = x0.y; xs[h][nb][2] = x0.z; xs[h][nb][3] = x0.w;
              xs[h][nb][4] = x1.x; xs[h][nb][5] = x1.y; xs[h][nb][6] = x1.z; xs[h][nb][7] = x1.w;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) lw[h][q] = hw[h][q] = 0u;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
#pragma unroll
              for (int q = 0; q < 8; ++q) xs[h][nb][q] = 0u;
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t a0, a1, a2, a3;
            e4m3x4_to_half2x2<HW>(lw[h][j], a0, a2);
            e4m3x4_to_half2x2<HW>(hw[h][j], a1, a3);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
              lm_mma(acc[2 * h + (j & 1)][nb], a0, a1, a2, a3, xs[h][nb][2 * j], xs[h][nb][2 * j + 1]);
          }
        }
      }
      // the stage is free once every lane's shared-memory reads are done
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
      // packed candidates: rows nlo / nhi, tokens 2t / 2t + 1 of each block
      const uint32_t ilo = 0xFFFFFFFFu - (uint32_t)((long long)nlo + a.vocab_offset);
      const uint32_t ihi = 0xFFFFFFFFu - (uint32_t)((long long)nhi + a.vocab_offset);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float slo_acc = (acc[0][nb][c] + acc[1][nb][c]) + (acc[2][nb][c] + acc[3][nb][c]);
          const float shi_acc = (acc[0][nb][2 + c] + acc[1][nb][2 + c]) +
                                (acc[2][nb][2 + c] + acc[3][nb][2 + c]);
          const __half vlo = __float2half_rn(slo_acc * slo);
          const __half vhi = __float2half_rn(shi_acc * shi);
          unsigned long long cand = 0ull;
          if (nlo < N && __half2float(vlo) > -FLT_MAX)
            cand = ((unsigned long long)f16_order_key(vlo) << 32) | ilo;
          if (nhi < N && __half2float(vhi) > -FLT_MAX)
            cand = lm_max(cand, ((unsigned long long)f16_order_key(vhi) << 32) | ihi);
          best[nb][c] = lm_max(best[nb][c], cand);
        }
      }
    }
    if (!ok) *abort_flag = 1;
    if (warp == 0 && lane == 0) trace_stamp(tr, 4);
    // reduce over the 8 row groups g (lanes t, t + 4, ..., t + 28)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1)
          best[nb][c] = lm_max(best[nb][c], __shfl_xor_sync(0xffffffffu, best[nb][c], o));
    if (g == 0) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        wbest[warp * 16 + nb * 8 + 2 * t] = best[nb][0];
        wbest[warp * 16 + nb * 8 + 2 * t + 1] = best[nb][1];
      }
    }
    lm_consumer_bar<NC>();
    if (tid < M) {
      unsigned long long v = 0ull;
#pragma unroll
      for (int w = 0; w < NC; ++w) v = lm_max(v, wbest[w * 16 + tid]);
      a.part[(size_t)b * M + tid] = v;
      __threadfence();  // this word is visible device-wide before the arrival below
    }
    lm_consumer_bar<NC>();
    if (warp == 0 && lane == 0) trace_stamp(tr, 6);
    // the last CTA to arrive combines every CTA's words (in CTA order: the
    // maximum does not depend on it) and clears the counter
    if (tid == 0) {
      __threadfence();
      const unsigned int prev = atomicAdd(a.counter, 1u);
      *last_flag = prev == (unsigned int)(G - 1) ? 1 : 0;
    }
    lm_consumer_bar<NC>();
    if (*last_flag) {
      // every consumer thread loads a share of the G x M words at once (one
      // L2 round trip), folds them per token into shared memory, then the
      // token maxima are written
      __threadfence();
      unsigned long long* tok_best = wbest;  // reused: [M] words
      if (tid < M) tok_best[tid] = 0ull;
      lm_consumer_bar<NC>();
      const int total = G * M;
      for (int i = tid; i < total; i += NC * 32) {
        const unsigned long long v = __ldcg(a.part + i);
        if (v) atomicMax(tok_best + (i % M), v);
      }
      lm_consumer_bar<NC>();
      if (tid < M) {
        const unsigned long long v = tok_best[tid];
        a.packed[tid] = v;
        if (a.ids) a.ids[tid] = v ? (long long)(0xFFFFFFFFull - (v & 0xFFFFFFFFull)) : 0ll;
      }
      if (tid == 0) *a.counter = 0u;
    }
  }
  __syncthreads();
  if (tid == 0 && *abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
  if (tid == 0) trace_stamp(tr, 7);
}

struct LmPlan {
  bool ok;
  int grid, stages, smem, off_x, off_bar;
};

// DDQ_LMH_MAX_M overrides the largest token count this kernel takes (0
// switches it off) for measurements.
int64_t lmh_max_m() {
  static const int64_t v = [] {
    const char* e = std::getenv("DDQ_LMH_MAX_M");
    return e ? (int64_t)std::atoll(e) : (int64_t)8;
  }();
  return v;
}

LmPlan lmh_plan(int64_t M, int64_t N, int64_t K, int sms) {
  LmPlan p{};
  // 1..8 tokens (at 9..16 the consumers' MMAs, not the weight stream, bound
  // it and the decode kernel's lm_head path measured faster)
  if (M < 1 || M > 8 || M > lmh_max_m() || N < 1 || K < 64 || K % 64 != 0 || K > 4096 ||
      sms <= 0)
    return p;
  if (N > 0x7fffffff - LM_TILE) return p;
  const int64_t tiles = (N + LM_TILE - 1) / LM_TILE;
  const int64_t grid = tiles < sms ? tiles : sms;
  const int64_t tile_bytes = LM_TILE * K;
  const int64_t x_bytes = M * K * 2;
  const int64_t off_x_max = LM_SMEM_MAX - ((x_bytes + 15) & ~15ll) - (16 * LM_MAX_STAGES + 32) -
                            8 * LM_MAX_CONSUMERS * 16 - 16;
  const int64_t stages = 2 * LM_NC;  // the ownership rule above needs exactly this many
  if (stages * tile_bytes > off_x_max) return p;
  const int64_t off_x = stages * tile_bytes;
  const int64_t off_bar = off_x + ((x_bytes + 15) & ~15ll);
  const int64_t total = off_bar + 16 * stages + 32 + 8 * LM_MAX_CONSUMERS * 16;
  if (total > LM_SMEM_MAX) return p;
  p.ok = true;
  p.grid = (int)grid;
  p.stages = (int)stages;
  p.smem = (int)total;
  p.off_x = (int)off_x;
  p.off_bar = (int)off_bar;
  return p;
}

bool lmh_hw_cvt() {
  static const bool v = [] {
    const char* e = std::getenv("DDQ_E4M3_CVT");
    return !(e && e[0] == 'i');
  }();
  return v;
}

template <int NB, int NC, bool HW>
int launch_lmh_t(const LmPlan& p, const LmArgs& a, cudaStream_t s) {
  static SmemAttrOnce attr;
  const int ast = ensure_smem_attr(attr, current_device(), w8a16_lmh_kernel<NB, NC, HW>, LM_SMEM_MAX);
  if (ast) return ast;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3((NC + 1) * 32);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_lmh_kernel<NB, NC, HW>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace

// The lm_head workspace starts with this kernel's area - the arrival counter
// (offset 0), then one word per CTA and token (offset 256) - sized for any
// shape on this device, so that the decode-kernel path for more tokens can
// keep its activation planes after it without touching the counter.
size_t lmh_area_bytes(int sms) {
  const size_t b = 256 + (size_t)(sms > 0 ? sms : 148) * 16 * 8;
  return (b + 4095) & ~(size_t)4095;
}

int launch_lmh(const __half* x, const uint8_t* wq, const float* scales, int M, int N, int K,
               int64_t vocab_offset, unsigned long long* packed, int64_t* ids, void* ws,
               size_t ws_bytes, unsigned long long timeout_ns, int debug_flags, cudaStream_t s) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  const LmPlan p = lmh_plan(M, N, K, sms);
  if (!p.ok) return DDQ_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(wq)) return DDQ_ERR_ALIGNMENT;
  if (!ws || ws_bytes < lmh_area_bytes(sms)) return DDQ_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return DDQ_ERR_ALIGNMENT;
  LmArgs a{};
  a.x = x;
  a.wq = wq;
  a.scales = scales;
  a.packed = packed;
  a.ids = reinterpret_cast<long long*>(ids);
  a.counter = reinterpret_cast<unsigned int*>(ws);
  a.part = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(ws) + 256);
  a.vocab_offset = vocab_offset;
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles = (N + LM_TILE - 1) / LM_TILE;
  a.stages = p.stages;
  a.off_x = p.off_x;
  a.off_bar = p.off_bar;
  a.timeout_ns = timeout_ns;
  a.trace = (debug_flags & 2) != 0;
  if (lmh_hw_cvt())
    return M <= 8 ? launch_lmh_t<1, LM_NC, true>(p, a, s) : launch_lmh_t<2, LM_NC, true>(p, a, s);
  return M <= 8 ? launch_lmh_t<1, LM_NC, false>(p, a, s) : launch_lmh_t<2, LM_NC, false>(p, a, s);
}

bool lmh_eligible(int64_t M, int64_t N, int64_t K, int sms) { return lmh_plan(M, N, K, sms).ok; }

}  // namespace ddq
