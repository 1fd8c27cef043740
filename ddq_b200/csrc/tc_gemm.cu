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
// Per CTA (192 threads, one 128 x BT output tile, one K range):
//   warp 0     TMA producer: e4m3 weight tile [128 x 64 B] (64-byte swizzle)
//              and activation tile [BT x 64 fp16] (128-byte swizzle) per stage
//   warp 1     MMA issuer: 4 x tcgen05.mma kind::f16 (K = 16) per stage,
//              tcgen05.commit releases the stage
//   warps 2-5  converters: e4m3 -> fp16 into the canonical 128-byte-swizzled
//              K-major A layout, then the epilogue (tcgen05.ld -> scale, bias,
//              fp16 store; or the packed greedy key for the lm_head)
// Split-K: CTAs of one tile write fp32 partials to the workspace; the last
// to arrive (atomic ticket) sums them in split order - deterministic - and
// runs the epilogue, then re-arms the ticket to zero.
// Every mbarrier wait is bounded; on timeout the CTA records DDQ_ERR_TIMEOUT
// in the device error word, drains its own TMA copies and MMAs, frees TMEM
// and exits.
#include <cudaTypedefs.h>

#include <cfloat>
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int TC_BN = 128;       // weight rows per tile (MMA M)
constexpr int TC_BK = 64;        // K elements per pipeline stage
constexpr int TC_THREADS = 192;  // 6 warps

template <int BT, int STAGES>
struct TcLayout {
  static constexpr int A_BYTES = TC_BN * TC_BK * 2;  // converted fp16 weight tile
  static constexpr int B_BYTES = BT * TC_BK * 2;     // activation tile
  static constexpr int W_BYTES = TC_BN * TC_BK;      // e4m3 weight tile
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_W = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_W + STAGES * W_BYTES;
  static constexpr int NBAR = 3 * STAGES + 2;  // full, empty, conv per stage; acc, drain
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_RED = OFF_MISC + 16;  // argmax reduction [4 warps][BT] u64
  static constexpr int BYTES = OFF_RED + 4 * BT * 8;
  static constexpr int ALLOC = BYTES + 1024;     // slack to align the base to 1024 B
  static_assert(B_BYTES % 1024 == 0, "activation stage must keep 1024-B alignment");
};

__device__ __forceinline__ float tc_load_bias(const void* bias, int bias_dtype, int n) {
  if (bias_dtype == DDQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (bias_dtype == DDQ_DTYPE_F32) return reinterpret_cast<const float*>(bias)[n];
  return 0.f;
}

__device__ __forceinline__ unsigned long long tc_pack_key(__half v, int64_t idx) {
  return ((unsigned long long)f16_order_key(v) << 32) |
         (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__device__ __forceinline__ void named_bar_epilogue() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Wait ignoring the abort flag (used only while winding down).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer_ns() - t0 > timeout_ns) return false;
  }
  return true;
}

struct TcArgs {
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  unsigned long long* packed;  // lm_head: per-token packed greedy key (ARGMAX)
  int64_t vocab_offset;
  float* ws_part;              // split-K partials
  unsigned* ws_cnt;            // split-K tickets (zero between calls)
  int M, N, K, kps;
  unsigned long long timeout_ns;
  int debug_flags;             // bit 0: never signal the accumulator (timeout test)
};

template <int BT, int STAGES, bool ARGMAX>
__global__ void __launch_bounds__(TC_THREADS, 1)
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_x, const TcArgs args) {
  using L = TcLayout<BT, STAGES>;
  constexpr uint32_t TMEM_COLS = BT < 32 ? 32 : BT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TC_BN, m0 = blockIdx.y * BT;
  const int split = blockIdx.z, nsplit = gridDim.z;
  const int KT = (args.K + TC_BK - 1) / TC_BK;
  const int kb = split * args.kps;
  const int nk = min(args.kps, KT - kb);  // >= 1 by construction of the plan

  const uint32_t bar_full = sbase + L::OFF_BAR;
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_conv = bar_empty + 8 * STAGES;
  const uint32_t bar_acc = bar_conv + 8 * STAGES;
  const uint32_t bar_drain = bar_acc + 8;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 8);
  const uint64_t tmo = args.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);
      ptx::mbar_init(bar_conv + 8 * s, 4);
    }
    ptx::mbar_init(bar_acc, 1);
    ptx::mbar_init(bar_drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_w);
    ptx::prefetch_tmap(&tm_x);
  }
  if (warp == 0) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_d = *tmem_holder;

  // Inputs written by a preceding grid are visible after this (PDL launch);
  // a no-op for an ordinary launch.
  ptx::pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!ptx::mbar_wait(bar_empty + 8 * s, ph ^ 1u, tmo, abort_flag)) break;
        ptx::mbar_arrive_expect_tx(bar_full + 8 * s, L::W_BYTES + L::B_BYTES);
        const int kc = (kb + i) * TC_BK;
        ptx::tma_load_2d(sbase + L::OFF_W + s * L::W_BYTES, &tm_w, kc, n0, bar_full + 8 * s);
        ptx::tma_load_2d(sbase + L::OFF_B + s * L::B_BYTES, &tm_x, kc, m0, bar_full + 8 * s);
        issued = i + 1;
      }
      if (*abort_flag) {
        // let every copy still in flight land before the CTA exits
        for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
          mbar_wait_drain(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u, tmo);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_f16_f32(TC_BN, BT);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        ok = ptx::mbar_wait(bar_full + 8 * s, ph, tmo, abort_flag) &&
             ptx::mbar_wait(bar_conv + 8 * s, ph, tmo, abort_flag);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t a0 = sbase + L::OFF_A + s * L::A_BYTES;
        const uint32_t b0 = sbase + L::OFF_B + s * L::B_BYTES;
#pragma unroll
        for (int j = 0; j < TC_BK / 16; ++j) {
          ptx::mma_f16_ss(tmem_d, ptx::smem_desc_sw128(a0 + 32 * j),
                          ptx::smem_desc_sw128(b0 + 32 * j), idesc, (i | j) != 0 ? 1u : 0u);
        }
        ptx::mma_commit(bar_empty + 8 * s);
      }
      if (ok && !(args.debug_flags & 1)) {
        ptx::mma_commit(bar_acc);
      } else {
        // wind down: wait for this thread's MMAs before TMEM is freed
        ptx::mma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0, tmo);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ converters
    const int t = threadIdx.x - 64;  // weight row of the tile this thread converts
    const int sw_w = (t >> 1) & 3;   // 64-byte swizzle phase of row t (e4m3 tile)
    const int sw_a = t & 7;          // 128-byte swizzle phase of row t (fp16 tile)
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!ptx::mbar_wait(bar_full + 8 * s, ph, tmo, abort_flag)) break;
      const uint8_t* wrow = smem + L::OFF_W + s * L::W_BYTES + t * 64;
      uint8_t* arow = smem + L::OFF_A + s * L::A_BYTES + t * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((c ^ sw_w) << 4));
        uint4 lo, hi;
        lo.x = e4m3x2_to_half2_bits((uint16_t)(v.x & 0xFFFF));
        lo.y = e4m3x2_to_half2_bits((uint16_t)(v.x >> 16));
        lo.z = e4m3x2_to_half2_bits((uint16_t)(v.y & 0xFFFF));
        lo.w = e4m3x2_to_half2_bits((uint16_t)(v.y >> 16));
        hi.x = e4m3x2_to_half2_bits((uint16_t)(v.z & 0xFFFF));
        hi.y = e4m3x2_to_half2_bits((uint16_t)(v.z >> 16));
        hi.z = e4m3x2_to_half2_bits((uint16_t)(v.w & 0xFFFF));
        hi.w = e4m3x2_to_half2_bits((uint16_t)(v.w >> 16));
        *reinterpret_cast<uint4*>(arow + (((2 * c) ^ sw_a) << 4)) = lo;
        *reinterpret_cast<uint4*>(arow + (((2 * c + 1) ^ sw_a) << 4)) = hi;
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_conv + 8 * s);
    }

    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;            // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;     // tile row == TMEM lane
    const int n = n0 + row;
    const int mvalid = min(BT, args.M - m0);
    const bool have_acc = ptx::mbar_wait(bar_acc, 0, tmo, abort_flag);
    if (have_acc) {
      ptx::tc_fence_after();
      const uint32_t taddr = tmem_d + ((uint32_t)(q * 32) << 16);
      constexpr int CH = BT < 32 ? 16 : 32;
      const float sc = n < args.N ? args.scales[n] : 0.f;
      const float bb = (n < args.N) ? tc_load_bias(args.bias, args.bias_dtype, n) : 0.f;
      unsigned long long* red = reinterpret_cast<unsigned long long*>(smem + L::OFF_RED);
      // lm_head: warp-wide max of the packed key of column j -> red[q][j]
      auto emit_key = [&](int j, float acc) {
        const __half v = __float2half_rn(acc * sc);
        unsigned long long k = (n < args.N && __half2float(v) > -FLT_MAX)
                                   ? tc_pack_key(v, (int64_t)n + args.vocab_offset) : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long u = __shfl_xor_sync(0xffffffffu, k, o);
          k = u > k ? u : k;
        }
        if (lane == 0) red[q * BT + j] = k;
      };
      bool final_tile = true;
      const int tile = blockIdx.y * gridDim.x + blockIdx.x;
      float* part = nullptr;
      if (nsplit > 1)
        part = args.ws_part + ((size_t)tile * nsplit + split) * (size_t)(TC_BN * BT);

#pragma unroll 1
      for (int c0 = 0; c0 < BT; c0 += CH) {
        uint32_t r[32];
        if (CH == 32) ptx::tmem_ld_32x32b_x32(taddr + c0, r);
        else ptx::tmem_ld_32x32b_x16(taddr + c0, r);
        ptx::tmem_ld_wait();
        if (c0 >= mvalid) continue;
        if (nsplit > 1) {
#pragma unroll
          for (int j = 0; j < CH; ++j)
            if (c0 + j < mvalid) part[(c0 + j) * TC_BN + row] = __uint_as_float(r[j]);
        } else if (ARGMAX) {
#pragma unroll
          for (int j = 0; j < CH; ++j)
            if (c0 + j < mvalid) emit_key(c0 + j, __uint_as_float(r[j]));
        } else {
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const int m = m0 + c0 + j;
            if (n < args.N && c0 + j < mvalid)
              args.y[(size_t)m * args.N + n] = __float2half_rn(fmaf(__uint_as_float(r[j]), sc, bb));
          }
        }
      }

      if (nsplit > 1) {
        // publish the partial, take a ticket; the last CTA reduces in split order
        __threadfence();
        named_bar_epilogue();
        if (t == 0) {
          const unsigned prev = atomicAdd(args.ws_cnt + tile, 1u);
          *last_flag = (prev == (unsigned)(nsplit - 1)) ? 1 : 0;
        }
        named_bar_epilogue();
        final_tile = *last_flag != 0;
        if (final_tile) {
          __threadfence();
          const float* base = args.ws_part + (size_t)tile * nsplit * (size_t)(TC_BN * BT);
#pragma unroll 1
          for (int j = 0; j < mvalid; ++j) {
            float acc = 0.f;
            for (int sp = 0; sp < nsplit; ++sp)
              acc += __ldcg(base + ((size_t)sp * BT + j) * TC_BN + row);
            if (ARGMAX) {
              emit_key(j, acc);
            } else if (n < args.N) {
              args.y[(size_t)(m0 + j) * args.N + n] = __float2half_rn(fmaf(acc, sc, bb));
            }
          }
          if (t == 0) args.ws_cnt[tile] = 0u;  // re-arm for the next call on this stream
        }
      }

      if (ARGMAX && final_tile) {
        // combine the 4 warps' maxima per token, one atomicMax per token row
        named_bar_epilogue();
        for (int j = t; j < mvalid; j += 128) {
          unsigned long long v = red[j];
          for (int w = 1; w < 4; ++w) v = red[w * BT + j] > v ? red[w * BT + j] : v;
          if (v) atomicMax(args.packed + m0 + j, v);
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_d, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
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

template <int BT, int STAGES, bool ARGMAX>
int launch_tc_t(const TcPlan& p, const __half* x, const uint8_t* wq, const TcArgs& a,
                cudaStream_t s) {
  using Lay = TcLayout<BT, STAGES>;
  auto kern = w8a16_tc_kernel<BT, STAGES, ARGMAX>;
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return DDQ_ERR_DEVICE;
  static bool attr_set[64] = {};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::ALLOC) !=
        cudaSuccess)
      return DDQ_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  CUtensorMap tm_w, tm_x;
  int st = make_tmap_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)a.K, (uint64_t)a.N,
                        (uint64_t)a.K, TC_BK, TC_BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (st) return st;
  st = make_tmap_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)a.K, (uint64_t)a.M,
                    (uint64_t)a.K * 2, TC_BK, BT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  dim3 grid((unsigned)((a.N + TC_BN - 1) / TC_BN), (unsigned)((a.M + BT - 1) / BT),
            (unsigned)p.splits);
  kern<<<grid, TC_THREADS, Lay::ALLOC, s>>>(tm_w, tm_x, a);
  return check_launch();
}

}  // namespace

TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int sms) {
  TcPlan p{};
  p.bt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const int64_t KT = (K + TC_BK - 1) / TC_BK;
  const int64_t tiles = ((N + TC_BN - 1) / TC_BN) * ((M + p.bt - 1) / p.bt);
  int64_t splits = 1, kps = KT;
  if (sms > 0 && tiles < sms && tiles <= kTicketSlots) {
    splits = sms / tiles;
    if (splits > KT) splits = KT;
    if (splits < 1) splits = 1;
    kps = (KT + splits - 1) / splits;
    splits = (KT + kps - 1) / kps;
  }
  p.splits = (int)splits;
  p.kps = (int)kps;
  p.tiles = tiles;
  if (splits > 1) {
    // [0, 4 KiB): one ticket per tile, always at the same place, so whatever
    // shape ran before, the tickets a call reads are the zeros the previous
    // call left behind.  Partials follow.
    p.ws_part_bytes = (size_t)tiles * splits * TC_BN * p.bt * sizeof(float);
    p.ws_bytes = kTicketBytes + p.ws_part_bytes;
  }
  return p;
}

int launch_tc(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, unsigned long long* packed, int64_t vocab_offset,
              int M, int N, int K, void* ws, size_t ws_bytes, unsigned long long timeout_ns,
              int debug_flags, cudaStream_t s) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  const TcPlan p = tc_plan(M, N, K, sms);
  if (p.ws_bytes > 0 && (ws == nullptr || ws_bytes < p.ws_bytes)) return DDQ_ERR_WORKSPACE;
  if (p.ws_bytes > 0 && (reinterpret_cast<uintptr_t>(ws) & 255u)) return DDQ_ERR_ALIGNMENT;
  if ((M + p.bt - 1) / p.bt > 65535) return DDQ_ERR_SHAPE;
  TcArgs a{};
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.packed = packed;
  a.vocab_offset = vocab_offset;
  a.ws_cnt = p.ws_bytes ? reinterpret_cast<unsigned*>(ws) : nullptr;
  a.ws_part = p.ws_bytes ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kTicketBytes)
                         : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.kps = p.kps;
  a.timeout_ns = timeout_ns;
  a.debug_flags = debug_flags;
  const bool am = packed != nullptr;
#define DDQ_TC_CASE(BT_, ST_)                                                           \
  case BT_:                                                                             \
    return am ? launch_tc_t<BT_, ST_, true>(p, x, wq, a, s)                             \
              : launch_tc_t<BT_, ST_, false>(p, x, wq, a, s);
  switch (p.bt) {
    DDQ_TC_CASE(16, 4)
    DDQ_TC_CASE(32, 4)
    DDQ_TC_CASE(64, 4)
    DDQ_TC_CASE(128, 4)
    DDQ_TC_CASE(256, 3)
    default:
      return DDQ_ERR_SHAPE;
  }
#undef DDQ_TC_CASE
}

}  // namespace ddq
