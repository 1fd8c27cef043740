// rt.cu - W8A16 GEMM for 17..64 tokens on the tcgen05 tensor cores, with
// every CTA's weight slice resident in shared memory before the grid
// dependency resolves.
//
// Semantics are those of the reference's f8_forward (gemm_FP8_d.cu:171-210):
//   y[m, n] = fp16( (sum_k x[m, k] * e4m3(W[n, k])) * scale[n] + bias[n] )
// with the sum in fp32; with the SwiGLU epilogue, z[m, j] = silu(g) * u of
// the fp16-rounded gate and up outputs (SwiGLU_d.cu:22-24), the weight being
// the 16-row interleave of gate and up that the decode and prefill kernels
// take (rows 32 b + i = gate row 16 b + i, rows 32 b + 16 + i = up row
// 16 b + i).
//
// Status: opt-in (ddq_set_debug bit 6), correct, and slower than the
// default paths.  In a chain of dependent calls on B200 it measured 7.3 us
// for q/k/v at 64 tokens (mma.sync resident slice: 4.9), 11.9 us for gate/up
// (split + e4m3 decode: 7.8) and 22.5 us for down (9.0).  Phase stamps and a
// standalone probe show where it goes: a tcgen05.mma of M = 64, N <= 72
// costs its issuing thread ~30 ns (tensor-pipe time ~10 ns), so K = 896 (56
// MMAs) needs ~1.7 us of issue from one thread, ~1 us from the three used
// here; the first activation atom lands ~0.5 us after the dependency; the
// epilogue over three accumulators and the barrier round trips add ~1.5 us.
// The design notes below are what was built.
//
// Why a kernel of its own: at 17..64 tokens the legacy mma.sync path runs out
// of tensor throughput (one m16n8k16 per about 8 SM cycles: 7.7 us of MMAs
// alone for the 9728 x 896 gate/up at 64 tokens), and the split-plane e4m3
// kernel (tc_decode.cu) adds a pre-pass launch and a 225 KB CTA that keeps
// the next GEMM's CTAs off the SM.  Here the tokens are the MMA's A operand
// (M = 64; token rows >= M arrive as zeros from the TMA box), the CTA's
// weight rows its B operand (N = the CTA's row count, a multiple of 8, at
// most 256), fp16 x fp16 -> fp32 in TMEM (kind::f16), K in 64-wide atoms
// (one 128-byte swizzle row):
//   before the grid dependency resolves
//     * one bulk copy of the CTA's contiguous e4m3 slice (one per row when K
//       is split), the per-row scale and bias, the TMEM allocation, and as
//       many weight atoms as the fp16 ring holds converted to fp16 in the
//       canonical 128-byte swizzled K-major layout (cvt.rn.f16x2.e4m3x2:
//       exact);
//   after it
//     warp 0      TMA loads of the activation atoms (64 tokens x 64 K, 8 KB)
//                 through a ring of 3..16 stages (as many as the shared-memory
//                 budget leaves: the fetch from L2 is latency-bound, so its
//                 rate grows with the atoms in flight)
//     warps 1-3   three MMA issuers (lane 0), 4 MMAs (K = 16) per atom on
//                 atoms i = w, w + 3, ... into their own 64 x R fp32
//                 accumulators, summed in order by the epilogue
//     warps 4-7   converters, a ring of fp16 weight atoms ahead of the MMAs
//                 (every atom where shared memory allows: each refill waits
//                 for an MMA to complete)
//     warps 4-7   then the epilogue: token m sits in TMEM lane
//                 (m mod 16) + 32 (m / 16) (the M = 64 data-path layout),
//                 weight row j in column j; scale, bias, fp16, stores.
// With K split over a cluster (large K: the activation stream per CTA stays
// near 20 atoms), each CTA parks its fp32 partial in its own shared memory
// and, after a cluster barrier, sums a share of the outputs over the
// cluster's partials in split order through distributed shared memory:
// deterministic, no workspace, no atomics.
// Shared memory stays within half an SM where both rings still fit there
// (the next GEMM's CTA can then be resident and fetch its own slice while
// this one runs), else the CTA takes the whole 227 KB.
// Every mbarrier wait is bounded; on timeout the CTA records
// DDQ_ERR_TIMEOUT, waits (bounded) for its own copies and MMAs, still takes
// part in the cluster barriers, writes nothing, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {
namespace {

constexpr int RT_THREADS = 256;
constexpr int RT_XS_MAX = 16;           // activation ring stages (the plan picks 3..16)
constexpr int RT_BS_MAX = 20;           // fp16 weight ring stages (up to every atom of a CTA)
constexpr int RT_XSTAGE = 64 * 128;     // 64 tokens x 64 fp16 (one swizzle atom)
constexpr int RT_ISSUERS = 3;           // MMA issuers: lane 0 of warps 1-3
constexpr int RT_CONV_THREADS = 128;    // warps 4-7
constexpr int RT_SMEM_MAX = 232448;     // 227 KB opt-in limit per CTA
constexpr int RT_SMEM_PAIR = 113 * 1024;  // two CTAs per SM
constexpr int RT_MAX_N = 256;           // MMA N limit (weight rows per CTA)
constexpr int kSmemPerSm = 233472;      // 228 KB of shared memory per SM
constexpr int kSmemReservedPerCta = 1024;

// barrier slots (8 bytes each) from off_bar
constexpr int RT_BAR_W = 0;                      // weight slice landed
constexpr int RT_BAR_XF = 1;                     // [xs] activation atom landed
constexpr int RT_BAR_XE = RT_BAR_XF + RT_XS_MAX; // [xs] activation stage free
constexpr int RT_BAR_BF = RT_BAR_XE + RT_XS_MAX; // [bs] fp16 weight atom ready
constexpr int RT_BAR_BE = RT_BAR_BF + RT_BS_MAX; // [bs] fp16 weight stage free
constexpr int RT_BAR_ACC = RT_BAR_BE + RT_BS_MAX; // accumulator complete
constexpr int RT_BAR_DRAIN = RT_BAR_ACC + 1;     // [RT_ISSUERS] MMA drain on exit
constexpr int RT_NBAR = RT_BAR_DRAIN + RT_ISSUERS;
constexpr int RT_BAR_BYTES = RT_NBAR * 8 + 16;   // + abort, drain flag, TMEM holder

struct RtArgs {
  const uint8_t* wq;
  const float* scales;
  const void* bias;
  int bias_dtype;
  __half* y;
  int M, N, K;
  int out_n;      // columns of y: N, or N / 2 with the SwiGLU epilogue
  int units;      // row units of unit_rows rows (8, or 32 with SwiGLU)
  int unit_rows;
  int row_ctas;   // CTAs per K split (gridDim.y)
  int splits;     // K splits = cluster size (gridDim.x)
  int atoms;      // K / 64
  int rmax;       // most rows any CTA takes
  int xs;         // activation ring stages
  int bs;         // fp16 weight ring stages
  int vec_y;      // y rows 16-byte aligned: vector stores
  int ncols;      // TMEM columns allocated (power of two >= 32)
  int acc_stride; // TMEM columns between the issuers' accumulators
  int off_b, off_x, off_sb, off_red, off_bar;  // shared-memory offsets (bytes)
  unsigned long long timeout_ns;
  int debug_flags;  // bit 1: phase stamps; bit 4: skip the accumulator-ready signal
};

__device__ __forceinline__ void rt_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ float rt_bias(const void* bias, int dt, int n) {
  if (dt == DDQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (dt == DDQ_DTYPE_F32) return reinterpret_cast<const float*>(bias)[n];
  return 0.f;
}

__device__ __forceinline__ uint32_t rt_pack(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Shared memory (from the 1024-byte aligned base):
//   0        the e4m3 weight slice [rows][kc] (kc = this CTA's K range); after
//            the MMAs, the fp32 partials [64][rmax] of a K split reuse it
//            unless off_red places them apart
//   off_b    bs fp16 weight atoms, rmax rows x 128 B each, swizzled
//   off_x    xs activation atoms, 64 rows x 128 B each, swizzled (TMA)
//   off_sb   scale[rmax], bias[rmax] fp32
//   off_bar  barriers, abort and drain flags, TMEM address
template <bool SWIGLU>
__global__ void __launch_bounds__(RT_THREADS, 2)
    w8a16_rt_kernel(const __grid_constant__ CUtensorMap tm_x, const RtArgs a) {
  extern __shared__ uint8_t rt_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(rt_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = a.splits;
  const int split = blockIdx.x;  // == rank in the cluster (cluster dims S x 1 x 1)
  const int rc = blockIdx.y;
  const int u0 = (int)((int64_t)rc * a.units / a.row_ctas);
  const int u1 = (int)((int64_t)(rc + 1) * a.units / a.row_ctas);
  const int r0 = u0 * a.unit_rows, R = (u1 - u0) * a.unit_rows;
  const int valid = min(R, a.N - r0);
  const int at0 = split * a.atoms / S, at1 = (split + 1) * a.atoms / S;
  const int nat = at1 - at0, kc = nat * 64, k0 = at0 * 64;
  const int K = a.K;
  const uint64_t tmo = a.timeout_ns;
  const uint32_t bar0 = sbase + (uint32_t)a.off_bar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + a.off_bar + RT_NBAR * 8);
  volatile int* drain_flag = abort_flag + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + a.off_bar + RT_NBAR * 8 + 8);
  const uint32_t bstage = (uint32_t)a.rmax * 128u;
  const bool tr = (a.debug_flags & 2) != 0;  // phase stamps (ddq_read_trace)

  if (tid == 0) {
    trace_stamp(tr, 0);
    ptx::mbar_init(bar(RT_BAR_W), 1);
    for (int i = 0; i < a.xs; ++i) {
      ptx::mbar_init(bar(RT_BAR_XF + i), 1);
      ptx::mbar_init(bar(RT_BAR_XE + i), 1);
    }
    for (int i = 0; i < a.bs; ++i) {
      ptx::mbar_init(bar(RT_BAR_BF + i), RT_CONV_THREADS / 32);
      ptx::mbar_init(bar(RT_BAR_BE + i), 1);
    }
    ptx::mbar_init(bar(RT_BAR_ACC), (uint32_t)(nat < RT_ISSUERS ? nat : RT_ISSUERS));
    for (int w = 0; w < RT_ISSUERS; ++w) ptx::mbar_init(bar(RT_BAR_DRAIN + w), 1);
    *abort_flag = 0;
    *drain_flag = 0;
    ptx::fence_mbar_init();
  }
  // TMEM before launch_dependents: a dependent kernel's CTA that shares the
  // SM then finds this CTA's columns taken, never the other way round
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), (uint32_t)a.ncols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_d = *tmem_holder;

  if (tid == 0) {
    // the weight slice (weights are never written by the kernel this one
    // depends on), then let the next kernel be scheduled
    ptx::mbar_arrive_expect_tx(bar(RT_BAR_W), (uint32_t)(valid * kc));
    if (S == 1) {
      rt_bulk_g2s(sbase, a.wq + (size_t)r0 * K, (uint32_t)(valid * K), bar(RT_BAR_W));
    } else {
      for (int r = 0; r < valid; ++r)
        rt_bulk_g2s(sbase + (uint32_t)(r * kc), a.wq + (size_t)(r0 + r) * K + k0, (uint32_t)kc,
                    bar(RT_BAR_W));
    }
    ptx::prefetch_tmap(&tm_x);
    trace_stamp(tr, 2);
    ptx::pdl_launch_dependents();
  }

  float* sc = reinterpret_cast<float*>(smem + a.off_sb);
  float* bi = sc + a.rmax;
  bool ok = true;
  if (warp == 0) {
    // ---------------------------------------------------- activation producer
    if (lane == 0) {
      ptx::pdl_wait();  // x comes from the previous kernel
      trace_stamp(tr, 3);
      int issued = 0;
      const int xs = a.xs;
      for (int i = 0; i < nat; ++i) {
        const int s = i % xs;
        if (i >= xs &&
            !ptx::mbar_wait(bar(RT_BAR_XE + s), (uint32_t)((i / xs) - 1) & 1u, tmo, abort_flag))
          break;
        ptx::mbar_arrive_expect_tx(bar(RT_BAR_XF + s), (uint32_t)RT_XSTAGE);
        ptx::tma_load_2d(sbase + (uint32_t)(a.off_x + s * RT_XSTAGE), &tm_x, k0 + i * 64, 0,
                         bar(RT_BAR_XF + s));
        ++issued;
      }
      trace_stamp(tr, 11);  // last activation load issued
      // every copy this CTA started has landed before it may exit
      for (int i = issued > xs ? issued - xs : 0; i < issued; ++i)
        ptx::mbar_wait(bar(RT_BAR_XF + i % xs), (uint32_t)(i / xs) & 1u, tmo, drain_flag);
      ptx::mbar_wait(bar(RT_BAR_W), 0u, tmo, drain_flag);
      trace_stamp(tr, 15);  // producer drained
    }
    __syncwarp();
  } else if (warp <= RT_ISSUERS) {
    // ---------------------------------------------------- MMA issuers
    // Issuing a tcgen05.mma costs its thread ~30 ns at these tile sizes
    // (measured), well above the tensor pipe's time for it, so three threads
    // issue: w takes atoms i = w, w + 3, ... into its own accumulator
    // (columns w * acc_stride), summed in order w = 0, 1, 2 by the epilogue.
    const int w = warp - 1;
    if (lane == 0 && w < nat) {
      ptx::pdl_wait();  // every wait below depends on the activations
      const uint32_t idesc = ptx::idesc_f16_f32(64, R);
      const uint32_t acc = tmem_d + (uint32_t)(w * a.acc_stride);
      for (int i = w; i < nat; i += RT_ISSUERS) {
        const int sb = i % a.bs, sx = i % a.xs;
        if (!ptx::mbar_wait(bar(RT_BAR_BF + sb), (uint32_t)(i / a.bs) & 1u, tmo, abort_flag) ||
            !ptx::mbar_wait(bar(RT_BAR_XF + sx), (uint32_t)(i / a.xs) & 1u, tmo, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (i == 0) trace_stamp(tr, 5);  // first atom of x and of fp16 weights ready
        if (i == nat / 2) trace_stamp(tr, 8);
        if (i == nat - 1) trace_stamp(tr, 9);
        const uint32_t xa = sbase + (uint32_t)(a.off_x + sx * RT_XSTAGE);
        const uint32_t ba = sbase + (uint32_t)a.off_b + (uint32_t)sb * bstage;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          ptx::mma_f16_ss(acc, ptx::smem_desc_sw128(xa + 32u * kk),
                          ptx::smem_desc_sw128(ba + 32u * kk), idesc, (i != w || kk) ? 1u : 0u);
        ptx::mma_commit(bar(RT_BAR_BE + sb));
        ptx::mma_commit(bar(RT_BAR_XE + sx));
      }
      if (w == 0) trace_stamp(tr, 4);  // issuer 0's last MMA issued
      if (ok && !(a.debug_flags & 16)) ptx::mma_commit(bar(RT_BAR_ACC));
      // this thread's MMAs are complete before TMEM or shared memory is reused
      ptx::mma_commit(bar(RT_BAR_DRAIN + w));
      ptx::mbar_wait(bar(RT_BAR_DRAIN + w), 0u, tmo, drain_flag);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------- converters
    const int ct = tid - 32 * (RT_ISSUERS + 1);
    for (int r = ct; r < R; r += RT_CONV_THREADS) {
      const int n = r0 + r;
      sc[r] = n < a.N ? a.scales[n] : 0.f;
      bi[r] = n < a.N ? rt_bias(a.bias, a.bias_dtype, n) : 0.f;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(RT_CONV_THREADS) : "memory");
    ok = ptx::mbar_wait(bar(RT_BAR_W), 0u, tmo, abort_flag);
    for (int i = 0; i < nat && ok; ++i) {
      const int sb = i % a.bs;
      if (i == a.bs) ptx::pdl_wait();  // later stages wait on MMAs, i.e. on x
      if (i >= a.bs &&
          !ptx::mbar_wait(bar(RT_BAR_BE + sb), (uint32_t)((i / a.bs) - 1) & 1u, tmo, abort_flag)) {
        ok = false;
        break;
      }
      // unit u: 16 e4m3 of row u / 4 (K 16 (u % 4) .. + 15 of atom i) -> two
      // 16-byte fp16 chunks 2 (u % 4) and 2 (u % 4) + 1 of the row's swizzled
      // 128 bytes (chunk c lands at c ^ (row mod 8)).  Rows >= valid convert
      // whatever the slice buffer holds: they only reach accumulator
      // columns that are never stored.
      const uint8_t* src = smem + i * 64;
      uint8_t* dst = smem + a.off_b + sb * bstage;
      for (int u = ct; u < R * 4; u += RT_CONV_THREADS) {
        const int r = u >> 2, c = u & 3, sw = r & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(src + r * kc + c * 16);
        uint4 lo, hi;
        e4m3x4_to_half2x2<true>(v.x, lo.x, lo.y);
        e4m3x4_to_half2x2<true>(v.y, lo.z, lo.w);
        e4m3x4_to_half2x2<true>(v.z, hi.x, hi.y);
        e4m3x4_to_half2x2<true>(v.w, hi.z, hi.w);
        uint8_t* drow = dst + (r >> 3) * 1024 + sw * 128;
        *reinterpret_cast<uint4*>(drow + (((2 * c) ^ sw) << 4)) = lo;
        *reinterpret_cast<uint4*>(drow + (((2 * c + 1) ^ sw) << 4)) = hi;
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(RT_BAR_BF + sb));
    }
    if (ct == 0) trace_stamp(tr, 10);  // this converter warp's last atom

    if (warp >= 4) {
      // ---------------------------------------------------- epilogue
      const int q = warp & 3;  // TMEM lane quarter this warp may read
      const int m = 16 * q + lane;
      const int ni = nat < RT_ISSUERS ? nat : RT_ISSUERS;  // accumulators written
      const bool got = ok && ptx::mbar_wait(bar(RT_BAR_ACC), 0u, tmo, abort_flag);
      if (ct == 0) trace_stamp(tr, 12);  // accumulators complete
      ptx::tc_fence_after();
      ptx::pdl_wait();  // y may be a buffer the previous kernel reads
      if (got) {
        const uint32_t tl = tmem_d + ((uint32_t)(32 * q) << 16);
        float* red = reinterpret_cast<float*>(smem + a.off_red);
        for (int c0 = 0; c0 < R; c0 += 32) {
          uint32_t v[32];
          __syncwarp();  // tcgen05.ld is warp-collective
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8)
            if (c0 + 8 * j8 < R) ptx::tmem_ld_32x32b_x8(tl + (uint32_t)(c0 + 8 * j8), v + 8 * j8);
          ptx::tmem_ld_wait();
          // the other issuers' accumulators, added in issuer order
          for (int w = 1; w < ni; ++w) {
            uint32_t u[32];
#pragma unroll
            for (int j8 = 0; j8 < 4; ++j8)
              if (c0 + 8 * j8 < R)
                ptx::tmem_ld_32x32b_x8(tl + (uint32_t)(w * a.acc_stride + c0 + 8 * j8), u + 8 * j8);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(u[j]));
          }
          if (c0 == 0 && ct == 0) trace_stamp(tr, 13);  // first chunk in registers
          if (lane < 16 && S > 1) {
            // fp32 partial of token row m (all 64; rows >= M hold zeros)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < R) red[m * a.rmax + c0 + j] = __uint_as_float(v[j]);
          }
          if (lane >= 16 || S > 1 || m >= a.M) continue;
          if constexpr (SWIGLU) {
            // columns c0 .. c0+15 gate, c0+16 .. c0+31 up (R is a multiple of 32)
            uint32_t o[8];
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              float z[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int jg = c0 + i + h, ju = jg + 16;
                const float g = __half2float(
                    __float2half_rn(fmaf(__uint_as_float(v[i + h]), sc[jg], bi[jg])));
                const float uu = __half2float(
                    __float2half_rn(fmaf(__uint_as_float(v[i + h + 16]), sc[ju], bi[ju])));
                z[h] = __fdividef(g, 1.0f + __expf(-g)) * uu;
              }
              o[i >> 1] = rt_pack(z[0], z[1]);
            }
            const int oc = (r0 + c0) >> 1;  // 16 output columns
            __half* yr = a.y + (size_t)m * a.out_n + oc;
            if (a.vec_y && oc + 16 <= a.out_n) {
              reinterpret_cast<uint4*>(yr)[0] = make_uint4(o[0], o[1], o[2], o[3]);
              reinterpret_cast<uint4*>(yr)[1] = make_uint4(o[4], o[5], o[6], o[7]);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (oc + i < a.out_n)
                  yr[i] = __ushort_as_half((unsigned short)(o[i >> 1] >> (16 * (i & 1))));
            }
          } else {
#pragma unroll
            for (int j8 = 0; j8 < 4; ++j8) {
              const int cb = c0 + 8 * j8;
              if (cb >= R) break;
              uint32_t o[4];
#pragma unroll
              for (int i = 0; i < 8; i += 2)
                o[i >> 1] = rt_pack(fmaf(__uint_as_float(v[8 * j8 + i]), sc[cb + i], bi[cb + i]),
                                    fmaf(__uint_as_float(v[8 * j8 + i + 1]), sc[cb + i + 1],
                                         bi[cb + i + 1]));
              const int n = r0 + cb;
              __half* yr = a.y + (size_t)m * a.N + n;
              if (a.vec_y && n + 8 <= a.N) {
                *reinterpret_cast<uint4*>(yr) = make_uint4(o[0], o[1], o[2], o[3]);
              } else {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (n + i < a.N)
                    yr[i] = __ushort_as_half((unsigned short)(o[i >> 1] >> (16 * (i & 1))));
              }
            }
          }
        }
      }
    }
    if (ct == 0) trace_stamp(tr, 14);  // epilogue stores issued
    __syncwarp();
  }

  if (S > 1) {
    // ---------------------------------------------------- split-K reduction
    // all partials parked; every CTA takes outputs [split E / S, (split+1) E / S)
    // of the M x R tile and sums them over the cluster in split order
    ptx::tc_fence_before();
    ptx::cluster_sync();
    bool any_abort = false;
    const uint32_t abort_addr = ptx::smem_u32(const_cast<int*>(abort_flag));
    for (int s = 0; s < S; ++s) any_abort |= ptx::ld_dsmem_u32(ptx::mapa_shared(abort_addr, s)) != 0;
    if (!any_abort) {
      ptx::pdl_wait();
      // groups of 4 columns; every split's 16 bytes in flight, then the sum
      // in split order
      const int R4 = R >> 2, E = a.M * R4;
      const int e0 = (int)((int64_t)split * E / S), e1 = (int)((int64_t)(split + 1) * E / S);
      const uint32_t red0 = sbase + (uint32_t)a.off_red;
      for (int e = e0 + tid; e < e1; e += RT_THREADS) {
        const int m = e / R4, j = (e - m * R4) * 4;
        const int n = r0 + j;
        if (n >= a.N) continue;
        const uint32_t off = red0 + (uint32_t)((m * a.rmax + j) * 4);
        float4 v[8];
#pragma unroll
        for (int s = 0; s < 8; ++s)
          if (s < S) v[s] = ptx::ld_dsmem_f4(ptx::mapa_shared(off, (uint32_t)s));
        float4 acc = v[0];
#pragma unroll
        for (int s = 1; s < 8; ++s) {
          if (s < S) {
            acc.x += v[s].x;
            acc.y += v[s].y;
            acc.z += v[s].z;
            acc.w += v[s].w;
          }
        }
        const uint32_t lo = rt_pack(fmaf(acc.x, sc[j], bi[j]), fmaf(acc.y, sc[j + 1], bi[j + 1]));
        const uint32_t hi =
            rt_pack(fmaf(acc.z, sc[j + 2], bi[j + 2]), fmaf(acc.w, sc[j + 3], bi[j + 3]));
        __half* yr = a.y + (size_t)m * a.N + n;
        if (a.vec_y && n + 4 <= a.N) {
          *reinterpret_cast<uint2*>(yr) = make_uint2(lo, hi);
        } else {
          const uint32_t w[2] = {lo, hi};
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (n + i < a.N) yr[i] = __ushort_as_half((unsigned short)(w[i >> 1] >> (16 * (i & 1))));
        }
      }
    }
    ptx::cluster_sync();  // no CTA leaves while another still reads its partials
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    trace_stamp(tr, 6);
    trace_stamp(tr, 7);
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_d, (uint32_t)a.ncols);
  }
  if (tid == 0 && *abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
}

}  // namespace

// ============================================================================
// Host side
// ============================================================================
namespace {

struct RtPlan {
  bool ok = false;
  int unit_rows = 8, units = 0, row_ctas = 0, splits = 1, atoms = 0, rmax = 0, ncols = 0;
  int xs = 3, bs = 2, acc_stride = 32;
  int off_b = 0, off_x = 0, off_sb = 0, off_red = 0, off_bar = 0, smem = 0;
};

int env_int(const char* name, int dflt) {
  const char* e = std::getenv(name);
  return e && *e ? std::atoi(e) : dflt;
}

// Token range the kernel takes (17..64 by default; DDQ_RT_MIN_M / DDQ_RT_MAX_M
// move it, DDQ_RT_MAX_M=0 switches the kernel off), read once.
int rt_min_m() {
  static const int v = env_int("DDQ_RT_MIN_M", 17);
  return v;
}
int rt_max_m() {
  static const int v = env_int("DDQ_RT_MAX_M", 64);
  return v < 64 ? v : 64;
}

RtPlan rt_layout(RtPlan p, int64_t kcmax) {
  const int64_t w_bytes = ((int64_t)p.rmax * kcmax + 1023) & ~1023ll;
  const int64_t b_bytes = (int64_t)p.bs * p.rmax * 128;
  const int64_t x_bytes = (int64_t)p.xs * RT_XSTAGE;
  const int64_t sb_bytes = (int64_t)2 * p.rmax * 4;
  const int64_t red_bytes = p.splits > 1 ? (int64_t)64 * p.rmax * 4 : 0;
  int64_t off = w_bytes;
  p.off_b = (int)off;
  off += b_bytes;
  p.off_x = (int)off;
  off += x_bytes;
  p.off_sb = (int)off;
  off += sb_bytes;
  p.off_red = 0;  // partials reuse the (then dead) weight slice
  if (red_bytes > w_bytes) {
    off = (off + 15) & ~15ll;
    p.off_red = (int)off;
    off += red_bytes;
  }
  off = (off + 15) & ~15ll;
  p.off_bar = (int)off;
  off += RT_BAR_BYTES;
  p.smem = (int)(off + 1024);  // slack for the 1024-byte alignment of the base
  return p;
}

// Rows: units of 8 (32 with SwiGLU, keeping each gate/up pair in one CTA)
// spread evenly over the CTAs of a split.  K: split over a cluster when the
// activation stream would pass 20 atoms per CTA (the MMAs read every atom of
// x once per CTA).  CTAs: one per SM and split while the shared memory of a
// CTA fits twice on an SM; where it does not, more (smaller) CTAs.
RtPlan rt_plan(int64_t M, int64_t N, int64_t K, int sms, bool swiglu) {
  RtPlan p;
  if (sms <= 0 || M < rt_min_m() || M > rt_max_m() || N <= 0 || K <= 0 || K % 64 != 0)
    return p;
  if (N > 0x7fffffff || K > 0x7fffffff) return p;
  p.unit_rows = swiglu ? 32 : 8;
  if (swiglu && N % 32 != 0) return p;
  p.atoms = (int)(K / 64);
  p.splits = (p.atoms + 19) / 20;
  if (p.splits > 8) return p;  // portable cluster size
  if (swiglu && p.splits > 1) return p;
  const int64_t units = (N + p.unit_rows - 1) / p.unit_rows;
  p.units = (int)units;
  const int64_t kcmax = (int64_t)((p.atoms + p.splits - 1) / p.splits) * 64;
  int64_t g = sms / p.splits;
  if (g < 1) g = 1;
  if (g > units) g = units;
  // Rings.  Refilling a stage of either ring waits for an MMA to complete;
  // an activation stage then waits for an L2 fetch as well (about 1 us from
  // issue to landing), a weight stage only for its conversion.  So the
  // activation ring gets its stages first - every atom of the CTA's K range
  // where the budget allows, at most 16 - and the weight ring what is left,
  // at most every atom; at least min(atoms, 8) and min(atoms, 4) stages.
  // Budget: half an SM where both rings fit in it (the next GEMM's CTA can
  // then be resident and fetch its slice meanwhile), else the whole 227 KB;
  // one CTA of this kernel per SM and split either way.  DDQ_RT_XS caps the
  // activation ring; DDQ_RT_PAIR=0 / 2 force the whole / the half-SM budget.
  if (g > sms / p.splits || (int64_t)((units + g - 1) / g) * p.unit_rows > RT_MAX_N) return p;
  p.row_ctas = (int)g;
  p.rmax = (int)((units + g - 1) / g) * p.unit_rows;
  const int nat_max = (p.atoms + p.splits - 1) / p.splits;
  int xs_cap = nat_max < RT_XS_MAX ? nat_max : RT_XS_MAX;
  static const int env_xs = env_int("DDQ_RT_XS", 0);
  if (env_xs > 0 && env_xs < xs_cap) xs_cap = env_xs;
  const int bs_cap = nat_max < RT_BS_MAX ? nat_max : RT_BS_MAX;
  const int xs_lo = xs_cap < 8 ? xs_cap : 8, bs_lo = bs_cap < 4 ? bs_cap : 4;
  static const int pair_mode = env_int("DDQ_RT_PAIR", 1);
  bool fits = false;
  for (int pass = 0; pass < 2 && !fits; ++pass) {
    const bool pair = pass == 0 ? pair_mode != 0 : pair_mode == 2;
    const int budget = pair ? RT_SMEM_PAIR : RT_SMEM_MAX;
    for (int xs = xs_cap; xs >= xs_lo && !fits; --xs) {
      for (int bs = bs_cap; bs >= bs_lo && !fits; --bs) {
        p.xs = xs;
        p.bs = bs;
        p = rt_layout(p, kcmax);
        fits = p.smem <= budget;
      }
    }
  }
  if (!fits) return p;
  // one accumulator per MMA issuer, 32-column aligned
  p.acc_stride = (p.rmax + 31) & ~31;
  const int nacc = nat_max < RT_ISSUERS ? nat_max : RT_ISSUERS;
  p.ncols = 32;
  while (p.ncols < nacc * p.acc_stride) p.ncols *= 2;
  // CTAs of this kernel that share an SM must never ask for more than the
  // SM's 512 TMEM columns between them (a CTA of a cluster that waited in
  // tcgen05.alloc for its neighbour could hold up the cluster barrier): at
  // most 512 / ncols of them may fit in shared memory
  const int per_sm = 512 / p.ncols;
  const int min_smem = kSmemPerSm / (per_sm + 1) - kSmemReservedPerCta + 1;
  if (p.smem < min_smem) p.smem = min_smem;
  p.ok = true;
  return p;
}

PFN_cuTensorMapEncodeTiled_v12000 rt_encoder() {
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

// x [M][K] fp16 as a 2-D tensor {K, M}; a box {64, 64} lands as one 64-token
// activation atom, token rows >= M read as zero.
int rt_tmap_x(CUtensorMap* m, const void* x, uint64_t K, uint64_t M) {
  auto enc = rt_encoder();
  if (!enc) return DDQ_ERR_DEVICE;
  cuuint64_t dims[2] = {K, M};
  cuuint64_t strides[1] = {K * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDQ_OK : DDQ_ERR_ALIGNMENT;
}

template <bool SWIGLU>
int launch_rt_t(const RtPlan& p, const CUtensorMap& tm_x, const RtArgs& a, cudaStream_t s) {
  static SmemAttrOnce attr;
  const int ast =
      ensure_smem_attr(attr, current_device(), w8a16_rt_kernel<SWIGLU>, RT_SMEM_MAX);
  if (ast) return ast;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.splits, (unsigned)p.row_ctas, 1);
  cfg.blockDim = dim3(RT_THREADS);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[na].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++na;
  if (p.splits > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = (unsigned)p.splits;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, w8a16_rt_kernel<SWIGLU>, tm_x, a) != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace

bool rt_eligible(int64_t M, int64_t N, int64_t K, int sms, bool swiglu) {
  return rt_plan(M, N, K, sms, swiglu).ok;
}

int launch_rt(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, bool swiglu,
              unsigned long long timeout_ns, cudaStream_t s, int debug_flags) {
  const int sms = device_sm_count(current_device());
  if (sms <= 0) return DDQ_ERR_DEVICE;
  if (!aligned16(x) || !aligned16(wq)) return DDQ_ERR_ALIGNMENT;
  const RtPlan p = rt_plan(M, N, K, sms, swiglu);
  if (!p.ok) return DDQ_ERR_SHAPE;
  CUtensorMap tm_x;
  const int st = rt_tmap_x(&tm_x, x, (uint64_t)K, (uint64_t)M);
  if (st) return st;
  RtArgs a{};
  a.wq = wq;
  a.scales = scales;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.M = M;
  a.N = N;
  a.K = K;
  a.out_n = swiglu ? N / 2 : N;
  a.units = p.units;
  a.unit_rows = p.unit_rows;
  a.row_ctas = p.row_ctas;
  a.splits = p.splits;
  a.atoms = p.atoms;
  a.rmax = p.rmax;
  a.xs = p.xs;
  a.bs = p.bs;
  a.vec_y = (a.out_n % 8 == 0) && aligned16(y);
  a.ncols = p.ncols;
  a.acc_stride = p.acc_stride;
  a.off_b = p.off_b;
  a.off_x = p.off_x;
  a.off_sb = p.off_sb;
  a.off_red = p.off_red;
  a.off_bar = p.off_bar;
  a.timeout_ns = timeout_ns;
  a.debug_flags = debug_flags;
  return swiglu ? launch_rt_t<true>(p, tm_x, a, s) : launch_rt_t<false>(p, tm_x, a, s);
}

}  // namespace ddq
