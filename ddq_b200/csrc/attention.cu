// attention.cu - one decode step of grouped-query attention with the rotary
// embedding and the KV-cache write fused in (replaces the reference's RoPE
// kernel, the cache copy and the attention call of a decode step:
// RoPe_d.cu:12-68, engine.py:126-130 and 225-251).
//
// For each sequence b and key/value head g (one CTA):
//   q_h  = fp16(rope(q_h, pos))   for the G query heads h of group g
//   k    = fp16(rope(k_g, pos)),  v = v_g        -> cache[b, g, pos, :]
//   o_h  = softmax_j( q_h . K[b, g, j, :] * scale ) V[b, g, j, :],  j = 0..pos
// Rotate-half RoPE in fp32 with the caller's cos/sin row for this position,
// rounded to fp16 as the unfused path rounds it; scores and softmax in fp32;
// o rounded to fp16.  The position is read on the device, so a captured CUDA
// graph replays it for every step.
//
// Two kernels:
//   decode_attention_mma_kernel<G>  64-wide heads (the Qwen2 shapes): K and V
//       chunks stream into shared memory through TMA, q K^T and P V run on
//       the tensor cores (mma.sync, fp16 operands, fp32 accumulation).
//   decode_attention_kernel<128>    128-wide heads: per-lane loads, the
//       arithmetic on the CUDA cores (lane = position for the scores, lane =
//       D / 32 head dimensions for the weighted sum).
// Both split the positions between the warps with an online softmax per query
// head and merge the warps' partial results in shared memory.
#include <cudaTypedefs.h>

#include <cfloat>
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "sm100_ptx.cuh"

namespace ddq {

constexpr int AT_GMAX = 8;  // query heads per key/value head, at most
// warps per CTA: 16 for 64-wide heads (one 32-position tile per warp for
// contexts up to 512), 8 for 128-wide heads (register budget)
__host__ __device__ constexpr int at_warps(int d) { return d == 64 ? 16 : 8; }

struct AtArgs {
  const __half* qkv;     // [B, (Hq + 2 Hkv) * D] row stride qkv_stride
  int64_t qkv_stride;
  __half* kc;            // [B, Hkv, cap, D] with batch stride cache_bstride
  __half* vc;
  int64_t cache_bstride;
  int cap;
  const float* cos;      // [D]
  const float* sin;      // [D]
  const int64_t* pos;    // device scalar
  __half* out;           // [B, Hq * D] row stride out_stride
  int64_t out_stride;
  int Hq, Hkv;
  float scale;
  int trace;             // debug flag bit 1: phase stamps (see ddq_read_trace)
  uint8_t* planes;       // split output: three e4m3 planes [3][B][Hq * D] (or null)
  float* xscale;         // and the token scales 2^-e [B]
  int kv_ready;          // pos and the cache rows before it are final before the
                         // previous kernel starts: load them ahead of the grid wait
};

template <int D>
__global__ void __launch_bounds__(at_warps(D) * 32, 1) decode_attention_kernel(const AtArgs a) {
  constexpr int NW = at_warps(D);
  constexpr int DH = D / 2;
  constexpr int DPL = D / 32;  // head dimensions per lane in the weighted sum
  const int b = blockIdx.x / a.Hkv, g = blockIdx.x % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ __align__(16) float q_s[AT_GMAX][D];
  __shared__ float m_s[NW][AT_GMAX], l_s[NW][AT_GMAX];
  __shared__ float acc_s[NW][AT_GMAX][D];

  ptx::pdl_wait();  // qkv comes from the previous kernel
  const int64_t p = *a.pos;
  if (p < 0 || p >= a.cap) return;  // the host checks the range; nothing to do otherwise
  const int L = (int)p + 1;
  const __half* row = a.qkv + (size_t)b * a.qkv_stride;
  const size_t head = (size_t)a.cap * D;
  __half* kc = a.kc + (size_t)b * a.cache_bstride + (size_t)g * head;
  __half* vc = a.vc + (size_t)b * a.cache_bstride + (size_t)g * head;

  // ---- rotary embedding of the G query heads and the new key; cache write
  for (int i = threadIdx.x; i < (G + 1) * DH; i += blockDim.x) {
    const int h = i / DH, d = i % DH;
    const __half* src = h < G ? row + (size_t)(g * G + h) * D
                              : row + (size_t)(a.Hq + g) * D;
    const float x1 = __half2float(src[d]), x2 = __half2float(src[d + DH]);
    // x * cos + rotate_half(x) * sin, each product rounded as torch rounds it
    const float y1 = __half2float(
        __float2half_rn(__fadd_rn(__fmul_rn(x1, a.cos[d]), __fmul_rn(-x2, a.sin[d]))));
    const float y2 = __half2float(
        __float2half_rn(__fadd_rn(__fmul_rn(x2, a.cos[d + DH]), __fmul_rn(x1, a.sin[d + DH]))));
    if (h < G) {
      q_s[h][d] = y1;
      q_s[h][d + DH] = y2;
    } else {
      kc[(size_t)p * D + d] = __float2half_rn(y1);
      kc[(size_t)p * D + d + DH] = __float2half_rn(y2);
    }
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    vc[(size_t)p * D + d] = row[(size_t)(a.Hq + a.Hkv + g) * D + d];
  __syncthreads();  // the cache row and q_s are visible to the whole CTA
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  // ---- scores and the weighted sum over this warp's 32-position tiles
  float m[AT_GMAX], l[AT_GMAX], acc[AT_GMAX][DPL];
#pragma unroll
  for (int h = 0; h < AT_GMAX; ++h) {
    m[h] = -FLT_MAX;
    l[h] = 0.f;
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc[h][t] = 0.f;
  }
  for (int t0 = warp * 32; t0 < L; t0 += NW * 32) {
    const int j = t0 + lane;
    const bool ok = j < L;
    float s[AT_GMAX];
#pragma unroll
    for (int h = 0; h < AT_GMAX; ++h) s[h] = 0.f;
    if (ok) {
      // the whole K row in flight at once, then G dot products against q
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * D);
      uint4 kv[D / 8];
#pragma unroll
      for (int c = 0; c < D / 8; ++c) kv[c] = kr[c];
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const __half2* hv = reinterpret_cast<const __half2*>(&kv[c]);
        float kf[8];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 f = __half22float2(hv[t]);
          kf[2 * t] = f.x;
          kf[2 * t + 1] = f.y;
        }
#pragma unroll
        for (int h = 0; h < AT_GMAX; ++h) {
          if (h < G) {
            const float4 qa = *reinterpret_cast<const float4*>(&q_s[h][c * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&q_s[h][c * 8 + 4]);
            float acc_s8 = s[h];
            acc_s8 = fmaf(qa.x, kf[0], acc_s8);
            acc_s8 = fmaf(qa.y, kf[1], acc_s8);
            acc_s8 = fmaf(qa.z, kf[2], acc_s8);
            acc_s8 = fmaf(qa.w, kf[3], acc_s8);
            acc_s8 = fmaf(qb.x, kf[4], acc_s8);
            acc_s8 = fmaf(qb.y, kf[5], acc_s8);
            acc_s8 = fmaf(qb.z, kf[6], acc_s8);
            acc_s8 = fmaf(qb.w, kf[7], acc_s8);
            s[h] = acc_s8;
          }
        }
      }
    }
    float pr[AT_GMAX];
#pragma unroll
    for (int h = 0; h < AT_GMAX; ++h) {
      pr[h] = 0.f;
      if (h >= G) continue;
      const float sv = ok ? s[h] * a.scale : -FLT_MAX;
      float tm = sv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
      const float mn = fmaxf(m[h], tm);
      const float corr = __expf(m[h] - mn);
      pr[h] = ok ? __expf(sv - mn) : 0.f;
      float ps = pr[h];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[h] = l[h] * corr + ps;
      m[h] = mn;
#pragma unroll
      for (int t = 0; t < DPL; ++t) acc[h][t] *= corr;
    }
    // weighted sum of V: 16 rows at a time, all their loads in flight first;
    // rows past the last position read as zero (their weights are zero too)
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += 16) {
      if (t0 + j0 >= L) break;
      float vf[16][DPL];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int pj = t0 + j0 + jj;
        const __half* vr = vc + (size_t)pj * D + lane * DPL;
        if (pj < L) {
          if constexpr (DPL == 2) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vr));
            vf[jj][0] = f.x;
            vf[jj][1] = f.y;
          } else {
            const uint2 u = *reinterpret_cast<const uint2*>(vr);
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            vf[jj][0] = f0.x;
            vf[jj][1] = f0.y;
            vf[jj][2] = f1.x;
            vf[jj][3] = f1.y;
          }
        } else {
#pragma unroll
          for (int t = 0; t < DPL; ++t) vf[jj][t] = 0.f;
        }
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
#pragma unroll
        for (int h = 0; h < AT_GMAX; ++h) {
          if (h >= G) continue;
          const float pj = __shfl_sync(0xffffffffu, pr[h], j0 + jj);
#pragma unroll
          for (int t = 0; t < DPL; ++t) acc[h][t] = fmaf(pj, vf[jj][t], acc[h][t]);
        }
      }
    }
  }

  // ---- merge the warps' partial softmax sums
#pragma unroll
  for (int h = 0; h < AT_GMAX; ++h) {
    if (h >= G) continue;
    if (lane == 0) {
      m_s[warp][h] = m[h];
      l_s[warp][h] = l[h];
    }
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc_s[warp][h][lane * DPL + t] = acc[h][t];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float mx = -FLT_MAX;
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, m_s[w][h]);
    float den = 0.f, num = 0.f;
    for (int w = 0; w < NW; ++w) {
      const float c = l_s[w][h] > 0.f ? __expf(m_s[w][h] - mx) : 0.f;
      den = fmaf(l_s[w][h], c, den);
      num = fmaf(acc_s[w][h][d], c, num);
    }
    a.out[(size_t)b * a.out_stride + (size_t)(g * G + h) * D + d] = __float2half_rn(num / den);
  }
}

// ----------------------------------------------------------------------------
// 64-wide heads: K and V stream into shared memory through TMA; both products
// run on the tensor cores.
// ----------------------------------------------------------------------------
// The positions are cut into 32-row chunks (4 KB of K + 4 KB of V, 128-byte
// swizzle, which keeps every 8x8 matrix load below free of bank conflicts).
// Warp w takes chunks w, w + 8, w + 16, ... through a ring of AM_DEPTH slots
// of its own, so up to 8 x AM_DEPTH chunks (768 positions) of a sequence are
// in flight at once, and refills a slot as soon as it has used it.  Before
// the grid dependency resolves, the CTA asks L2 for rows 0..pos of its K and
// V (a prefetch only: what the kernel uses is read after the wait).
//
// Per chunk and warp (mma.sync m16n8k16, fp16 operands, fp32 accumulation),
// with the G <= 8 query heads on MMA rows 0..7:
//   S[h, j]  = q_h . K[j]            16 MMAs (4 tiles of 8 positions x 4 K steps)
//   online softmax of S * scale per head, fp32, in registers (quad shuffles)
//   O[h, :] += P[h, :] V             16 MMAs (8 tiles of 8 dims x 2 K steps)
// q (the RoPE output, rounded to fp16 as the unfused path rounds it), K and
// V are fp16, so every product is exact.  Each weight p is carried as
// p_hi = fp16(p) on MMA row h and p_lo = fp16(p - p_hi) on row h + 8 of the
// same fragment: about 22 bits of p reach the weighted sum at no extra MMA
// (O = rows 0..7 + rows 8..15).  Rows past the last position are masked in S
// and zeroed in the V tile before use (the cache there may hold anything,
// and 0 x NaN is NaN).
constexpr int AM_NW = 8;          // warps
constexpr int AM_DEPTH = 3;       // ring slots per warp
constexpr int AM_ROWS = 32;       // positions per chunk
constexpr int AM_CHUNK = AM_ROWS * 64 * 2;  // bytes of K (and of V) per chunk

struct AmSmem {
  uint8_t ring[AM_NW * AM_DEPTH][2][AM_CHUNK];  // [slot][K | V]
  float acc[AM_NW][AT_GMAX][64];
  __half q[AT_GMAX][64];
  __align__(16) __half knew[64];  // the new cache row (patched into its chunk's tile)
  __align__(16) __half vnew[64];
  float m[AM_NW][AT_GMAX], l[AM_NW][AT_GMAX];
  float amax_w[AM_NW];   // split output: each head's |o| maximum
  float amax_r[8];       // and each CTA's of the cluster (one per KV head)
  unsigned long long full[AM_NW * AM_DEPTH];
  unsigned long long bar_amax;  // the other CTAs' maxima have arrived
  int abort_flag;
};

// byte offset of 16-byte chunk j of row r in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t at2_swz(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

__device__ __forceinline__ void am_ldsm(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void am_ldsm_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// d += A (16 x 16, row-major fragment a0..a3) * B (16 x 8, column fragment b0, b1)
__device__ __forceinline__ void am_mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t am_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// SPLIT: instead of (or besides) fp16 o, emit the o projection's B operand:
// the three e4m3 planes of the token's o row under a power-of-two scale, as
// the decode GEMM's split pre-pass would make them from fp16 o.  The row of a
// token spans its Hkv CTAs, launched as one cluster: each pushes its |o|
// maximum to the others (4 bytes into their shared memory, counted on their
// barrier) and splits its own heads.
template <int G, bool SPLIT>
__global__ void __launch_bounds__(AM_NW * 32, 1)
    decode_attention_mma_kernel(const __grid_constant__ CUtensorMap tm_k,
                                const __grid_constant__ CUtensorMap tm_v, const AtArgs a,
                                unsigned long long timeout_ns) {
  constexpr int D = 64, DH = 32;
  static_assert(G >= 1 && G <= 8, "query heads per group");
  extern __shared__ uint8_t am_raw[];
  AmSmem& sm = *reinterpret_cast<AmSmem*>((reinterpret_cast<uintptr_t>(am_raw) + 1023) &
                                          ~static_cast<uintptr_t>(1023));
  const int b = blockIdx.x / a.Hkv, g = blockIdx.x % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const bool tr = a.trace != 0;
  if (threadIdx.x == 0) trace_stamp(tr, 0);
  __half* kc = a.kc + (size_t)b * a.cache_bstride + (size_t)g * a.cap * D;
  __half* vc = a.vc + (size_t)b * a.cache_bstride + (size_t)g * a.cap * D;
  if (threadIdx.x == 0) {
    for (int s = 0; s < AM_NW * AM_DEPTH; ++s) ptx::mbar_init(ptx::smem_u32(&sm.full[s]), 1);
    if (SPLIT) {
      ptx::mbar_init(ptx::smem_u32(&sm.bar_amax), 1);
      ptx::mbar_arrive_expect_tx(ptx::smem_u32(&sm.bar_amax), (uint32_t)(4 * (a.Hkv - 1)));
    }
    sm.abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
  } else if (threadIdx.x == 32 && !a.kv_ready) {
    // L2 prefetch of rows 0..pos while the previous kernel finishes; the
    // position read here may be stale, which only makes the hint less useful
    const int64_t ph = *a.pos;
    if (ph >= 0 && ph < a.cap) {
      const uint32_t bytes = (uint32_t)(ph + 1) * (uint32_t)(D * 2);
      for (uint32_t off = 0; off < bytes; off += 32768u) {
        const uint32_t n = bytes - off < 32768u ? bytes - off : 32768u;
        ptx::bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(kc) + off, n);
        ptx::bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(vc) + off, n);
      }
    }
  }
  const uint32_t ring0 = ptx::smem_u32(&sm.ring[0][0][0]);
  auto issue = [&](int c) {  // chunk c into its slot of this warp's ring
    const int s = warp * AM_DEPTH + (c / AM_NW) % AM_DEPTH;
    const uint32_t full = ptx::smem_u32(&sm.full[s]);
    const uint32_t dst = ring0 + (uint32_t)(s * 2 * AM_CHUNK);
    ptx::mbar_arrive_expect_tx(full, 2u * AM_CHUNK);
    ptx::tma_load_4d(dst, &tm_k, 0, c * AM_ROWS, g, b, full);
    ptx::tma_load_4d(dst + AM_CHUNK, &tm_v, 0, c * AM_ROWS, g, b, full);
  };
  // With kv_ready the position and every cache row this step reads (except
  // the new one, patched in shared memory below) were final before the
  // previous kernel started: the first ring of chunks streams in while that
  // kernel still runs.
  int64_t p_early = -1;
  bool early = false;
  if (a.kv_ready) {
    __syncthreads();  // barriers initialised
    p_early = *a.pos;
    if (p_early >= 0 && p_early < a.cap) {
      early = true;
      const int n0 = ((int)p_early + AM_ROWS) / AM_ROWS;  // chunks of rows 0..pos
      if (lane == 0)
        for (int i = 0; i < AM_DEPTH; ++i) {
          const int c = warp + i * AM_NW;
          if (c < n0) issue(c);
        }
    }
  }
  ptx::pdl_wait();  // qkv comes from the previous kernel; earlier cache rows are complete
  if (threadIdx.x == 0) trace_stamp(tr, 1);
  // one memory round trip: the position, this group's q / k / v values and
  // the rotary rows are all requested before any of them is used
  const __half* row = a.qkv + (size_t)b * a.qkv_stride;
  constexpr int NT = AM_NW * 32;
  constexpr int NRI = ((G + 1) * DH + NT - 1) / NT;  // rotary pairs per thread
  float x1[NRI], x2[NRI], c1[NRI], s1[NRI], c2[NRI], s2[NRI];
  const int64_t p = a.kv_ready ? p_early : *a.pos;
#pragma unroll
  for (int r = 0; r < NRI; ++r) {
    const int i = threadIdx.x + r * NT;
    if (i < (G + 1) * DH) {
      const int h = i / DH, d = i % DH;
      const __half* src = h < G ? row + (size_t)(g * G + h) * D : row + (size_t)(a.Hq + g) * D;
      x1[r] = __half2float(src[d]);
      x2[r] = __half2float(src[d + DH]);
      c1[r] = a.cos[d];
      s1[r] = a.sin[d];
      c2[r] = a.cos[d + DH];
      s2[r] = a.sin[d + DH];
    }
  }
  const __half vnew = threadIdx.x < D ? row[(size_t)(a.Hq + a.Hkv + g) * D + threadIdx.x]
                                      : __float2half_rn(0.f);
  if (p < 0 || p >= a.cap) return;  // the host checks the range; nothing to do otherwise
  const int L = (int)p + 1;
  const int nchunks = (L + AM_ROWS - 1) / AM_ROWS;
  const int last = nchunks - 1;  // the chunk that holds the new row
  __syncthreads();  // barriers initialised
  // split output: the cluster's barriers are ready before any CTA pushes
  // (the matching wait comes after the merge)
  if (SPLIT) ptx::cluster_arrive_relaxed();

  // every chunk can be requested now: the new row is not read back from the
  // cache (its stale copy in the last chunk's tile is overwritten in shared
  // memory), so the copies overlap the rotary embedding below
  if (lane == 0 && !early)
    for (int i = 0; i < AM_DEPTH; ++i) {
      const int c = warp + i * AM_NW;
      if (c < nchunks) issue(c);
    }

  // ---- rotary embedding of the G query heads and the new key; cache write
#pragma unroll
  for (int r = 0; r < NRI; ++r) {
    const int i = threadIdx.x + r * NT;
    if (i < (G + 1) * DH) {
      const int h = i / DH, d = i % DH;
      // x * cos + rotate_half(x) * sin, each product rounded as torch rounds it
      const __half y1 = __float2half_rn(__fadd_rn(__fmul_rn(x1[r], c1[r]), __fmul_rn(-x2[r], s1[r])));
      const __half y2 = __float2half_rn(__fadd_rn(__fmul_rn(x2[r], c2[r]), __fmul_rn(x1[r], s2[r])));
      if (h < G) {
        sm.q[h][d] = y1;
        sm.q[h][d + DH] = y2;
      } else {
        kc[(size_t)p * D + d] = y1;
        kc[(size_t)p * D + d + DH] = y2;
        sm.knew[d] = y1;
        sm.knew[d + DH] = y2;
      }
    }
  }
  for (int i = threadIdx.x; i < (AT_GMAX - G) * D; i += blockDim.x)
    sm.q[G + i / D][i % D] = __float2half_rn(0.f);
  if (threadIdx.x < D) {
    vc[(size_t)p * D + threadIdx.x] = vnew;
    sm.vnew[threadIdx.x] = vnew;
  }
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(tr, 2);
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  // q fragments (rows 0..7 = heads; rows 8..15 of the A operand are zero)
  uint32_t qa[4][2];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    qa[kk][0] = *reinterpret_cast<const uint32_t*>(&sm.q[gid][16 * kk + 2 * tig]);
    qa[kk][1] = *reinterpret_cast<const uint32_t*>(&sm.q[gid][16 * kk + 8 + 2 * tig]);
  }
  float m_r = -FLT_MAX, l_r = 0.f;  // running max and sum of head gid
  float o[8][4];                    // O tiles: rows gid (p_hi part), gid + 8 (p_lo part)
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;

  int it = 0;
  for (int c = warp; c < nchunks; c += AM_NW, ++it) {
    const int s = warp * AM_DEPTH + it % AM_DEPTH;
    if (!ptx::mbar_wait(ptx::smem_u32(&sm.full[s]), (uint32_t)((it / AM_DEPTH) & 1), timeout_ns,
                        &sm.abort_flag))
      break;
    if (threadIdx.x == 0 && it == 0) trace_stamp(tr, 3);
    const uint32_t ks = ring0 + (uint32_t)(s * 2 * AM_CHUNK), vs = ks + AM_CHUNK;
    const int jn = min(AM_ROWS, L - c * AM_ROWS);  // positions of this chunk in use
    if (c == last) {
      // the new row (position jn - 1 of this chunk) from shared memory; the
      // rows after it are zeroed in the V tile
      uint8_t* krow = &sm.ring[s][0][0];
      uint8_t* vrow = &sm.ring[s][1][0];
      const int rp = jn - 1;
      if (lane < 16) {
        const int j = lane & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(lane < 8 ? &sm.knew[8 * j] : &sm.vnew[8 * j]);
        *reinterpret_cast<uint4*>((lane < 8 ? krow : vrow) + at2_swz(rp, j)) = v;
      }
      for (int idx = lane; idx < (AM_ROWS - jn) * 8; idx += 32)
        *reinterpret_cast<uint4*>(vrow + (jn + idx / 8) * 128 + (idx % 8) * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
    }
    // S = Q K^T: tile nt holds positions 8 nt + 2 tig (+1) of head gid
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) {
        uint32_t r[4];
        am_ldsm(ks + at2_swz(8 * nt + (lane & 7), 4 * kh + (lane >> 3)), r);
        am_mma(sc[nt], qa[2 * kh][0], 0u, qa[2 * kh][1], 0u, r[0], r[1]);
        am_mma(sc[nt], qa[2 * kh + 1][0], 0u, qa[2 * kh + 1][1], 0u, r[2], r[3]);
      }
    }
    // online softmax of head gid over the chunk (the quad of lanes shares the row)
    float sv[4][2];
    float mx = -FLT_MAX;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sv[nt][e] = 8 * nt + 2 * tig + e < jn ? sc[nt][e] * a.scale : -FLT_MAX;
        mx = fmaxf(mx, sv[nt][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m_r, mx);
    const float corr = __expf(m_r - mn);
    float ps = 0.f;
    uint32_t phi[4], plo[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const float p0 = 8 * nt + 2 * tig < jn ? __expf(sv[nt][0] - mn) : 0.f;
      const float p1 = 8 * nt + 2 * tig + 1 < jn ? __expf(sv[nt][1] - mn) : 0.f;
      ps += p0 + p1;
      const __half2 hi = __floats2half2_rn(p0, p1);
      const float2 hf = __half22float2(hi);
      phi[nt] = *reinterpret_cast<const uint32_t*>(&hi);
      plo[nt] = am_h2(p0 - hf.x, p1 - hf.y);  // exact difference, then rounded
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_r = l_r * corr + ps;
    m_r = mn;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      o[nd][0] *= corr;
      o[nd][1] *= corr;
      o[nd][2] *= corr;
      o[nd][3] *= corr;
    }
    // O += P V: K step k2 covers positions 16 k2 .. 16 k2 + 15
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int mi = lane >> 3;
        uint32_t r[4];
        am_ldsm_t(vs + at2_swz(16 * k2 + (mi & 1) * 8 + (lane & 7), 2 * np + (mi >> 1)), r);
        am_mma(o[2 * np], phi[2 * k2], plo[2 * k2], phi[2 * k2 + 1], plo[2 * k2 + 1], r[0], r[1]);
        am_mma(o[2 * np + 1], phi[2 * k2], plo[2 * k2], phi[2 * k2 + 1], plo[2 * k2 + 1], r[2],
               r[3]);
      }
    }
    // the slot is free: fetch this warp's chunk AM_DEPTH steps ahead into it
    __syncwarp();
    ptx::fence_proxy_async_smem();
    const int cn = c + AM_NW * AM_DEPTH;
    if (cn < nchunks && lane == 0) issue(cn);
  }
  // after a timeout, wait (bounded) for copies still landing in this warp's slots
  if (lane == 0 && sm.abort_flag) {
    for (int k = 0; k < AM_DEPTH; ++k) {
      const int j = it + k;
      if (warp + j * AM_NW >= nchunks) break;
      const uint32_t full = ptx::smem_u32(&sm.full[warp * AM_DEPTH + j % AM_DEPTH]);
      const long long t0 = clock64();
      while (!ptx::mbar_try_wait(full, (uint32_t)((j / AM_DEPTH) & 1))) {
        if (clock64() - t0 > (long long)(timeout_ns * 2ull)) break;
      }
    }
  }

  // ---- merge the warps' partial softmax sums
  if (threadIdx.x == 0) trace_stamp(tr, 4);
  if (gid < G) {
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      sm.acc[warp][gid][8 * nd + 2 * tig] = o[nd][0] + o[nd][2];
      sm.acc[warp][gid][8 * nd + 2 * tig + 1] = o[nd][1] + o[nd][3];
    }
    if (tig == 0) {
      sm.m[warp][gid] = m_r;
      sm.l[warp][gid] = l_r;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(tr, 5);
  // warp h merges head h: lane w < 8 holds warp w's max and sum, every lane
  // two head dimensions; the weights are summed in warp order
  static_assert(AT_GMAX <= AM_NW, "one warp per query head in the merge");
  float2 oz = make_float2(0.f, 0.f);  // this lane's two fp16-rounded o values (split output)
  if (warp < G) {
    const int h = warp;
    const float mw = lane < AM_NW ? sm.m[lane][h] : -FLT_MAX;
    const float lw = lane < AM_NW ? sm.l[lane][h] : 0.f;
    float mx = mw;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mx = __shfl_sync(0xffffffffu, mx, 0);
    const float cw = lw > 0.f ? __expf(mw - mx) : 0.f;
    float den = 0.f, n0 = 0.f, n1 = 0.f;
#pragma unroll
    for (int w = 0; w < AM_NW; ++w) {
      const float c = __shfl_sync(0xffffffffu, cw, w);
      const float l = __shfl_sync(0xffffffffu, lw, w);
      const float2 av = *reinterpret_cast<const float2*>(&sm.acc[w][h][2 * lane]);
      den = fmaf(l, c, den);
      n0 = fmaf(av.x, c, n0);
      n1 = fmaf(av.y, c, n1);
    }
    const __half2 o2 = __floats2half2_rn(n0 / den, n1 / den);
    if (a.out) {
      __half* dst = a.out + (size_t)b * a.out_stride + (size_t)(g * G + h) * D + 2 * lane;
      if ((reinterpret_cast<uintptr_t>(dst) & 3u) == 0) {
        *reinterpret_cast<__half2*>(dst) = o2;
      } else {  // caller's output row stride is odd
        dst[0] = __low2half(o2);
        dst[1] = __high2half(o2);
      }
    }
    if (SPLIT) {
      oz = __half22float2(o2);
      const float am = warp_max(fmaxf(fabsf(oz.x), fabsf(oz.y)));
      if (lane == 0) sm.amax_w[warp] = am;
    }
  }
  if (SPLIT) {
    // ---- the o projection's operand: row maximum over the cluster, then
    // the same three-plane split as the GEMM's pre-pass, on fp16 o
    __syncthreads();
    ptx::cluster_wait();
    const uint32_t rank = ptx::cluster_ctarank();
    const uint32_t bar = ptx::smem_u32(&sm.bar_amax);
    if (threadIdx.x == 0) {
      float cta = 0.f;
      for (int w = 0; w < G; ++w) cta = fmaxf(cta, sm.amax_w[w]);
      sm.amax_r[rank] = cta;
      const uint32_t slot = ptx::smem_u32(&sm.amax_r[rank]);
      for (int r = 0; r < a.Hkv; ++r)
        if (r != (int)rank)
          ptx::st_async_b32(ptx::mapa_shared(slot, (uint32_t)r), __float_as_uint(cta),
                            ptx::mapa_shared(bar, (uint32_t)r));
    }
    __syncthreads();
    // never skipped: no CTA may leave while another can still store into it
    // (after an abort this is a bounded drain)
    bool got = a.Hkv == 1 || ptx::mbar_wait_cluster(bar, 0u, timeout_ns, &sm.abort_flag);
    if (!got) {
      const long long t0 = clock64();
      while (!ptx::mbar_try_wait_cluster(bar, 0u)) {
        if (clock64() - t0 > (long long)(timeout_ns * 2ull)) break;
      }
    }
    if (got && warp < G) {
      float amax = 0.f;
      for (int r = 0; r < a.Hkv; ++r) amax = fmaxf(amax, sm.amax_r[r]);
      const int e = split_shift(amax);
      const float up = ldexpf(1.f, e);
      const float z0 = oz.x * up, z1 = oz.y * up;  // exact: power-of-two scale
      const uint16_t b1 = float2_to_e4m3x2(z0, z1);
      const float2 d1 = e4m3x2_to_float2(b1);
      const float r0 = z0 - d1.x, r1 = z1 - d1.y;
      const uint16_t b2 = float2_to_e4m3x2(r0, r1);
      const float2 d2 = e4m3x2_to_float2(b2);
      const uint16_t b3 = float2_to_e4m3x2(r0 - d2.x, r1 - d2.y);
      const size_t K = (size_t)a.Hq * D;
      const size_t plane = (size_t)gridDim.x / a.Hkv * K;
      uint8_t* dst = a.planes + (size_t)b * K + (size_t)(g * G + warp) * D + 2 * lane;
      *reinterpret_cast<uint16_t*>(dst) = b1;
      *reinterpret_cast<uint16_t*>(dst + plane) = b2;
      *reinterpret_cast<uint16_t*>(dst + 2 * plane) = b3;
      if (rank == 0 && threadIdx.x == 0) a.xscale[b] = ldexpf(1.f, -e);
    }
  }
  if (threadIdx.x == 0 && sm.abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
  if (threadIdx.x == 0) trace_stamp(tr, 6);
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 at_encoder() {
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

// [B][Hkv][cap][64] fp16 as a 4-D tensor {64, cap, Hkv, B}; box {64, 32, 1, 1}
int at_cache_map(CUtensorMap* m, const void* base, int cap, int Hkv, int B, int64_t bstride) {
  auto enc = at_encoder();
  if (!enc) return DDQ_ERR_DEVICE;
  cuuint64_t dims[4] = {64, (cuuint64_t)cap, (cuuint64_t)Hkv, (cuuint64_t)B};
  cuuint64_t strides[3] = {128, (cuuint64_t)cap * 128, (cuuint64_t)bstride * 2};
  cuuint32_t box[4] = {64, AM_ROWS, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDQ_OK : DDQ_ERR_ALIGNMENT;
}
}  // namespace

int launch_decode_attention(const __half* qkv, int64_t qkv_stride, __half* kc, __half* vc,
                            int64_t cache_bstride, int cap, const float* cos, const float* sin,
                            const int64_t* pos, __half* out, int64_t out_stride, uint8_t* planes,
                            float* xscale, int B, int Hq, int Hkv, int D, float scale,
                            unsigned long long timeout_ns, int debug_flags, int flags,
                            cudaStream_t s) {
  if (B < 1 || Hkv < 1 || Hq < Hkv || Hq % Hkv != 0 || Hq / Hkv > AT_GMAX || cap < 1)
    return DDQ_ERR_SHAPE;
  if (D != 64 && D != 128) return DDQ_ERR_SHAPE;
  const bool split = planes != nullptr;
  // the split output: 64-wide heads, one cluster of Hkv CTAs per token (portable size)
  if (split && (D != 64 || Hkv > 8 || !xscale)) return DDQ_ERR_SHAPE;
  if (!split && !out) return DDQ_ERR_INVALID_ARGUMENT;
  if (!aligned16(kc) || !aligned16(vc) || (cache_bstride % 8) != 0) return DDQ_ERR_ALIGNMENT;
  if (split && !aligned16(planes)) return DDQ_ERR_ALIGNMENT;
  AtArgs a{qkv, qkv_stride, kc, vc, cache_bstride, cap, cos, sin, pos, out, out_stride, Hq, Hkv,
           scale, (debug_flags & 2) != 0 ? 1 : 0, planes, xscale, (flags & 1) != 0 ? 1 : 0};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * Hkv));
  cfg.blockDim = dim3(at_warps(D) * 32);
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = (unsigned)Hkv;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = split ? 2 : 1;
  cudaError_t e;
  if (D == 64) {
    // TMA-streamed tensor-core variant (the cache must be 16-byte aligned per batch)
    CUtensorMap tk, tv;
    int st = at_cache_map(&tk, kc, cap, Hkv, B, cache_bstride);
    if (st) return st;
    st = at_cache_map(&tv, vc, cap, Hkv, B, cache_bstride);
    if (st) return st;
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return DDQ_ERR_DEVICE;
    static SmemAttrOnce attr[2][AT_GMAX];
    const int smem = (int)sizeof(AmSmem) + 1024;
    cfg.blockDim = dim3(AM_NW * 32);
    cfg.dynamicSmemBytes = smem;
    auto go = [&](auto kern, int gi) -> int {
      const int ast = ensure_smem_attr(attr[split ? 1 : 0][gi], dev, kern, smem);
      if (ast) return ast;
      e = cudaLaunchKernelEx(&cfg, kern, tk, tv, a, timeout_ns);
      return DDQ_OK;
    };
    int rc = DDQ_OK;
    switch (Hq / Hkv) {
#define DDQ_AT_G(G_)                                                                          \
  case G_:                                                                                    \
    rc = split ? go(decode_attention_mma_kernel<G_, true>, G_ - 1)                            \
               : go(decode_attention_mma_kernel<G_, false>, G_ - 1);                          \
    if (rc) return rc;                                                                        \
    break;
      DDQ_AT_G(1) DDQ_AT_G(2) DDQ_AT_G(3) DDQ_AT_G(4)
      DDQ_AT_G(5) DDQ_AT_G(6) DDQ_AT_G(7) DDQ_AT_G(8)
#undef DDQ_AT_G
      default:
        return DDQ_ERR_SHAPE;
    }
  } else {
    e = cudaLaunchKernelEx(&cfg, decode_attention_kernel<128>, a);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return DDQ_ERR_LAUNCH;
  }
  return check_launch();
}

}  // namespace ddq
