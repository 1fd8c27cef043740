// attention.cu - one decode step of grouped-query attention with the rotary
// embedding and the KV-cache write fused in (replaces the reference's RoPE
// kernel, the cache copy and the attention call of a decode step:
// RoPe_d.cu:12-68, engine.py:126-130 and 225-251).
//
// For each sequence b and key/value head g (one CTA, 256 threads):
//   q_h  = fp16(rope(q_h, pos))   for the G query heads h of group g
//   k    = fp16(rope(k_g, pos)),  v = v_g        -> cache[b, g, pos, :]
//   o_h  = softmax_j( q_h . K[b, g, j, :] * scale ) V[b, g, j, :],  j = 0..pos
// Rotate-half RoPE in fp32 with the caller's cos/sin row for this position,
// rounded to fp16 as the unfused path rounds it; scores, softmax and the
// weighted sum in fp32; o rounded to fp16.  The position is read on the
// device, so a captured CUDA graph replays it for every step.
//
// Work split: the warps (16 for 64-wide heads) take 32-position tiles in
// turn (lane = position for the scores, lane = D / 32 head dimensions for the
// weighted sum of V) with an online softmax per query head; the CTA merges
// the warps' partial results in shared memory.  Every K row and every group
// of 16 V rows is requested before it is used, so a warp waits on memory once
// per step instead of once per row.  K rows are read once per CTA, by one lane each (128
// contiguous bytes); V rows once, coalesced across the warp.  The step reads
// the cache at HBM rate; the arithmetic runs on the CUDA cores.
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
// 64-wide heads: the K and V rows stream into shared memory through TMA.
// ----------------------------------------------------------------------------
// Per-lane global loads left the kernel waiting on memory (one latency per
// row group, a few warps per SM).  Here the positions are cut into 32-row
// chunks (4 KB of K + 4 KB of V); warp w owns ring slot w and the chunks
// w, w + 16, ...; each warp's lane 0 issues the TMA copies of its next chunk
// as soon as it has finished with the slot, so up to 16 chunks per CTA are in
// flight.  The copies use the 128-byte swizzle, which keeps both access
// patterns free of bank conflicts: lane = position reads its K row, lane =
// two head dimensions reads a V row.
constexpr int AT2_NW = 16;        // warps = ring slots
constexpr int AT2_ROWS = 32;      // positions per chunk
constexpr int AT2_CHUNK = AT2_ROWS * 64 * 2;  // bytes of K (and of V) per chunk

struct At2Smem {
  uint8_t ring[AT2_NW][2][AT2_CHUNK];          // [slot][K | V]
  float q[AT_GMAX][64];
  float acc[AT2_NW][AT_GMAX][64];
  float m[AT2_NW][AT_GMAX], l[AT2_NW][AT_GMAX];
  float p[AT2_NW][AT_GMAX][AT2_ROWS];           // per warp: this chunk's weights
  unsigned long long full[AT2_NW];
  int abort_flag;
};

// byte offset of 16-byte chunk j of row r in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t at2_swz(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

template <int G>
__global__ void __launch_bounds__(AT2_NW * 32, 1)
    decode_attention_tma_kernel(const __grid_constant__ CUtensorMap tm_k,
                                const __grid_constant__ CUtensorMap tm_v, const AtArgs a,
                                unsigned long long timeout_ns) {
  constexpr int D = 64, DH = 32;
  extern __shared__ uint8_t at2_raw[];
  At2Smem& sm = *reinterpret_cast<At2Smem*>((reinterpret_cast<uintptr_t>(at2_raw) + 1023) &
                                            ~static_cast<uintptr_t>(1023));
  const int b = blockIdx.x / a.Hkv, g = blockIdx.x % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int w = 0; w < AT2_NW; ++w) ptx::mbar_init(ptx::smem_u32(&sm.full[w]), 1);
    sm.abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
  }
  ptx::pdl_wait();  // qkv comes from the previous kernel
  const int64_t p = *a.pos;
  if (p < 0 || p >= a.cap) return;  // the host checks the range; nothing to do otherwise
  const int L = (int)p + 1;
  const int nchunks = (L + AT2_ROWS - 1) / AT2_ROWS;
  const __half* row = a.qkv + (size_t)b * a.qkv_stride;
  __half* kc = a.kc + (size_t)b * a.cache_bstride + (size_t)g * a.cap * D;
  __half* vc = a.vc + (size_t)b * a.cache_bstride + (size_t)g * a.cap * D;

  // ---- rotary embedding of the G query heads and the new key; cache write
  for (int i = threadIdx.x; i < (G + 1) * DH; i += blockDim.x) {
    const int h = i / DH, d = i % DH;
    const __half* src = h < G ? row + (size_t)(g * G + h) * D : row + (size_t)(a.Hq + g) * D;
    const float x1 = __half2float(src[d]), x2 = __half2float(src[d + DH]);
    // x * cos + rotate_half(x) * sin, each product rounded as torch rounds it
    const float y1 = __half2float(
        __float2half_rn(__fadd_rn(__fmul_rn(x1, a.cos[d]), __fmul_rn(-x2, a.sin[d]))));
    const float y2 = __half2float(
        __float2half_rn(__fadd_rn(__fmul_rn(x2, a.cos[d + DH]), __fmul_rn(x1, a.sin[d + DH]))));
    if (h < G) {
      sm.q[h][d] = y1;
      sm.q[h][d + DH] = y2;
    } else {
      kc[(size_t)p * D + d] = __float2half_rn(y1);
      kc[(size_t)p * D + d + DH] = __float2half_rn(y2);
    }
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    vc[(size_t)p * D + d] = row[(size_t)(a.Hq + a.Hkv + g) * D + d];
  ptx::fence_proxy_async_global();  // the new cache row is read back through TMA
  __syncthreads();
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  const uint32_t full = ptx::smem_u32(&sm.full[warp]);
  const uint32_t kdst = ptx::smem_u32(&sm.ring[warp][0][0]);
  const uint32_t vdst = ptx::smem_u32(&sm.ring[warp][1][0]);
  auto issue = [&](int c) {
    ptx::mbar_arrive_expect_tx(full, 2u * AT2_CHUNK);
    ptx::tma_load_4d(kdst, &tm_k, 0, c * AT2_ROWS, g, b, full);
    ptx::tma_load_4d(vdst, &tm_v, 0, c * AT2_ROWS, g, b, full);
  };
  if (lane == 0 && warp < nchunks) issue(warp);

  float m[G], l[G], acc[G][2];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -FLT_MAX;
    l[h] = 0.f;
    acc[h][0] = acc[h][1] = 0.f;
  }
  float* pw = &sm.p[warp][0][0];
  int phase = 0, pending = warp < nchunks ? 1 : 0;
  for (int c = warp; c < nchunks; c += AT2_NW, phase ^= 1) {
    if (!ptx::mbar_wait(full, (uint32_t)phase, timeout_ns, &sm.abort_flag)) break;
    pending = 0;
    const uint8_t* ks = &sm.ring[warp][0][0];
    const uint8_t* vs = &sm.ring[warp][1][0];
    const int t0 = c * AT2_ROWS;
    const bool ok = t0 + lane < L;
    // scores: lane = position, its K row from the swizzled tile
    float s[G];
#pragma unroll
    for (int h = 0; h < G; ++h) s[h] = 0.f;
#pragma unroll
    for (int cc = 0; cc < D / 8; ++cc) {
      const uint4 u = *reinterpret_cast<const uint4*>(ks + at2_swz(lane, cc));
      const __half2* hv = reinterpret_cast<const __half2*>(&u);
      float kf[8];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(hv[t]);
        kf[2 * t] = f.x;
        kf[2 * t + 1] = f.y;
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float4 qa = *reinterpret_cast<const float4*>(&sm.q[h][cc * 8]);
        const float4 qb = *reinterpret_cast<const float4*>(&sm.q[h][cc * 8 + 4]);
        float v = s[h];
        v = fmaf(qa.x, kf[0], v);
        v = fmaf(qa.y, kf[1], v);
        v = fmaf(qa.z, kf[2], v);
        v = fmaf(qa.w, kf[3], v);
        v = fmaf(qb.x, kf[4], v);
        v = fmaf(qb.y, kf[5], v);
        v = fmaf(qb.z, kf[6], v);
        v = fmaf(qb.w, kf[7], v);
        s[h] = v;
      }
    }
    // online softmax per query head; this chunk's weights go to shared memory
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float sv = ok ? s[h] * a.scale : -FLT_MAX;
      float tm = sv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
      const float mn = fmaxf(m[h], tm);
      const float corr = __expf(m[h] - mn);
      const float pv = ok ? __expf(sv - mn) : 0.f;
      pw[h * AT2_ROWS + lane] = pv;
      float ps = pv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[h] = l[h] * corr + ps;
      m[h] = mn;
      acc[h][0] *= corr;
      acc[h][1] *= corr;
    }
    __syncwarp();
    // weighted sum: lane = head dimensions 2 lane, 2 lane + 1 of each V row;
    // rows past the last position are skipped (the cache there is not ours)
    const int jn = min(AT2_ROWS, L - t0);
    const uint32_t voff = (uint32_t)(lane >> 2), vsub = (uint32_t)(lane & 3) * 4;
#pragma unroll
    for (int j4 = 0; j4 < AT2_ROWS; j4 += 4) {
      if (j4 >= jn) break;
      float2 vf[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        vf[t] = j4 + t < jn ? __half22float2(*reinterpret_cast<const __half2*>(
                                  vs + at2_swz(j4 + t, (int)voff) + vsub))
                            : make_float2(0.f, 0.f);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float4 p4 = *reinterpret_cast<const float4*>(pw + h * AT2_ROWS + j4);
        const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          acc[h][0] = fmaf(pp[t], vf[t].x, acc[h][0]);
          acc[h][1] = fmaf(pp[t], vf[t].y, acc[h][1]);
        }
      }
    }
    // the slot and the weights are free: fetch this warp's next chunk
    __syncwarp();
    ptx::fence_proxy_async_smem();
    if (c + AT2_NW < nchunks) {
      if (lane == 0) issue(c + AT2_NW);
      pending = 1;
    }
  }
  // after a timeout, wait (bounded) for a copy still landing in this slot
  if (pending && lane == 0) {
    const long long t0 = clock64();
    while (!ptx::mbar_try_wait(full, (uint32_t)phase)) {
      if (clock64() - t0 > (long long)(timeout_ns * 2ull)) break;
    }
  }

  // ---- merge the warps' partial softmax sums
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (lane == 0) {
      sm.m[warp][h] = m[h];
      sm.l[warp][h] = l[h];
    }
    sm.acc[warp][h][2 * lane] = acc[h][0];
    sm.acc[warp][h][2 * lane + 1] = acc[h][1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float mx = -FLT_MAX;
    for (int w = 0; w < AT2_NW; ++w) mx = fmaxf(mx, sm.m[w][h]);
    float den = 0.f, num = 0.f;
    for (int w = 0; w < AT2_NW; ++w) {
      const float cw = sm.l[w][h] > 0.f ? __expf(sm.m[w][h] - mx) : 0.f;
      den = fmaf(sm.l[w][h], cw, den);
      num = fmaf(sm.acc[w][h][d], cw, num);
    }
    a.out[(size_t)b * a.out_stride + (size_t)(g * G + h) * D + d] = __float2half_rn(num / den);
  }
  if (threadIdx.x == 0 && sm.abort_flag) record_device_error(DDQ_ERR_TIMEOUT);
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
  cuuint32_t box[4] = {64, AT2_ROWS, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDQ_OK : DDQ_ERR_ALIGNMENT;
}
}  // namespace

int launch_decode_attention(const __half* qkv, int64_t qkv_stride, __half* kc, __half* vc,
                            int64_t cache_bstride, int cap, const float* cos, const float* sin,
                            const int64_t* pos, __half* out, int64_t out_stride, int B, int Hq,
                            int Hkv, int D, float scale, unsigned long long timeout_ns,
                            cudaStream_t s) {
  if (B < 1 || Hkv < 1 || Hq < Hkv || Hq % Hkv != 0 || Hq / Hkv > AT_GMAX || cap < 1)
    return DDQ_ERR_SHAPE;
  if (D != 64 && D != 128) return DDQ_ERR_SHAPE;
  if (!aligned16(kc) || !aligned16(vc) || (cache_bstride % 8) != 0) return DDQ_ERR_ALIGNMENT;
  AtArgs a{qkv, qkv_stride, kc, vc, cache_bstride, cap, cos, sin, pos, out, out_stride, Hq, Hkv,
           scale};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * Hkv));
  cfg.blockDim = dim3(at_warps(D) * 32);
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (D == 64) {
    // TMA-streamed variant (the cache must be 16-byte aligned per batch)
    CUtensorMap tk, tv;
    int st = at_cache_map(&tk, kc, cap, Hkv, B, cache_bstride);
    if (st) return st;
    st = at_cache_map(&tv, vc, cap, Hkv, B, cache_bstride);
    if (st) return st;
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return DDQ_ERR_DEVICE;
    static bool attr_set[AT_GMAX][64] = {};
    const int smem = (int)sizeof(At2Smem) + 1024;
    cfg.blockDim = dim3(AT2_NW * 32);
    cfg.dynamicSmemBytes = smem;
    switch (Hq / Hkv) {
#define DDQ_AT_G(G_)                                                                     \
  case G_:                                                                               \
    if (!attr_set[G_ - 1][dev]) {                                                        \
      if (cudaFuncSetAttribute(decode_attention_tma_kernel<G_>,                          \
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=     \
          cudaSuccess)                                                                   \
        return DDQ_ERR_LAUNCH;                                                           \
      attr_set[G_ - 1][dev] = true;                                                      \
    }                                                                                    \
    e = cudaLaunchKernelEx(&cfg, decode_attention_tma_kernel<G_>, tk, tv, a, timeout_ns); \
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
