// common.cuh - shared device helpers for the sm_100a W8A16 kernels.
#pragma once

#include <cfloat>
#include <mutex>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/ddq_b200.h"

namespace ddq {

// ----------------------------------------------------------------------------
// e4m3fn <-> fp16/fp32 with the hardware converters (sm_89+).
// Every e4m3fn value is exactly representable in fp16, so the decode is exact.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3x2_to_half2_bits(uint16_t two_bytes) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two_bytes, __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t two_bytes) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two_bytes, __NV_E4M3);
  __half2 hh;
  hh = *reinterpret_cast<__half2*>(&h);
  return __half22float2(hh);
}

// Two e4m3fn bytes of v (the pair selected by `sel`: 0x4140 = bytes 0,1;
// 0x4342 = bytes 2,3) -> two fp16 holding exactly e4m3 value * 2^-8, in the
// byte order of v.  Integer arithmetic only (byte permute, and, add, shift),
// so it runs on the full-rate ALU pipes instead of the converter:
//   e4m3 s.eeee.mmm -> fp16 bits s.0eeee.mmm0000000; the 5-bit fp16 exponent
//   field then reads e with bias 15 instead of 7, i.e. the value times 2^-8,
//   and e4m3 subnormals (e = 0) land on fp16 subnormals with the same factor.
//   The sign moves from bit 7 to bit 15 by adding (b & 0x80) before the
//   shift: bit 7 + bit 7 carries into bit 8.
// Caller multiplies the fp32 result by 256 (exact).  The NaN codes 0x7F/0xFF
// come out as +-1.875 (i.e. +-480 after the factor) instead of NaN; the
// quantizer never produces them from finite weights.
__device__ __forceinline__ uint32_t e4m3x2_to_half2_bits_x2m8(uint32_t v, uint32_t sel) {
  const uint32_t t = __byte_perm(v, 0u, sel);  // 0x00_b1_00_b0
  return (t + (t & 0x00800080u)) << 7;
}

// The four e4m3fn bytes of w -> two fp16x2 words (bytes 0,1 -> lo; 2,3 -> hi).
// HW: the hardware converter (cvt.rn.f16x2.e4m3x2, exact: every e4m3fn value
// is an fp16 value), one instruction per pair; otherwise the integer-ALU form
// above, four instructions per pair, whose results are the values times 2^-8.
// kE4m3ToF16Scale<HW> is the factor that restores the value (1 or 256).
template <bool HW>
__device__ __forceinline__ void e4m3x4_to_half2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  if constexpr (HW) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
  } else {
    lo = e4m3x2_to_half2_bits_x2m8(w, 0x4140u);
    hi = e4m3x2_to_half2_bits_x2m8(w, 0x4342u);
  }
}
template <bool HW>
constexpr float kE4m3ToF16Scale = HW ? 1.f : 256.f;

// Two fp32 values -> two e4m3fn bytes (a -> low byte), round to nearest even,
// saturating to +-448.  For |v| <= 464 this equals torch's float8_e4m3fn cast.
__device__ __forceinline__ uint16_t float2_to_e4m3x2(float a, float b) {
  float2 f = make_float2(a, b);
  return (uint16_t)__nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
}

// Monotone 16-bit key of an fp16 value: larger fp16 -> larger key.
// Split 8 fp32 values (already scaled by 2^e) into three e4m3 planes; the
// bytes keep the element order (element 0 -> lowest byte).
__device__ __forceinline__ void split8(const float* z, uint2& p1, uint2& p2, uint2& p3) {
  uint32_t o1[2] = {0u, 0u}, o2[2] = {0u, 0u}, o3[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float z0 = z[2 * i], z1 = z[2 * i + 1];
    const uint16_t b1 = float2_to_e4m3x2(z0, z1);
    const float2 d1 = e4m3x2_to_float2(b1);
    const float r0 = z0 - d1.x, r1 = z1 - d1.y;  // exact (Sterbenz)
    const uint16_t b2 = float2_to_e4m3x2(r0, r1);
    const float2 d2 = e4m3x2_to_float2(b2);
    const uint16_t b3 = float2_to_e4m3x2(r0 - d2.x, r1 - d2.y);
    const int word = i >> 1, sh = (i & 1) * 16;
    o1[word] |= (uint32_t)b1 << sh;
    o2[word] |= (uint32_t)b2 << sh;
    o3[word] |= (uint32_t)b3 << sh;
  }
  p1 = make_uint2(o1[0], o1[1]);
  p2 = make_uint2(o2[0], o2[1]);
  p3 = make_uint2(o3[0], o3[1]);
}

// Power-of-two shift e of a token row for the three-plane split: with the row
// maximum amax = f * 2^ex (f in [0.5, 1)), z = x * 2^e has max |z| in
// [128, 256), the top binade of e4m3 below its 448 limit; 0 for an all-zero
// or non-finite row.
__device__ __forceinline__ int split_shift(float amax) {
  int ex = 0;
  const bool finite = amax > 0.f && amax <= FLT_MAX;
  if (finite) frexpf(amax, &ex);
  return finite ? 8 - ex : 0;
}

__device__ __forceinline__ uint32_t f16_order_key(__half h) {
  uint16_t b = __half_as_ushort(h);
  return (b & 0x8000u) ? (uint32_t)(uint16_t)(~b) : (uint32_t)(b | 0x8000u);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Device error word set by bounded waits that give up (read by ddq_device_error).
extern __device__ int g_device_error;

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// Phase trace (debug flag bit 1): %globaltimer stamps per CTA, read back with
// ddq_read_trace().  kTraceSlots stamps for each of the first kTraceCtas CTAs.
constexpr int kTraceCtas = 2048;
constexpr int kTraceSlots = 16;
extern __device__ unsigned long long g_trace[kTraceCtas * kTraceSlots];

__device__ __forceinline__ void trace_stamp(bool on, int slot) {
  if (!on) return;
  const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (cta < (unsigned)kTraceCtas) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_trace[cta * kTraceSlots + slot] = t;
  }
}

// ----------------------------------------------------------------------------
// Host-side helpers
// ----------------------------------------------------------------------------
int device_sm_count(int device);
int current_device();
int check_launch();
bool pdl_enabled();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Limit of every device-side bounded wait and the debug flags, as set by
// ddq_set_debug (capi.cu).
unsigned long long wait_timeout_ns();
int debug_flags();

// Raises a kernel's dynamic shared-memory limit once per device, safe under
// concurrent first calls from several host threads (std::call_once per
// device).  cudaFuncSetAttribute is not a stream operation, so the first
// launch of each kernel on a device must come before any stream capture.
// A failure is cleared from the runtime's error state and returned to every
// later caller.
constexpr int kMaxDev = 64;
struct SmemAttrOnce {
  std::once_flag once[kMaxDev];
  int status[kMaxDev] = {};
};
template <typename Kernel>
int ensure_smem_attr(SmemAttrOnce& o, int dev, Kernel kern, int bytes) {
  if (dev < 0 || dev >= kMaxDev) return DDQ_ERR_DEVICE;
  std::call_once(o.once[dev], [&] {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess) {
      cudaGetLastError();
      o.status[dev] = DDQ_ERR_LAUNCH;
    } else {
      o.status[dev] = DDQ_OK;
    }
  });
  return o.status[dev];
}

}  // namespace ddq
