// launch.cuh - internal launcher declarations shared by the C-ABI dispatcher.
#pragma once
#include "common.cuh"

namespace ddq {

int launch_skinny(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                  int bias_dtype, __half* y, int M, int N, int K, cudaStream_t s);
int launch_skinny_argmax(const __half* x, const uint8_t* wq, const float* scales,
                         unsigned long long* packed, int64_t vocab_offset, int M, int N, int K,
                         cudaStream_t s);
int launch_generic(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                   int bias_dtype, __half* y, int64_t M, int64_t N, int64_t K, cudaStream_t s);
int launch_argmax_f16(const __half* logits, int64_t B, int64_t V, int64_t* out, cudaStream_t s);
// Largest split-K factor: the splits of one tile form a thread-block cluster
// (8 = the portable cluster size).
constexpr int64_t kMaxSplits = 8;

struct TcPlan {
  int bt;            // token tile (MMA N)
  int splits;        // split-K factor (grid.z)
  int kps;           // 64-wide K steps per split
  int64_t tiles;     // 128 x bt output tiles
  size_t ws_part_bytes;
  size_t ws_bytes;   // global workspace needed (0: split-K reduces in shared memory)
};
TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int sms);
int launch_tc(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, unsigned long long* packed, int64_t vocab_offset,
              int M, int N, int K, void* ws, size_t ws_bytes, unsigned long long timeout_ns,
              int debug_flags, cudaStream_t s);
// Decode-shape path (tc_decode.cu): activations split into three e4m3 planes,
// e4m3 x e4m3 tensor-core GEMM.  Needs a workspace for the planes.
struct DecPlan {
  int bt;             // token tile: 16, 32 or 64
  int splits;         // split-K factor (cluster size)
  int kps;            // K stages (dc_stage_k(bt) bytes each) per split
  int sms;
  size_t plane_bytes; // 3 * M * K
  size_t ws_bytes;    // planes + per-token scales
};
DecPlan dec_plan(int64_t M, int64_t N, int64_t K, int sms, bool no_split = false);
int launch_dec(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
               int bias_dtype, __half* y, unsigned long long* packed, int64_t vocab_offset, int M,
               int N, int K, void* ws, size_t ws_bytes, unsigned long long timeout_ns,
               int debug_flags, cudaStream_t s, bool swiglu = false,
               const uint8_t* ext_planes = nullptr, const float* ext_xscale = nullptr,
               int64_t* ids = nullptr, unsigned int* counter = nullptr);
// With packed (the greedy epilogue) and no ext_planes, the split pre-pass
// zeroes packed[0, M) before the GEMM's atomicMax; with ids and counter (a
// zero word the call leaves at zero) the GEMM's last CTA also writes ids.
// 1..16 tokens, K % 64 == 0: each SM's weight slice resident in shared memory
// before the grid dependency, mma.sync on fp16 activations (thin.cu).  No
// workspace.  thin_eligible says whether launch_thin takes the shape.
bool thin_eligible(int64_t M, int64_t N, int64_t K, int sms);
int launch_thin(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
                int bias_dtype, __half* y, int M, int N, int K, unsigned long long timeout_ns,
                cudaStream_t s, int debug_flags = 0);
// 1..16 tokens, K % 64 == 0: each CTA's contiguous weight slice resident in
// shared memory (one bulk copy) before the grid dependency, weights on the
// mma.sync A operand, dependents triggered at entry (rs.cu).  No workspace.
// 17..64 tokens on the tcgen05 tensor cores with resident weight slices
// converted to fp16 before the grid dependency (rt.cu); optional SwiGLU
// epilogue over the 16-row gate/up interleave.  No workspace.
bool rt_eligible(int64_t M, int64_t N, int64_t K, int sms, bool swiglu);
int launch_rt(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, bool swiglu,
              unsigned long long timeout_ns, cudaStream_t s, int debug_flags);

bool rs_eligible(int64_t M, int64_t N, int64_t K, int sms);
int launch_rs(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, unsigned long long timeout_ns,
              cudaStream_t s, int debug_flags = 0);
// Fused lm_head argmax for 1..16 tokens streaming 16-row weight tiles with one
// bulk copy each (lmh.cu).  Its workspace area (arrival counter + per-CTA
// words, lmh_area_bytes) leads the lm_head workspace and must be zero before
// the first call; every call leaves the counter at zero.
bool lmh_eligible(int64_t M, int64_t N, int64_t K, int sms);
size_t lmh_area_bytes(int sms);
int launch_lmh(const __half* x, const uint8_t* wq, const float* scales, int M, int N, int K,
               int64_t vocab_offset, unsigned long long* packed, int64_t* ids, void* ws,
               size_t ws_bytes, unsigned long long timeout_ns, int debug_flags, cudaStream_t s);
// Prefill shapes: exact e4m3 -> fp16 weight expansion into the workspace
// (N * K * 2 bytes), then the fp16 tensor-core GEMM (tc_prefill.cu).
size_t pf_workspace_bytes(int64_t N, int64_t K);
// QKV epilogue with RoPE and the KV-cache write (head_dim 64): the weight
// rows are [Hq q heads | Hkv k heads | Hkv v heads] x 64, GEMM token row m is
// sequence b = m / S, token s = m % S, at cache position start + s.
struct PfRope {
  __half* kc;             // [B, Hkv, cap, 64], batch stride cache_bstride
  __half* vc;
  int64_t cache_bstride;
  int cap;
  const float* cos;       // [S, 64] for positions start .. start + S - 1
  const float* sin;
  int start;
  __half* q_out;          // [B * S, Hq, 64]
  __half* k_out;          // [B * S, Hkv, 64] or null
  __half* v_out;
  int S, Hq, Hkv;
};

int launch_pf(const __half* x, const uint8_t* wq, const float* scales, const void* bias,
              int bias_dtype, __half* y, int M, int N, int K, void* ws, size_t ws_bytes,
              unsigned long long timeout_ns, int debug_flags, cudaStream_t s,
              bool swiglu = false, const PfRope* rope = nullptr);
// A workspace was used by a call other than a double-buffered prefill GEMM
// (the next prefill call on it must not expand ahead of the previous kernel);
// a call on a capturing stream also marks it as used in a CUDA graph.
void ws_note_other_use(const void* ws, cudaStream_t s);
// Prefill: RoPE of q and k, q in token-major layout, k/v into the cache (rope.cu).
int launch_prefill_rope_kv(const __half* qkv, int64_t qkv_stride, __half* kc, __half* vc,
                           int64_t cache_bstride, int cap, const float* cos, const float* sin,
                           int start, __half* q_out, __half* k_out, __half* v_out, int B,
                           int S, int Hq, int Hkv, int D, cudaStream_t s);
// Decode-step attention with RoPE and the KV-cache write fused (attention.cu).
int launch_decode_attention(const __half* qkv, int64_t qkv_stride, __half* kc, __half* vc,
                            int64_t cache_bstride, int cap, const float* cos, const float* sin,
                            const int64_t* pos, __half* out, int64_t out_stride, uint8_t* planes,
                            float* xscale, int B, int Hq, int Hkv, int D, float scale,
                            unsigned long long timeout_ns, int debug_flags, int flags,
                            cudaStream_t s);
// Residual add + RMSNorm, optionally followed by the three-plane split of the
// result for a decode GEMM (norm.cu).
int launch_add_rmsnorm_split(const __half* x, const __half* delta, const float* w, float eps,
                             __half* x_out, __half* h, uint8_t* planes, float* xscale, int M,
                             int H, cudaStream_t s);
// Residual add + RMSNorm (norm.cu).
int launch_add_rmsnorm(const __half* x, const __half* delta, const float* w, float eps,
                       __half* x_out, __half* h, int M, int H, cudaStream_t s);
int launch_unpack_argmax(const unsigned long long* packed, int64_t M, int64_t* ids, cudaStream_t s);

}  // namespace ddq
