/*
 * ddq_b200.h - C ABI of the B200 (sm_100a) W8A16 projection-GEMM library.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream
 * (passed as void*, i.e. a cudaStream_t; NULL = legacy default stream),
 * launches asynchronously on that stream and returns a ddq_status.  Nothing
 * here allocates device memory; nothing synchronises the device.  Mutable
 * global state: per-device cached attributes (SM count, the driver's
 * tensor-map encoder, kernels' shared-memory limits), the device error word
 * read by ddq_device_error(), the debug settings of ddq_set_debug(), and a
 * host-side table keyed by workspace address that records, for prefill-shape
 * calls, which of the workspace's two fp16 buffers the next call uses and
 * whether the previous call on it was an eager prefill call (see
 * ddq_w8a16_gemm_workspace_size).  All of it is guarded for concurrent host
 * threads.
 *
 * Data formats (all row-major, contiguous):
 *   x      fp16  [M, K]   activations
 *   wq     uint8 [N, K]   e4m3fn weight bytes (K contiguous)
 *   scales fp32  [N]      per-output-channel scale: w ~= e4m3(wq) * scale
 *   bias   fp16 or fp32 [N], or NULL
 *   y      fp16  [M, N]
 *
 * Each declaration names the reference interface it replaces
 * (hdahroug/ddq, file:line).
 */
#ifndef DDQ_B200_H
#define DDQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The Python mirror turns a non-zero status into a
 * RuntimeError carrying ddq_status_string(), as the reference's TORCH_CHECK
 * does (gemm_FP8_d.cu:151-152, 173-180, 190). */
typedef enum ddq_status {
  DDQ_OK = 0,
  DDQ_ERR_INVALID_ARGUMENT = 1, /* NULL pointer, negative size, bad dtype code */
  DDQ_ERR_SHAPE = 2,            /* inconsistent or unsupported M/N/K */
  DDQ_ERR_ALIGNMENT = 3,        /* pointer not aligned as the kernel needs */
  DDQ_ERR_WORKSPACE = 4,        /* workspace missing or smaller than required */
  DDQ_ERR_DEVICE = 5,           /* no sm_100 device / attribute query failed */
  DDQ_ERR_LAUNCH = 6,           /* CUDA launch error (cudaGetLastError) */
  DDQ_ERR_TIMEOUT = 7           /* a device-side bounded wait gave up */
} ddq_status;

/* Element type codes for bias / weight inputs. */
enum {
  DDQ_DTYPE_NONE = 0,
  DDQ_DTYPE_F16 = 1,
  DDQ_DTYPE_F32 = 2
};

/* Human-readable text of a status code (static storage). */
const char* ddq_status_string(int status);

/* Library version, (major << 16) | minor. */
int ddq_version(void);

/*
 * Quantize a weight matrix to e4m3fn with a per-row fp32 scale.
 * Replaces: quantize() + quantize_kernel, gemm_FP8_d.cu:150-167, 66-86.
 *   scale[n] = max_k |w[n,k]| / 448   (1.0 for an all-zero row)
 *   wq[n,k]  = e4m3fn(w[n,k] / scale[n]), IEEE fp32 division, round to
 *              nearest even (torch's float8_e4m3fn cast; the reference
 *              encoder rounds ties half-up instead, gemm_FP8_d.cu:56).
 * w_dtype is DDQ_DTYPE_F16 (the reference's only input, :151) or
 * DDQ_DTYPE_F32.
 */
int ddq_quantize_e4m3(const void* w, int w_dtype, int64_t N, int64_t K,
                      uint8_t* wq, float* scales, void* stream);

/*
 * Bytes of device workspace ddq_w8a16_gemm needs for this shape (0 if none).
 * Decode shapes (M <= 64) keep the activations split into three e4m3 planes
 * and the per-token scales there; prefill shapes (M >= 128 by default) keep
 * the weight expanded to fp16 (N * K * 2 bytes; the size reported is two such
 * buffers at fixed offsets, 0 and half the workspace, which consecutive
 * prefill calls alternate; one buffer also works, without the overlap
 * below).  The contents need no initialisation.  One workspace sized for the
 * largest shape serves any sequence of shapes; calls sharing it must be
 * ordered on one stream.  The pointer must be 256-byte aligned.
 * Overlap: an eager prefill call (its stream not capturing) whose previous
 * call on the same workspace was also an eager prefill call expands its
 * weight before the previous kernel finishes (that kernel reads the other
 * buffer).  A call made while its stream captures a CUDA graph never does,
 * and marks the workspace: no later call on that address expands early,
 * since a replayed graph runs kernels between eager calls that the library
 * does not see.
 */
size_t ddq_w8a16_gemm_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * y = fp16( x @ (e4m3(wq) * scale)^T + bias ), fp32 accumulation.
 * Replaces: f8_forward() + fp8_gemm_kernel, gemm_FP8_d.cu:171-210, 94-146,
 * and, at the engine's dispatch point, gemm_d.cu:36-87 (cuBLAS + the
 * separate add_bias_kernel, here folded into the epilogue).
 * bias_dtype: DDQ_DTYPE_NONE (bias may be NULL), _F16 (the reference's only
 * bias type, gemm_FP8_d.cu:191) or _F32.
 * Requirements: M >= 0, N >= 1, K >= 1; the fast paths need K % 16 == 0 and
 * 16-byte aligned x / wq (a generic CUDA kernel covers the rest).
 * Kernels by shape (16-byte aligned x and wq, K % 16 == 0):
 *   1..16 tokens, and 17..64 with few MMAs per CTA, where a CTA's weight
 *     slice and the activations fit in shared memory: one mma.sync kernel
 *     on a resident weight slice (the thin kernel takes the 1..16-token
 *     shapes that one does not);
 *   other M <= 64: the activation-split pre-pass plus the e4m3 tcgen05 GEMM
 *     (with ddq_set_debug bit 6, 17..64 tokens with K % 64 == 0 run an
 *     opt-in single tcgen05 kernel instead - tokens on the MMA's A operand,
 *     each CTA's weight rows converted to fp16 in shared memory before the
 *     grid dependency - correct, but slower in dependent chains);
 *   larger M: the prefill kernels.
 * The workspace is used by the last two only.  While ddq_set_debug's
 * injection flags are
 * set, the first group also takes the split + decode kernels.  Summation order differs between these kernels, so the
 * same row can round differently at different M (all within the fp32
 * tolerance); each kernel is bitwise reproducible.
 */
int ddq_w8a16_gemm(const void* x, const uint8_t* wq, const float* scales,
                   const void* bias, int bias_dtype, void* y,
                   int64_t M, int64_t N, int64_t K,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Number of kernels one ddq_w8a16_gemm call of this shape (16-byte aligned
 * x / wq) launches on the current device: 1 or 2.  A diagnostic for launch
 * counts in benchmarks; no reference counterpart.
 */
int ddq_w8a16_gemm_kernel_count(int64_t M, int64_t N, int64_t K);

/*
 * Allocation-free variant of ddq_w8a16_gemm for decode shapes.  It has no
 * counterpart in the reference; it exists for callers that cannot allocate
 * device memory where they call a projection (a host that pre-plans and owns
 * every allocation, a serving runtime that bans cudaMalloc on its request
 * path, code recording a CUDA graph).  Same inputs and output as
 * ddq_w8a16_gemm; it always runs the activation split + e4m3 decode kernel
 * (ddq_w8a16_gemm's kernel for these shapes except the ones its thin kernel
 * takes, where the two agree within the fp32 tolerance, not bit for bit).
 * The scratch lives in a 1 MiB device array inside the library (held by
 * every GPU that loads it, until the process exits) instead of a caller
 * workspace.
 * Limits: 1 <= M <= 64, K % 16 == 0, 16-byte aligned x and wq, and
 * 3*M*K (rounded up to 256) + 4*M <= 1048576 bytes; larger sizes return
 * DDQ_ERR_WORKSPACE (M > 64 or K % 16 != 0: DDQ_ERR_SHAPE).
 * The first call on a device looks up the array's device address (with that
 * device current), and so does the first call after the device's context
 * changed (cudaDeviceReset); make those calls before any stream capture.
 * Bounded waits use the limit and debug flags set by ddq_set_debug, as
 * ddq_w8a16_gemm does.  All calls share the array: calls that may overlap on
 * the GPU (different streams, or several host threads) race - order them on
 * one stream.
 */
int ddq_w8a16_gemm_noalloc(const void* x, const uint8_t* wq, const float* scales,
                           const void* bias, int bias_dtype, void* y,
                           int64_t M, int64_t N, int64_t K, void* stream);

/*
 * Gate/up projection with the SwiGLU epilogue, no [M, 2I] intermediate:
 *   g = fp16( x @ (e4m3(Wg) * sg)^T + bg ),  u = fp16( x @ (e4m3(Wu) * su)^T + bu )
 *   z[m, j] = fp16( silu(g[m, j]) * u[m, j] )            (fp32 math)
 * Replaces: engine.py:189-193 (gate_proj, up_proj, then swiglu_naive,
 * SwiGLU_d.cu:12-26); no reference counterpart fuses them.
 * wq_gu [2I, K] (and scales_gu, bias [2I]) interleave gate and up in blocks of
 * 16 rows: rows 32 b + i = gate row 16 b + i, rows 32 b + 16 + i = up row
 * 16 b + i (0 <= i < 16).  I % 16 == 0, K % 16 == 0, 16-byte aligned x, wq_gu
 * and z [M, I].  Kernels: M <= 64, the split pre-pass and the e4m3 decode
 * GEMM (with ddq_set_debug bit 6, 17..64 tokens with K % 64 == 0 run the
 * opt-in tcgen05 resident-slice kernel); larger M, the prefill kernels.
 * Workspace:
 * ddq_w8a16_gemm_swiglu_workspace_size bytes, used as for ddq_w8a16_gemm.
 */
size_t ddq_w8a16_gemm_swiglu_workspace_size(int64_t M, int64_t I, int64_t K);
int ddq_w8a16_gemm_swiglu(const void* x, const uint8_t* wq_gu, const float* scales_gu,
                          const void* bias, int bias_dtype, void* z,
                          int64_t M, int64_t I, int64_t K,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * One decode step of grouped-query attention with RoPE and the KV-cache write
 * fused in.  Replaces, for a decode step: the q/k RoPE (RoPe_d.cu:12-68), the
 * cache write (engine.py:126-130) and the attention (engine.py:225-251).
 *   qkv   fp16 [B, (Hq + 2 Hkv) * D], row stride qkv_stride (elements): q heads,
 *         then k heads, then v heads (the stacked QKV projection's output)
 *   k_cache, v_cache  fp16 [B, Hkv, capacity, D], batch stride in elements
 *   cos, sin  fp32 [D]: the rotary row of this step's position
 *   pos   device int64 scalar, 0 <= pos < capacity (read on the device)
 *   out   fp16 [B, Hq * D], row stride out_stride
 * Writes cache[b, g, pos] = (rope(k_g), v_g), then
 *   out[b, h] = softmax_j(rope(q_h) . K[b, h / (Hq/Hkv), j] * scale) V[...],
 * j = 0..pos, in fp32.  Hq % Hkv == 0, Hq / Hkv <= 8, D = 64 or 128.
 */
int ddq_decode_attention(const void* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                         int64_t cache_batch_stride, int64_t capacity, const float* cos,
                         const float* sin, const int64_t* pos, void* out, int64_t out_stride,
                         int64_t B, int64_t Hq, int64_t Hkv, int64_t D, float scale,
                         void* stream);

/*
 * ddq_decode_attention with the o projection's operand as its output: the
 * three e4m3 planes [3][B][Hq * D] of each token's o row under a power-of-two
 * scale and the token scales 2^-e [B] (xscale), exactly as the decode GEMM's
 * split pre-pass makes them from fp16 o, for ddq_w8a16_gemm_planes.  No
 * reference counterpart (it removes the pre-pass between attention and the o
 * projection).  out (fp16 o) is optional (NULL: not written).  D = 64,
 * Hkv <= 8 (the Hkv CTAs of a token run as one thread-block cluster); planes
 * 16-byte aligned.  flags bit 0 (kv_ready): the caller guarantees that *pos
 * and the cache rows before it were final before the kernel issued just
 * before this call on the stream started (as in a decode loop, where earlier
 * steps wrote them); the kernel then loads them while that kernel still runs.
 */
int ddq_decode_attention_split(const void* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                               int64_t cache_batch_stride, int64_t capacity, const float* cos,
                               const float* sin, const int64_t* pos, void* out,
                               int64_t out_stride, uint8_t* planes, float* xscale, int64_t B,
                               int64_t Hq, int64_t Hkv, int64_t D, float scale, int flags,
                               void* stream);

/*
 * Prefill rotary embedding and KV-cache write for a chunk of S tokens per
 * sequence starting at cache position `start`.  Replaces, for a prefill
 * chunk, the RoPE kernel on q and k (RoPe_d.cu:12-68, called from
 * engine.py:219-220) and the cache write (engine.py:126-130, 222).
 *   qkv    fp16 [B * S, (Hq + 2 Hkv) * D] token rows (b major), row stride
 *          qkv_stride (elements, multiple of 8): q heads, k heads, v heads
 *   k_cache, v_cache  fp16 [B, Hkv, capacity, D], batch stride in elements
 *   cos, sin  fp32 [S, D]: the rotary rows of positions start .. start + S - 1
 *   q_out  fp16 [B, S, Hq, D] (contiguous)
 *   k_out, v_out  fp16 [B, S, Hkv, D] (contiguous) or NULL: token-major copies
 *          of the new key and value rows (attention inputs whose strides do not
 *          depend on the cache capacity)
 * Writes q_out[b, s, h] = rope(q_h), cache[b, g, start + s] = (rope(k_g), v_g)
 * (and k_out[b, s, g], v_out[b, s, g]) with rope(x) = x cos + rotate_half(x) sin
 * in fp32, rounded to fp16.
 * D = 64 or 128; start + S <= capacity; every pointer 16-byte aligned.
 */
int ddq_prefill_rope_kv(const void* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                        int64_t cache_batch_stride, int64_t capacity, const float* cos,
                        const float* sin, int64_t start, void* q_out, void* k_out, void* v_out,
                        int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D, void* stream);

/*
 * The q/k/v projection of a prefill chunk with RoPE and the KV-cache write in
 * its epilogue: bit for bit ddq_w8a16_gemm(x, wq, scales, bias) -> qkv [B * S,
 * (Hq + 2 Hkv) * D] followed by ddq_prefill_rope_kv(qkv, ...), without writing
 * or re-reading qkv.  Replaces, for a prefill chunk, the q/k/v projections
 * (engine.py:215-217; f8_forward + fp8_gemm_kernel, gemm_FP8_d.cu:171-210,
 * 94-146) with the RoPE kernel on q and k after them (RoPe_d.cu:12-68,
 * engine.py:219-220) and the cache write (engine.py:126-130, 222).
 *   x       fp16 [B * S, K] token rows (b major)
 *   wq, scales, bias, bias_dtype   as ddq_w8a16_gemm with N = (Hq + 2 Hkv) * D
 *   k_cache, v_cache, cache_batch_stride, capacity, cos, sin, start, q_out,
 *   k_out, v_out   as ddq_prefill_rope_kv
 *   workspace  at least ddq_w8a16_gemm_workspace_size(B * S, N, K) bytes,
 *              256-byte aligned
 * Alignment: x and wq 16 bytes; q_out, k_out, v_out, the caches, cos and sin
 * 32 bytes (whole-sector accesses), cache_batch_stride a multiple of 16.
 * Returns DDQ_ERR_SHAPE (nothing launched) where the fused kernel does not
 * take the shape: D != 64, or B * S below the prefill kernel's minimum
 * (ddq_w8a16_gemm_kernel_count(B * S, N, K) == 2 with B * S > 64); the caller
 * then runs the two calls it replaces.
 */
int ddq_w8a16_gemm_qkv_rope_kv(const void* x, const uint8_t* wq, const float* scales,
                               const void* bias, int bias_dtype, int64_t B, int64_t S, int64_t K,
                               int64_t Hq, int64_t Hkv, int64_t D, void* k_cache, void* v_cache,
                               int64_t cache_batch_stride, int64_t capacity, const float* cos,
                               const float* sin, int64_t start, void* q_out, void* k_out,
                               void* v_out, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Residual add + RMSNorm over rows of H (H % 8 == 0, 16-byte aligned rows):
 *   s = fp16(x + delta)   (delta may be NULL: s = x); written to x_out if
 *                         non-NULL (x_out may be x)
 *   h = fp16( s * rsqrt(mean(s^2) + eps) * w )   fp32 math, w fp32 [H]
 * Replaces: qwen2_rmsnorm_kernel (RMSnorm_d.cu:23-87) and the residual add
 * before it (engine.py:254-256).
 */
int ddq_add_rmsnorm(const void* x, const void* delta, const float* w, float eps,
                    void* x_out, void* h, int64_t M, int64_t H, void* stream);

/*
 * Residual add + RMSNorm as ddq_add_rmsnorm, followed by the split of h that
 * the decode GEMM takes as its operand (what ddq_w8a16_gemm's pre-pass does
 * with x): per row a power-of-two scale 2^e with max |h * 2^e| in [128, 256),
 * and h * 2^e = p1 + p2 + p3 in three e4m3 planes.
 *   planes  e4m3 [3][M][H] (16-byte aligned), xscale fp32 [M] = 2^-e
 *   h       fp16 [M, H], optional (NULL: not stored)
 * H % 16 == 0 and H <= 2048.  Replaces, on the decode path, the RMSNorm
 * before a projection (RMSnorm_d.cu:23-87) and the projection's own split.
 */
int ddq_add_rmsnorm_split(const void* x, const void* delta, const float* w, float eps,
                          void* x_out, void* h, uint8_t* planes, float* xscale,
                          int64_t M, int64_t H, void* stream);

/*
 * The decode-shape GEMM (M <= 64) on activations already split by
 * ddq_add_rmsnorm_split: same result as ddq_w8a16_gemm on the h they came
 * from (or, with swiglu != 0, as ddq_w8a16_gemm_swiglu with N = 2I rows and
 * y = z [M, N/2]).  Replaces: gemm_FP8_d.cu:171-210 for a projection whose
 * input is produced by an RMSNorm.  No workspace.
 */
int ddq_w8a16_gemm_planes(const uint8_t* planes, const float* xscale, const uint8_t* wq,
                          const float* scales, const void* bias, int bias_dtype, void* y,
                          int64_t M, int64_t N, int64_t K, int swiglu, void* stream);

/*
 * Greedy argmax over fp16 logits [B, V] -> int64 [B]; ties go to the
 * lowest index.  Replaces: sampler_d.cu:10-70 (argmax_kernel + forward).
 */
int ddq_argmax_f16(const void* logits, int64_t B, int64_t V, int64_t* out,
                   void* stream);

/*
 * Bytes of workspace ddq_lm_head_argmax needs.  It starts with two arrival
 * counters (bytes 0 and 64: the last CTA to arrive combines the results, of
 * the streaming kernel and of the decode kernel) and one word per CTA and
 * token of the streaming kernel (its tokens: see below), followed by the
 * activation planes of the decode-kernel path used for more tokens.
 * Zero-fill it once before its first use; every call leaves the counters at
 * zero.  Keep it for ddq_lm_head_argmax calls only (other entry points
 * would overwrite the counters), one workspace per stream.
 */
size_t ddq_lm_head_argmax_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * Fused lm_head GEMM + greedy argmax over one vocabulary shard:
 *   logits[m, n] = fp16( x[m,:] . (e4m3(wq[n,:]) * scale[n]) )   (no bias)
 *   packed[m]    = max over n of  (ordered_fp16(logits[m,n]) << 32)
 *                                 | (0xFFFFFFFF - (n + vocab_offset))
 * i.e. the largest fp16 logit, ties to the lowest global index, encoded so
 * that a MAX over packed values of several shards (an NCCL all-gather or
 * all-reduce MAX) yields the global greedy token.  ids[m] (may be NULL)
 * receives the decoded global index of this shard's best logit.
 * The logits are never written to memory.  1..16 tokens with K % 64 == 0
 * (K <= 4096) run one kernel that streams 16-row weight tiles and writes
 * packed[] and ids[] itself; other shapes run the activation split (which
 * also zeroes packed[]) and the decode kernel with an argmax epilogue, whose
 * last CTA writes ids[] (with the workspace's counter; a call whose chunks
 * of 64 tokens include one below the decode kernel's minimum runs a memset
 * and an unpack kernel instead).
 * Replaces: engine.py:338 (lm_head via gemm_d) + engine.py:345/351
 * (sampler_d.forward on the last position), sampler_d.cu:10-49.
 */
int ddq_lm_head_argmax(const void* x, const uint8_t* wq, const float* scales,
                       int64_t M, int64_t N, int64_t K, int64_t vocab_offset,
                       uint64_t* packed, int64_t* ids,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * Decode packed (key, index) words produced by ddq_lm_head_argmax (or their
 * element-wise MAX across shards) into int64 token ids.
 */
int ddq_unpack_argmax(const uint64_t* packed, int64_t M, int64_t* ids,
                      void* stream);

/*
 * Read (and clear) the device error word that bounded device-side waits set
 * when they give up.  Synchronises `stream`.  *code = 0 means no error.
 */
int ddq_device_error(int* code, void* stream);

/*
 * Test hook (no reference counterpart): set the limit of every device-side
 * bounded wait (0 = the 1 s default) and debug flags for later launches in
 * this process.  flags bit 0 makes the tensor-core decode and prefill
 * kernels skip the accumulator-ready signal, so their epilogue waits run out
 * and report
 * DDQ_ERR_TIMEOUT through ddq_device_error() without faulting the GPU;
 * bit 1 turns on the phase trace read by ddq_read_trace(); bit 6 switches
 * on the opt-in 17..64-token tcgen05 resident-slice kernel, and bit 4 makes
 * that kernel skip its accumulator-ready signal the same way; bits 2 and 3
 * have no effect of their own.  While bit 0 or bit 2 is set, the shapes of
 * the resident-slice and thin kernels run the split + decode kernels instead
 * (bit 2 alone selects exactly that, e.g. to compare a fused producer's
 * planes with the GEMM's own pre-pass); while bit 3 is set, the mma.sync
 * resident-slice kernel's shapes go to the thin kernel where it takes them
 * (to test that kernel); with any bit but 1, 4, 6 and 7 set, the opt-in
 * kernel takes no shape.  Bit 7 runs the prefill GEMMs that use CTA pairs
 * (512 tokens and more, N >= 2048) on single CTAs, to compare the two.
 * A wait that runs out is followed by a second bounded wait for the CTA's own
 * copies in flight; should that one run out too, the CTA exits with copies
 * outstanding and the context's further behaviour is undefined (it has not
 * happened in any test: the copies read valid memory and complete).
 */
int ddq_set_debug(int flags, uint64_t wait_timeout_ns);

/*
 * Tracing hook (no reference counterpart): with debug flag bit 1 set, each of
 * the first 2048 CTAs of a tensor-core launch writes %globaltimer stamps (ns)
 * into 16 slots: 0 entry, 1 set-up done, 2 first weight loads issued, 3 first
 * weight tile landed (decode kernel: activation producer past the grid
 * dependency), 4 last MMA issued, 5 accumulator ready, 6 epilogue done,
 * 7 exit; decode kernel in split-K mode also 8 partials sent, 9 the other
 * ranks' partials received, 10 partials reduced; the thin kernel writes 0,
 * 2 (weight copies issued), 3 (grid dependency resolved), 5 (weights and
 * activations landed), 4 (MMAs done), 6 and 7; other slots stay 0.  This copies the
 * stamps of the first max_ctas CTAs (16 uint64 each) to host memory `dst`
 * and synchronises `stream`.
 */
int ddq_read_trace(uint64_t* dst, int max_ctas, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DDQ_B200_H */
