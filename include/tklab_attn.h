/*
 * tklab_attn.h — C ABI of the B200 (sm_100a) flash-attention library
 * (libtklab_attn.so).  Plain pointers, sizes and a CUDA stream handle; no
 * PyTorch types.  Every entry point validates its arguments, launches
 * asynchronously on `stream` (a cudaStream_t, NULL = legacy default stream)
 * and returns a status code (TK_OK = 0).  Errors detected on the device
 * (a bounded wait that ran out) are recorded in a per-device status word
 * read by tk_attn_device_status().
 *
 * Layout contract (same as the reference module): Q, K, V, O, dO, dQ, dK,
 * dV are contiguous (batch, heads, seq, head_dim) tensors of one 16-bit
 * type; the log-sum-exp and delta buffers are contiguous fp32
 * (batch, heads, seq).  The log-sum-exp is base 2 and includes the softmax
 * scale: lse = log2(sum_n exp2(scale * log2(e) * q.k_n)).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   tk_attn_fwd         src/tklab/kernels/flash_attention.py:296-347
 *                       (_launch_forward and its launch of
 *                        _flash_attention_forward_kernel, :120-264)
 *   tk_attn_bwd_pre     src/tklab/kernels/flash_attention.py:560-569
 *                       (_attn_bwd_preprocess_kernel launch, :368-395)
 *   tk_attn_bwd         src/tklab/kernels/flash_attention.py:570-606
 *                       (_attn_bwd_dkdv_kernel :398-466 and
 *                        _attn_bwd_dq_kernel :469-533 launches)
 *   tk_attn_bwd_fused / tk_attn_dq_convert
 *                       the two launches of tk_attn_bwd, exposed separately
 *   tk_attn_fwd_ws / tk_attn_fwd_workspace_bytes
 *                       _launch_forward (src/tklab/kernels/flash_attention.py:
 *                       296-347) with optional scratch for a key-split
 *                       schedule of problems with too few query tiles to
 *                       fill the device; the reference launches one program
 *                       per query tile and has no such schedule
 *   tk_attn_bwd_workspace_bytes
 *                       the fp32 dQ accumulator size; the reference needs
 *                       no workspace because its dQ pass recomputes P
 *                       (src/tklab/kernels/flash_attention.py:589-606)
 */
#ifndef TKLAB_ATTN_H_
#define TKLAB_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TK_API __attribute__((visibility("default")))
#else
#define TK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of Q/K/V/O/dO/dQ/dK/dV. */
#define TK_DTYPE_F16 0
#define TK_DTYPE_BF16 1

/* Status codes. */
#define TK_OK 0
#define TK_ERR_INVALID_ARGUMENT 1
#define TK_ERR_UNSUPPORTED 2
#define TK_ERR_MISALIGNED 3
#define TK_ERR_LAUNCH 4
#define TK_ERR_TENSOR_MAP 5
#define TK_ERR_DEVICE_TIMEOUT 6 /* low byte; bits 8.. carry the wait site */
#define TK_ERR_NO_DRIVER 7
#define TK_ERR_TOO_LARGE 8
#define TK_ERR_OUT_OF_MEMORY 9 /* device memory the library needs could not be committed */

/* Forward attention.  o receives softmax(scale * q k^T) v (causal: key n
 * attends query m only when n <= m).  lse may be NULL; otherwise it
 * receives the base-2 log-sum-exp of every query row.  head_dim must be a
 * multiple of 8 from 8 to 256 (widths other than 64, 128 and 256 run the
 * next wider kernel with the missing columns zero-filled on load and clipped
 * on store; 136..192 run a 192-column and 200..256 a 256-column kernel); q,
 * k, v, o must be 16-byte aligned. */
TK_API int tk_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int64_t batch,
                int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                void* stream);

/* Bytes of scratch tk_attn_fwd_ws can use for this problem on the current
 * device: nonzero when the problem has too few work items for the device's
 * SMs and its longest item would set the time (few (batch, head) slabs,
 * long sequences; head_dim up to 128).  Such problems are then run as
 * chunks of the key range, whose fp32 partial outputs and log-sum-exps are
 * written to the scratch and merged by a second kernel.  0: tk_attn_fwd_ws
 * runs exactly tk_attn_fwd.  Returns 0 for invalid arguments too. */
TK_API size_t tk_attn_fwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                          int dtype, int causal);

/* tk_attn_fwd with scratch for the key-split schedule.  workspace NULL (or
 * workspace_bytes 0): identical to tk_attn_fwd.  Otherwise workspace must
 * be 256-byte aligned device memory of at least
 * tk_attn_fwd_workspace_bytes(...) bytes (TK_ERR_INVALID_ARGUMENT if
 * smaller, TK_ERR_MISALIGNED if unaligned), private to this call until it
 * completes on `stream`.  The result agrees with tk_attn_fwd's within
 * fp32 rounding before the final rounding to the 16-bit output. */
TK_API int tk_attn_fwd_ws(const void* q, const void* k, const void* v, void* o, float* lse, int64_t batch,
                          int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Backward preprocessing: delta[b,h,m] = sum_d o[b,h,m,d] * d_o[b,h,m,d]
 * (fp32), and, when dq_accum is not NULL, the fp32 dQ accumulator
 * (batch*heads*seq*head_dim floats, 16-byte aligned) cleared to zero. */
TK_API int tk_attn_bwd_pre(const void* o, const void* d_o, float* delta, float* dq_accum, int64_t batch,
                    int64_t heads, int64_t seq, int64_t head_dim, int dtype, void* stream);

/* Backward attention from the saved lse and the delta of tk_attn_bwd_pre.
 * dq_accum must hold zeros on entry (tk_attn_bwd_pre clears it); it is used
 * as an fp32 workspace and then converted into dq.  dk and dv are written
 * directly.  All of q, k, v, d_o, dq, dk, dv must be 16-byte aligned.
 * head_dim: multiples of 8 up to 256 (136..256 on a kernel that gives each
 * 128-key tile two CTAs, one per 128-column half of dk, dv and dq). */
TK_API int tk_attn_bwd(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                const float* delta, float* dq_accum, void* dq, void* dk, void* dv, int64_t batch,
                int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                void* stream);

/* The two launches of tk_attn_bwd, for callers that schedule them apart:
 * tk_attn_bwd_fused runs the fused recompute kernel (dK and dV written,
 * scaled dQ contributions added into dq_accum), tk_attn_dq_convert turns the
 * n-element fp32 accumulator into dq (n a multiple of 8). */
TK_API int tk_attn_bwd_fused(const void* q, const void* k, const void* v, const void* d_o,
                             const float* lse, const float* delta, float* dq_accum, void* dk,
                             void* dv, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                             int dtype, int causal, float scale, void* stream);
TK_API int tk_attn_dq_convert(const float* dq_accum, void* dq, int64_t n, int dtype, void* stream);

/* The backward for callers that cannot allocate device memory (plugins whose
 * host gives them no allocator, frameworks that own every device byte through
 * their own pool, allocation-free hot loops).  Same inputs and outputs as
 * tk_attn_bwd_pre + tk_attn_bwd, but delta and the fp32 dQ accumulator live
 * in a 64 MiB array compiled into the library instead of caller buffers, so
 * nothing is allocated.  head_dim 64 or 128.  Limit:
 * batch*heads*seq*(head_dim+1) <= 16,777,216, else TK_ERR_TOO_LARGE before
 * any launch.  The array is shared by all calls
 * on a device: calls whose kernels overlap on the GPU race on it; each call
 * clears the accumulator it needs.  Every argument is checked before the
 * array is touched or anything launches.  The first call on a device looks
 * up the array's device address — make it before any stream capture; if
 * the device cannot commit the 64 MiB there (lazy module loading) the call
 * returns TK_ERR_OUT_OF_MEMORY.  Every GPU that loads this part of the
 * library holds the 64 MiB until exit.
 * No counterpart in the reference (its backward allocates through torch). */
TK_API int tk_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                               const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                               int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                               int dtype, int causal, float scale, void* stream);

/* Deterministic backward: dQ is produced by a query-stationary kernel that
 * keeps it in tensor memory and adds the key tiles in one fixed order, with
 * no atomics, so repeated calls give bitwise identical dq; dk and dv come
 * from the fused kernel with its dQ path compiled out (bitwise identical to
 * tk_attn_bwd's dk and dv).  No fp32 accumulator, no conversion pass.
 * Replaces the reference's two backward launches `_attn_bwd_dkdv_kernel` and
 * `_attn_bwd_dq_kernel` (src/tklab/kernels/flash_attention.py:570-606),
 * which are deterministic the same way.
 *   tk_attn_bwd_dkdv          dK, dV from q, k, v, dO, lse and delta
 *   tk_attn_bwd_dq            dQ (input dtype, scale applied)
 *   tk_attn_bwd_deterministic delta (tk_attn_bwd_pre without the clear), then
 *                             both of the above */
TK_API int tk_attn_bwd_dkdv(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                            const float* delta, void* dk, void* dv, int64_t batch, int64_t heads, int64_t seq,
                            int64_t head_dim, int dtype, int causal, float scale, void* stream);
TK_API int tk_attn_bwd_dq(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                          const float* delta, void* dq, int64_t batch, int64_t heads, int64_t seq,
                          int64_t head_dim, int dtype, int causal, float scale, void* stream);
TK_API int tk_attn_bwd_deterministic(const void* q, const void* k, const void* v, const void* o,
                                     const void* d_o, const float* lse, float* delta, void* dq, void* dk,
                                     void* dv, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                     int dtype, int causal, float scale, void* stream);

/* Rotate-half RoPE fused into the attention (the reference applies it as a
 * separate op, `rope` in src/tklab/kernels/rope.py:310-316, whose kernels
 * :27-160 fix the arithmetic; this is the step before attention).  Tables
 * cos and sin are (seq, head_dim/2) fp32, indexed by the position only and
 * shared by every batch and head; head_dim must be 64 or 128.
 *   tk_attn_fwd_rope        o = attention(R q, R k, v): K is rotated once
 *                           into the caller's k_rot workspace (same shape as
 *                           k; it holds R k on return), and the forward kernel
 *                           rotates each Q tile in shared memory after its
 *                           load; rotated values are rounded to dtype, as the
 *                           reference's separate rope output is; lse as in
 *                           tk_attn_fwd
 *   tk_rope_rotate          out = R x (transpose: R^T x) for a contiguous
 *                           (batch, heads, seq, head_dim) tensor; out may be x.
 *                           The backward runs tk_attn_bwd_pre and
 *                           tk_attn_bwd_fused on R q, R k, then
 *   tk_attn_dq_convert_rope dq = R^T dq_accum rounded to dtype (in place of
 *                           tk_attn_dq_convert), and tk_rope_rotate with
 *                           transpose on dk. */
TK_API int tk_attn_fwd_rope(const void* q, const void* k, const void* v, const float* cos, const float* sin,
                            void* k_rot, void* o, float* lse, int64_t batch, int64_t heads, int64_t seq,
                            int64_t head_dim, int dtype, int causal, float scale, void* stream);
TK_API int tk_rope_rotate(const void* x, void* out, const float* cos, const float* sin, int64_t batch,
                          int64_t heads, int64_t seq, int64_t head_dim, int dtype, int transpose, void* stream);
TK_API int tk_attn_dq_convert_rope(const float* dq_accum, void* dq, const float* cos, const float* sin,
                                   int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int dtype,
                                   void* stream);

/* Grouped-query-attention decode: one query token per query head, q_heads =
 * G * kv_heads (query head h reads KV head h / G), contiguous KV cache.
 * The reference specifies this workload as a model only
 * (docs/research/gqa_decode_model.md: "Canonical decode workload",
 * "Semantic GQA mapping"); it has no kernel.
 *   q, o     (batch, q_heads, head_dim)         16-bit
 *   k, v     (batch, kv_heads, seq_kv, head_dim) 16-bit
 *   kv_lens  (batch) int32 valid keys per batch (clamped to [0, seq_kv]),
 *            or NULL for all seq_kv; a batch with none gets o = 0, lse = -inf
 *   lse      (batch, q_heads) fp32 base-2 log-sum-exp (scale included), or NULL
 *   o = softmax(q . K^T * scale) V over the valid keys.  G in {1, 2, 4, 8,
 *   16}, head_dim 64 or 128.  Split-KV with a combine pass; the partials live
 *   in `workspace`, at least tk_gqa_decode_workspace_bytes(...) bytes.
 *   G = 4, 8 or 16 runs the tensor-core kernel (128-key
 *   tiles by TMA, S^T = K q^T and O^T = V^T P^T on tcgen05); the rest the
 *   CUDA-core kernel (64-key chunks by bulk copy). */
TK_API size_t tk_gqa_decode_workspace_bytes(int64_t batch, int64_t q_heads, int64_t seq_kv, int64_t head_dim);
TK_API int tk_gqa_decode(const void* q, const void* k, const void* v, const int32_t* kv_lens, void* o, float* lse,
                         void* workspace, size_t workspace_bytes, int64_t batch, int64_t q_heads,
                         int64_t kv_heads, int64_t seq_kv, int64_t head_dim, int dtype, float scale, void* stream);
/* Process-wide choice of the decode kernel: -1 (default) tensor cores where
 * supported, 0 always the CUDA-core kernel, 1 the same as -1.  For A/B
 * measurements and tests; returns TK_ERR_INVALID_ARGUMENT otherwise. */
TK_API int tk_gqa_decode_set_path(int mode);

/* Bytes of the fp32 dQ accumulator tk_attn_bwd needs (0 on bad sizes). */
TK_API size_t tk_attn_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim);

/* Synchronise `stream`, then read and clear the current device's status
 * word (TK_OK when no kernel reported an error since the last read). */
TK_API int tk_attn_device_status(int* status_out, void* stream);

/* Upper bound, in nanoseconds, of every wait inside the kernels (default
 * 2e9).  A wait that runs out records TK_ERR_DEVICE_TIMEOUT and the kernel
 * drains and exits instead of hanging. */
TK_API int tk_attn_set_wait_timeout_ns(unsigned long long timeout_ns);

/* Launch a one-CTA kernel that waits on a barrier nothing ever arrives at,
 * bounded by timeout_ns: exercises the device-timeout path without any
 * fault.  The status word then reads TK_ERR_DEVICE_TIMEOUT. */
TK_API int tk_attn_selftest_wait_timeout(unsigned long long timeout_ns, void* stream);

/* Human-readable name of a status code. */
TK_API const char* tk_attn_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* TKLAB_ATTN_H_ */
