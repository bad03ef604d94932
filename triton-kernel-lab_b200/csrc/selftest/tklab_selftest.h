/* C ABI of libtklab_selftest.so: test-only probes of the building blocks the
 * attention kernels rely on.  Not part of the attention library and not a
 * counterpart of anything in the reference; only the tests load it.  Status
 * codes are those of tklab_attn.h. */
#ifndef TKLAB_SELFTEST_H_
#define TKLAB_SELFTEST_H_

#include <stdint.h>

#if defined(__GNUC__)
#define TKS_API __attribute__((visibility("default")))
#else
#define TKS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* One 128 x n x 128 tcgen05 product in the operand form `mode` uses inside
 * the attention kernels, written as fp32 row-major c.
 *   mode 0: c[128][128] = a[128][128] . b[128][128]^T   (both K-major)
 *   mode 1: c[128][n]   = a[128][128] . b[128][n]       (a read from TMEM)
 *   mode 2: c[128][n]   = a[128][128]^T . b[128][n]     (both MN-major)
 *   mode 3: c[128][n]   = a[128][128] . b[128][n]       (a K-major, b MN-major)
 * n is 64 or 128 (ignored for mode 0). */
TKS_API int tk_selftest_umma(const void* a, const void* b, float* c, int mode, int n, int dtype, void* stream);

/* y[i] = the packed FMA-pipe base-2 exponential the softmax phases use
 * (exp2_fma_pair), evaluated on x[i], i < n.  x and y are device fp32. */
TKS_API int tk_selftest_exp2_fma(const float* x, float* y, int64_t n, void* stream);

/* Host-side view of the forward's key-split schedule
 * (csrc/attn_fwd_split_plan.h, the code the attention library runs), for
 * CPU tests.  tk_selftest_fwd_split_plan: 1 when a (bh, seq, head_dim,
 * causal) forward on a device with `sms` SMs is split, with out[0..5] =
 * chunk length in key tiles, chunks per item at most, units (CTAs), first
 * row of a multi-chunk item, workspace bytes, query tiles per work item;
 * 0 when it is not split.  No device is touched. */
TKS_API int tk_selftest_fwd_split_plan(int64_t bh, int64_t seq, int64_t head_dim, int causal, int sms,
                                       int64_t* out);

/* The forward kernel's decode of split unit u: out[0..2] = slab, query-tile
 * group, chunk.  Host code only. */
TKS_API void tk_selftest_fwd_split_decode(int u, int bh, int n_ctiles, int causal, int kt, int split_l, int* out);

/* Synchronise `stream`, then read and clear this library's device status
 * word (the first error a probe kernel recorded). */
TKS_API int tk_selftest_status(int* status_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TKLAB_SELFTEST_H_ */
