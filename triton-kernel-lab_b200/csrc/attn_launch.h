// Internal launch interface between the C ABI (attn_capi.cu) and the kernel
// translation units.  Host-only; plain structs, no torch types.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace tk {

struct FwdArgs {
  const CUtensorMap* tm_q;
  const CUtensorMap* tm_k;
  const CUtensorMap* tm_v;
  const CUtensorMap* tm_o;
  void* o;     // output, (B*H, S, D) 16-bit (persistent mode stores it directly)
  float* lse;  // nullptr: do not store the statistic
  int64_t BH, S, D;
  bool bf16;
  int causal;
  float scale_log2;
  unsigned long long timeout_ns;
  int* status;
  cudaStream_t stream;
  // Rotate-half RoPE tables (S, D/2) fp32 applied to Q and K inside the
  // kernel; both nullptr for plain attention.  Last, so positional
  // initialisers of the fields above stay valid.
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  // Optional scratch for the key-split schedule of problems with too few
  // work items to fill the device (attn_fwd_split_bytes gives the size; 0
  // or nullptr: never split).  Unused with RoPE.
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
};

// Forward for 128 < head_dim <= 256 (attn_fwd_d256_sm100.cu): a Q map with
// 128-row boxes, K and V maps with 64-row boxes; O (B*H, S, D) 16-bit is
// stored directly.
struct FwdD256Args {
  const CUtensorMap* tm_q;
  const CUtensorMap* tm_k;
  const CUtensorMap* tm_v;
  void* o;
  float* lse;
  int64_t BH, S, D;
  bool bf16;
  int causal;
  float scale_log2;
  unsigned long long timeout_ns;
  int* status;
  cudaStream_t stream;
};

struct BwdPreArgs {
  const void* o;
  const void* d_o;
  float* delta;
  float* dq_accum;  // zeroed here; nullptr skips the clear
  int64_t BH, S, D;
  bool bf16;
  cudaStream_t stream;
};

struct BwdArgs {
  const CUtensorMap* tm_q;
  const CUtensorMap* tm_k;
  const CUtensorMap* tm_v;
  const CUtensorMap* tm_do;
  const CUtensorMap* tm_dk;
  const CUtensorMap* tm_dv;
  const CUtensorMap* tm_dq;  // fp32 dQ accumulator, reduced into by TMA
  const float* lse;
  const float* delta;
  int64_t BH, S, D;
  bool bf16;
  int causal;
  float scale;       // softmax scale, applied to dQ and dK
  float scale_log2;  // scale * log2(e), used to recompute P
  unsigned long long timeout_ns;
  int* status;
  cudaStream_t stream;
};

// Backward for 128 < head_dim <= 256 (attn_bwd_d256_sm100.cu): Q and dO maps
// with 64-row boxes, K, dK and dV maps with 128-row boxes, the fp32 dQ
// accumulator map with {32, 64} boxes; V is read directly (row-major,
// (B*H, S, D) 16-bit) into tensor memory.
struct BwdD256Args {
  const CUtensorMap* tm_q;
  const CUtensorMap* tm_k;
  const CUtensorMap* tm_do;
  const CUtensorMap* tm_dk;
  const CUtensorMap* tm_dv;
  const CUtensorMap* tm_dq;
  const void* v;
  const float* lse;
  const float* delta;
  int64_t BH, S, D;
  bool bf16;
  int causal;
  float scale;
  float scale_log2;
  unsigned long long timeout_ns;
  int* status;
  cudaStream_t stream;
};

// Deterministic dQ kernel (query-stationary, no atomics).
struct BwdDqArgs {
  const CUtensorMap* tm_q;
  const CUtensorMap* tm_k;
  const CUtensorMap* tm_v;
  const CUtensorMap* tm_do;
  const CUtensorMap* tm_dq;  // 16-bit dQ output
  const float* lse;
  const float* delta;
  int64_t BH, S, D;
  bool bf16;
  int causal;
  float scale;
  float scale_log2;
  unsigned long long timeout_ns;
  int* status;
  cudaStream_t stream;
};

struct DqConvertArgs {
  const float* dq_accum;
  void* dq;
  int64_t n;  // elements
  bool bf16;
  cudaStream_t stream;
};

struct RopeRotateArgs {
  const void* x;
  void* out;  // may alias x
  const float* cos;
  const float* sin;
  int64_t rows;  // batch * heads * S
  int64_t S, D;
  bool bf16;
  bool transpose;
  cudaStream_t stream;
};

struct DqConvertRopeArgs {
  const float* dq_accum;
  void* dq;
  const float* cos;
  const float* sin;
  int64_t rows;  // batch * heads * S
  int64_t S, D;
  bool bf16;
  cudaStream_t stream;
};

struct GqaDecodeArgs {
  const void* q;       // (B, Hkv * G, D)
  const void* k;       // (B, Hkv, L, D)
  const void* v;       // (B, Hkv, L, D)
  const int* kv_lens;  // (B) valid keys per batch, or nullptr (all L)
  void* o;             // (B, Hkv * G, D)
  float* lse;          // (B, Hkv * G) base-2 log-sum-exp, or nullptr
  float* part_o;       // workspace (B, Hkv * G, splits, D)
  float* part_ml;      // workspace (B, Hkv * G, splits, 2)
  int64_t B, Hkv, G, L, D;
  int splits;  // from gqa_decode_splits (CUDA cores) or gqa_decode_splits_tc (tensor cores)
  bool bf16;
  float scale_log2;
  unsigned long long timeout_ns;
  int* status;
  cudaStream_t stream;
  // Tensor-core kernel (gqa_decode_tc_sm100.cu): maps over q as (B*Hq, D)
  // rows with 16-row boxes and over K, V as (B*Hkv, L, D) with 128-row boxes;
  // all nullptr selects the CUDA-core kernel.  Last, so positional
  // initialisers of the fields above stay valid.
  const CUtensorMap* tm_q = nullptr;
  const CUtensorMap* tm_k = nullptr;
  const CUtensorMap* tm_v = nullptr;
};

int launch_attn_fwd(const FwdArgs& a);
// Bytes of workspace the forward's key-split schedule needs for this problem
// on a device with `sms` SMs (0: the problem is not split).
size_t attn_fwd_split_bytes(int64_t BH, int64_t S, int64_t D, int causal, int sms);
int launch_attn_fwd_d256(const FwdD256Args& a);
int gqa_decode_splits(int64_t B, int64_t Hkv, int64_t L, int sm_count);
int gqa_decode_keys_per_split(int64_t L, int n_splits);
int launch_gqa_decode(const GqaDecodeArgs& a);
bool gqa_decode_tc_supported(int64_t D, int64_t G);
int gqa_decode_splits_tc(int64_t B, int64_t Hkv, int64_t L, int64_t D, int sm_count);
int launch_gqa_decode_tc_split(const GqaDecodeArgs& a);
int launch_rope_rotate(const RopeRotateArgs& a);
int launch_dq_convert_rope(const DqConvertRopeArgs& a);
int launch_attn_bwd_pre(const BwdPreArgs& a);
int launch_attn_bwd(const BwdArgs& a);
int launch_attn_bwd_d256(const BwdD256Args& a);
// The fused backward with its dQ path compiled out (dK and dV only; a.tm_dq
// is not read).
int launch_attn_bwd_dkdv(const BwdArgs& a);
int launch_attn_bwd_dq(const BwdDqArgs& a);
int launch_attn_dq_convert(const DqConvertArgs& a);
int launch_wait_timeout_selftest(unsigned long long timeout_ns, int* status, cudaStream_t stream);

// One-time set-up of a kernel on the current device, guarded by a mutex:
// checks the registers per thread the kernel was built with against
// `expect_regs` (when > 0: the setmaxnreg splits inside the kernels assume
// that exact launch allocation), raises its dynamic shared-memory limit to
// `smem_bytes`, and caches the device's SM count (returned through
// `sm_count` when not null).  Errors are cleared from the runtime's
// last-error slot before returning.
int prepare_kernel(const void* kernel, int smem_bytes, int expect_regs, int* sm_count);

}  // namespace tk
