// C ABI of libtklab_attn.so (declared in include/tklab_attn.h): argument
// validation, TMA tensor-map encoding and kernel dispatch.  Host code only
// besides the per-device status word.
#include <cudaTypedefs.h>

#include <climits>
#include <cmath>
#include <cstdint>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/tklab_attn.h"
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace {

// Device status word: kernels record the first error they hit here.
__device__ int g_tk_status_word = 0;

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
std::mutex g_mu;
unsigned long long g_timeout_ns = 2000000000ull;
// GQA decode kernel choice: -1 tensor cores where supported (G = 4, 8 or
// 16), 0 always the CUDA-core kernel, 1 the same as -1.
int g_decode_path = -1;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int status_ptr(int** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return tk::kErrNoDriver;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tk_status_word) != cudaSuccess) {
      cudaGetLastError();
      return tk::kErrNoDriver;
    }
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  *out = g_status_ptr[dev];
  return tk::kOk;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int dtype,
                int64_t max_head_dim = 128) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return tk::kErrInvalidArgument;
  // Any head_dim up to the kernel's width whose rows are 16-byte multiples:
  // the kernels for 64, 128 and 256 run it with the tensor maps declaring the
  // true width (loads zero-fill the missing columns, stores and reductions
  // clip them).  Only the forward has a 256-wide kernel.
  if (head_dim < 8 || head_dim > max_head_dim || head_dim % 8 != 0) return tk::kErrUnsupported;
  if (dtype != TK_DTYPE_F16 && dtype != TK_DTYPE_BF16) return tk::kErrUnsupported;
  const int64_t bh = batch * heads;
  if (bh > INT_MAX || seq > INT_MAX) return tk::kErrTooLarge;
  const int64_t tiles = (seq + 127) / 128;
  if (tiles * bh > INT_MAX) return tk::kErrTooLarge;
  return tk::kOk;
}

// 3-D map over a contiguous (B*H, S, D) 16-bit tensor: box {64, box_rows, 1}
// (128 rows unless a kernel tiles the sequence by 64), 128-byte swizzle, zero
// fill outside the tensor (ragged S tails).
int make_map(CUtensorMap* map, const void* base, int64_t bh, int64_t seq, int64_t head_dim,
             int dtype, uint32_t box_rows = 128) {
  auto fn = encode_fn();
  if (fn == nullptr) return tk::kErrNoDriver;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(seq),
                        static_cast<cuuint64_t>(bh)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim * 2),
                           static_cast<cuuint64_t>(seq * head_dim * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map,
                  dtype == TK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? tk::kOk : tk::kErrTensorMap;
}

// 3-D map over the contiguous fp32 (B*H, S, D) dQ accumulator: box
// {32, 128, 1} (128-byte rows) with the 128-byte swizzle; used as the target
// of TMA bulk reduce-add.
int make_map_f32(CUtensorMap* map, const float* base, int64_t bh, int64_t seq, int64_t head_dim,
                 uint32_t box_rows = 128) {
  auto fn = encode_fn();
  if (fn == nullptr) return tk::kErrNoDriver;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(seq),
                        static_cast<cuuint64_t>(bh)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim * 4),
                           static_cast<cuuint64_t>(seq * head_dim * 4)};
  cuuint32_t box[3] = {32, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? tk::kOk : tk::kErrTensorMap;
}

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace

namespace tk {

int prepare_kernel(const void* kernel, int smem_bytes, int expect_regs, int* sm_count) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    cudaGetLastError();
    return kErrNoDriver;
  }
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> prepared;  // (kernel, device) -> SM count
  std::lock_guard<std::mutex> lock(mu);
  auto it = prepared.find({kernel, dev});
  if (it == prepared.end()) {
    if (expect_regs > 0) {
      cudaFuncAttributes attr;
      if (cudaFuncGetAttributes(&attr, kernel) != cudaSuccess || attr.numRegs != expect_regs) {
        cudaGetLastError();
        return kErrLaunch;
      }
    }
    int sms = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
      cudaGetLastError();
      return kErrLaunch;
    }
    it = prepared.emplace(std::make_pair(kernel, dev), sms).first;
  }
  if (sm_count != nullptr) *sm_count = it->second;
  return kOk;
}

}  // namespace tk

extern "C" {

int tk_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int64_t batch,
                int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                void* stream) {
  return tk_attn_fwd_ws(q, k, v, o, lse, batch, heads, seq, head_dim, dtype, causal, scale, nullptr, 0, stream);
}

size_t tk_attn_fwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int dtype,
                                   int causal) {
  if (check_shape(batch, heads, seq, head_dim, dtype, 256) != tk::kOk || head_dim > 128) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return tk::attn_fwd_split_bytes(batch * heads, seq, head_dim, causal ? 1 : 0, sms);
}

int tk_attn_fwd_ws(const void* q, const void* k, const void* v, void* o, float* lse, int64_t batch,
                   int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype, 256)) return rc;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return tk::kErrMisaligned;
  if (lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u)) return tk::kErrMisaligned;
  if (workspace == nullptr) workspace_bytes = 0;
  if (workspace_bytes > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255u)) return tk::kErrMisaligned;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  const int64_t bh = batch * heads;
  CUtensorMap mq, mk, mv, mo;
  if (head_dim > 128) {
    // 136..256: one 128-row query tile per CTA against 64-key tiles.
    if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype)) return rc;
    if (int rc = make_map(&mk, k, bh, seq, head_dim, dtype, 64)) return rc;
    if (int rc = make_map(&mv, v, bh, seq, head_dim, dtype, 64)) return rc;
    tk::FwdD256Args a{&mq, &mk, &mv, o, lse, bh, seq, head_dim, dtype == TK_DTYPE_BF16, causal ? 1 : 0,
                      scale * kLog2e, g_timeout_ns, status, static_cast<cudaStream_t>(stream)};
    return tk::launch_attn_fwd_d256(a);
  }
  if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mk, k, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mv, v, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mo, o, bh, seq, head_dim, dtype)) return rc;
  tk::FwdArgs a{&mq, &mk, &mv, &mo, o, lse, bh, seq, head_dim, dtype == TK_DTYPE_BF16,
                causal ? 1 : 0, scale * kLog2e, g_timeout_ns, status,
                static_cast<cudaStream_t>(stream)};
  a.workspace = workspace_bytes > 0 ? workspace : nullptr;
  a.workspace_bytes = workspace_bytes;
  return tk::launch_attn_fwd(a);
}

int tk_attn_bwd_pre(const void* o, const void* d_o, float* delta, float* dq_accum, int64_t batch,
                    int64_t heads, int64_t seq, int64_t head_dim, int dtype, void* stream) {
  if (o == nullptr || d_o == nullptr || delta == nullptr) return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype, 256)) return rc;
  if (!aligned16(o) || !aligned16(d_o)) return tk::kErrMisaligned;
  if (reinterpret_cast<uintptr_t>(delta) & 3u) return tk::kErrMisaligned;
  if (dq_accum != nullptr && !aligned16(dq_accum)) return tk::kErrMisaligned;
  tk::BwdPreArgs a{o, d_o, delta, dq_accum, batch * heads, seq, head_dim, dtype == TK_DTYPE_BF16,
                   static_cast<cudaStream_t>(stream)};
  return tk::launch_attn_bwd_pre(a);
}

int tk_attn_bwd_fused(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                      const float* delta, float* dq_accum, void* dk, void* dv, int64_t batch,
                      int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                      void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || d_o == nullptr || lse == nullptr ||
      delta == nullptr || dq_accum == nullptr || dk == nullptr || dv == nullptr)
    return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype, 256)) return rc;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(d_o) || !aligned16(dk) ||
      !aligned16(dv) || !aligned16(dq_accum))
    return tk::kErrMisaligned;
  if ((reinterpret_cast<uintptr_t>(lse) & 3u) || (reinterpret_cast<uintptr_t>(delta) & 3u))
    return tk::kErrMisaligned;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  const int64_t bh = batch * heads;
  CUtensorMap mq, mk, mv, mdo, mdk, mdv, mdq;
  if (head_dim > 128) {
    // 136..256: two CTAs per 128-key tile, one head-dim half each; 64-query steps.
    if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype, 64)) return rc;
    if (int rc = make_map(&mk, k, bh, seq, head_dim, dtype)) return rc;
    if (int rc = make_map(&mdo, d_o, bh, seq, head_dim, dtype, 64)) return rc;
    if (int rc = make_map(&mdk, dk, bh, seq, head_dim, dtype)) return rc;
    if (int rc = make_map(&mdv, dv, bh, seq, head_dim, dtype)) return rc;
    if (int rc = make_map_f32(&mdq, dq_accum, bh, seq, head_dim, 64)) return rc;
    tk::BwdD256Args a{&mq, &mk, &mdo, &mdk, &mdv, &mdq, v, lse, delta, bh, seq, head_dim,
                      dtype == TK_DTYPE_BF16, causal ? 1 : 0, scale, scale * kLog2e, g_timeout_ns, status,
                      static_cast<cudaStream_t>(stream)};
    return tk::launch_attn_bwd_d256(a);
  }
  if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mk, k, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mv, v, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdo, d_o, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdk, dk, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdv, dv, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map_f32(&mdq, dq_accum, bh, seq, head_dim)) return rc;
  tk::BwdArgs a{&mq,  &mk,   &mv,      &mdo,       &mdk,   &mdv, &mdq, lse, delta,
                bh,   seq,   head_dim, dtype == TK_DTYPE_BF16, causal ? 1 : 0, scale,
                scale * kLog2e, g_timeout_ns, status, static_cast<cudaStream_t>(stream)};
  return tk::launch_attn_bwd(a);
}

int tk_attn_fwd_rope(const void* q, const void* k, const void* v, const float* cos, const float* sin, void* k_rot,
                     void* o, float* lse, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int dtype,
                     int causal, float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || cos == nullptr || sin == nullptr ||
      k_rot == nullptr)
    return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype)) return rc;
  if (head_dim != 64 && head_dim != 128) return tk::kErrUnsupported;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(cos) || !aligned16(sin) ||
      !aligned16(k_rot))
    return tk::kErrMisaligned;
  if (lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u)) return tk::kErrMisaligned;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  const int64_t bh = batch * heads;
  // K once, into the caller's workspace (every CTA streams every K tile);
  // Q inside the kernel, once per query tile.
  tk::RopeRotateArgs rk{k, k_rot, cos, sin, bh * seq, seq, head_dim, dtype == TK_DTYPE_BF16, false,
                        static_cast<cudaStream_t>(stream)};
  if (int rc = tk::launch_rope_rotate(rk)) return rc;
  CUtensorMap mq, mk, mv, mo;
  if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mk, k_rot, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mv, v, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mo, o, bh, seq, head_dim, dtype)) return rc;
  tk::FwdArgs a{&mq, &mk, &mv, &mo, o, lse, bh, seq, head_dim, dtype == TK_DTYPE_BF16,
                causal ? 1 : 0, scale * kLog2e, g_timeout_ns, status,
                static_cast<cudaStream_t>(stream), cos, sin};
  return tk::launch_attn_fwd(a);
}

int tk_rope_rotate(const void* x, void* out, const float* cos, const float* sin, int64_t batch, int64_t heads,
                   int64_t seq, int64_t head_dim, int dtype, int transpose, void* stream) {
  if (x == nullptr || out == nullptr || cos == nullptr || sin == nullptr) return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype)) return rc;
  if (head_dim != 64 && head_dim != 128) return tk::kErrUnsupported;
  if (!aligned16(x) || !aligned16(out) || !aligned16(cos) || !aligned16(sin)) return tk::kErrMisaligned;
  tk::RopeRotateArgs a{x, out, cos, sin, batch * heads * seq, seq, head_dim, dtype == TK_DTYPE_BF16,
                       transpose != 0, static_cast<cudaStream_t>(stream)};
  return tk::launch_rope_rotate(a);
}

int tk_attn_dq_convert_rope(const float* dq_accum, void* dq, const float* cos, const float* sin, int64_t batch,
                            int64_t heads, int64_t seq, int64_t head_dim, int dtype, void* stream) {
  if (dq_accum == nullptr || dq == nullptr || cos == nullptr || sin == nullptr) return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype)) return rc;
  if (head_dim != 64 && head_dim != 128) return tk::kErrUnsupported;
  if (!aligned16(dq_accum) || !aligned16(dq) || !aligned16(cos) || !aligned16(sin)) return tk::kErrMisaligned;
  tk::DqConvertRopeArgs a{dq_accum, dq, cos, sin, batch * heads * seq, seq, head_dim, dtype == TK_DTYPE_BF16,
                          static_cast<cudaStream_t>(stream)};
  return tk::launch_dq_convert_rope(a);
}

size_t tk_gqa_decode_workspace_bytes(int64_t batch, int64_t q_heads, int64_t seq_kv, int64_t head_dim) {
  if (batch <= 0 || q_heads <= 0 || seq_kv <= 0 || head_dim <= 0) return 0;
  // Upper bound over every kv_heads and device: one split per 64-key chunk.
  const int64_t splits = (seq_kv + 63) / 64;
  const int64_t rows = batch * q_heads * splits;
  return static_cast<size_t>(rows) * static_cast<size_t>(head_dim + 2) * sizeof(float);
}

int tk_gqa_decode(const void* q, const void* k, const void* v, const int32_t* kv_lens, void* o, float* lse,
                  void* workspace, size_t workspace_bytes, int64_t batch, int64_t q_heads, int64_t kv_heads,
                  int64_t seq_kv, int64_t head_dim, int dtype, float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || workspace == nullptr)
    return tk::kErrInvalidArgument;
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || seq_kv <= 0) return tk::kErrInvalidArgument;
  if (q_heads % kv_heads != 0) return tk::kErrInvalidArgument;
  const int64_t group = q_heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8 && group != 16) return tk::kErrUnsupported;
  if (head_dim != 64 && head_dim != 128) return tk::kErrUnsupported;
  if (dtype != TK_DTYPE_F16 && dtype != TK_DTYPE_BF16) return tk::kErrUnsupported;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  if (batch > 65535 || kv_heads > 65535 || seq_kv > INT_MAX) return tk::kErrTooLarge;
  if (batch * kv_heads * seq_kv * head_dim > (int64_t{1} << 40)) return tk::kErrTooLarge;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(workspace))
    return tk::kErrMisaligned;
  if ((lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u)) ||
      (kv_lens != nullptr && (reinterpret_cast<uintptr_t>(kv_lens) & 3u)))
    return tk::kErrMisaligned;
  if (workspace_bytes < tk_gqa_decode_workspace_bytes(batch, q_heads, seq_kv, head_dim)) return tk::kErrTooLarge;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();  // do not leave the error for the next launch check
    return tk::kErrNoDriver;
  }
  const bool use_tc = g_decode_path != 0 && tk::gqa_decode_tc_supported(head_dim, group) &&
                      batch * q_heads <= INT_MAX;
  const int splits = use_tc ? tk::gqa_decode_splits_tc(batch, kv_heads, seq_kv, head_dim, sms)
                            : tk::gqa_decode_splits(batch, kv_heads, seq_kv, sms);
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + batch * q_heads * splits * head_dim;
  tk::GqaDecodeArgs a{q, k, v, kv_lens, o, lse, part_o, part_ml, batch, kv_heads, group, seq_kv, head_dim,
                      splits, dtype == TK_DTYPE_BF16, scale * kLog2e, g_timeout_ns, status,
                      static_cast<cudaStream_t>(stream)};
  CUtensorMap mq, mk, mv;
  if (use_tc) {
    if (int rc = make_map(&mq, q, 1, batch * q_heads, head_dim, dtype, 16)) return rc;
    if (int rc = make_map(&mk, k, batch * kv_heads, seq_kv, head_dim, dtype)) return rc;
    if (int rc = make_map(&mv, v, batch * kv_heads, seq_kv, head_dim, dtype)) return rc;
    a.tm_q = &mq;
    a.tm_k = &mk;
    a.tm_v = &mv;
  }
  return tk::launch_gqa_decode(a);
}

int tk_gqa_decode_set_path(int mode) {
  if (mode < -1 || mode > 1) return tk::kErrInvalidArgument;
  g_decode_path = mode;
  return tk::kOk;
}

int tk_attn_dq_convert(const float* dq_accum, void* dq, int64_t n, int dtype, void* stream) {
  if (dq_accum == nullptr || dq == nullptr || n <= 0 || n % 8 != 0) return tk::kErrInvalidArgument;
  if (dtype != TK_DTYPE_F16 && dtype != TK_DTYPE_BF16) return tk::kErrUnsupported;
  if (!aligned16(dq_accum) || !aligned16(dq)) return tk::kErrMisaligned;
  tk::DqConvertArgs c{dq_accum, dq, n, dtype == TK_DTYPE_BF16, static_cast<cudaStream_t>(stream)};
  return tk::launch_attn_dq_convert(c);
}

int tk_attn_bwd(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                const float* delta, float* dq_accum, void* dq, void* dk, void* dv, int64_t batch,
                int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                void* stream) {
  if (dq == nullptr) return tk::kErrInvalidArgument;
  if (!aligned16(dq)) return tk::kErrMisaligned;
  if (int rc = tk_attn_bwd_fused(q, k, v, d_o, lse, delta, dq_accum, dk, dv, batch, heads, seq,
                                 head_dim, dtype, causal, scale, stream))
    return rc;
  return tk_attn_dq_convert(dq_accum, dq, batch * heads * seq * head_dim, dtype, stream);
}

int tk_attn_bwd_dkdv(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                     const float* delta, void* dk, void* dv, int64_t batch, int64_t heads, int64_t seq,
                     int64_t head_dim, int dtype, int causal, float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || d_o == nullptr || lse == nullptr ||
      delta == nullptr || dk == nullptr || dv == nullptr)
    return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype)) return rc;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(d_o) || !aligned16(dk) || !aligned16(dv))
    return tk::kErrMisaligned;
  if ((reinterpret_cast<uintptr_t>(lse) & 3u) || (reinterpret_cast<uintptr_t>(delta) & 3u))
    return tk::kErrMisaligned;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  const int64_t bh = batch * heads;
  CUtensorMap mq, mk, mv, mdo, mdk, mdv;
  if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mk, k, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mv, v, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdo, d_o, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdk, dk, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdv, dv, bh, seq, head_dim, dtype)) return rc;
  tk::BwdArgs a{&mq,  &mk,   &mv,      &mdo,       &mdk,   &mdv, nullptr, lse, delta,
                bh,   seq,   head_dim, dtype == TK_DTYPE_BF16, causal ? 1 : 0, scale,
                scale * kLog2e, g_timeout_ns, status, static_cast<cudaStream_t>(stream)};
  return tk::launch_attn_bwd_dkdv(a);
}

int tk_attn_bwd_dq(const void* q, const void* k, const void* v, const void* d_o, const float* lse,
                   const float* delta, void* dq, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                   int dtype, int causal, float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || d_o == nullptr || lse == nullptr ||
      delta == nullptr || dq == nullptr)
    return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype)) return rc;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(d_o) || !aligned16(dq))
    return tk::kErrMisaligned;
  if ((reinterpret_cast<uintptr_t>(lse) & 3u) || (reinterpret_cast<uintptr_t>(delta) & 3u))
    return tk::kErrMisaligned;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  const int64_t bh = batch * heads;
  CUtensorMap mq, mk, mv, mdo, mdq;
  if (int rc = make_map(&mq, q, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mk, k, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mv, v, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdo, d_o, bh, seq, head_dim, dtype)) return rc;
  if (int rc = make_map(&mdq, dq, bh, seq, head_dim, dtype)) return rc;
  tk::BwdDqArgs a{&mq, &mk, &mv, &mdo, &mdq, lse, delta, bh, seq, head_dim, dtype == TK_DTYPE_BF16,
                  causal ? 1 : 0, scale, scale * kLog2e, g_timeout_ns, status,
                  static_cast<cudaStream_t>(stream)};
  return tk::launch_attn_bwd_dq(a);
}

int tk_attn_bwd_deterministic(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                              const float* lse, float* delta, void* dq, void* dk, void* dv, int64_t batch,
                              int64_t heads, int64_t seq, int64_t head_dim, int dtype, int causal, float scale,
                              void* stream) {
  // Everything the three launches check, before the first of them runs.
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || d_o == nullptr || lse == nullptr ||
      delta == nullptr || dq == nullptr || dk == nullptr || dv == nullptr)
    return tk::kErrInvalidArgument;
  if (int rc = check_shape(batch, heads, seq, head_dim, dtype)) return rc;
  if (!std::isfinite(scale) || scale <= 0.0f) return tk::kErrInvalidArgument;
  for (const void* p : {q, k, v, o, d_o, static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv)})
    if (!aligned16(p)) return tk::kErrMisaligned;
  if ((reinterpret_cast<uintptr_t>(lse) & 3u) || (reinterpret_cast<uintptr_t>(delta) & 3u))
    return tk::kErrMisaligned;
  if (int rc = tk_attn_bwd_pre(o, d_o, delta, nullptr, batch, heads, seq, head_dim, dtype, stream)) return rc;
  if (int rc = tk_attn_bwd_dkdv(q, k, v, d_o, lse, delta, dk, dv, batch, heads, seq, head_dim, dtype, causal,
                                scale, stream))
    return rc;
  return tk_attn_bwd_dq(q, k, v, d_o, lse, delta, dq, batch, heads, seq, head_dim, dtype, causal, scale, stream);
}

size_t tk_attn_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim) {
  if (batch <= 0 || heads <= 0 || seq <= 0 || head_dim <= 0) return 0;
  return static_cast<size_t>(batch) * static_cast<size_t>(heads) * static_cast<size_t>(seq) *
         static_cast<size_t>(head_dim) * sizeof(float);
}

int tk_attn_device_status(int* status_out, void* stream) {
  if (status_out == nullptr) return tk::kErrInvalidArgument;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return tk::kErrLaunch;
  int value = 0;
  if (cudaMemcpy(&value, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return tk::kErrLaunch;
  const int zero = 0;
  if (cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return tk::kErrLaunch;
  *status_out = value;
  return tk::kOk;
}

int tk_attn_set_wait_timeout_ns(unsigned long long timeout_ns) {
  if (timeout_ns == 0) return tk::kErrInvalidArgument;
  g_timeout_ns = timeout_ns;
  return tk::kOk;
}

int tk_attn_selftest_wait_timeout(unsigned long long timeout_ns, void* stream) {
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return tk::kErrInvalidArgument;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  return tk::launch_wait_timeout_selftest(timeout_ns, status, static_cast<cudaStream_t>(stream));
}

const char* tk_attn_status_string(int status) {
  switch (status & 0xff) {
    case TK_OK: return "ok";
    case TK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TK_ERR_UNSUPPORTED: return "unsupported dtype or head_dim";
    case TK_ERR_MISALIGNED: return "misaligned pointer";
    case TK_ERR_LAUNCH: return "CUDA launch failure";
    case TK_ERR_TENSOR_MAP: return "TMA tensor map encoding failed";
    case TK_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case TK_ERR_NO_DRIVER: return "CUDA driver or device unavailable";
    case TK_ERR_TOO_LARGE: return "problem size exceeds the supported range";
    case TK_ERR_OUT_OF_MEMORY: return "device memory could not be committed";
    default: return "unknown status";
  }
}

}  // extern "C"
