// tk_attn_bwd_noalloc: the attention backward for callers that cannot
// allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits or unsafe —
// under a host framework or runtime that owns every device byte through its
// own pool and forbids allocations behind its back, inside a plugin whose
// host gives it no allocator, or in a latency-critical loop where an
// allocation could synchronise the device.  The regular backward
// (tk_attn_bwd_pre + tk_attn_bwd) needs two scratch buffers from the caller:
// delta (B*H*S floats) and the fp32 dQ accumulator (B*H*S*D floats).  This
// entry point takes the same inputs and outputs but keeps that scratch in a
// fixed array compiled into the library, so it allocates nothing.  It
// accepts head_dim 64 or 128.
//
// Limits and sharing:
//   * capacity: kScratchFloats = 16 Mi floats (64 MiB).  A problem fits when
//     batch*heads*seq*(head_dim + 1) <= 16,777,216; larger ones are rejected
//     with TK_ERR_TOO_LARGE before anything is launched.  Every GPU on which
//     the library's module is loaded holds these 64 MiB until the process
//     exits.
//   * the array is shared by every call on a device and keeps the last
//     call's contents.  The dQ accumulator is cleared at the start of each
//     call (by the preprocessing kernel, which also rewrites delta), so
//     successive calls are independent — but two calls whose kernels
//     overlap on the GPU (different streams, no ordering between them) race
//     on the same scratch and corrupt each other's dQ.  Order such calls on
//     one stream or with events.
//   * the first call on a device looks up the device address of the array
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture.  The 64 MiB are committed
//     when the library's module is loaded on the device — with lazy module
//     loading, at that first call — and if the device cannot hold them the
//     call returns TK_ERR_OUT_OF_MEMORY (the CUDA error is cleared, so later
//     calls of the library do not see it).
//   * every argument is checked (pointers, shape, dtype, scale, alignment,
//     capacity) before the scratch is touched or anything is launched, so a
//     refused call never disturbs the scratch of an earlier call still
//     running.
#include <cmath>
#include <cstdint>
#include <mutex>

#include "../../include/tklab_attn.h"
#include "sm100_primitives.cuh"

namespace {

constexpr size_t kScratchFloats = size_t{1} << 24;  // 64 MiB of fp32

// Scratch for the no-allocation backward: the dQ accumulator first (16-byte
// vector atomics need its 256-byte alignment), delta right after it.  In host
// code this name is only a stand-in for the symbol: the kernels are handed
// the device address looked up below, never the host-side name.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return TK_ERR_NO_DRIVER;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    float* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();  // clear the sticky-free error so later launches do not report it
      return err == cudaErrorMemoryAllocation ? TK_ERR_OUT_OF_MEMORY : TK_ERR_NO_DRIVER;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return TK_OK;
}

}  // namespace

extern "C" int tk_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                   const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                   int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                   int dtype, int causal, float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || d_o == nullptr ||
      lse == nullptr || dq == nullptr || dk == nullptr || dv == nullptr)
    return TK_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || heads <= 0 || seq <= 0) return TK_ERR_INVALID_ARGUMENT;
  if (head_dim != 64 && head_dim != 128) return TK_ERR_UNSUPPORTED;
  if (dtype != TK_DTYPE_F16 && dtype != TK_DTYPE_BF16) return TK_ERR_UNSUPPORTED;
  if (!std::isfinite(scale) || scale <= 0.0f) return TK_ERR_INVALID_ARGUMENT;
  for (const void* p : {q, k, v, o, d_o, static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv)})
    if (reinterpret_cast<uintptr_t>(p) & 15u) return TK_ERR_MISALIGNED;
  if (reinterpret_cast<uintptr_t>(lse) & 3u) return TK_ERR_MISALIGNED;
  // Capacity check before anything touches the device.
  const size_t rows = static_cast<size_t>(batch) * static_cast<size_t>(heads) * static_cast<size_t>(seq);
  if (rows > kScratchFloats) return TK_ERR_TOO_LARGE;
  const size_t accum_floats = rows * static_cast<size_t>(head_dim);
  if (accum_floats + rows > kScratchFloats) return TK_ERR_TOO_LARGE;
  float* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  float* dq_accum = scratch;
  float* delta = scratch + accum_floats;  // accum_floats is a multiple of 64: stays aligned
  if (int rc = tk_attn_bwd_pre(o, d_o, delta, dq_accum, batch, heads, seq, head_dim, dtype, stream))
    return rc;
  return tk_attn_bwd(q, k, v, d_o, lse, delta, dq_accum, dq, dk, dv, batch, heads, seq, head_dim,
                     dtype, causal, scale, stream);
}
