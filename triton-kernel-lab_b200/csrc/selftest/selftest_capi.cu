// C ABI of the test-only library libtklab_selftest.so (selftest/tklab_selftest.h):
// argument checks, its own device status word and tensor maps, dispatch.
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "../../../include/tklab_attn.h"
#include "../attn_fwd_split_plan.h"
#include "../sm100_primitives.cuh"
#include "tklab_selftest.h"
#include "tklab_selftest_impl.h"

namespace {

__device__ int g_tks_status_word = 0;

constexpr int kMaxDevices = 64;
constexpr int kKernelSlots = 4;
int* g_status_ptr[kMaxDevices] = {};
bool g_attr_set[kMaxDevices][kKernelSlots] = {};
std::mutex g_mu;
constexpr unsigned long long kTimeoutNs = 2000000000ull;

int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= kMaxDevices) {
    cudaGetLastError();
    return tk::kErrNoDriver;
  }
  return tk::kOk;
}

int status_ptr(int** out) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tks_status_word) != cudaSuccess) {
      cudaGetLastError();
      return tk::kErrNoDriver;
    }
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  *out = g_status_ptr[dev];
  return tk::kOk;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D map over a row-major 128 x cols 16-bit matrix: box {64, 128}, 128-byte
// swizzle, as the attention kernels' operand tiles.
int make_map(CUtensorMap* map, const void* base, int64_t cols, int dtype) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (fn == nullptr) {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
              cudaSuccess &&
          q == cudaDriverEntryPointSuccess)
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  }
  if (fn == nullptr) return tk::kErrNoDriver;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), 128, 1};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 2), static_cast<cuuint64_t>(cols * 2 * 128)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype == TK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? tk::kOk : tk::kErrTensorMap;
}

}  // namespace

namespace tk {

int set_smem_attr_once(const void* kernel, int bytes, int slot) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (slot < 0 || slot >= kKernelSlots) return kErrInvalidArgument;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_attr_set[dev][slot]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
      cudaGetLastError();
      return kErrLaunch;
    }
    g_attr_set[dev][slot] = true;
  }
  return kOk;
}

}  // namespace tk

extern "C" {

int tk_selftest_umma(const void* a, const void* b, float* c, int mode, int n, int dtype, void* stream) {
  if (a == nullptr || b == nullptr || c == nullptr) return tk::kErrInvalidArgument;
  if (mode < 0 || mode > 3) return tk::kErrInvalidArgument;
  if (mode == 0) n = 128;
  if (n != 64 && n != 128) return tk::kErrUnsupported;
  if (dtype != TK_DTYPE_F16 && dtype != TK_DTYPE_BF16) return tk::kErrUnsupported;
  if (!aligned16(a) || !aligned16(b) || !aligned16(c)) return tk::kErrMisaligned;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  CUtensorMap ma, mb;
  if (int rc = make_map(&ma, a, 128, dtype)) return rc;
  if (int rc = make_map(&mb, b, n, dtype)) return rc;
  return tk::launch_umma_diag(&ma, &mb, static_cast<const uint32_t*>(a), c, mode, n, dtype == TK_DTYPE_BF16,
                              kTimeoutNs, status, static_cast<cudaStream_t>(stream));
}

int tk_selftest_exp2_fma(const float* x, float* y, int64_t n, void* stream) {
  if (x == nullptr || y == nullptr || n <= 0) return tk::kErrInvalidArgument;
  if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(y) & 3u)) return tk::kErrMisaligned;
  return tk::launch_exp2_fma_pair(x, y, n, static_cast<cudaStream_t>(stream));
}

int tk_selftest_fwd_split_plan(int64_t bh, int64_t seq, int64_t head_dim, int causal, int sms, int64_t* out) {
  if (out == nullptr || head_dim <= 0 || head_dim > 128) return 0;
  const tk::FwdKernelShape k = tk::fwd_kernel_shape(head_dim);
  tk::FwdSplitPlan p;
  if (!tk::plan_fwd_split_impl(k.kT, k.min_blocks, k.width, seq, bh, causal ? 1 : 0, sms, p)) return 0;
  out[0] = p.split_l;
  out[1] = p.cmax;
  out[2] = p.units;
  out[3] = p.row0;
  out[4] = static_cast<int64_t>(p.bytes);
  out[5] = k.kT;
  return 1;
}

void tk_selftest_fwd_split_decode(int u, int bh, int n_ctiles, int causal, int kt, int split_l, int* out) {
  if (out != nullptr) tk::fwd_split_decode(u, bh, n_ctiles, causal, kt, split_l, out);
}

int tk_selftest_status(int* status_out, void* stream) {
  if (status_out == nullptr) return tk::kErrInvalidArgument;
  int* status = nullptr;
  if (int rc = status_ptr(&status)) return rc;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return tk::kErrLaunch;
  int value = 0;
  if (cudaMemcpy(&value, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return tk::kErrLaunch;
  const int zero = 0;
  if (cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return tk::kErrLaunch;
  *status_out = value;
  return tk::kOk;
}

}  // extern "C"
