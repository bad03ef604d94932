// Test-only library (libtklab_selftest.so), not part of the attention
// library: a diagnostic single-tile tcgen05 GEMM.  It runs one 128 x n x 128 product with
// exactly the operand forms the attention kernels use, so a test can check
// each convention (descriptor fields, swizzle, TMEM A-operand packing) in
// isolation against a host matmul:
//   mode 0  C = A B^T   A [128][128] K-major, B [128][128] K-major   (S = Q K^T)
//   mode 1  C = A B     A from TMEM (packed 16-bit), B [128][n] MN-major  (O += P V)
//   mode 2  C = A^T B   A stored [128 k][128 m] MN-major, B [128][n] MN-major  (dQ = dS K)
//   mode 3  C = A B     A [128][128] K-major, B [128][n] MN-major    (dK += dS^T Q)
#include "../sm100_primitives.cuh"
#include "tklab_selftest_impl.h"

namespace tk {
namespace {

constexpr int kDiagSmem = 32768 * 2 + 1024;

__global__ void __launch_bounds__(128, 1)
    umma_diag_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const uint32_t* __restrict__ a_words, float* __restrict__ c, int mode, int n,
                     int bf16, unsigned long long timeout_ns, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  uint8_t* sA = smem;
  uint8_t* sB = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint64_t* bar_load = bars;
  uint64_t* bar_mma = bars + 1;
  uint64_t* bar_a = bars + 2;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + 65536 + 64);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(bar_load, 1);
    mbar_init(bar_mma, 1);
    mbar_init(bar_a, 4);
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc(&ctl->tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int row = warp * 32 + lane;

  if (threadIdx.x == 0) {
    const int a_blocks = 2;
    const int b_blocks = (mode == 0) ? 2 : n / 64;
    mbar_arrive_expect_tx(bar_load, (a_blocks + b_blocks) * kBlockBytes);
    for (int b = 0; b < a_blocks; ++b) tma_load_3d(sA + b * kBlockBytes, &tm_a, bar_load, b * 64, 0, 0);
    for (int b = 0; b < b_blocks; ++b) tma_load_3d(sB + b * kBlockBytes, &tm_b, bar_load, b * 64, 0, 0);
  }
  if (mode == 1) {
    // Every thread writes its own A row into TMEM columns [128, 192).
    uint32_t w0[32], w1[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      w0[i] = a_words[row * 64 + i];
      w1[i] = a_words[row * 64 + 32 + i];
    }
    tmem_st32(t_lane + 128, w0);
    tmem_st32(t_lane + 160, w1);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_a);
  }
  if (threadIdx.x == 0) {
    bool ok = mbar_wait(bar_load, 0, ctl, timeout_ns, status, 20);
    if (ok && mode == 1) ok = mbar_wait(bar_a, 0, ctl, timeout_ns, status, 21);
    if (ok) {
      tc_fence_after();
      const uint32_t fmt = bf16 ? 1u : 0u;
      const uint32_t a_s = smem_u32(sA), b_s = smem_u32(sB);
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t acc = kk > 0 ? 1u : 0u;
        if (mode == 0) {
          umma_ss(tmem, sdesc_kmajor(a_s, 128, kk * 16), sdesc_kmajor(b_s, 128, kk * 16),
                  idesc_f16(fmt, 128, 128, 0, 0), acc);
        } else if (mode == 1) {
          umma_ts(tmem, tmem + 128 + kk * 8, sdesc_mnmajor(b_s, 128, kk * 16), idesc_f16(fmt, 128, n, 0, 1),
                  acc);
        } else if (mode == 2) {
          umma_ss(tmem, sdesc_mnmajor(a_s, 128, kk * 16), sdesc_mnmajor(b_s, 128, kk * 16),
                  idesc_f16(fmt, 128, n, 1, 1), acc);
        } else {
          umma_ss(tmem, sdesc_kmajor(a_s, 128, kk * 16), sdesc_mnmajor(b_s, 128, kk * 16),
                  idesc_f16(fmt, 128, n, 0, 1), acc);
        }
      }
      umma_commit(bar_mma);
    }
  }
  __syncwarp();
  if (mbar_wait(bar_mma, 0, ctl, timeout_ns, status, 22)) {
    tc_fence_after();
    const int ncols = (mode == 0) ? 128 : n;
    for (int cb = 0; cb < ncols / 32; ++cb) {
      uint32_t v[32];
      tmem_ld32(t_lane + cb * 32, v);
      tmem_wait_ld();
      reg_fence(v);
      for (int i = 0; i < 32; ++i) c[row * ncols + cb * 32 + i] = __uint_as_float(v[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

int launch_umma_diag(const CUtensorMap* tm_a, const CUtensorMap* tm_b, const uint32_t* a_words, float* c,
                     int mode, int n, bool bf16, unsigned long long timeout_ns, int* status,
                     cudaStream_t stream) {
  if (int rc = set_smem_attr_once(reinterpret_cast<const void*>(umma_diag_kernel), kDiagSmem, 0)) return rc;
  umma_diag_kernel<<<1, 128, kDiagSmem, stream>>>(*tm_a, *tm_b, a_words, c, mode, n, bf16 ? 1 : 0,
                                                  timeout_ns, status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace tk
