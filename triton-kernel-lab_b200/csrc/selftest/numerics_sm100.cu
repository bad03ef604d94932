// Test-only library (libtklab_selftest.so): evaluates the FMA-pipe base-2
// exponential of the softmax phases (exp2_fma_pair) on arbitrary inputs, so
// a test can check it against its stated error bound and clamp.
#include "../sm100_primitives.cuh"
#include "tklab_selftest_impl.h"

namespace tk {
namespace {

__global__ void exp2_fma_pair_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  const int64_t pairs = (n + 1) / 2;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e0 = 2 * i;
    const bool has_hi = e0 + 1 < n;
    const float x0 = x[e0];
    const float x1 = has_hi ? x[e0 + 1] : x0;
    float p0, p1;
    exp2_fma_pair(x0, x1, p0, p1);
    y[e0] = p0;
    if (has_hi) y[e0 + 1] = p1;
  }
}

}  // namespace

int launch_exp2_fma_pair(const float* x, float* y, int64_t n, cudaStream_t stream) {
  const int64_t pairs = (n + 1) / 2;
  const int threads = 256;
  const int64_t blocks64 = (pairs + threads - 1) / threads;
  const int blocks = static_cast<int>(blocks64 < 4096 ? blocks64 : 4096);
  exp2_fma_pair_kernel<<<blocks, threads, 0, stream>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace tk
