// Backward helper kernels (HBM-bound, no tensor cores):
//   * preprocess: delta[row] = sum_d O[row, d] * dO[row, d] in fp32, and the
//     fp32 dQ accumulator cleared in the same pass.  Semantics follow the
//     reference `_attn_bwd_preprocess_kernel`
//     (src/tklab/kernels/flash_attention.py:368-395).
//   * dq convert: dQ = dtype(dq_accum) once every key tile has added its share.
//   * a wait self-test that waits on an mbarrier nothing arrives at, so the
//     bounded-wait / error-status path can be exercised without a fault.
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

constexpr int kPreThreads = 256;

__device__ __forceinline__ float dot8(uint4 a, uint4 b, bool bf16) {
  const uint32_t av[4] = {a.x, a.y, a.z, a.w};
  const uint32_t bv[4] = {b.x, b.y, b.z, b.w};
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 fa, fb;
    if (bf16) {
      fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&av[i]));
      fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bv[i]));
    } else {
      fa = __half22float2(*reinterpret_cast<const __half2*>(&av[i]));
      fb = __half22float2(*reinterpret_cast<const __half2*>(&bv[i]));
    }
    acc = fmaf(fa.x, fb.x, acc);
    acc = fmaf(fa.y, fb.y, acc);
  }
  return acc;
}

// Each group of G = DP/8 threads owns one row of d8 = head_dim/8 16-byte
// chunks (d8 <= G; DP is 64, 128 or 256, the padded width); thread g of the group
// reads chunk g of O and dO (128-bit loads) and clears the matching 32 bytes
// of the dQ accumulator, threads g >= d8 idle.
template <int DP>
__global__ void __launch_bounds__(kPreThreads)
    attn_bwd_pre_kernel(const uint4* __restrict__ o, const uint4* __restrict__ d_o,
                        float* __restrict__ delta, float4* __restrict__ dq_accum, long long rows, int d8,
                        int bf16) {
  constexpr int kGroup = DP / 8;
  const long long tid = static_cast<long long>(blockIdx.x) * kPreThreads + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * kPreThreads;
  const int g = threadIdx.x % kGroup;
  // Uniform trip count across the warp so the shuffles below stay converged.
  const long long total = rows * kGroup;
  const long long iters = (total + stride - 1) / stride;
  for (long long it = 0; it < iters; ++it) {
    const long long idx = tid + it * stride;
    const bool live = idx < total;
    const long long row = idx / kGroup;
    float part = 0.0f;
    if (live && g < d8) {
      const uint4 a = o[row * d8 + g];
      const uint4 b = d_o[row * d8 + g];
      part = dot8(a, b, bf16 != 0);
      if (dq_accum != nullptr) {
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        dq_accum[row * (2 * d8) + 2 * g] = z;
        dq_accum[row * (2 * d8) + 2 * g + 1] = z;
      }
    }
#pragma unroll
    for (int off = kGroup / 2; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    if (live && g == 0) delta[row] = part;
  }
}

__global__ void __launch_bounds__(256)
    dq_convert_kernel(const float4* __restrict__ src, uint4* __restrict__ dst, long long n8,
                      int bf16) {
  const long long stride = static_cast<long long>(gridDim.x) * 256;
  for (long long i = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x; i < n8; i += stride) {
    const float4 a = src[2 * i];
    const float4 b = src[2 * i + 1];
    uint4 w;
    if (bf16) {
      w.x = pack2<true>(a.x, a.y);
      w.y = pack2<true>(a.z, a.w);
      w.z = pack2<true>(b.x, b.y);
      w.w = pack2<true>(b.z, b.w);
    } else {
      w.x = pack2<false>(a.x, a.y);
      w.y = pack2<false>(a.z, a.w);
      w.z = pack2<false>(b.x, b.y);
      w.w = pack2<false>(b.z, b.w);
    }
    dst[i] = w;
  }
}

__global__ void wait_timeout_selftest_kernel(unsigned long long timeout_ns, int* status) {
  __shared__ uint64_t bar;
  __shared__ CtaControl ctl;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    ctl.abort = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait must give up after timeout_ns.
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &ctl, timeout_ns, status, 15);
  __syncthreads();
}

int grid_for(long long work, int threads) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();  // a launch on a device that cannot be queried reports its own error
    sms = 148;
  }
  long long blocks = (work + threads - 1) / threads;
  const long long cap = static_cast<long long>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

}  // namespace

int launch_attn_bwd_pre(const BwdPreArgs& a) {
  const long long rows = a.BH * a.S;
  if (a.D < 8 || a.D > 256 || a.D % 8 != 0) return kErrUnsupported;
  const int d8 = static_cast<int>(a.D / 8);
  if (a.D > 128) {
    const int grid = grid_for(rows * 32, kPreThreads);
    attn_bwd_pre_kernel<256><<<grid, kPreThreads, 0, a.stream>>>(
        static_cast<const uint4*>(a.o), static_cast<const uint4*>(a.d_o), a.delta,
        reinterpret_cast<float4*>(a.dq_accum), rows, d8, a.bf16 ? 1 : 0);
  } else if (a.D <= 64) {
    const int grid = grid_for(rows * 8, kPreThreads);
    attn_bwd_pre_kernel<64><<<grid, kPreThreads, 0, a.stream>>>(
        static_cast<const uint4*>(a.o), static_cast<const uint4*>(a.d_o), a.delta,
        reinterpret_cast<float4*>(a.dq_accum), rows, d8, a.bf16 ? 1 : 0);
  } else {
    const int grid = grid_for(rows * 16, kPreThreads);
    attn_bwd_pre_kernel<128><<<grid, kPreThreads, 0, a.stream>>>(
        static_cast<const uint4*>(a.o), static_cast<const uint4*>(a.d_o), a.delta,
        reinterpret_cast<float4*>(a.dq_accum), rows, d8, a.bf16 ? 1 : 0);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_attn_dq_convert(const DqConvertArgs& a) {
  if (a.n % 8 != 0) return kErrInvalidArgument;
  const long long n8 = a.n / 8;
  const int grid = grid_for(n8, 256);
  dq_convert_kernel<<<grid, 256, 0, a.stream>>>(reinterpret_cast<const float4*>(a.dq_accum),
                                                static_cast<uint4*>(a.dq), n8, a.bf16 ? 1 : 0);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_wait_timeout_selftest(unsigned long long timeout_ns, int* status, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(timeout_ns, status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace tk
