// Elementwise rotate-half RoPE kernels for the RoPE attention backward
// (HBM-bound: one read and one write of each element):
//   rope_rotate_kernel     out = R x or R^T x for (rows, D) 16-bit tensors
//                          (rows = batch*heads*S, position = row % S); out
//                          may alias x
//   dq_convert_rope_kernel dQ = R^T dQ_acc: the fp32 dQ accumulator of the
//                          rotated problem rotated back and rounded to dtype
// Semantics: rope_sm100.cuh (reference src/tklab/kernels/rope.py:27-160).
#include "attn_launch.h"
#include "rope_sm100.cuh"

namespace tk {
namespace {

// One thread per (row, pair of 16-byte chunks): a row has D/16 chunk pairs.
template <bool kBf16, bool kTranspose>
__global__ void __launch_bounds__(256) rope_rotate_kernel(const uint4* __restrict__ x, uint4* out,
                                                          const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t, long long rows, int S,
                                                          int D) {
  const int half = D / 2;
  const int pairs = half / 8;
  const long long n = rows * pairs;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long u = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; u < n; u += stride) {
    const long long row = u / pairs;
    const int k = static_cast<int>(u % pairs);
    const int pos = static_cast<int>(row % S);
    const long long ia = (row * D + 8 * k) / 8;  // uint4 index of the first-half chunk
    const long long ib = ia + half / 8;
    float a[8], b[8];
    unpack8<kBf16>(x[ia], a);
    unpack8<kBf16>(x[ib], b);
    const size_t t = static_cast<size_t>(pos) * half + 8 * k;
    rope_rotate8<kTranspose>(a, b, cos_t + t, sin_t + t);
    out[ia] = pack8<kBf16>(a);
    out[ib] = pack8<kBf16>(b);
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(256) dq_convert_rope_kernel(const float4* __restrict__ acc, uint4* __restrict__ dq,
                                                              const float* __restrict__ cos_t,
                                                              const float* __restrict__ sin_t, long long rows,
                                                              int S, int D) {
  const int half = D / 2;
  const int pairs = half / 8;
  const long long n = rows * pairs;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long u = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; u < n; u += stride) {
    const long long row = u / pairs;
    const int k = static_cast<int>(u % pairs);
    const int pos = static_cast<int>(row % S);
    const long long fa = (row * D + 8 * k) / 4;  // float4 index of the first-half chunk
    const long long fb = fa + half / 4;
    const float4 a0 = acc[fa], a1 = acc[fa + 1], b0 = acc[fb], b1 = acc[fb + 1];
    float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const size_t t = static_cast<size_t>(pos) * half + 8 * k;
    rope_rotate8<true>(a, b, cos_t + t, sin_t + t);
    dq[fa / 2] = pack8<kBf16>(a);
    dq[fb / 2] = pack8<kBf16>(b);
  }
}

int rope_grid(long long n) {
  const long long blocks = (n + 255) / 256;
  return static_cast<int>(blocks < 148LL * 16 ? (blocks > 0 ? blocks : 1) : 148LL * 16);
}

}  // namespace

int launch_rope_rotate(const RopeRotateArgs& a) {
  if (a.D != 64 && a.D != 128) return kErrUnsupported;
  const long long n = a.rows * (a.D / 16);
  const int grid = rope_grid(n);
  auto x = static_cast<const uint4*>(a.x);
  auto out = static_cast<uint4*>(a.out);
  if (a.bf16) {
    if (a.transpose)
      rope_rotate_kernel<true, true><<<grid, 256, 0, a.stream>>>(x, out, a.cos, a.sin, a.rows, a.S, a.D);
    else
      rope_rotate_kernel<true, false><<<grid, 256, 0, a.stream>>>(x, out, a.cos, a.sin, a.rows, a.S, a.D);
  } else {
    if (a.transpose)
      rope_rotate_kernel<false, true><<<grid, 256, 0, a.stream>>>(x, out, a.cos, a.sin, a.rows, a.S, a.D);
    else
      rope_rotate_kernel<false, false><<<grid, 256, 0, a.stream>>>(x, out, a.cos, a.sin, a.rows, a.S, a.D);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_dq_convert_rope(const DqConvertRopeArgs& a) {
  if (a.D != 64 && a.D != 128) return kErrUnsupported;
  const long long n = a.rows * (a.D / 16);
  const int grid = rope_grid(n);
  auto acc = static_cast<const float4*>(static_cast<const void*>(a.dq_accum));
  auto dq = static_cast<uint4*>(a.dq);
  if (a.bf16)
    dq_convert_rope_kernel<true><<<grid, 256, 0, a.stream>>>(acc, dq, a.cos, a.sin, a.rows, a.S, a.D);
  else
    dq_convert_rope_kernel<false><<<grid, 256, 0, a.stream>>>(acc, dq, a.cos, a.sin, a.rows, a.S, a.D);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace tk
