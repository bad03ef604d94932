// Rotate-half rotary position embedding (RoPE) for the attention kernels.
//
// Semantics follow the reference `_rope_forward_kernel` /
// `_rope_backward_kernel` (src/tklab/kernels/rope.py:27-74, :77-160): for a
// row x at position p with half width h and angle tables cos, sin of shape
// (positions, h), in fp32 and rounded to the element type on output,
//   out[c]     = x[c] cos[p][c] - x[c+h] sin[p][c]
//   out[c + h] = x[c+h] cos[p][c] + x[c] sin[p][c]
// and the transpose (the backward of the rotation) negates the sine.
//
// Here the row is one (batch, head, position) row of Q or K, the tables are
// indexed by the position only (shared across batch and heads) and are fp32.
#pragma once

#include "sm100_primitives.cuh"

namespace tk {

// Eight 16-bit elements (one 16-byte chunk) to fp32 and back.
template <bool kBf16>
__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (kBf16) {
      f[2 * i] = __uint_as_float(u[i] << 16);
      f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    } else {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
}

template <bool kBf16>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack2<kBf16>(f[0], f[1]), pack2<kBf16>(f[2], f[3]), pack2<kBf16>(f[4], f[5]),
                    pack2<kBf16>(f[6], f[7]));
}

// Rotate eight (first, second) pairs in place with the angles of columns
// c..c+7 of position row `cs` / `sn` (fp32, 32-byte aligned).  kTranspose
// applies the inverse rotation.
template <bool kTranspose>
__device__ __forceinline__ void rope_rotate8(float (&a)[8], float (&b)[8], const float* cs, const float* sn) {
  const float4 c0 = *reinterpret_cast<const float4*>(cs);
  const float4 c1 = *reinterpret_cast<const float4*>(cs + 4);
  const float4 s0 = *reinterpret_cast<const float4*>(sn);
  const float4 s1 = *reinterpret_cast<const float4*>(sn + 4);
  const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (kTranspose) s[i] = -s[i];
    const float x1 = a[i], x2 = b[i];
    a[i] = x1 * c[i] - x2 * s[i];
    b[i] = x2 * c[i] + x1 * s[i];
  }
}

// Rotate, in shared memory, row r of a 128-row tile stored in the
// 128-byte-swizzled column-block layout (D = 64 or 128 columns), whose
// position is `pos` (rows at or past `S`, zero-filled by the tile load, are
// left alone).  Column c pairs with c + D/2: for D = 128 the two 16-byte
// chunks sit at the same offset of the two column blocks, for D = 64 in
// chunks k and k + 4 of the one block.  One thread rotates its whole row
// (the calling warpgroup has a thread per row and registers to keep every
// load of the row in flight).
template <int D, bool kBf16>
__device__ __forceinline__ void rope_rotate_row(uint8_t* tile, int r, int pos, int S, const float* __restrict__ cos_t,
                                                const float* __restrict__ sin_t) {
  constexpr int kHalf = D / 2;
  if (pos >= S) return;
  const float* cs = cos_t + static_cast<size_t>(pos) * kHalf;
  const float* sn = sin_t + static_cast<size_t>(pos) * kHalf;
#pragma unroll
  for (int k = 0; k < kHalf / 8; ++k) {
    uint4* pa = reinterpret_cast<uint4*>(tile + swz_offset(r, 8 * k, kTileRows));
    uint4* pb = reinterpret_cast<uint4*>(tile + swz_offset(r, 8 * k + kHalf, kTileRows));
    float a[8], b[8];
    unpack8<kBf16>(*pa, a);
    unpack8<kBf16>(*pb, b);
    rope_rotate8<false>(a, b, cs + 8 * k, sn + 8 * k);
    *pa = pack8<kBf16>(a);
    *pb = pack8<kBf16>(b);
  }
}

}  // namespace tk
