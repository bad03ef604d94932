// Grouped-query-attention decode on sm_100a: one query token per query head,
// Hq = G * Hkv query heads sharing each key/value head (query head h reads
// KV head h / G), a contiguous KV cache (B, Hkv, L, D) of 16-bit elements and
// an optional per-batch valid length.  The workload the reference specifies
// in docs/research/gqa_decode_model.md ("Canonical decode workload",
// "Semantic GQA mapping"): useful work 4 B Hq L D FLOPs against
// 2 sKV B Hkv L D bytes of unique KV payload, i.e. about 2G/sKV FLOP/B — an
// HBM-bound problem at every practical G, so no tensor cores (M = G <= 16).
//
// Split-KV (flash-decoding):
//   gqa_decode_split_kernel  one CTA per (batch, KV head, split): a split is
//     a run of 64-key sub-chunks (enough splits for about four CTAs per SM).
//     Per sub-chunk one thread copies its K and V rows into shared memory
//     with two bulk copies (cp.async.bulk, mbarrier completion, bounded
//     wait); the 4 warps then compute the G x 64 scores (lanes own D/32
//     head-dim columns, warp reductions), the online softmax per query head
//     in base 2, and P.V (lanes own head-dim columns, warps split the keys,
//     summed through shared memory at the end in a fixed order: decode is
//     bitwise reproducible).  Each query head's partial
//     (max m, sum l, unnormalised o) goes to a workspace.
//   gqa_decode_combine_kernel one warp per (batch, query head): merges the
//     chunk partials, o = sum 2^(m_s - M) o_s / sum 2^(m_s - M) l_s, writes
//     o in the input dtype and the base-2 log-sum-exp M + log2(sum ...).
// Semantics: softmax(q . K^T / sqrt(D)) V per query head over its KV head's
// first kv_len[b] keys (all L when no lengths are given).
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

constexpr int kDecChunk = 64;  // keys per CTA
constexpr int kDecThreads = 128;
constexpr int kDecMaxG = 16;

__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <bool kBf16>
__device__ __forceinline__ float to_f32(uint16_t h) {
  if constexpr (kBf16) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
  } else {
    return __half2float(__ushort_as_half(h));
  }
}

// A lane's N (2 or 4) consecutive 16-bit elements of a shared-memory row, in
// one 4- or 8-byte load, to fp32.
template <int N, bool kBf16>
__device__ __forceinline__ void load_cols(const uint16_t* p, float (&f)[N]) {
  uint32_t w[N / 2];
  if constexpr (N == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x;
    w[1] = u.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    if constexpr (kBf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
}

template <int D, int G, bool kBf16>
__global__ void __launch_bounds__(kDecThreads)
    gqa_decode_split_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                            const uint16_t* __restrict__ v, const int* __restrict__ kv_lens,
                            float* __restrict__ part_o, float* __restrict__ part_ml, int Hkv, int L, int n_splits,
                            int keys_per_split, float scale_log2, unsigned long long timeout_ns, int* status) {
  constexpr int kCols = D / 32;  // head-dim columns per lane
  __shared__ __align__(128) uint16_t sK[kDecChunk * D];
  __shared__ __align__(128) uint16_t sV[kDecChunk * D];
  __shared__ float sS[G][kDecChunk];
  __shared__ float sMrun[G], sLrun[G], sAlpha[G];
  __shared__ float sO[G][D];
  __shared__ __align__(8) uint64_t bar;
  __shared__ CtaControl ctl;

  const int split = blockIdx.x, hkv = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = kv_lens != nullptr ? min(max(kv_lens[b], 0), L) : L;
  const int first = split * keys_per_split;
  const int last = min(len, first + keys_per_split);  // this CTA's keys: [first, last)
  const size_t kv_head = static_cast<size_t>(b) * Hkv + hkv;
  // Query head g of this KV head is h = hkv * G + g.
  const size_t q_head0 = static_cast<size_t>(b) * Hkv * G + static_cast<size_t>(hkv) * G;
  const size_t part0 = (q_head0 * n_splits + split);  // (head, split) row; a head's rows are n_splits apart

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    ctl.abort = 0;
    fence_mbarrier_init();
  }
  for (int i = threadIdx.x; i < G * D; i += kDecThreads) (&sO[0][0])[i] = 0.0f;
  if (threadIdx.x < G) {
    sMrun[threadIdx.x] = -INFINITY;
    sLrun[threadIdx.x] = 0.0f;
  }
  // Query rows of the G heads, scaled by scale*log2(e), D/32 columns per lane.
  float qr[G][kCols];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < kCols; ++c)
      qr[g][c] = to_f32<kBf16>(q[(q_head0 + g) * D + lane * kCols + c]) * scale_log2;
  float o[G][kCols];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < kCols; ++c) o[g][c] = 0.0f;
  __syncthreads();

  bool ok = true;
  uint32_t phase = 0;
  // 64-key sub-chunks of [first, last), one at a time through shared memory
  // (several CTAs per SM overlap each other's copies and arithmetic), with an
  // online softmax across them: the running maximum / sum per query head live
  // in shared memory, each warp rescales its own partial output rows.
  for (int key0 = first; ok && key0 < last; key0 += kDecChunk, phase ^= 1u) {
    const int n_keys = min(kDecChunk, last - key0);
    if (threadIdx.x == 0) {
      const uint32_t bytes = static_cast<uint32_t>(n_keys) * D * 2;
      mbar_arrive_expect_tx(&bar, 2 * bytes);
      bulk_load_1d(sK, k + (kv_head * L + key0) * D, bytes, &bar);
      bulk_load_1d(sV, v + (kv_head * L + key0) * D, bytes, &bar);
    }
    ok = mbar_wait(&bar, phase, &ctl, timeout_ns, status, 30);
    ok = __syncthreads_and(ok);
    if (!ok) {
      if (threadIdx.x == 0) {
        // The copies did not complete in time: wait once more, bounded, for
        // them to land before this CTA's shared memory is released.
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(smem_u32(&bar), phase) && global_timer_ns() - t0 < timeout_ns) {
        }
      }
      break;
    }
    // Scores s[g][j] = q_g . k_j (base-2 scaled).  A warp takes 32/G keys at
    // a time: every lane holds its D/32-column partial of all 32 (key, head)
    // dot products, and a reduce-scatter over the 32 lanes (five halving
    // exchanges, 31 shuffles) leaves lane l with the complete dot product
    // number l (key l / G of the group, head l % G) — one shuffle per dot
    // product instead of five.
    constexpr int kGroupKeys = 32 / G;
    for (int grp = warp; grp * kGroupKeys < n_keys; grp += 4) {
      float val[32];
#pragma unroll
      for (int kk = 0; kk < kGroupKeys; ++kk) {
        // Rows past n_keys hold stale data: their dot products are computed
        // and dropped.
        const int j = grp * kGroupKeys + kk;
        float kc[kCols];
        load_cols<kCols, kBf16>(&sK[j * D + lane * kCols], kc);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float acc = 0.0f;
#pragma unroll
          for (int c = 0; c < kCols; ++c) acc = fmaf(qr[g][c], kc[c], acc);
          val[kk * G + g] = acc;
        }
      }
#pragma unroll
      for (int step = 0; step < 5; ++step) {
        const int off = 16 >> step;  // partner lane distance = half the live values
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
          const float keep = upper ? val[off + i] : val[i];
          const float send = upper ? val[i] : val[off + i];
          val[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const int j = grp * kGroupKeys + lane / G;
      if (j < n_keys) sS[lane % G][j] = val[0];
    }
    __syncthreads();
    // Online softmax per query head: warp w handles heads w, w + 4, ...
    for (int g = warp; g < G; g += 4) {
      const float s0 = lane < n_keys ? sS[g][lane] : -INFINITY;
      const float s1 = lane + 32 < n_keys ? sS[g][lane + 32] : -INFINITY;
      float mc = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
      const float m_old = sMrun[g];
      const float m_new = fmaxf(m_old, mc);
      const float p0 = lane < n_keys ? ex2(s0 - m_new) : 0.0f;
      const float p1 = lane + 32 < n_keys ? ex2(s1 - m_new) : 0.0f;
      float lc = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) lc += __shfl_xor_sync(0xffffffffu, lc, off);
      sS[g][lane] = p0;
      sS[g][lane + 32] = p1;
      __syncwarp();
      if (lane == 0) {
        const float alpha = (m_old == -INFINITY) ? 0.0f : ex2(m_old - m_new);
        sAlpha[g] = alpha;
        sLrun[g] = sLrun[g] * alpha + lc;
        sMrun[g] = m_new;
      }
    }
    __syncthreads();
    // o = alpha o + sum_j p_j v_j over this warp's keys, lanes own columns.
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float alpha = sAlpha[g];
#pragma unroll
      for (int c = 0; c < kCols; ++c) o[g][c] *= alpha;
    }
    for (int j = warp; j < n_keys; j += 4) {
      float vc[kCols];
      load_cols<kCols, kBf16>(&sV[j * D + lane * kCols], vc);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = sS[g][j];
        const uint64_t p2 = f2_pack(p, p);
#pragma unroll
        for (int c = 0; c < kCols; c += 2) {
          // Two columns per packed fp32x2 fma.
          f2_unpack(ffma2(p2, f2_pack(vc[c], vc[c + 1]), f2_pack(o[g][c], o[g][c + 1])), o[g][c], o[g][c + 1]);
        }
      }
    }
    // sK, sV and sS are reused by the next sub-chunk.
    __syncthreads();
  }
  // The combine kernel may start launching; it reads the partials only after
  // this grid has completed.
  pdl_launch_dependents();
  if (!ok || first >= last) {
    // Failed copy, or no keys (past this batch's length): a neutral partial
    // (m = -inf, l = 0, o = 0).
    for (int i = threadIdx.x; i < G * D; i += kDecThreads)
      part_o[(part0 + static_cast<size_t>(i / D) * n_splits) * D + i % D] = 0.0f;
    if (threadIdx.x < G) {
      part_ml[(part0 + static_cast<size_t>(threadIdx.x) * n_splits) * 2 + 0] = -INFINITY;
      part_ml[(part0 + static_cast<size_t>(threadIdx.x) * n_splits) * 2 + 1] = 0.0f;
    }
    return;
  }
  // Sum the four warps' partial rows in shared memory, in a fixed order
  // (warp 0, 1, 2, 3), so the result is the same from run to run.
#pragma unroll 1
  for (int w = 0; w < 4; ++w) {
    if (warp == w) {
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < kCols; ++c) sO[g][lane * kCols + c] += o[g][c];
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < G * D; i += kDecThreads) {
    const int g = i / D, d = i % D;
    part_o[(part0 + static_cast<size_t>(g) * n_splits) * D + d] = sO[g][d];
  }
  if (threadIdx.x < G) {
    part_ml[(part0 + static_cast<size_t>(threadIdx.x) * n_splits) * 2 + 0] = sMrun[threadIdx.x];
    part_ml[(part0 + static_cast<size_t>(threadIdx.x) * n_splits) * 2 + 1] = sLrun[threadIdx.x];
  }
}

template <int D, bool kBf16>
__global__ void __launch_bounds__(128)
    gqa_decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                              uint16_t* __restrict__ out, float* __restrict__ lse, long long n_heads, int n_splits) {
  constexpr int kCols = D / 32;
  // Launched as a programmatic dependent of the split kernel: wait for its
  // partials before reading them.
  pdl_wait_prerequisites();
  const long long head = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (head >= n_heads) return;
  const float* ml = part_ml + head * n_splits * 2;
  float m = -INFINITY;
  for (int s = lane; s < n_splits; s += 32) m = fmaxf(m, ml[2 * s]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float l = 0.0f;
  float acc[kCols];
#pragma unroll
  for (int c = 0; c < kCols; ++c) acc[c] = 0.0f;
  for (int s = 0; s < n_splits; ++s) {
    const float ms = ml[2 * s];
    const float w = (ms == -INFINITY) ? 0.0f : ex2(ms - m);
    l += w * ml[2 * s + 1];
    const float* os = part_o + (head * n_splits + s) * D + lane * kCols;
#pragma unroll
    for (int c = 0; c < kCols; ++c) acc[c] = fmaf(w, os[c], acc[c]);
  }
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
  for (int c = 0; c < kCols; c += 2)
    *reinterpret_cast<uint32_t*>(out + head * D + lane * kCols + c) = pack2<kBf16>(acc[c] * inv, acc[c + 1] * inv);
  if (lse != nullptr && lane == 0) lse[head] = (l > 0.0f) ? m + lg2(l) : -INFINITY;
}

// The combine kernel as a programmatic dependent launch: its CTAs may be
// scheduled while the split kernel's last CTAs finish, hiding the launch
// latency (it waits for the split grid to complete before reading).
template <int D, bool kBf16>
cudaError_t launch_combine(const GqaDecodeArgs& a, unsigned blocks, long long n_heads, int n_splits) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gqa_decode_combine_kernel<D, kBf16>, static_cast<const float*>(a.part_o),
                            static_cast<const float*>(a.part_ml), static_cast<uint16_t*>(a.o), a.lse, n_heads,
                            n_splits);
}

template <int D, int G, bool kBf16>
int launch_split(const GqaDecodeArgs& a, int n_splits) {
  dim3 grid(static_cast<unsigned>(n_splits), static_cast<unsigned>(a.Hkv), static_cast<unsigned>(a.B));
  const int keys_per_split = gqa_decode_keys_per_split(a.L, n_splits);
  gqa_decode_split_kernel<D, G, kBf16><<<grid, kDecThreads, 0, a.stream>>>(
      static_cast<const uint16_t*>(a.q), static_cast<const uint16_t*>(a.k), static_cast<const uint16_t*>(a.v),
      a.kv_lens, a.part_o, a.part_ml, static_cast<int>(a.Hkv), static_cast<int>(a.L), n_splits, keys_per_split,
      a.scale_log2, a.timeout_ns, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

template <int D, bool kBf16>
int launch_d(const GqaDecodeArgs& a, int n_splits) {
  switch (a.G) {
    case 1: return launch_split<D, 1, kBf16>(a, n_splits);
    case 2: return launch_split<D, 2, kBf16>(a, n_splits);
    case 4: return launch_split<D, 4, kBf16>(a, n_splits);
    case 8: return launch_split<D, 8, kBf16>(a, n_splits);
    case 16: return launch_split<D, 16, kBf16>(a, n_splits);
    default: return kErrUnsupported;
  }
}

}  // namespace

// Splits per (batch, KV head): enough CTAs for about four per SM over the
// whole problem, each a run of whole 64-key sub-chunks (never fewer keys
// than one sub-chunk per split, so short caches keep one split per chunk).
int gqa_decode_splits(int64_t B, int64_t Hkv, int64_t L, int sm_count) {
  const int64_t chunks = (L + kDecChunk - 1) / kDecChunk;
  const int64_t heads = B * Hkv;
  const int64_t want = (4LL * sm_count + heads - 1) / heads;
  const int64_t splits = want < 1 ? 1 : (want > chunks ? chunks : want);
  const int64_t per = ((chunks + splits - 1) / splits) * kDecChunk;  // keys per split, whole chunks
  return static_cast<int>((L + per - 1) / per);
}

int gqa_decode_keys_per_split(int64_t L, int n_splits) {
  const int64_t chunks = (L + kDecChunk - 1) / kDecChunk;
  return static_cast<int>(((chunks + n_splits - 1) / n_splits) * kDecChunk);
}

int launch_gqa_decode(const GqaDecodeArgs& a) {
  if (a.D != 64 && a.D != 128) return kErrUnsupported;
  if (a.G < 1 || a.G > kDecMaxG) return kErrUnsupported;
  const int n_splits = a.splits;
  int rc;
  if (a.tm_k != nullptr)
    rc = launch_gqa_decode_tc_split(a);
  else if (a.D == 64)
    rc = a.bf16 ? launch_d<64, true>(a, n_splits) : launch_d<64, false>(a, n_splits);
  else
    rc = a.bf16 ? launch_d<128, true>(a, n_splits) : launch_d<128, false>(a, n_splits);
  if (rc != kOk) return rc;
  const long long n_heads = a.B * a.Hkv * a.G;
  const unsigned blocks = static_cast<unsigned>((n_heads + 3) / 4);
  cudaError_t err;
  if (a.D == 64)
    err = a.bf16 ? launch_combine<64, true>(a, blocks, n_heads, n_splits)
                 : launch_combine<64, false>(a, blocks, n_heads, n_splits);
  else
    err = a.bf16 ? launch_combine<128, true>(a, blocks, n_heads, n_splits)
                 : launch_combine<128, false>(a, blocks, n_heads, n_splits);
  return err == cudaSuccess && cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace tk
