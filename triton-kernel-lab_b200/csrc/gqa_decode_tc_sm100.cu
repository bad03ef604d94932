// GQA decode with the products on the tensor cores (tcgen05), head_dim 64 or
// 128 (the layout is sized for 128: at 64 only the first 64-column block of
// each K, V and q tile is loaded).
//
// The same workload and partial format as gqa_decode_sm100.cu (one query
// token per query head, G query heads per KV head, contiguous (B, Hkv, L, D)
// cache, optional per-batch length; reference specification
// docs/research/gqa_decode_model.md), laid out so that the CUDA cores only
// run the softmax:
//
// * One CTA = (batch, KV head, split), a split being a run of 128-key tiles.
//   K and V tiles arrive by TMA through rings of three stages at head_dim
//   128 (one CTA per SM) or two at 64 (two CTAs per SM): warp 0 loads K and
//   the G query rows, warp 2 V; 96-192 KB of the cache in flight per SM.
// * Scores transposed, S^T = K Q^T: M = 128 keys (TMEM lanes), N = 16 query
//   heads (G padded with the following rows of q, whose columns are never
//   read), K = 128 head-dim elements: 8 MMAs into one of two 16-column TMEM
//   buffers.
// * Softmax warps 4-7, thread t = key t of the tile: base-2 online softmax
//   with the scale folded in.  The running maxima
//   move only when some score of the tile lies more than 2^8 above its
//   head's running maximum (one barrier with an OR reduction per tile
//   decides); then the tile maxima come from a warp reduce-scatter and a
//   4-warp exchange through shared memory and O is rescaled.  Row sums are
//   kept per thread and reduced once at the end in a fixed order.  P^T is
//   written as 16-bit values into shared memory (K-major, 16 head rows x 128
//   keys, 128-byte swizzle), the B operand of
// * O^T += V^T P^T: M = 128 head-dim rows (V read as an MN-major A operand
//   straight from its TMA tile), N = 16, K = 128 keys: 8 MMAs into 16 TMEM
//   columns; thread t owns head-dim element t of every head's output.
// * The unnormalised partial o, the running maximum m and the sum l of each
//   query head go to the workspace in the format gqa_decode_combine_kernel
//   merges.
//
// Every mbarrier wait is bounded; the softmax warps reach the same named
// barriers in every tile (whether a tile rescales is decided by a barrier
// reduction, so it is the same in every warp) and once at the end whatever
// happens, so a timeout never leaves a warp waiting on a barrier the others
// skipped.
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

constexpr int kTcKeys = 128;  // keys per tile (the M of S^T)
constexpr int kTcD = 128;  // shared-memory layout and O^T rows are sized for head_dim 128
constexpr int kTcN = 16;  // query heads per MMA (G padded)
constexpr int kTcThreads = 256;
constexpr int kTcBlockBytes = kTcKeys * kSwizzleBytes;  // one 64-column block of a K/V tile
constexpr int kTcQBlockBytes = kTcN * kSwizzleBytes;
constexpr int kTcPBytes = kTcN * kTcKeys * 2;  // 4 KB

// Shared-memory layout per head_dim.  Barriers first; then the K and V rings
// (stages of 128 keys x D); then q, P (two buffers) and the reduction
// scratch.  O^T's second 64-row block reads 16 KB past each V stage (its rows
// are never read): inside the stage at D = 128 (32 KB stages, the second
// column block), the next stage or the q/P region at D = 64, which is padded
// so that the read stays inside the allocation and never touches a barrier.
// D = 64: two stages, about 81 KB, two CTAs per SM; D = 128: three stages,
// about 206 KB, one CTA per SM.
template <int D>
struct TcCfg {
  static constexpr int kStages = D == 64 ? 2 : 3;
  static constexpr int kMinBlocks = D == 64 ? 2 : 1;
  static constexpr int kTileBytes = kTcKeys * D * 2;
  static constexpr int kQBytes = kTcN * D * 2;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_ready[2], pv_done, o_final
  static constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 2;
  static constexpr int kOffBar = 0;
  static constexpr int kOffCtl = kOffBar + kNumBars * 8;
  static constexpr int kOffK = 1024;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffQ = kOffV + kStages * kTileBytes;
  static constexpr int kOffP = kOffQ + ((kQBytes + 1023) / 1024) * 1024;  // two buffers
  static constexpr int kOffRed = kOffP + 2 * kTcPBytes;  // float [2][4][16] tile maxima
  static constexpr int kOffSum = kOffRed + 2 * 4 * kTcN * 4;  // float [4][16] row sums
  static constexpr int kEnd = kOffSum + 4 * kTcN * 4;
  static constexpr int kPadEnd = kOffV + kStages * kTileBytes + kTcBlockBytes;
  static constexpr int kSmemBytes = kEnd > kPadEnd ? kEnd : kPadEnd;
  static_assert(kOffCtl + 64 <= kOffK, "barriers overlap the K ring");
};
constexpr uint32_t kColO = 32;  // S^T buffers at columns 0 and 16
constexpr uint32_t kTcTmemCols = 64;
constexpr float kTcRescale = 8.0f;

__device__ __forceinline__ bool warp_wait_tc(uint64_t* bar, uint32_t parity, CtaControl* ctl, uint64_t timeout_ns,
                                             int* status, int site) {
  const bool ok = mbar_wait(bar, parity, ctl, timeout_ns, status, site);
  return __all_sync(0xffffffffu, ok);
}

template <bool kBf16>
__device__ __forceinline__ uint16_t to16(float x) {
  if constexpr (kBf16) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  } else {
    return __half_as_ushort(__float2half_rn(x));
  }
}

// Barrier over `threads` threads (named barrier `id`) that also returns
// whether `pred` was true in any of them (bar.red.or).
__device__ __forceinline__ bool named_barrier_or(int id, int threads, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return out != 0;
}

// Maximum over the warp of each of G per-lane values, scattered: lane l
// returns the maximum of value l / (32 / G).  A reduce-scatter (each step
// sends half of the values still held and keeps the other half) followed by
// plain butterflies: G - 1 + log2(32 / G) shuffles instead of 5 G.
template <int G>
__device__ __forceinline__ float warp_max_scatter(float (&v)[G], int lane) {
#pragma unroll
  for (int c = G, m = 16; c > 1; c >>= 1, m >>= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < c / 2; ++i) {
      const float send = upper ? v[i] : v[i + c / 2];
      const float keep = upper ? v[i + c / 2] : v[i];
      v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, m));
    }
  }
#pragma unroll
  for (int m = 32 / G / 2; m > 0; m >>= 1) v[0] = fmaxf(v[0], __shfl_xor_sync(0xffffffffu, v[0], m));
  return v[0];
}

template <int D, int G, bool kBf16>
__global__ void __launch_bounds__(kTcThreads, TcCfg<D>::kMinBlocks)
    gqa_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const int* __restrict__ kv_lens,
                         float* __restrict__ part_o, float* __restrict__ part_ml, int Hkv, int L, int n_splits,
                         int keys_per_split, float scale_log2, unsigned long long timeout_ns, int* status) {
  static_assert(G >= 1 && G <= kTcN, "query heads per KV head must fit one MMA's N");
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  using C = TcCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x, hkv = blockIdx.y, b = blockIdx.z;
  const int len = kv_lens != nullptr ? min(max(kv_lens[b], 0), L) : L;
  const int first = split * keys_per_split;
  const int last = min(len, first + keys_per_split);  // this CTA's keys: [first, last)
  const int n_tiles = last > first ? (last - first + kTcKeys - 1) / kTcKeys : 0;
  const int kv_slab = b * Hkv + hkv;
  const int q_row0 = kv_slab * G;  // query head hkv * G + g of batch b is row b * Hq + hkv * G + g
  const size_t part0 = static_cast<size_t>(q_row0) * n_splits + split;

  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sP = smem + C::kOffP;
  float* sRed = reinterpret_cast<float*>(smem + C::kOffRed);
  float* sSum = reinterpret_cast<float*>(smem + C::kOffSum);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + C::kStages;
  uint64_t* v_full = k_empty + C::kStages;
  uint64_t* v_empty = v_full + C::kStages;
  uint64_t* s_full = v_empty + C::kStages;
  uint64_t* p_ready = s_full + 2;
  uint64_t* pv_done = p_ready + 2;
  uint64_t* o_final = pv_done + 1;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kOffCtl);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_final, 1);
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  // P^T rows G..15 stay zero (their O^T columns are never read, but they are
  // computed, so keep them finite).
  for (int i = threadIdx.x; i < 2 * kTcPBytes / 16; i += kTcThreads)
    reinterpret_cast<uint4*>(sP)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 Q and K, warp 2 V ----------------
    if (lane == 0 && n_tiles > 0) {
      const bool is_k = warp == 0;
      const CUtensorMap* map = is_k ? &tm_k : &tm_v;
      uint8_t* ring = is_k ? sK : sV;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      if (is_k) {
        mbar_arrive_expect_tx(q_full, kTcN * D * 2);
#pragma unroll
        for (int blk = 0; blk < D / 64; ++blk)
          tma_load_3d(sQ + blk * kTcQBlockBytes, &tm_q, q_full, blk * 64, q_row0, 0);
      }
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % C::kStages;
        const uint32_t ph = (j / C::kStages) & 1;
        if (!mbar_wait(&empty[st], ph ^ 1, ctl, timeout_ns, status, is_k ? 1 : 2)) break;
        mbar_arrive_expect_tx(&full[st], kTcKeys * D * 2);
#pragma unroll
        for (int blk = 0; blk < D / 64; ++blk)
          tma_load_3d(ring + st * C::kTileBytes + blk * kTcBlockBytes, map, &full[st], blk * 64,
                      first + j * kTcKeys, kv_slab);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (n_tiles > 0) {
      const bool leader = elect_one();
      const uint32_t fmt = kBf16 ? 1u : 0u;
      const uint32_t idesc_s = idesc_f16(fmt, kTcKeys, kTcN, 0, 0);
      // O^T has M = 128 rows for both head dims: at D = 64 the second
      // 64-row block reads the unused half of the V stage (its rows of O^T
      // are never read), which keeps the 128-lane accumulator layout.
      const uint32_t idesc_o = idesc_f16(fmt, kTcD, kTcN, 1, 0);
      const uint32_t q_lo = sdesc_lo_kmajor(smem_u32(sQ));
      const uint32_t k_lo0 = sdesc_lo_kmajor(smem_u32(sK));
      const uint32_t v_lo0 = sdesc_lo_mnmajor(smem_u32(sV), kTcKeys);
      const uint32_t p_lo0 = sdesc_lo_kmajor(smem_u32(sP));
      constexpr uint32_t kStageLo = C::kTileBytes >> 4;
      constexpr uint32_t kPLo = kTcPBytes >> 4;
      // S^T(j) = K_j Q^T into buffer j & 1.
      auto issue_s = [&](int j) -> bool {
        const int st = j % C::kStages;
        if (!warp_wait_tc(&k_full[st], (j / C::kStages) & 1, ctl, timeout_ns, status, 3)) return false;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss_w(tmem + 16u * (j & 1), k_lo0 + st * kStageLo + kmajor_koff(kTcKeys, kk * 16),
                      q_lo + kmajor_koff(kTcN, kk * 16), idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[j & 1]);
          umma_commit(&k_empty[st]);
        }
        __syncwarp();
        return true;
      };
      bool ok = warp_wait_tc(q_full, 0, ctl, timeout_ns, status, 4) && issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        // The next tile's scores run while the softmax works on this one
        // (its S buffer was released by p_ready(j - 1), waited below last
        // iteration).
        if (j + 1 < n_tiles && !(ok = issue_s(j + 1))) break;
        if (!(ok = warp_wait_tc(&p_ready[j & 1], (j >> 1) & 1, ctl, timeout_ns, status, 5))) break;
        const int st = j % C::kStages;
        if (!(ok = warp_wait_tc(&v_full[st], (j / C::kStages) & 1, ctl, timeout_ns, status, 6))) break;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kTcKeys / 16; ++kk)
            umma_ss_w(tmem + kColO, v_lo0 + st * kStageLo + mnmajor_koff(kk * 16),
                      p_lo0 + (j & 1) * kPLo + kmajor_koff(kTcN, kk * 16), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&v_empty[st]);
          umma_commit(pv_done);
          if (j + 1 == n_tiles) umma_commit(o_final);
        }
        __syncwarp();
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax and epilogue: thread t = key t / head-dim t ----------------
    const int q4 = warp & 3;
    const int t = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    float m_run[G], lsum[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      lsum[g] = 0.0f;
    }
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      // Every warp reaches the barriers of every tile, failed or not.
      ok = ok && warp_wait_tc(&s_full[j & 1], (j >> 1) & 1, ctl, timeout_ns, status, 7);
      float x[G];
      bool jump = false;
      if (ok) {
        tc_fence_after();
        uint32_t s[16];
        tmem_ld16(t_lane + 16u * (j & 1), s);
        tmem_wait_ld();
        reg_fence16(s);
        const bool valid = first + j * kTcKeys + t < last;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          x[g] = valid ? __uint_as_float(s[g]) * scale_log2 : -INFINITY;
          jump = jump || x[g] > m_run[g] + kTcRescale;
        }
      }
      // Common case: no score of the tile is more than 2^8 above its head's
      // running maximum, so P = 2^(x - m_run) as it is (no tile maximum, no
      // exchange).  Otherwise (the first tile, or a head whose scores jumped)
      // the tile maxima are computed and the running maxima moved.
      const bool rescale = named_barrier_or(1, 128, jump);
      float alpha[G];
#pragma unroll
      for (int g = 0; g < G; ++g) alpha[g] = 1.0f;
      if (rescale) {
        float* red = sRed + (j & 1) * 4 * kTcN;  // [head][warp]
        if (ok) {
          float wm[G];
#pragma unroll
          for (int g = 0; g < G; ++g) wm[g] = x[g];
          const float hm = warp_max_scatter<G>(wm, lane);
          if ((lane & (32 / G - 1)) == 0) red[(lane / (32 / G)) * 4 + q4] = hm;
        }
        named_barrier_sync(1, 128);
        if (ok) {
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float4 w4 = *reinterpret_cast<const float4*>(red + g * 4);
            const float m_new = fmaxf(m_run[g], fmaxf(fmaxf(w4.x, w4.y), fmaxf(w4.z, w4.w)));
            alpha[g] = m_run[g] == -INFINITY ? 0.0f : ex2(m_run[g] - m_new);
            m_run[g] = m_new;
          }
          if (j > 0) {
            // P(j-1) V must be in O before O is rescaled.
            ok = warp_wait_tc(pv_done, (j - 1) & 1, ctl, timeout_ns, status, 8);
            if (ok) {
              tc_fence_after();
              uint32_t o[16];
              tmem_ld16(t_lane + kColO, o);
              tmem_wait_ld();
              reg_fence16(o);
#pragma unroll
              for (int g = 0; g < G; ++g) o[g] = __float_as_uint(__uint_as_float(o[g]) * alpha[g]);
              tmem_st16(t_lane + kColO, o);
            }
          }
        }
      }
      if (!ok) continue;
      uint8_t* pbuf = sP + (j & 1) * kTcPBytes;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = ex2(x[g] - m_run[g]);
        lsum[g] = fmaf(lsum[g], alpha[g], p);
        *reinterpret_cast<uint16_t*>(pbuf + swz_offset(g, t, kTcN)) = to16<kBf16>(p);
      }
      fence_proxy_async_smem();
      if (rescale && j > 0) tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[j & 1]);
    }
    // The combine kernel may start launching; it reads the partials only
    // after this grid has completed.
    pdl_launch_dependents();
    // Row sums: warp butterflies, then the four warps in a fixed order.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int g = 0; g < G; ++g) lsum[g] += __shfl_xor_sync(0xffffffffu, lsum[g], off);
#pragma unroll
    for (int g = 0; g < G; ++g)
      if (lane == g) sSum[q4 * kTcN + g] = lsum[g];
    named_barrier_sync(1, 128);
    if (n_tiles > 0 && ok) ok = warp_wait_tc(o_final, 0, ctl, timeout_ns, status, 9);
    if (n_tiles > 0 && ok) {
      tc_fence_after();
      uint32_t o[16];
      tmem_ld16(t_lane + kColO, o);
      tmem_wait_ld();
      reg_fence16(o);
      if (t < D)
#pragma unroll
        for (int g = 0; g < G; ++g) part_o[(part0 + static_cast<size_t>(g) * n_splits) * D + t] = __uint_as_float(o[g]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (t == g) {
          const float l = ((sSum[g] + sSum[kTcN + g]) + sSum[2 * kTcN + g]) + sSum[3 * kTcN + g];
          part_ml[(part0 + static_cast<size_t>(g) * n_splits) * 2 + 0] = m_run[g];
          part_ml[(part0 + static_cast<size_t>(g) * n_splits) * 2 + 1] = l;
        }
      }
    } else {
      // No keys in this split, or a wait that ran out: a neutral partial.
      if (t < D)
#pragma unroll
        for (int g = 0; g < G; ++g) part_o[(part0 + static_cast<size_t>(g) * n_splits) * D + t] = 0.0f;
      if (t < G) {
        part_ml[(part0 + static_cast<size_t>(t) * n_splits) * 2 + 0] = -INFINITY;
        part_ml[(part0 + static_cast<size_t>(t) * n_splits) * 2 + 1] = 0.0f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

template <int D, int G, bool kBf16>
int launch_tc_t(const GqaDecodeArgs& a, int n_splits, int keys_per_split) {
  using C = TcCfg<D>;
  static_assert(C::kSmemBytes <= 232448, "decode shared memory exceeds the sm_100 limit");
  auto kern = gqa_decode_tc_kernel<D, G, kBf16>;
  if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern), C::kSmemBytes, 0, nullptr)) return rc;
  dim3 grid(static_cast<unsigned>(n_splits), static_cast<unsigned>(a.Hkv), static_cast<unsigned>(a.B));
  kern<<<grid, kTcThreads, C::kSmemBytes, a.stream>>>(*a.tm_q, *a.tm_k, *a.tm_v, a.kv_lens, a.part_o, a.part_ml,
                                                     static_cast<int>(a.Hkv), static_cast<int>(a.L), n_splits,
                                                     keys_per_split, a.scale_log2, a.timeout_ns, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

template <int D, bool kBf16>
int launch_tc_g(const GqaDecodeArgs& a, int n_splits, int keys_per_split) {
  switch (a.G) {
    case 4: return launch_tc_t<D, 4, kBf16>(a, n_splits, keys_per_split);
    case 8: return launch_tc_t<D, 8, kBf16>(a, n_splits, keys_per_split);
    case 16: return launch_tc_t<D, 16, kBf16>(a, n_splits, keys_per_split);
    default: return kErrUnsupported;
  }
}

}  // namespace

bool gqa_decode_tc_supported(int64_t D, int64_t G) { return (D == 64 || D == 128) && (G == 4 || G == 8 || G == 16); }

// Splits per (batch, KV head) for the tensor-core kernel (one CTA per SM at
// head_dim 128, two at 64): the count that minimises a simple makespan model
// — waves of CTAs times (128-key tiles per split + a prologue worth about one
// and a half tiles) — so the last wave is not left mostly empty and short
// splits do not pay the prologue too often.
int gqa_decode_splits_tc(int64_t B, int64_t Hkv, int64_t L, int64_t D, int sm_count) {
  const int64_t tiles = (L + kTcKeys - 1) / kTcKeys;
  const int64_t heads = B * Hkv;
  sm_count *= D == 64 ? TcCfg<64>::kMinBlocks : TcCfg<128>::kMinBlocks;
  const int64_t cap = tiles < 1024 ? tiles : 1024;
  int64_t best = 1;
  double best_cost = -1.0;
  for (int64_t s = 1; s <= cap; ++s) {
    const int64_t per = (tiles + s - 1) / s;
    const int64_t used = (tiles + per - 1) / per;  // splits that hold keys
    if (used != s) continue;
    // At head_dim 64 a tile is half the bytes, so a one-tile split's fixed
    // costs (prologue, partials, combine) outweigh what it spreads.
    if (D == 64 && per < 2 && tiles >= 2) continue;
    const int64_t waves = (heads * s + sm_count - 1) / sm_count;
    const double cost = static_cast<double>(waves) * (static_cast<double>(per) + 1.5);
    if (best_cost < 0.0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return static_cast<int>(best);
}

int gqa_decode_keys_per_split_tc(int64_t L, int n_splits) {
  const int64_t tiles = (L + kTcKeys - 1) / kTcKeys;
  return static_cast<int>(((tiles + n_splits - 1) / n_splits) * kTcKeys);
}

int launch_gqa_decode_tc_split(const GqaDecodeArgs& a) {
  if (!gqa_decode_tc_supported(a.D, a.G) || a.tm_q == nullptr || a.tm_k == nullptr || a.tm_v == nullptr)
    return kErrUnsupported;
  const int kps = gqa_decode_keys_per_split_tc(a.L, a.splits);
  if (a.D == 64) return a.bf16 ? launch_tc_g<64, true>(a, a.splits, kps) : launch_tc_g<64, false>(a, a.splits, kps);
  return a.bf16 ? launch_tc_g<128, true>(a, a.splits, kps) : launch_tc_g<128, false>(a, a.splits, kps);
}

}  // namespace tk
