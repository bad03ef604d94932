// Flash-attention forward for head dims 136..256 on sm_100a (B200).
//
// Same semantics as attn_fwd_sm100.cu (reference
// src/tklab/kernels/flash_attention.py:54-117, :120-264: base-2 online
// softmax with the scale folded in, P rounded to the input dtype for P.V,
// O = acc / row_sum, LSE = m + log2(l)), laid out for a head of W = 192
// (head dims 136..192) or 256 (200..256) columns:
//
// * Persistent: one CTA per SM walks work units (causal: a head's heaviest
//   query tile paired with its lightest; non-causal: one tile), each item a
//   128-row query tile against 64-key tiles.  The next item's Q load and
//   first S products overlap the current item's epilogue.
// * Tensor memory (512 columns): O [0,W), S in two 64-column buffers
//   [256,320) and [320,384) so S(j+1) runs while the softmax works on S(j);
//   P(j) goes back packed over the first 32 columns of its S buffer and
//   feeds the P.V MMA (M=128, N=W, K=16 per instruction) from TMEM.
// * Shared memory: Q (W/64 blocks of 16 KB), K and V rings of two 64-key
//   stages (W/64 blocks of 8 KB each): 192 KB at W = 256, 144 KB at 192.
// * 8 warps: warp 0 TMA producer, warp 1 TMEM allocator and MMA issuer
//   (converged warp, one elected lane issues), warps 4..7 softmax (thread t
//   owns query row t = TMEM lane t) and epilogue (O / l from TMEM straight
//   to global memory; TMEM O released as soon as it is loaded).
// * MMA order per item: S(0), S(1), then per key tile j: P(j).V_j, S(j+2)
//   into the buffer P(j) was read from; the item's last S releases Q.  O is
//   rescaled only when a row's running maximum moves by more than 2^8 (lazy
//   rescale), and then after waiting for P(j-1).V to complete (pv_done).
// * head_dim below W (a multiple of 8) runs the kernel with the tensor maps
//   declaring the true width: loads zero-fill, the stores skip the columns.
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

constexpr int kKeyTile = 64;
constexpr int kD256Threads = 256;
// q_full, q_empty, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2],
// p_ready[2], pv_done, o_final, o_empty
constexpr int kNumBars = 2 + 8 + 2 + 2 + 3;

// Layout for a kernel width of NB column blocks of 64 (NB = 3: head dims
// 136..192, NB = 4: 200..256): shared memory Q (NB x 16 KB), K and V rings
// of two 64-key stages (NB x 8 KB each); TMEM O in [0, 64 NB), S buffers at
// columns 256 and 320.
template <int NB>
struct WideCfg {
  static constexpr int kW = 64 * NB;
  static constexpr int kQBytes = kTileRows * kW * 2;
  static constexpr int kKVBytes = kKeyTile * kW * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + 2 * kKVBytes;
  static constexpr int kBarOff = kVOff + 2 * kKVBytes;
  static constexpr int kCtlOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kCtlOff + 64;
};
constexpr int kKVBlockBytes = kKeyTile * kSwizzleBytes;  // 8 KB: one 64-column block of a key tile
constexpr uint32_t kColO = 0;
constexpr uint32_t kColS = 256;  // two buffers of 64 columns
constexpr float kRescale = 8.0f;

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, CtaControl* ctl, uint64_t timeout_ns,
                                          int* status, int site) {
  const bool ok = mbar_wait(bar, parity, ctl, timeout_ns, status, site);
  return __all_sync(0xffffffffu, ok);
}

// Work units: causal — a head's query tiles paired heaviest with lightest
// (tile n-1-p, then tile p; the middle tile alone when n is odd), so every
// unit costs about the same; non-causal — one query tile.  Units are ordered
// head-major so the CTAs running at one time share few heads' K and V in L2.
__device__ __forceinline__ int wide_unit_items(int causal, int n_qtiles, int p) {
  return (causal && 2 * p + 1 != n_qtiles) ? 2 : 1;
}
__device__ __forceinline__ int wide_item_qtile(int causal, int n_qtiles, int p, int i) {
  return causal ? (i == 0 ? n_qtiles - 1 - p : p) : p;
}

template <int NB, bool kBf16>
__global__ void __launch_bounds__(kD256Threads, 1)
    attn_fwd_d256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, uint16_t* __restrict__ out,
                         float* __restrict__ lse, int S, int n_qtiles, int units_per_head, int n_units, int causal,
                         int d_real, float scale_log2, unsigned long long timeout_ns, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  using C = WideCfg<NB>;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_ktiles = (S + kKeyTile - 1) / kKeyTile;

  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;
  uint64_t* k_full = q_empty + 1;
  uint64_t* k_empty = k_full + 2;
  uint64_t* v_full = k_empty + 2;
  uint64_t* v_empty = v_full + 2;
  uint64_t* s_full = v_empty + 2;
  uint64_t* p_ready = s_full + 2;
  uint64_t* pv_done = p_ready + 2;
  uint64_t* o_final = pv_done + 1;
  uint64_t* o_empty = o_final + 1;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kCtlOff);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_final, 1);
    mbar_init(o_empty, 4);
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // Every role walks the same item sequence: `it` counts this CTA's items,
  // `g0` its key tiles before the current item (ring stages, S buffers and
  // barrier phases run on these counters across items).
  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      bool ok = true;
      int it = 0, g0 = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
        const int bh = u / units_per_head, p = u % units_per_head;
        const int ni = wide_unit_items(causal, n_qtiles, p);
        for (int i = 0; ok && i < ni; ++i, ++it) {
          const int m0 = wide_item_qtile(causal, n_qtiles, p, i) * kTileRows;
          const int n_kv = causal ? min((m0 + kTileRows + kKeyTile - 1) / kKeyTile, n_ktiles) : n_ktiles;
          // Q of the previous item is free once its last S product is done.
          if (!(ok = mbar_wait(q_empty, (it & 1) ^ 1, ctl, timeout_ns, status, 10))) break;
          mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
          for (int b = 0; b < NB; ++b) tma_load_3d(sQ + b * kBlockBytes, &tm_q, q_full, b * 64, m0, bh);
          for (int j = 0; j < n_kv; ++j) {
            const int g = g0 + j;
            const int st = g & 1;
            const uint32_t ph = (g >> 1) & 1;
            if (!(ok = mbar_wait(&k_empty[st], ph ^ 1, ctl, timeout_ns, status, 1))) break;
            mbar_arrive_expect_tx(&k_full[st], C::kKVBytes);
#pragma unroll
            for (int b = 0; b < NB; ++b)
              tma_load_3d(sK + st * C::kKVBytes + b * kKVBlockBytes, &tm_k, &k_full[st], b * 64, j * kKeyTile, bh);
            if (!(ok = mbar_wait(&v_empty[st], ph ^ 1, ctl, timeout_ns, status, 2))) break;
            mbar_arrive_expect_tx(&v_full[st], C::kKVBytes);
#pragma unroll
            for (int b = 0; b < NB; ++b)
              tma_load_3d(sV + st * C::kKVBytes + b * kKVBlockBytes, &tm_v, &v_full[st], b * 64, j * kKeyTile, bh);
          }
          g0 += n_kv;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const bool leader = elect_one();
    const uint32_t fmt = kBf16 ? 1u : 0u;
    const uint32_t idesc_s = idesc_f16(fmt, 128, kKeyTile, 0, 0);
    const uint32_t idesc_pv = idesc_f16(fmt, 128, C::kW, 0, 1);
    const uint32_t q_lo = sdesc_lo_kmajor(smem_u32(sQ));
    const uint32_t k_lo0 = sdesc_lo_kmajor(smem_u32(sK));
    const uint32_t v_lo0 = sdesc_lo_mnmajor(smem_u32(sV), kKeyTile);
    constexpr uint32_t kStageLo = C::kKVBytes >> 4;
    // S(g) = Q K^T into S buffer g & 1 (W/16 MMAs of K = 16); the item's last
    // one also releases Q.
    auto issue_s = [&](int g, bool last_of_item) -> bool {
      const int st = g & 1;
      if (!warp_wait(&k_full[st], (g >> 1) & 1, ctl, timeout_ns, status, 3)) return false;
      tc_fence_after();
      if (leader) {
        const uint32_t k_lo = k_lo0 + st * kStageLo;
#pragma unroll
        for (int kk = 0; kk < C::kW / 16; ++kk)
          umma_ss_w(tmem + kColS + 64u * st, q_lo + kmajor_koff(kTileRows, kk * 16),
                    k_lo + kmajor_koff(kKeyTile, kk * 16), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        if (last_of_item) umma_commit(q_empty);
      }
      __syncwarp();
      return true;
    };
    bool ok = true;
    int it = 0, g0 = 0;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
      const int p = u % units_per_head;
      const int ni = wide_unit_items(causal, n_qtiles, p);
      for (int i = 0; ok && i < ni; ++i, ++it) {
        const int m0 = wide_item_qtile(causal, n_qtiles, p, i) * kTileRows;
        const int n_kv = causal ? min((m0 + kTileRows + kKeyTile - 1) / kKeyTile, n_ktiles) : n_ktiles;
        if (!(ok = warp_wait(q_full, it & 1, ctl, timeout_ns, status, 4))) break;
        if (!(ok = issue_s(g0, n_kv == 1))) break;
        if (n_kv > 1 && !(ok = issue_s(g0 + 1, n_kv == 2))) break;
        for (int j = 0; j < n_kv; ++j) {
          const int g = g0 + j;
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!(ok = warp_wait(&p_ready[st], ph, ctl, timeout_ns, status, 5))) break;
          if (!(ok = warp_wait(&v_full[st], ph, ctl, timeout_ns, status, 6))) break;
          // The first product of an item overwrites O: the previous item's
          // epilogue must have read it.
          if (j == 0 && it > 0 && !(ok = warp_wait(o_empty, (it - 1) & 1, ctl, timeout_ns, status, 11))) break;
          tc_fence_after();
          if (leader) {
            // O += P(j) V_j: P packed in the first 32 columns of S buffer st.
            const uint32_t v_lo = v_lo0 + st * kStageLo;
#pragma unroll
            for (int kk = 0; kk < kKeyTile / 16; ++kk)
              umma_ts_w(tmem + kColO, tmem + kColS + 64u * st + kk * 8, v_lo + mnmajor_koff(kk * 16), idesc_pv,
                        (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&v_empty[st]);
            umma_commit(pv_done);
            if (j + 1 == n_kv) umma_commit(o_final);
          }
          __syncwarp();
          if (j + 2 < n_kv && !(ok = issue_s(g + 2, j + 3 == n_kv))) break;
        }
        g0 += n_kv;
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax and epilogue ----------------
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    bool ok = true;
    int it = 0, g0 = 0;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
      const int bh = u / units_per_head, p = u % units_per_head;
      const int ni = wide_unit_items(causal, n_qtiles, p);
      for (int i = 0; ok && i < ni; ++i, ++it) {
        const int m0 = wide_item_qtile(causal, n_qtiles, p, i) * kTileRows;
        const int n_kv = causal ? min((m0 + kTileRows + kKeyTile - 1) / kKeyTile, n_ktiles) : n_ktiles;
        const int row_g = m0 + r;
        float m_run = -INFINITY, l_run = 0.0f;
        for (int j = 0; ok && j < n_kv; ++j) {
          const int g = g0 + j;
          const int st = g & 1;
          if (!(ok = warp_wait(&s_full[st], (g >> 1) & 1, ctl, timeout_ns, status, 7))) break;
          tc_fence_after();
          const uint32_t s_addr = t_lane + kColS + 64u * st;
          uint32_t s[2][32];
          tmem_ld32(s_addr, s[0]);
          tmem_ld32(s_addr + 32, s[1]);
          tmem_wait_ld();
          reg_fence(s[0]);
          reg_fence(s[1]);
          const int n0 = j * kKeyTile;
          int lim = S - n0;
          if (causal) lim = min(lim, row_g - n0 + 1);
          float mx = -INFINITY;
#pragma unroll
          for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              if (b * 32 + c >= lim) s[b][c] = __float_as_uint(-INFINITY);
              mx = fmaxf(mx, __uint_as_float(s[b][c]));
            }
          const float m_new = fmaxf(m_run, mx * scale_log2);
          const bool need = m_new > m_run + kRescale;
          const float m_use = need ? m_new : m_run;
          const float alpha = (m_run == -INFINITY) ? 0.0f : ex2(m_run - m_use);
          const float ms = (m_use == -INFINITY) ? 0.0f : m_use;
          if (j > 0 && __any_sync(0xffffffffu, need)) {
            // P(j-1).V must be in O before it is rescaled (pv_done counts
            // every product of every item: (g-1)&1 is its phase).
            if (!(ok = warp_wait(pv_done, (g - 1) & 1, ctl, timeout_ns, status, 8))) break;
            tc_fence_after();
#pragma unroll 1
            for (int cb = 0; cb < C::kW / 32; ++cb) {
              uint32_t o[32];
              tmem_ld32(t_lane + kColO + cb * 32, o);
              tmem_wait_ld();
              reg_fence(o);
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st32(t_lane + kColO + cb * 32, o);
            }
          }
          float sum = 0.0f;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            uint32_t pk[16];
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float p0 = ex2(fmaf(__uint_as_float(s[b][c]), scale_log2, -ms));
              const float p1 = ex2(fmaf(__uint_as_float(s[b][c + 1]), scale_log2, -ms));
              sum += p0 + p1;
              pk[c >> 1] = pack2<kBf16>(p0, p1);
            }
            tmem_st16(s_addr + b * 16, pk);
          }
          l_run = l_run * alpha + sum;
          m_run = m_use;
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_ready[st]);
        }
        g0 += n_kv;
        if (!ok) break;
        // Epilogue: O / l from TMEM straight to global memory, one row per
        // thread, 16-byte pieces (rows past S and columns past the true
        // head_dim skipped); TMEM O is released for the next item's first
        // product as soon as the last column block is loaded.
        if (!(ok = warp_wait(o_final, it & 1, ctl, timeout_ns, status, 9))) break;
        tc_fence_after();
        const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        const bool row_ok = row_g < S;
        uint16_t* orow = out + (static_cast<size_t>(bh) * S + (row_ok ? row_g : 0)) * d_real;
#pragma unroll 1
        for (int cb = 0; cb < C::kW / 32; ++cb) {
          uint32_t o[32];
          tmem_ld32(t_lane + kColO + cb * 32, o);
          tmem_wait_ld();
          reg_fence(o);
          if (cb + 1 == C::kW / 32) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
          }
          if (row_ok) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int col = cb * 32 + q * 8;
              if (col < d_real) {
                uint4 w;
                w.x = pack2<kBf16>(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
                w.y = pack2<kBf16>(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
                w.z = pack2<kBf16>(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
                w.w = pack2<kBf16>(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
                *reinterpret_cast<uint4*>(orow + col) = w;
              }
            }
          }
        }
        if (lse != nullptr && row_ok) lse[static_cast<size_t>(bh) * S + row_g] = m_run + lg2(l_run);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NB, bool kBf16>
int launch_d256_t(const FwdD256Args& a) {
  using C = WideCfg<NB>;
  static_assert(C::kSmemBytes <= 232448, "wide-head forward shared memory exceeds the sm_100 limit");
  auto kern = attn_fwd_d256_kernel<NB, kBf16>;
  int sms = 0;
  if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern), C::kSmemBytes, 0, &sms)) return rc;
  const int n_qtiles = static_cast<int>((a.S + kTileRows - 1) / kTileRows);
  const int units_per_head = a.causal ? (n_qtiles + 1) / 2 : n_qtiles;
  const long long n_units = static_cast<long long>(units_per_head) * a.BH;
  if (n_units > INT32_MAX) return kErrTooLarge;
  // One persistent CTA per SM (shared memory and TMEM allow no second one).
  const int grid = static_cast<int>(n_units < sms ? n_units : sms);
  kern<<<grid, kD256Threads, C::kSmemBytes, a.stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_v, static_cast<uint16_t*>(a.o), a.lse, static_cast<int>(a.S), n_qtiles,
      units_per_head, static_cast<int>(n_units), a.causal, static_cast<int>(a.D), a.scale_log2, a.timeout_ns,
      a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_attn_fwd_d256(const FwdD256Args& a) {
  if (a.D > 256 || a.o == nullptr) return kErrUnsupported;
  if (a.D <= 192) return a.bf16 ? launch_d256_t<3, true>(a) : launch_d256_t<3, false>(a);
  return a.bf16 ? launch_d256_t<4, true>(a) : launch_d256_t<4, false>(a);
}

}  // namespace tk
