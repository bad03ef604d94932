// Flash-attention forward for head dims 136..256 on sm_100a (B200).
//
// Same semantics as attn_fwd_sm100.cu (reference
// src/tklab/kernels/flash_attention.py:54-117, :120-264: base-2 online
// softmax with the scale folded in, P rounded to the input dtype for P.V,
// O = acc / row_sum, LSE = m + log2(l)), laid out for a head of W = 192
// (head dims 136..192) or 256 (200..256) columns:
//
// * One CTA = one 128-row query tile of one (batch, head); keys in tiles of
//   64.  Tensor memory (512 columns): O [0,W), S in two 64-column buffers
//   [256,320) and [320,384) so S(j+1) runs while the softmax works on S(j);
//   P(j) goes back packed over the first 32 columns of its S buffer and
//   feeds the P.V MMA (M=128, N=W, K=16 per instruction) from TMEM.
// * Shared memory: Q (W/64 blocks of 16 KB), K and V rings of two 64-key
//   stages (W/64 blocks of 8 KB each): 192 KB at W = 256, 144 KB at 192.
// * 8 warps: warp 0 TMA producer, warp 1 TMEM allocator and MMA issuer
//   (converged warp, one elected lane issues), warps 4..7 softmax (thread t
//   owns query row t = TMEM lane t) and epilogue.
// * MMA order: S(0), S(1), then per key tile j: P(j).V_j, S(j+2) into the
//   buffer P(j) was read from.  O is rescaled only when a row's running
//   maximum moves by more than 2^8 (lazy rescale), and then after waiting
//   for P(j-1).V to complete (pv_done).
// * head_dim below W (a multiple of 8) runs the kernel with the tensor maps
//   declaring the true width: loads zero-fill, the store clips.
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

constexpr int kKeyTile = 64;
constexpr int kD256Threads = 256;
// q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2],
// p_ready[2], pv_done, o_final
constexpr int kNumBars = 1 + 8 + 2 + 2 + 2;

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

template <int NB, bool kBf16>
__global__ void __launch_bounds__(kD256Threads, 1)
    attn_fwd_d256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                         float* __restrict__ lse, int S, int n_qtiles, int causal, int d_real, float scale_log2,
                         unsigned long long timeout_ns, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Head-major, heaviest query tile of a head first.
  const int bh = static_cast<int>(blockIdx.x) / n_qtiles;
  const int qt = n_qtiles - 1 - static_cast<int>(blockIdx.x) % n_qtiles;
  const int m0 = qt * kTileRows;
  const int n_ktiles = (S + kKeyTile - 1) / kKeyTile;
  const int n_kv = causal ? min((m0 + kTileRows + kKeyTile - 1) / kKeyTile, n_ktiles) : n_ktiles;

  using C = WideCfg<NB>;
  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + 2;
  uint64_t* v_full = k_empty + 2;
  uint64_t* v_empty = v_full + 2;
  uint64_t* s_full = v_empty + 2;
  uint64_t* p_ready = s_full + 2;
  uint64_t* pv_done = p_ready + 2;
  uint64_t* o_final = pv_done + 1;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kCtlOff);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
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
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
    tma_prefetch_map(&tm_o);
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
      for (int b = 0; b < NB; ++b) tma_load_3d(sQ + b * kBlockBytes, &tm_q, q_full, b * 64, m0, bh);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1, ctl, timeout_ns, status, 1)) break;
        mbar_arrive_expect_tx(&k_full[st], C::kKVBytes);
#pragma unroll
        for (int b = 0; b < NB; ++b)
          tma_load_3d(sK + st * C::kKVBytes + b * kKVBlockBytes, &tm_k, &k_full[st], b * 64, j * kKeyTile, bh);
        if (!mbar_wait(&v_empty[st], ph ^ 1, ctl, timeout_ns, status, 2)) break;
        mbar_arrive_expect_tx(&v_full[st], C::kKVBytes);
#pragma unroll
        for (int b = 0; b < NB; ++b)
          tma_load_3d(sV + st * C::kKVBytes + b * kKVBlockBytes, &tm_v, &v_full[st], b * 64, j * kKeyTile, bh);
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
    // S(j) = Q K_j^T into S buffer j&1 (16 MMAs of K = 16 over the 256 columns).
    auto issue_s = [&](int j) -> bool {
      const int st = j & 1;
      if (!warp_wait(&k_full[st], (j >> 1) & 1, ctl, timeout_ns, status, 3)) return false;
      tc_fence_after();
      if (leader) {
        const uint32_t k_lo = k_lo0 + st * kStageLo;
#pragma unroll
        for (int kk = 0; kk < C::kW / 16; ++kk)
          umma_ss_w(tmem + kColS + 64u * st, q_lo + kmajor_koff(kTileRows, kk * 16),
                    k_lo + kmajor_koff(kKeyTile, kk * 16), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
      }
      __syncwarp();
      return true;
    };
    bool ok = warp_wait(q_full, 0, ctl, timeout_ns, status, 4);
    if (ok && n_kv > 0) ok = issue_s(0);
    if (ok && n_kv > 1) ok = issue_s(1);
    for (int j = 0; ok && j < n_kv; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!(ok = warp_wait(&p_ready[st], ph, ctl, timeout_ns, status, 5))) break;
      if (!(ok = warp_wait(&v_full[st], ph, ctl, timeout_ns, status, 6))) break;
      tc_fence_after();
      if (leader) {
        // O += P(j) V_j: P packed in the first 32 columns of S buffer j&1.
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
      if (j + 2 < n_kv && !(ok = issue_s(j + 2))) break;
    }
  } else if (warp >= 4) {
    // ---------------- softmax and epilogue ----------------
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int row_g = m0 + r;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; ok && j < n_kv; ++j) {
      const int st = j & 1;
      if (!(ok = warp_wait(&s_full[st], (j >> 1) & 1, ctl, timeout_ns, status, 7))) break;
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
        // P(j-1).V must be in O before it is rescaled.
        if (!(ok = warp_wait(pv_done, (j - 1) & 1, ctl, timeout_ns, status, 8))) break;
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
    // Epilogue: O / l staged through Q (dead once every product has
    // completed, which o_final implies), then one TMA store per column block
    // (rows past S and columns past the true head_dim are clipped).  Every
    // warp of the warpgroup reaches the barrier below once, on failure too.
    if (ok) ok = warp_wait(o_final, 0, ctl, timeout_ns, status, 9);
    if (ok) {
      tc_fence_after();
      const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll 1
      for (int cb = 0; cb < C::kW / 32; ++cb) {
        uint32_t o[32];
        tmem_ld32(t_lane + kColO + cb * 32, o);
        tmem_wait_ld();
        reg_fence(o);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint4 w;
          w.x = pack2<kBf16>(__uint_as_float(o[ch * 8 + 0]) * inv_l, __uint_as_float(o[ch * 8 + 1]) * inv_l);
          w.y = pack2<kBf16>(__uint_as_float(o[ch * 8 + 2]) * inv_l, __uint_as_float(o[ch * 8 + 3]) * inv_l);
          w.z = pack2<kBf16>(__uint_as_float(o[ch * 8 + 4]) * inv_l, __uint_as_float(o[ch * 8 + 5]) * inv_l);
          w.w = pack2<kBf16>(__uint_as_float(o[ch * 8 + 6]) * inv_l, __uint_as_float(o[ch * 8 + 7]) * inv_l);
          *reinterpret_cast<uint4*>(sQ + swz_offset(r, cb * 32 + ch * 8, kTileRows)) = w;
        }
      }
      fence_proxy_async_smem();
    }
    named_barrier_sync(1, 128);
    if (ok && q4 == 0 && lane == 0 && !ctl->abort) {
      // A store may clip a partial column block but never starts past the
      // tensor's true width.
      for (int b = 0; b < NB && b * 64 < d_real; ++b) tma_store_3d(&tm_o, sQ + b * kBlockBytes, b * 64, m0, bh);
      tma_store_commit();
      tma_store_wait_read_all();
    }
    if (ok && lse != nullptr && row_g < S) lse[static_cast<size_t>(bh) * S + row_g] = m_run + lg2(l_run);
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
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return kErrLaunch;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
      return kErrLaunch;
    attr_set[dev] = true;
  }
  const int n_qtiles = static_cast<int>((a.S + kTileRows - 1) / kTileRows);
  const long long grid = static_cast<long long>(n_qtiles) * a.BH;
  if (grid > INT32_MAX) return kErrTooLarge;
  kern<<<static_cast<unsigned>(grid), kD256Threads, C::kSmemBytes, a.stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_v, *a.tm_o, a.lse, static_cast<int>(a.S), n_qtiles, a.causal, static_cast<int>(a.D),
      a.scale_log2, a.timeout_ns, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_attn_fwd_d256(const FwdD256Args& a) {
  if (a.D > 256) return kErrUnsupported;
  if (a.D <= 192) return a.bf16 ? launch_d256_t<3, true>(a) : launch_d256_t<3, false>(a);
  return a.bf16 ? launch_d256_t<4, true>(a) : launch_d256_t<4, false>(a);
}

}  // namespace tk
