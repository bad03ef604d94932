// Deterministic dQ for the flash-attention backward on sm_100a: one CTA owns
// a 128-row query tile of one (batch, head), keeps dQ in tensor memory and
// streams the key/value tiles, so dQ is the sum over key tiles in one fixed
// order with no atomics — bitwise reproducible from run to run.
//
// Semantics follow the reference `_attn_bwd_dq_kernel`
// (src/tklab/kernels/flash_attention.py:469-533): for each key block (causal:
// up to the diagonal, :513) recompute
//   P  = exp2(scale*log2(e) * Q.K^T - LSE2)      dP = dO.V^T
//   dS = P * (dP - delta)                       dQ += dS.K
// with dS rounded to the input dtype for its product (:530), the diagonal
// and the ragged key tail masked (:523-526), and dQ scaled by the softmax
// scale at the end (:532).
//
// 12 warps in three warpgroups (setmaxnreg 56 / 224 / 224):
//   WG0  warp 0   TMA producer of Q and dO (once) and the K ring
//        warp 1   TMEM allocator and tcgen05.mma issuer (converged warp, one
//                 elected lane issues)
//        warp 2   TMA producer of the V ring
//   WG1, WG2  keys 0..63 (WG1) and 64..127 (WG2) of every key tile; thread
//             t owns query row t (TMEM lane t).  Per key tile: load its
//             halves of S and dP, release them, form P and dS in registers,
//             write dS packed to 16 bits into TMEM (the A operand of
//             dQ += dS.K).  Epilogue: each stores one column half of dQ.
// Tensor memory: S [0,128), dP [128,256), dQ [256,256+D), dS in two 64-column
// buffers from 256+D (tile j uses buffer j&1).
// MMA order per key tile j: S(j+1) and dP(j+1) as soon as the compute warps
// have read S(j) and dP(j), then dQ += dS(j).K(j), so the products of the next
// tile run while the compute warps work on the current one; S/dP go first
// because the compute warps wait for them next.  A tcgen05.commit tracks every
// earlier MMA of the issuing thread, and dQ(j-1) is issued before S(j+1), so
// the completion of S(j+1) (sdp_full) also means dQ(j-1) has read dS buffer
// (j+1)&1: the compute warps need no separate "dS free" wait.  (Issuing dQ
// from a second warp was measured slower: its MMAs then interleave with
// S(j+1)/dP(j+1) and delay the products the compute warps wait for.)
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

// Exponential pairs of every 8 computed on the FMA pipe in unmasked tiles
// (2 of 8: deterministic backward 3.53 -> 3.37 ms at C3).
#ifndef TK_DQ_EMU_PAIRS_PER8
#define TK_DQ_EMU_PAIRS_PER8 2
#endif
constexpr int kDqEmuPairsPer8 = TK_DQ_EMU_PAIRS_PER8;

template <int D>
struct DqCfg {
  // K_j stays until dQ(j) has read it, so its ring is one deeper than V's.
  static constexpr int kKStages = (D == 64) ? 4 : 3;
  static constexpr int kVStages = (D == 64) ? 4 : 2;
  static constexpr int kTileBytes = kTileRows * D * 2;
  static constexpr int kQOff = 0;
  static constexpr int kDOOff = kQOff + kTileBytes;
  static constexpr int kKOff = kDOOff + kTileBytes;
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kVStages * kTileBytes;
  // qdo_full, kv_full[KS], k_empty[KS], v_empty[VS], sdp_full, sdp_free,
  // ds_ready[2], dq_done.  K_j and V_j land on one barrier, kv_full[j % KS]
  // (two producer arrivals plus both tiles' bytes), so the MMA warp polls
  // once per tile for its operands.
  static constexpr int kNumBars = 1 + 2 * kKStages + kVStages + 5;
  static constexpr int kCtlOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kCtlOff + 64;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColDP = 128;
  static constexpr uint32_t kColDQ = 256;
  static constexpr uint32_t kColDS = 256 + D;  // two buffers of 64 columns
  static_assert(kColDS + 128 <= kTmemCols, "tensor memory overflow");
};

constexpr int kDqThreads = 384;
// Launch allocation 168 registers x 384 threads; the control warpgroup keeps
// 56 and each compute warpgroup gets 224 (56 + 2 x 224 = 3 x 168).
constexpr int kDqLaunchRegs = 168;
constexpr int kDqRegsCtrl = 56;
constexpr int kDqRegsCompute = 224;
static_assert(kDqRegsCtrl + 2 * kDqRegsCompute <= 3 * kDqLaunchRegs, "register split exceeds the launch");

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, CtaControl* ctl, uint64_t timeout_ns,
                                          int* status, int site) {
  const bool ok = mbar_wait(bar, parity, ctl, timeout_ns, status, site);
  return __all_sync(0xffffffffu, ok);
}

template <int D, bool kBf16>
__global__ void __launch_bounds__(kDqThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse,
                       const float* __restrict__ delta, int S, int BH, int n_tiles, int causal, float scale,
                       float scale_log2, unsigned long long timeout_ns, int* status) {
  using C = DqCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  // Head-major order, heaviest query tile (most key tiles under a causal
  // mask) of each head first.
  const int bh = static_cast<int>(blockIdx.x) / n_tiles;
  const int qi = n_tiles - 1 - static_cast<int>(blockIdx.x) % n_tiles;
  const int m0 = qi * kTileRows;
  const int n_kv = causal ? qi + 1 : n_tiles;

  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sDO = smem + C::kDOOff;
  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* qdo_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* k_empty = kv_full + C::kKStages;
  uint64_t* v_empty = k_empty + C::kKStages;
  uint64_t* sdp_full = v_empty + C::kVStages;
  uint64_t* sdp_free = sdp_full + 1;
  // ds_ready[2], by tile parity like the dS buffers it hands over: the MMA
  // warp issues S/dP(t) before it takes dS(t-1), so the compute warps can
  // finish tiles t-1 and t before it looks; one barrier would then be two
  // phases ahead of its parity wait.  Tile t+2, the next user of
  // ds_ready[t & 1], needs S/dP(t+2), issued only after dS(t) was taken.
  uint64_t* ds_ready = sdp_free + 1;
  uint64_t* dq_done = ds_ready + 2;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kCtlOff);

  if (threadIdx.x == 0) {
    mbar_init(qdo_full, 1);
    for (int i = 0; i < C::kKStages; ++i) {
      mbar_init(&kv_full[i], 2);  // the K and the V producer
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < C::kVStages; ++i) mbar_init(&v_empty[i], 1);
    mbar_init(sdp_full, 1);
    mbar_init(sdp_free, 8);  // every warp of both compute warpgroups
    mbar_init(&ds_ready[0], 8);
    mbar_init(&ds_ready[1], 8);
    mbar_init(dq_done, 1);
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
    tma_prefetch_map(&tm_do);
    tma_prefetch_map(&tm_dq);
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (wg == 0) {
    warpgroup_reg_dec<kDqRegsCtrl>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      mbar_arrive_expect_tx(qdo_full, 2 * C::kTileBytes);
#pragma unroll
      for (int b = 0; b < D / 64; ++b) {
        tma_load_3d(sQ + b * kBlockBytes, &tm_q, qdo_full, b * 64, m0, bh);
        tma_load_3d(sDO + b * kBlockBytes, &tm_do, qdo_full, b * 64, m0, bh);
      }
      for (int j = 0; j < n_kv; ++j) {
        const int ks = j % C::kKStages;
        if (!mbar_wait(&k_empty[ks], ((j / C::kKStages) & 1) ^ 1, ctl, timeout_ns, status, 1)) break;
        mbar_arrive_expect_tx(&kv_full[ks], C::kTileBytes);
#pragma unroll
        for (int b = 0; b < D / 64; ++b)
          tma_load_3d(sK + ks * C::kTileBytes + b * kBlockBytes, &tm_k, &kv_full[ks], b * 64, j * kTileRows, bh);
      }
    } else if (warp == 2 && lane == 0) {
      // ---------------- V producer: its own thread, so a V load never waits
      // behind a K slot (K_j is held until dQ(j), V_j only until dP(j)).
      // kv_full[j % KS] cannot receive tile j+KS's arrivals before tile j's
      // phase completes: K_{j+KS} waits for dQ(j) and V_{j+KS} for
      // dP(j+KS-VS), both issued only after that phase. ----------------
      for (int j = 0; j < n_kv; ++j) {
        const int vs = j % C::kVStages;
        if (!mbar_wait(&v_empty[vs], ((j / C::kVStages) & 1) ^ 1, ctl, timeout_ns, status, 2)) break;
        uint64_t* full = &kv_full[j % C::kKStages];
        mbar_arrive_expect_tx(full, C::kTileBytes);
#pragma unroll
        for (int b = 0; b < D / 64; ++b)
          tma_load_3d(sV + vs * C::kTileBytes + b * kBlockBytes, &tm_v, full, b * 64, j * kTileRows, bh);
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      const bool leader = elect_one();
      const uint32_t fmt = kBf16 ? 1u : 0u;
      const uint32_t idesc_s = idesc_f16(fmt, 128, 128, 0, 0);
      const uint32_t idesc_dq = idesc_f16(fmt, 128, D, 0, 1);
      const uint32_t q_lo = sdesc_lo_kmajor(smem_u32(sQ));
      const uint32_t do_lo = sdesc_lo_kmajor(smem_u32(sDO));
      const uint32_t k_lo0 = sdesc_lo_kmajor(smem_u32(sK));
      const uint32_t k_mn_lo0 = sdesc_lo_mnmajor(smem_u32(sK), kTileRows);
      const uint32_t v_lo0 = sdesc_lo_kmajor(smem_u32(sV));
      constexpr uint32_t kTileLo = C::kTileBytes >> 4;
      // tcgen05.mma issue blocks at about the tensor core's execution rate
      // and only a few MMAs queue ahead of it, so every barrier poll of this
      // warp between two MMA batches risks idling the tensor core.  The loop
      // therefore has at most two polls after the S/dP batch (the next
      // tile's operands and ds_ready) and one after the dQ batch (sdp_free),
      // each normally satisfied already and covered by the queued MMAs.
      // One copy of each step and rolled MMA loops keep the code compact:
      // this warp sleeps while the compute warps stream long unrolled bodies
      // through the instruction cache.
      //
      // Step t: S(t) and dP(t) once the compute warps have read S(t-1) and
      // dP(t-1), then dQ += dS(t-1) K_{t-1}.
      bool ok = warp_wait(qdo_full, 0, ctl, timeout_ns, status, 5);
      if (ok && n_kv > 0) ok = warp_wait(&kv_full[0], 0, ctl, timeout_ns, status, 3);
      for (int t = 0; ok && t <= n_kv; ++t) {
        if (t < n_kv) {
          const int ks = t % C::kKStages, vs = t % C::kVStages;
          if (t > 0 && !(ok = warp_wait(sdp_free, (t - 1) & 1, ctl, timeout_ns, status, 6))) break;
          tc_fence_after();
          if (leader) {
            const uint32_t k_lo = k_lo0 + ks * kTileLo;
            const uint32_t v_lo = v_lo0 + vs * kTileLo;
#pragma unroll 1
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = kmajor_koff(kTileRows, kk * 16);
              const uint32_t acc = kk > 0 ? 1u : 0u;
              umma_ss_w(tmem + C::kColS, q_lo + off, k_lo + off, idesc_s, acc);
              umma_ss_w(tmem + C::kColDP, do_lo + off, v_lo + off, idesc_s, acc);
            }
            umma_commit(sdp_full);
            umma_commit(&v_empty[vs]);  // V_t is only read by dP(t)
          }
          __syncwarp();
          const int tn = t + 1;
          if (tn < n_kv &&
              !(ok = warp_wait(&kv_full[tn % C::kKStages], (tn / C::kKStages) & 1, ctl, timeout_ns, status, 4)))
            break;
        }
        if (t > 0) {
          // dQ += dS(j) K_j with dS(j) packed in TMEM buffer j&1.
          const int j = t - 1;
          const int ks = j % C::kKStages;
          if (!(ok = warp_wait(&ds_ready[j & 1], (j >> 1) & 1, ctl, timeout_ns, status, 7))) break;
          tc_fence_after();
          if (leader) {
            const uint32_t k_mn_lo = k_mn_lo0 + ks * kTileLo;
            const uint32_t ds_col = tmem + C::kColDS + 64u * (j & 1);
#pragma unroll 1
            for (int kk = 0; kk < kTileRows / 16; ++kk)
              umma_ts_w(tmem + C::kColDQ, ds_col + kk * 8, k_mn_lo + mnmajor_koff(kk * 16), idesc_dq,
                        (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&k_empty[ks]);  // K_j was read by S(j) and dQ(j)
            if (t == n_kv) umma_commit(dq_done);
          }
          __syncwarp();
        }
      }
    }
  } else {
    warpgroup_reg_inc<kDqRegsCompute>();
    // ---------------- compute warpgroup h: keys 64h..64h+63 of each tile ----------------
    const int h = wg - 1;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row within the tile (TMEM lane)
    const int row_g = m0 + r;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t s_cols = t_lane + C::kColS + 64u * h;
    const uint32_t dp_cols = t_lane + C::kColDP + 64u * h;
    const uint32_t ds_cols = t_lane + C::kColDS + 32u * h;
    // Padded query rows (row_g >= S) get LSE = +inf, so P = dS = 0.
    const bool row_ok = row_g < S;
    const float lse_r = row_ok ? lse[static_cast<size_t>(bh) * S + row_g] : INFINITY;
    const float delta_r = row_ok ? delta[static_cast<size_t>(bh) * S + row_g] : 0.0f;
    const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
    const uint64_t nlse2 = f2_pack(-lse_r, -lse_r);
    const uint64_t ndelta2 = f2_pack(-delta_r, -delta_r);
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!(ok = warp_wait(sdp_full, j & 1, ctl, timeout_ns, status, 8))) break;
      tc_fence_after();
      uint32_t s[2][32], dp[2][32];
      tmem_ld32(s_cols, s[0]);
      tmem_ld32(s_cols + 32, s[1]);
      tmem_ld32(dp_cols, dp[0]);
      tmem_ld32(dp_cols + 32, dp[1]);
      tmem_wait_ld();
      reg_fence(s[0]);
      reg_fence(s[1]);
      reg_fence(dp[0]);
      reg_fence(dp[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sdp_free);
      // Keys of this half: n0 + c.  Masked: keys past the sequence and, on
      // the causal diagonal, keys after the query.
      const int n0 = j * kTileRows + 64 * h;
      int lim = S - n0;
      if (causal) lim = min(lim, row_g - n0 + 1);
      const bool masked = __any_sync(0xffffffffu, lim < 64);
      uint32_t pk[2][16];
#pragma unroll
      for (int b = 0; b < 2; ++b) {
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          // Pairs of keys per packed fp32x2 instruction.
          float x0, x1;
          f2_unpack(ffma2(f2_pack(__uint_as_float(s[b][c]), __uint_as_float(s[b][c + 1])), scale2, nlse2), x0, x1);
          float p0, p1;
          // Unmasked tiles put kDqEmuPairsPer8 of every 8 exponential pairs
          // on the FMA pipe (exp2_fma_pair) so the MUFU does not set the pace.
          if (!masked && ((c >> 1) & 7) >= 8 - kDqEmuPairsPer8) {
            exp2_fma_pair(x0, x1, p0, p1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          if (masked) {
            if (b * 32 + c >= lim) p0 = 0.0f;
            if (b * 32 + c + 1 >= lim) p1 = 0.0f;
          }
          float d0, d1;
          f2_unpack(fmul2(f2_pack(p0, p1),
                          fadd2(f2_pack(__uint_as_float(dp[b][c]), __uint_as_float(dp[b][c + 1])), ndelta2)),
                    d0, d1);
          pk[b][c >> 1] = pack2<kBf16>(d0, d1);
        }
      }
      // dS buffer j&1 was last read by dQ(j-2), complete since sdp_full(j).
      tmem_st16(ds_cols + 64u * (j & 1), pk[0]);
      tmem_st16(ds_cols + 64u * (j & 1) + 16, pk[1]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_ready[j & 1]);
    }
    // Epilogue: dQ * scale -> the input dtype, staged through the Q buffer
    // (dead once the last S product has completed, which dq_done implies);
    // each warpgroup stages one column half, then one thread stores the tile
    // (rows >= S and columns past the true head_dim are clipped by the map).
    if (ok) ok = warp_wait(dq_done, 0, ctl, timeout_ns, status, 10);
    if (ok) {
      tc_fence_after();
      constexpr int kHalfD = D / 2;
#pragma unroll
      for (int cb = 0; cb < kHalfD / 32; ++cb) {
        uint32_t v[32];
        tmem_ld32(t_lane + C::kColDQ + kHalfD * h + cb * 32, v);
        tmem_wait_ld();
        reg_fence(v);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint4 w;
          w.x = pack2<kBf16>(__uint_as_float(v[ch * 8 + 0]) * scale, __uint_as_float(v[ch * 8 + 1]) * scale);
          w.y = pack2<kBf16>(__uint_as_float(v[ch * 8 + 2]) * scale, __uint_as_float(v[ch * 8 + 3]) * scale);
          w.z = pack2<kBf16>(__uint_as_float(v[ch * 8 + 4]) * scale, __uint_as_float(v[ch * 8 + 5]) * scale);
          w.w = pack2<kBf16>(__uint_as_float(v[ch * 8 + 6]) * scale, __uint_as_float(v[ch * 8 + 7]) * scale);
          *reinterpret_cast<uint4*>(sQ + swz_offset(r, kHalfD * h + cb * 32 + ch * 8, kTileRows)) = w;
        }
      }
      fence_proxy_async_smem();
    }
    // Both compute warpgroups reach this barrier exactly once.
    named_barrier_sync(1, 256);
    if (h == 0 && q4 == 0 && lane == 0 && !ctl->abort) {
#pragma unroll
      for (int b = 0; b < D / 64; ++b) tma_store_3d(&tm_dq, sQ + b * kBlockBytes, b * 64, m0, bh);
      tma_store_commit();
      tma_store_wait_read_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int D, bool kBf16>
int launch_dq_t(const BwdDqArgs& a) {
  using C = DqCfg<D>;
  static_assert(C::kSmemBytes <= 232448, "dQ kernel shared memory exceeds the sm_100 limit");
  auto kern = attn_bwd_dq_kernel<D, kBf16>;
  // The setmaxnreg split inside the kernel assumes exactly kDqLaunchRegs
  // registers per thread at launch; a build that differs is refused.
  if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern), C::kSmemBytes, kDqLaunchRegs, nullptr))
    return rc;
  const int n_tiles = static_cast<int>((a.S + kTileRows - 1) / kTileRows);
  const long long grid = static_cast<long long>(n_tiles) * a.BH;
  kern<<<static_cast<unsigned>(grid), kDqThreads, C::kSmemBytes, a.stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_v, *a.tm_do, *a.tm_dq, a.lse, a.delta, static_cast<int>(a.S),
      static_cast<int>(a.BH), n_tiles, a.causal, a.scale, a.scale_log2, a.timeout_ns, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_attn_bwd_dq(const BwdDqArgs& a) {
  if (a.D <= 64) return a.bf16 ? launch_dq_t<64, true>(a) : launch_dq_t<64, false>(a);
  if (a.D <= 128) return a.bf16 ? launch_dq_t<128, true>(a) : launch_dq_t<128, false>(a);
  return kErrUnsupported;
}

}  // namespace tk
