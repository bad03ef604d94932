// Flash-attention forward for sm_100a (B200): TMA-fed Q/K/V tiles, tcgen05
// MMAs accumulating S = Q.K^T and O += P.V in tensor memory, online softmax
// in base 2 with the scale folded in, causal tile skipping and a separate
// masked path for the diagonal / ragged-tail key tiles.
//
// Semantics follow the reference Triton kernel
// (src/tklab/kernels/flash_attention.py:54-117 `_attention_inner` and
// :120-264 `_flash_attention_forward_kernel`): scores are scaled by
// scale*log2(e) before the running maximum, probabilities are exp2 of the
// scaled score minus the running maximum, P is rounded to the input dtype
// for the P.V product, O = acc / row_sum, and the optional statistic is the
// base-2 log-sum-exp `row_max + log2(row_sum)` (:254-264).
//
// At head_dim 128 a work item is two consecutive 128-row query tiles (A and
// B) of one (batch, head); the CTA streams the key/value tiles once for both,
// 12 warps, one CTA per SM.  At head_dim 64 an item is one query tile (A
// only): 8 warps, 256 tensor-memory columns and 80 KB of shared memory, so
// two CTAs share an SM and each tile's S -> softmax -> P.V chain runs on its
// own MMA warp instead of taking turns with a second tile on one (the same
// math per row; 2-21 % faster at head_dim 64 than two tiles per CTA).  Large
// causal problems and short ones run persistent CTAs (one or two per SM)
// over balanced units of items (the next item's Q load and first products
// overlap the current epilogue); otherwise one CTA runs one item.  Warpgroups,
// registers rebalanced with setmaxnreg:
//   WG0  warp 0   TMA producer (Q_A and Q_B per item, then K and V tiles
//                 through two rings)
//        warp 1   TMEM allocator and tcgen05.mma issuer (the warp runs the
//                 loop converged, one elected lane issues)
//   WG1  warps 4..7   softmax of tile A: thread t owns query row t (TMEM
//                     lane t); also rescales O_A when its running maximum
//                     moves, and runs tile A's epilogue (O_A / row_sum
//                     stored from registers straight to global memory by
//                     persistent CTAs, staged through Q_A for one TMA store
//                     otherwise)
//   WG2  warps 8..11  the same for tile B (head_dim 128 only)
// Tensor memory: O_A, O_B (D columns each), then S_A and S_B (128 columns
// each); at head_dim 64 O_A and S_A in 256 columns.  P is written back as packed 16-bit pairs over the
// first 64 columns of its tile's S and consumed from TMEM by the P.V MMA.
// MMA issue order per key tile j: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), so
// while the softmax of one tile runs the tensor core works on the other
// tile.  S_X(j+1) is issued after PV_X(j), so once a softmax warpgroup sees
// S_X(j+1) complete it may rescale O_X without a separate barrier.
// Problems with too few items to fill the device, whose longest item would
// set the kernel's time, may run in the key-split mode (kOrderSplit below,
// with a caller workspace): chunks of an item's key range in separate CTAs,
// merged by attn_fwd_combine_kernel.
#include <algorithm>
#include <type_traits>

#include "attn_fwd_split_plan.h"
#include "attn_launch.h"
#include "rope_sm100.cuh"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

template <int D>
struct FwdCfg {
  // Query tiles per CTA (and softmax warpgroups), CTAs per SM.
  static constexpr int kT = (D == 64) ? 1 : 2;
  static constexpr int kMinBlocks = (kT == 1) ? 2 : 1;
  static constexpr int kThreads = 128 * (1 + kT);
  // Launch allocation kLaunchRegs x kThreads; after setmaxnreg the control
  // warpgroup keeps 56 and each softmax warpgroup gets kRegsSoftmax
  // (56 + kT x kRegsSoftmax = (1 + kT) x kLaunchRegs), so the increases are
  // always satisfiable; two 256-thread CTAs x 128 registers fill an SM.
  static constexpr int kLaunchRegs = (kT == 1) ? 128 : 168;
  static constexpr int kRegsCtrl = 56;
  static constexpr int kRegsSoftmax = (kT == 1) ? 200 : 224;
  static_assert(kRegsCtrl + kT * kRegsSoftmax <= (1 + kT) * kLaunchRegs, "register split exceeds the launch");
  static constexpr int kStages = 2;
  static constexpr int kTileBytes = kTileRows * D * 2;
  static constexpr int kQOff = 0;  // Q_A (, Q_B)
  static constexpr int kKOff = kQOff + kT * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  // q_full, q_empty, k_full[S], k_empty[S], v_full[S], v_empty[S],
  // s_full[2], p_ready[2], o_final[2], q_rot[2] (the last only used with
  // RoPE)
  static constexpr int kNumBars = 2 + 4 * kStages + 8;
  static constexpr int kCtlOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kCtlOff + 64;
  static constexpr uint32_t kTmemCols = (kT == 1) ? 256 : 512;
  // O of tile x at column x * D, S of tile x at kT D + 128 x.
  static constexpr uint32_t kColO0 = 0;
  static constexpr uint32_t kColS0 = kT * D;
};

// The running maximum used for P is only moved when the true maximum exceeds
// it by more than this (base-2 units), so P <= 2^8 and O is rescaled rarely.
// The result is unchanged mathematically because O and row_sum always share
// the same reference maximum.
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, CtaControl* ctl,
                                          uint64_t timeout_ns, int* status, int site) {
  const bool ok = mbar_wait(bar, parity, ctl, timeout_ns, status, site);
  return __all_sync(0xffffffffu, ok);
}

// Of every 8 column pairs of an unmasked tile, this many take their exp2 on
// the FMA pipe (exp2_fma_pair, packed fp32x2 arithmetic) and the rest on the
// MUFU, which alone would bound a tile at 1024 cycles (16384 exponentials at
// 16 per clock per SM) while the rest of the softmax needs about three issue
// slots per element.
#ifndef TK_FWD_EMU_PAIRS_PER8
#define TK_FWD_EMU_PAIRS_PER8 3
#endif
constexpr int kEmuPairsPer8 = TK_FWD_EMU_PAIRS_PER8;

template <bool kMasked>
__device__ __forceinline__ void max_chunk(uint32_t (&s)[32], int col0, int lim, float (&mx)[8]) {
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    float v0 = __uint_as_float(s[c]), v1 = __uint_as_float(s[c + 1]);
    if constexpr (kMasked) {
      if (col0 + c >= lim) {
        v0 = -INFINITY;
        s[c] = __float_as_uint(v0);
      }
      if (col0 + c + 1 >= lim) {
        v1 = -INFINITY;
        s[c + 1] = __float_as_uint(v1);
      }
    }
    mx[(c >> 1) & 7] = fmax3(mx[(c >> 1) & 7], v0, v1);
  }
}

// Online-softmax step for one row and one 128-key tile of S at s_addr (TMEM):
// loads S (two halves, the second overlapping the first half's maximum),
// updates the running maximum / sum, returns the rescale factor of the
// previous accumulator (alpha) and whether the maximum moved (need), and
// writes P (16-bit pairs) over the first 64 TMEM columns at s_addr.
template <bool kBf16, bool kMasked>
__device__ __forceinline__ void softmax_tile(uint32_t s_addr, int lim, float scale_log2, float& m_run,
                                             float& l_run, float& alpha, bool& need) {
  uint32_t s[4][32];
  tmem_ld32(s_addr, s[0]);
  tmem_ld32(s_addr + 32, s[1]);
  tmem_wait_ld();
  reg_fence(s[0]);
  reg_fence(s[1]);
  tmem_ld32(s_addr + 64, s[2]);
  tmem_ld32(s_addr + 96, s[3]);
  float mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
  max_chunk<kMasked>(s[0], 0, lim, mx);
  max_chunk<kMasked>(s[1], 32, lim, mx);
  tmem_wait_ld();
  reg_fence(s[2]);
  reg_fence(s[3]);
  max_chunk<kMasked>(s[2], 64, lim, mx);
  max_chunk<kMasked>(s[3], 96, lim, mx);
  const float mxa = fmax3(mx[0], mx[1], mx[2]), mxb = fmax3(mx[3], mx[4], mx[5]);
  const float m_tile = fmax3(mxa, mxb, fmaxf(mx[6], mx[7]));
  const float m_new = fmaxf(m_run, m_tile * scale_log2);
  need = m_new > m_run + kRescaleThreshold;
  const float m_use = need ? m_new : m_run;
  alpha = (m_run == -INFINITY) ? 0.0f : ex2(m_run - m_use);
  const float ms = (m_use == -INFINITY) ? 0.0f : m_use;
  // x = s * scale_log2 - max and the row sum run on packed pairs.
  const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
  const uint64_t negm2 = f2_pack(-ms, -ms);
  uint64_t sum2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 32; c += 2) {
      float x0, x1;
      f2_unpack(ffma2(f2_pack(__uint_as_float(s[b][c]), __uint_as_float(s[b][c + 1])), scale2, negm2), x0, x1);
      float p0, p1;
      // Masked tiles keep every exponential on the MUFU so that masked
      // entries are exactly zero.
      if (!kMasked && ((c >> 1) & 7) >= 8 - kEmuPairsPer8) {
        exp2_fma_pair(x0, x1, p0, p1);
      } else {
        p0 = ex2(x0);
        p1 = ex2(x1);
      }
      sum2[(c >> 1) & 1] = fadd2(sum2[(c >> 1) & 1], f2_pack(p0, p1));
      pk[c >> 1] = pack2<kBf16>(p0, p1);
    }
    tmem_st16(s_addr + b * 16, pk);
  }
  float sa0, sa1, sb0, sb1;
  f2_unpack(sum2[0], sa0, sa1);
  f2_unpack(sum2[1], sb0, sb1);
  l_run = l_run * alpha + ((sa0 + sa1) + (sb0 + sb1));
  m_run = m_use;
}

// Work is split into units of one or two query-tile pairs ("items"), walked
// by every CTA with a stride of gridDim.x.  Modes:
//   kOrderHead   one item per unit, head-major (the pairs of one head are
//                adjacent, so resident CTAs share a few heads' K/V in L2),
//                heaviest pair of a head first;
//   kOrderLpt    one item per unit, heaviest pairs of every head first (when
//                all heads' K/V fit in L2 together);
//   kOrderPaired unit u of head bh holds the pairs ct = n_ctiles-1-p and
//                ct = p, so every causal unit costs the same number of key
//                tiles and a static stride over units keeps persistent CTAs
//                balanced.
//   kOrderSplit  (few, long items: the longest would set the kernel's time)
//                unit = one chunk of at most split_l key tiles of one item,
//                enumerated chunk level by chunk level (every item's chunk 0,
//                then chunk 1 of the items that have one, ...), heaviest
//                query tiles first within a head.  Items with more than one
//                chunk write O / row_sum of each chunk in fp32 and its base-2
//                log-sum-exp to a workspace; attn_fwd_combine_kernel merges
//                them.  The last chunk of an item also carries tile B's extra
//                (diagonal) key tile, so every chunk has work for both tiles.
// The launcher runs one CTA per unit (hardware scheduling) in the first two
// modes and the split mode, and one persistent CTA per SM in the third.
constexpr int kOrderHead = 0;
constexpr int kOrderLpt = 1;
constexpr int kOrderPaired = 2;
constexpr int kOrderSplit = 3;

__device__ __forceinline__ int fwd_unit_items(int u, int n_ctiles, int mode) {
  if (mode != kOrderPaired) return 1;
  const int p = u % ((n_ctiles + 1) / 2);
  return (p == n_ctiles - 1 - p) ? 1 : 2;
}

__device__ __forceinline__ void fwd_unit_item(int u, int sub, int BH, int n_ctiles, int mode, int& bh, int& ct) {
  if (mode == kOrderPaired) {
    const int n_pairs = (n_ctiles + 1) / 2;
    bh = u / n_pairs;
    const int p = u % n_pairs;
    ct = (sub == 0) ? n_ctiles - 1 - p : p;
  } else if (mode == kOrderLpt) {
    bh = u % BH;
    ct = n_ctiles - 1 - u / BH;
  } else {
    bh = u / n_ctiles;
    ct = n_ctiles - 1 - u % n_ctiles;
  }
}

// One item as a role sees it: slab, query-tile group, first key tile and the
// number of key tiles of tile A / tile B from there.
struct FwdItem {
  int bh, ct, j0, n_a, n_b, chunk;
  bool split;  // one of several chunks: partial result to the workspace
};

// split_item: the CTA's (bh, ct, chunk) in shared memory, decoded by
// fwd_split_decode (split mode only).
template <int kT, bool kSplit>
__device__ __forceinline__ FwdItem fwd_item(int u, int sub, int BH, int n_ctiles, int n_ntiles, int causal,
                                            int mode, int split_l, const int* split_item) {
  FwdItem f;
  f.chunk = 0;
  if constexpr (kSplit) {
    f.bh = split_item[0];
    f.ct = split_item[1];
    f.chunk = split_item[2];
  } else {
    fwd_unit_item(u, sub, BH, n_ctiles, mode, f.bh, f.ct);
  }
  const int na = causal ? min(kT * f.ct + 1, n_ntiles) : n_ntiles;
  const int nb = causal ? min(kT * f.ct + kT, n_ntiles) : n_ntiles;
  if constexpr (kSplit) {
    f.j0 = f.chunk * split_l;
    const int ea = min(f.j0 + split_l, na);
    const int eb = (ea == na) ? nb : ea;
    f.n_a = ea - f.j0;
    f.n_b = eb - f.j0;
    f.split = na > split_l;
  } else {
    f.j0 = 0;
    f.n_a = na;
    f.n_b = nb;
    f.split = false;
  }
  return f;
}

// kRope: rotate-half RoPE (tables rope_cos / rope_sin, (S, D/2) fp32) is
// applied to each item's Q tiles in shared memory after their TMA load and
// before the S products read them, by the softmax warpgroups (thread r
// rotates row r of its own tile) at the start of the item, where they would
// otherwise wait for S(0).  K arrives rotated (the caller rotates it once:
// every CTA streams every K tile, so rotating K here would repeat the work
// once per query tile).
// kSplit: the key-split schedule (mode kOrderSplit, chunk partials to
// o_part / lse_part); the regular kernels carry none of its code.
template <int D, bool kBf16, bool kRope, bool kSplit>
__global__ void __launch_bounds__(FwdCfg<D>::kThreads, FwdCfg<D>::kMinBlocks)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    uint16_t* __restrict__ out, float* __restrict__ lse, const float* __restrict__ rope_cos,
                    const float* __restrict__ rope_sin,
                    int S, int BH, int n_ctiles, int causal, int mode, int n_units, int d_real, float scale_log2,
                    unsigned long long timeout_ns, int* status, int split_l, int split_cmax,
                    float* __restrict__ o_part, float* __restrict__ lse_part) {
  using C = FwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  const int n_ntiles = (S + kTileRows - 1) / kTileRows;

  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + C::kStages;
  uint64_t* v_full = k_empty + C::kStages;
  uint64_t* v_empty = v_full + C::kStages;
  uint64_t* s_full = v_empty + C::kStages;  // [2]
  uint64_t* p_ready = s_full + 2;           // [2]
  uint64_t* o_final = p_ready + 2;          // [2]
  uint64_t* q_rot = o_final + 2;           // [2]: Q_x rotated (RoPE)
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kCtlOff);
  int* split_item = reinterpret_cast<int*>(smem + C::kCtlOff + 16);  // [3], split mode

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_final[i], 1);
    }
    mbar_init(&q_rot[0], 4);  // the four warps of softmax warpgroup x
    mbar_init(&q_rot[1], 4);
    ctl->abort = 0;
    if constexpr (kSplit) fwd_split_decode(blockIdx.x, BH, n_ctiles, causal, C::kT, split_l, split_item);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
    tma_prefetch_map(&tm_o);
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // Every role walks the same item sequence: units blockIdx.x, +gridDim.x,
  // ...; barrier phases follow running counters (items, key tiles, S and P
  // tiles per query tile) so consecutive items pipeline into each other.
  if (wg == 0) {
    warpgroup_reg_dec<C::kRegsCtrl>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t g = 0;  // key tiles loaded so far
      int it = 0;      // items so far
      bool ok = true;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
        const int n_sub = fwd_unit_items(u, n_ctiles, mode);
        for (int sub = 0; ok && sub < n_sub; ++sub, ++it) {
          const FwdItem f = fwd_item<C::kT, kSplit>(u, sub, BH, n_ctiles, n_ntiles, causal, mode, split_l, split_item);
          const int bh = f.bh;
          const int m0 = f.ct * C::kT * kTileRows;
          const int n_kv_b = f.n_b;
          // Q_A and Q_B are free once the previous item's last S product
          // has completed.
          if (it > 0 && !(ok = mbar_wait(q_empty, (it - 1) & 1, ctl, timeout_ns, status, 13))) break;
          mbar_arrive_expect_tx(q_full, C::kT * C::kTileBytes);
#pragma unroll
          for (int x = 0; x < C::kT; ++x)
#pragma unroll
            for (int b = 0; b < D / 64; ++b)
              tma_load_3d(sQ + x * C::kTileBytes + b * kBlockBytes, &tm_q, q_full, b * 64, m0 + x * kTileRows, bh);
          // kr: first row of the key tile being loaded.
          int kr = f.j0 * kTileRows;
          for (int left = n_kv_b; left > 0; --left, ++g, kr += kTileRows) {
            const int st = g % C::kStages;
            const uint32_t ph = (g / C::kStages) & 1;
            if (!(ok = mbar_wait(&k_empty[st], ph ^ 1, ctl, timeout_ns, status, 1))) break;
            mbar_arrive_expect_tx(&k_full[st], C::kTileBytes);
#pragma unroll
            for (int b = 0; b < D / 64; ++b)
              tma_load_3d(sK + st * C::kTileBytes + b * kBlockBytes, &tm_k, &k_full[st], b * 64, kr, bh);
            if (!(ok = mbar_wait(&v_empty[st], ph ^ 1, ctl, timeout_ns, status, 2))) break;
            mbar_arrive_expect_tx(&v_full[st], C::kTileBytes);
#pragma unroll
            for (int b = 0; b < D / 64; ++b)
              tma_load_3d(sV + st * C::kTileBytes + b * kBlockBytes, &tm_v, &v_full[st], b * 64, kr, bh);
          }
        }
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      // The whole warp runs the loop (waits included) so that addresses and
      // descriptors stay warp-uniform; one elected lane issues each
      // tcgen05.mma / commit.  Descriptors are precomputed low words plus
      // compile-time offsets (one add per operand per MMA).
      const bool leader = elect_one();
      const uint32_t idesc_qk = idesc_f16(kBf16 ? 1u : 0u, 128, 128, 0, 0);
      const uint32_t idesc_pv = idesc_f16(kBf16 ? 1u : 0u, 128, D, 0, 1);
      const uint32_t q_lo0 = sdesc_lo_kmajor(smem_u32(sQ));
      const uint32_t k_lo0 = sdesc_lo_kmajor(smem_u32(sK));
      const uint32_t v_lo0 = sdesc_lo_mnmajor(smem_u32(sV), kTileRows);
      constexpr uint32_t kTileLo = C::kTileBytes >> 4;  // low-word step between tiles
      auto issue_s = [&](int x, int st) {
        const uint32_t q_lo = q_lo0 + x * kTileLo;
        const uint32_t k_lo = k_lo0 + st * kTileLo;
        const uint32_t d = tmem + C::kColS0 + 128u * x;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss_w(d, q_lo + kmajor_koff(kTileRows, kk * 16), k_lo + kmajor_koff(kTileRows, kk * 16), idesc_qk,
                      kk > 0 ? 1u : 0u);
          umma_commit(&s_full[x]);
        }
        __syncwarp();
      };
      auto issue_pv = [&](int x, int st, bool accumulate) {
        const uint32_t v_lo = v_lo0 + st * kTileLo;
        const uint32_t p_col = tmem + C::kColS0 + 128u * x;
        const uint32_t d = tmem + C::kColO0 + D * x;
        const uint32_t acc0 = accumulate ? 1u : 0u;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kTileRows / 16; ++kk)
            umma_ts_w(d, p_col + kk * 8, v_lo + mnmajor_koff(kk * 16), idesc_pv, kk > 0 ? 1u : acc0);
        }
        __syncwarp();
      };
      auto commit = [&](uint64_t* bar) {
        if (leader) umma_commit(bar);
        __syncwarp();
      };
      uint32_t g = 0;             // key tiles consumed so far
      uint32_t pa = 0, pb = 0;    // P tiles of A / B consumed so far
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
        const int n_sub = fwd_unit_items(u, n_ctiles, mode);
        for (int sub = 0; ok && sub < n_sub; ++sub, ++it) {
          // Key tiles are counted from the item's first one (f.j0).
          const FwdItem f = fwd_item<C::kT, kSplit>(u, sub, BH, n_ctiles, n_ntiles, causal, mode, split_l, split_item);
          const int n_kv_a = f.n_a;
          const int n_kv_b = f.n_b;
          // S_x(0) overwrites the previous item's P_x, whose P.V was issued
          // earlier on this thread: the tensor pipe keeps that order.
          if (!(ok = warp_wait(kRope ? &q_rot[0] : q_full, it & 1, ctl, timeout_ns, status, 3))) break;
          {
            const int st0 = g % C::kStages;
            if (!(ok = warp_wait(&k_full[st0], (g / C::kStages) & 1, ctl, timeout_ns, status, 4))) break;
            tc_fence_after();
            issue_s(0, st0);
            if constexpr (C::kT == 2) {
              if (kRope) {
                if (!(ok = warp_wait(&q_rot[1], it & 1, ctl, timeout_ns, status, 14))) break;
                tc_fence_after();
              }
              issue_s(1, st0);
            }
            commit(&k_empty[st0]);
            if (n_kv_b == 1) commit(q_empty);
          }
          for (int j = 0; ok && j < n_kv_b; ++j) {
            const uint32_t gj = g + j, gj1 = gj + 1;
            const int st = gj % C::kStages;
            const uint32_t ph = (gj / C::kStages) & 1;
            const int st1 = gj1 % C::kStages;
            const uint32_t ph1 = (gj1 / C::kStages) & 1;
            const int j1 = j + 1;
            bool v_ready = false, k_ready = false;
            if (j < n_kv_a) {
              // P_A(j) ready also means tile A's warps finished reading the
              // previous item's O_A (the epilogue precedes it).
              if (!(ok = warp_wait(&p_ready[0], pa & 1, ctl, timeout_ns, status, 5))) break;
              ++pa;
              if (!(ok = warp_wait(&v_full[st], ph, ctl, timeout_ns, status, 6))) break;
              v_ready = true;
              tc_fence_after();
              issue_pv(0, st, j > 0);
              if (j1 < n_kv_a) {
                if (!(ok = warp_wait(&k_full[st1], ph1, ctl, timeout_ns, status, 7))) break;
                k_ready = true;
                issue_s(0, st1);
              } else {
                commit(&o_final[0]);
              }
            }
            if constexpr (C::kT == 2) {
              if (!(ok = warp_wait(&p_ready[1], pb & 1, ctl, timeout_ns, status, 8))) break;
              ++pb;
              if (!v_ready && !(ok = warp_wait(&v_full[st], ph, ctl, timeout_ns, status, 9))) break;
              tc_fence_after();
              issue_pv(1, st, j > 0);
              commit(&v_empty[st]);
              if (j1 < n_kv_b) {
                if (!k_ready && !(ok = warp_wait(&k_full[st1], ph1, ctl, timeout_ns, status, 10))) break;
                issue_s(1, st1);
                commit(&k_empty[st1]);
                if (j1 == n_kv_b - 1) commit(q_empty);  // the item's last S product
              } else {
                commit(&o_final[1]);
              }
            } else {
              // One tile (n_kv_a == n_kv_b): P_A(j).V read V_j and S_A(j+1)
              // read K_{j+1}.
              commit(&v_empty[st]);
              if (j1 < n_kv_b) {
                commit(&k_empty[st1]);
                if (j1 == n_kv_b - 1) commit(q_empty);  // the item's last S product
              }
            }
          }
          g += n_kv_b;
        }
      }
    }
  } else {
    warpgroup_reg_inc<C::kRegsSoftmax>();
    // ---------------- softmax / correction / epilogue of tile x ----------------
    const int x = wg - 1;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t s_addr = t_lane + C::kColS0 + 128u * x;
    const uint32_t o_addr = t_lane + C::kColO0 + D * x;
    // 32-byte stores when every row starts on a 32-byte boundary.
    const bool wide_store = (d_real % 16) == 0 && (reinterpret_cast<uintptr_t>(out) & 31u) == 0;
    uint32_t cs = 0;  // S tiles of this query tile consumed so far
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
      const int n_sub = fwd_unit_items(u, n_ctiles, mode);
      for (int sub = 0; ok && sub < n_sub; ++sub, ++it) {
        int bh, m0, n_kv_x, n_first;
        {
          const FwdItem f = fwd_item<C::kT, kSplit>(u, sub, BH, n_ctiles, n_ntiles, causal, mode, split_l, split_item);
          bh = f.bh;
          m0 = f.ct * C::kT * kTileRows;
          n_kv_x = (x == 0) ? f.n_a : f.n_b;
          n_first = f.j0 * kTileRows;  // first key of the item
        }
        const int row_g = m0 + x * kTileRows + r;
        if constexpr (kRope) {
          // Rotate this thread's row of Q_x once the item's Q has landed.
          // (No early exit: after a failed wait the warps still reach the
          // epilogue's warpgroup barrier.)
          if (ok) ok = warp_wait(q_full, it & 1, ctl, timeout_ns, status, 15);
          if (ok) {
            rope_rotate_row<D, kBf16>(sQ + x * C::kTileBytes, r, row_g, S, rope_cos, rope_sin);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_rot[x]);
          }
        }
        float m_run = -INFINITY, l_run = 0.0f;
        for (int j = 0; ok && j < n_kv_x; ++j, ++cs) {
          if (!(ok = warp_wait(&s_full[x], cs & 1, ctl, timeout_ns, status, 11))) break;
          tc_fence_after();
          const int n0 = n_first + j * kTileRows;
          int lim = S - n0;
          if (causal) lim = min(lim, row_g - n0 + 1);
          float alpha;
          bool need;
          if (__any_sync(0xffffffffu, lim < kTileRows))
            softmax_tile<kBf16, true>(s_addr, lim, scale_log2, m_run, l_run, alpha, need);
          else
            softmax_tile<kBf16, false>(s_addr, lim, scale_log2, m_run, l_run, alpha, need);
          // S_x(j) completing implies P_x(j-1).V has completed, so O_x can be
          // rescaled here, before P_x(j) is released to the MMA warp.
          if (j >= 1 && __any_sync(0xffffffffu, need)) {
#pragma unroll
            for (int cb = 0; cb < D / 32; ++cb) {
              uint32_t o[32];
              tmem_ld32(o_addr + cb * 32, o);
              tmem_wait_ld();
              reg_fence(o);
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st32(o_addr + cb * 32, o);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_ready[x]);
        }
        // Epilogue.  The next item's P_x(0) is released only after the O_x
        // loads below, which keeps the MMA warp from overwriting O_x early.
        // ok is warp-uniform; after a failed wait the epilogue is skipped
        // but the warpgroup barrier below is still reached.
        if (ok) ok = warp_wait(&o_final[x], it & 1, ctl, timeout_ns, status, 12);
        if (ok) tc_fence_after();
        const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        const bool row_ok = row_g < S;
        // (Split state re-derived here rather than held through the key loop.)
        const int n_kv_item_a = causal ? min(m0 / kTileRows + 1, n_ntiles) : n_ntiles;
        const bool split_out = kSplit && n_kv_item_a > split_l;
        if (kSplit && split_out) {
          // One chunk of a split item: O_x / row_sum of this chunk in fp32
          // (all D columns; those past the true head_dim are zero) and its
          // base-2 log-sum-exp, for attn_fwd_combine_kernel.
          const size_t prow = (static_cast<size_t>(bh) * split_cmax + split_item[2]) * S + row_g;
          float* orow = o_part + prow * D;
#pragma unroll
          for (int cb = 0; ok && cb < D / 32; ++cb) {
            uint32_t o[32];
            tmem_ld32(o_addr + cb * 32, o);
            tmem_wait_ld();
            reg_fence(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * inv_l);
            if (row_ok) {
#pragma unroll
              for (int q = 0; q < 4; ++q) st_global_v8(orow + cb * 32 + q * 8, &o[q * 8]);
            }
          }
          if (ok && row_ok) lse_part[prow] = m_run + lg2(l_run);
        } else if (mode != kOrderPaired) {
          // One item per CTA: O_x / row_sum staged through Q_x (dead once O_x
          // is final) and written by one TMA store, which clips rows past S
          // and columns past the true head_dim.
          uint8_t* stage = sQ + x * C::kTileBytes;
#pragma unroll
          for (int cb = 0; ok && cb < D / 32; ++cb) {
            uint32_t o[32];
            tmem_ld32(o_addr + cb * 32, o);
            tmem_wait_ld();
            reg_fence(o);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
              uint4 w;
              w.x = pack2<kBf16>(__uint_as_float(o[ch * 8 + 0]) * inv_l, __uint_as_float(o[ch * 8 + 1]) * inv_l);
              w.y = pack2<kBf16>(__uint_as_float(o[ch * 8 + 2]) * inv_l, __uint_as_float(o[ch * 8 + 3]) * inv_l);
              w.z = pack2<kBf16>(__uint_as_float(o[ch * 8 + 4]) * inv_l, __uint_as_float(o[ch * 8 + 5]) * inv_l);
              w.w = pack2<kBf16>(__uint_as_float(o[ch * 8 + 6]) * inv_l, __uint_as_float(o[ch * 8 + 7]) * inv_l);
              *reinterpret_cast<uint4*>(stage + swz_offset(r, cb * 32 + ch * 8, kTileRows)) = w;
            }
          }
          fence_proxy_async_smem();
          // Every warp of the warpgroup reaches this barrier exactly once
          // (one item per CTA in this mode), on failure too.
          named_barrier_sync(1 + x, 128);
          // (Tile B of a short sequence may lie wholly past S: nothing to store.)
          if (ok && q4 == 0 && lane == 0 && !ctl->abort && m0 + x * kTileRows < S) {
#pragma unroll
            for (int b = 0; b < D / 64; ++b)
              tma_store_3d(&tm_o, stage + b * kBlockBytes, b * 64, m0 + x * kTileRows, bh);
            tma_store_commit();
            tma_store_wait_read_all();
          }
        } else {
          // Persistent CTAs: Q_x is already loading the next item, so O_x /
          // row_sum goes from registers straight to global memory, one row
          // per thread (rows past S, columns past the true head_dim skipped).
          uint16_t* orow = out + (static_cast<size_t>(bh) * S + row_g) * d_real;
#pragma unroll
          for (int cb = 0; ok && cb < D / 32; ++cb) {
            uint32_t o[32];
            tmem_ld32(o_addr + cb * 32, o);
            tmem_wait_ld();
            reg_fence(o);
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              w[e] = pack2<kBf16>(__uint_as_float(o[2 * e]) * inv_l, __uint_as_float(o[2 * e + 1]) * inv_l);
            if (row_ok) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int col = cb * 32 + hh * 16;
                if (wide_store && col < d_real) {
                  st_global_v8(orow + col, &w[hh * 8]);
                } else if (!wide_store) {
#pragma unroll
                  for (int q = 0; q < 2; ++q)
                    if (col + q * 8 < d_real)
                      *reinterpret_cast<uint4*>(orow + col + q * 8) = make_uint4(
                          w[hh * 8 + q * 4], w[hh * 8 + q * 4 + 1], w[hh * 8 + q * 4 + 2], w[hh * 8 + q * 4 + 3]);
                }
              }
            }
          }
        }
        if (ok && lse != nullptr && row_ok && !split_out) lse[static_cast<size_t>(bh) * S + row_g] = m_run + lg2(l_run);
      }
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

// Merges the chunks of split items: for a row whose item has nch > 1 chunks
// with outputs O_c (already divided by their own row sums) and base-2
// log-sum-exps L_c, M = max_c L_c, w_c = 2^(L_c - M),
// O = sum_c w_c O_c / sum_c w_c and LSE = M + log2(sum_c w_c).  One warp per
// row (lane c holds chunk c's L_c; nch <= 32); rows of single-chunk items
// were written by the forward itself.
template <int D, bool kBf16>
__global__ void __launch_bounds__(256)
    attn_fwd_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part,
                            uint16_t* __restrict__ out, float* __restrict__ lse, int S, int row0, long long n_rows,
                            int causal, int kT, int split_l, int split_cmax, int n_ntiles, int d_real) {
  const long long wrow = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wrow >= n_rows) return;
  const int rows_per = S - row0;
  const int bh = static_cast<int>(wrow / rows_per);
  const int m = row0 + static_cast<int>(wrow % rows_per);
  const int ct = m / (kT * kTileRows);
  const int na = causal ? min(kT * ct + 1, n_ntiles) : n_ntiles;
  const int nch = (na + split_l - 1) / split_l;
  if (nch <= 1) return;
  const size_t base = static_cast<size_t>(bh) * split_cmax * S + m;  // chunk c at base + c S
  constexpr int kPer = D / 32;  // columns per lane
  using Vec = typename std::conditional<kPer == 4, float4, float2>::type;
  // Every load of a group of 8 chunks (and the statistic) is issued before
  // any of them is used, so a warp waits for one memory latency per group
  // rather than one per chunk.
  constexpr int kGroup = 8;
  Vec v[kGroup];
  const float lc = (lane < nch) ? lse_part[base + static_cast<size_t>(lane) * S] : -INFINITY;
  auto load_group = [&](int c0) {
#pragma unroll
    for (int i = 0; i < kGroup; ++i)
      if (c0 + i < nch)
        v[i] = *reinterpret_cast<const Vec*>(o_part + (base + static_cast<size_t>(c0 + i) * S) * D + lane * kPer);
  };
  load_group(0);
  float mx = lc;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float w = (lane < nch) ? ex2(lc - mx) : 0.0f;
  float sum = w;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.0f;
  for (int c0 = 0; c0 < nch; c0 += kGroup) {
    if (c0 > 0) load_group(c0);
#pragma unroll
    for (int i = 0; i < kGroup; ++i) {
      const float wc = __shfl_sync(0xffffffffu, w, (c0 + i) & 31);
      if (c0 + i < nch) {
        acc[0] += wc * v[i].x;
        acc[1] += wc * v[i].y;
        if constexpr (kPer == 4) {
          acc[2] += wc * reinterpret_cast<const float4&>(v[i]).z;
          acc[3] += wc * reinterpret_cast<const float4&>(v[i]).w;
        }
      }
    }
  }
  const float inv = 1.0f / sum;
  // head_dim is a multiple of 8, so a lane's columns are all inside it or all
  // past it, and rows start on 16-byte boundaries.
  if (lane * kPer < d_real) {
    uint16_t* dst = out + (static_cast<size_t>(bh) * S + m) * d_real + lane * kPer;
    if constexpr (kPer == 4) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<kBf16>(acc[0] * inv, acc[1] * inv),
                                                  pack2<kBf16>(acc[2] * inv, acc[3] * inv));
    } else {
      *reinterpret_cast<uint32_t*>(dst) = pack2<kBf16>(acc[0] * inv, acc[1] * inv);
    }
  }
  if (lse != nullptr && lane == 0) lse[static_cast<size_t>(bh) * S + m] = mx + lg2(sum);
}

// The key-split schedule.  Used only when the regular one would not be
// persistent, its longest item has at least 48 key tiles and at least twice
// the average load of a resident CTA (the device is less than half busy on
// average while that item runs): chunks of split_l key tiles, the length
// chosen by simulating the schedule (split_makespan), at most 32 chunks per
// item.  Measured on one B200 with a fixed length (about two chunks' worth
// of tile-A key tiles per resident CTA, at least 16; split against unsplit,
// bf16, L2 flushed, interleaved): (B, H, S) = (1, 2, 8192) causal 1.94x,
// (1, 4, 8192) causal 1.17x, (1, 2, 16384) causal 1.41x (head_dim 128) and
// 1.34x (64), (1, 1, 16384) non-causal 1.53x, (1, 1, 32768) causal 1.65x
// (128) and 1.53x (64); 3 or 4 chunks' worth per CTA were equal or slower,
// and (1, 4, 8192)'s 320 chunks of 16 tiles took three full rounds of the
// 148 SMs, which the simulated choice avoids.  Problems only moderately underfilled (C4's 4
// heads per GPU, longest item 1.15x the average load; (1, 8, 4096) with 31
// key tiles) ran 6-18 % slower when split under a looser rule: the fp32
// partial outputs and the merge cost more than the balance gains.

static_assert(kSplitTileRows == kTileRows, "the split plan and the kernel use the same tile size");
static_assert(fwd_kernel_shape(64).kT == FwdCfg<64>::kT && fwd_kernel_shape(64).min_blocks == FwdCfg<64>::kMinBlocks &&
                  fwd_kernel_shape(128).kT == FwdCfg<128>::kT &&
                  fwd_kernel_shape(128).min_blocks == FwdCfg<128>::kMinBlocks,
              "the split plan's view of the kernels matches their configuration");

template <int D>
bool plan_fwd_split(int64_t S, int64_t BH, int causal, int sms, FwdSplitPlan& p) {
  using C = FwdCfg<D>;
  return plan_fwd_split_impl(C::kT, C::kMinBlocks, D, S, BH, causal, sms, p);
}

template <int D, bool kBf16, bool kRope>
int launch_fwd_t(const FwdArgs& a) {
  using C = FwdCfg<D>;
  static_assert(C::kSmemBytes <= 232448, "forward shared memory exceeds the sm_100 limit");
  auto kern_regular = attn_fwd_kernel<D, kBf16, kRope, false>;
  auto kern_split = attn_fwd_kernel<D, kBf16, false, true>;
  // The setmaxnreg split inside the kernel assumes exactly C::kLaunchRegs
  // registers per thread at launch; a build that differs is refused.
  int sms = 0;
  if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern_regular), C::kSmemBytes, C::kLaunchRegs, &sms))
    return rc;
  const int n_ctiles = static_cast<int>((a.S + C::kT * kTileRows - 1) / (C::kT * kTileRows));
  const long long n_items = static_cast<long long>(n_ctiles) * a.BH;
  const long long n_pair_units = static_cast<long long>((n_ctiles + 1) / 2) * a.BH;
  int mode;
  long long n_units, grid;
  // Persistent: the resident CTAs (one or two per SM) walk equal-cost paired
  // units, so the next item's Q load and first products overlap the current
  // epilogue; at least two units per resident CTA keep the last round's
  // imbalance small.  Measured (interleaved A/B, bit-identical O): non-causal
  // items only gain when they are short (at most four key tiles, where a
  // CTA's prologue and epilogue weigh most: 6-21 % at S = 384-512, 1-11 %
  // slower at S = 1024-8192, where the register-to-global epilogue costs
  // more than the overlap saves); causal items at head_dim 128 at every
  // length; causal single-tile items (head_dim 64) up to S = 2048 (7-19 %),
  // beyond which two hardware-scheduled CTAs per SM balance better (9 % at
  // S = 16384).
  const long long resident = static_cast<long long>(C::kMinBlocks) * sms;
  FwdSplitPlan plan;
  const bool split = !kRope && a.workspace != nullptr && a.workspace_bytes > 0 &&
                     plan_fwd_split<D>(a.S, a.BH, a.causal, sms, plan);
  if (split && a.workspace_bytes < plan.bytes) return kErrInvalidArgument;
  if (split) {
    if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern_split), C::kSmemBytes, C::kLaunchRegs, nullptr))
      return rc;
  }
  auto kern = split ? kern_split : kern_regular;
  const bool persist_shape =
      a.S <= 4 * kTileRows || (a.causal && (C::kT == 2 || a.S <= 16 * kTileRows));
  if (split) {
    mode = kOrderSplit;
    n_units = plan.units;
    grid = plan.units;
  } else if (n_ctiles > 1 && n_pair_units >= 2LL * resident && persist_shape) {
    mode = kOrderPaired;
    n_units = n_pair_units;
    grid = resident;
  } else {
    // One CTA per item, scheduled by the hardware.  Heaviest-first across
    // heads only pays when it cannot thrash L2: K and V of all heads
    // together must stay well inside the 126 MB L2.
    const double kv_bytes = 2.0 * static_cast<double>(a.BH) * static_cast<double>(a.S) * D * 2.0;
    mode = (a.causal && kv_bytes <= 80.0e6) ? kOrderLpt : kOrderHead;
    n_units = n_items;
    grid = n_items;
  }
  if (n_units > INT32_MAX || grid > INT32_MAX) return kErrTooLarge;
  kern<<<static_cast<unsigned>(grid), C::kThreads, C::kSmemBytes, a.stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_v, *a.tm_o, static_cast<uint16_t*>(a.o), a.lse, a.rope_cos, a.rope_sin,
      static_cast<int>(a.S),
      static_cast<int>(a.BH), n_ctiles, a.causal, mode, static_cast<int>(n_units), static_cast<int>(a.D),
      a.scale_log2, a.timeout_ns, a.status, split ? plan.split_l : 0, split ? plan.cmax : 0,
      split ? static_cast<float*>(a.workspace) : nullptr,
      split ? reinterpret_cast<float*>(static_cast<uint8_t*>(a.workspace) + plan.part_bytes) : nullptr);
  if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
  if (split) {
    const long long n_rows = a.BH * (a.S - plan.row0);
    const long long blocks = (n_rows * 32 + 255) / 256;
    if (n_rows > 0) {
      attn_fwd_combine_kernel<D, kBf16><<<static_cast<unsigned>(blocks), 256, 0, a.stream>>>(
          static_cast<const float*>(a.workspace),
          reinterpret_cast<const float*>(static_cast<const uint8_t*>(a.workspace) + plan.part_bytes),
          static_cast<uint16_t*>(a.o), a.lse, static_cast<int>(a.S), plan.row0, n_rows, a.causal, C::kT,
          plan.split_l, plan.cmax, static_cast<int>((a.S + kTileRows - 1) / kTileRows), static_cast<int>(a.D));
      if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
    }
  }
  return kOk;
}

}  // namespace

size_t attn_fwd_split_bytes(int64_t BH, int64_t S, int64_t D, int causal, int sms) {
  FwdSplitPlan p;
  if (D <= 0 || D > 128) return 0;
  const bool split = (D <= 64) ? plan_fwd_split<64>(S, BH, causal, sms, p) : plan_fwd_split<128>(S, BH, causal, sms, p);
  return split ? p.bytes : 0;
}

int launch_attn_fwd(const FwdArgs& a) {
  // head_dim <= 64 runs the 64-column kernel, 64 < head_dim <= 128 the
  // 128-column one; the tensor maps carry the true width.
  if (a.rope_cos != nullptr || a.rope_sin != nullptr) {
    // RoPE pairs column c with c + D/2 of full tiles: head_dim 64 or 128.
    if (a.rope_cos == nullptr || a.rope_sin == nullptr) return kErrInvalidArgument;
    if (a.D == 64) return a.bf16 ? launch_fwd_t<64, true, true>(a) : launch_fwd_t<64, false, true>(a);
    if (a.D == 128) return a.bf16 ? launch_fwd_t<128, true, true>(a) : launch_fwd_t<128, false, true>(a);
    return kErrUnsupported;
  }
  if (a.D <= 64) return a.bf16 ? launch_fwd_t<64, true, false>(a) : launch_fwd_t<64, false, false>(a);
  if (a.D <= 128) return a.bf16 ? launch_fwd_t<128, true, false>(a) : launch_fwd_t<128, false, false>(a);
  return kErrUnsupported;
}

}  // namespace tk
