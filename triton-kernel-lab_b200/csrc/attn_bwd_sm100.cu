// Flash-attention backward for sm_100a (B200): one fused recompute kernel that
// produces dK and dV for a 128-key tile and reduces its dQ contributions into
// an fp32 accumulator, all five contractions on tcgen05 with TMEM
// accumulators.
//
// Semantics follow the reference kernels `_attn_bwd_dkdv_kernel` and
// `_attn_bwd_dq_kernel` (src/tklab/kernels/flash_attention.py:398-533):
//   P  = exp2(scale*log2(e) * Q.K^T - LSE2)     (LSE2 = base-2 log-sum-exp)
//   dV += P^T dO            dP = dO V^T        dS = P * (dP - delta)
//   dK += dS^T Q (times scale)                 dQ += dS K (times scale)
// with P and dS rounded to the input dtype for their products (:459-462,530),
// causal blocks below the diagonal skipped (:438, :513) and the diagonal and
// ragged tails masked (:454-457, :523-526).  The reference runs dK/dV and dQ
// as two kernels that both recompute P (14 N^2 d MMA flops); here dQ is
// produced by the same CTA (10 N^2 d) and reduced across key tiles by the
// TMA unit (bulk tensor reduce-add from shared memory).
//
// One CTA owns a 128-key tile (K, V resident in smem) of one (batch, head)
// and walks 128-query steps.  The transposed products are computed directly
// (S^T = K Q^T, dP^T = V dO^T) so TMEM lane n holds key n.  16 warps in four
// warpgroups, registers rebalanced with setmaxnreg:
//   WG0  warp 0   producer: TMA for K, V, dO_i (1 stage); plain loads of
//                 LSE/delta
//        warp 1   TMEM allocator and tcgen05.mma issuer (the warp runs the
//                 loop converged, one elected lane issues)
//        warp 2   issues the TMA reduce-add of each staged dQ tile
//        warp 3   producer of the Q tiles
//   WG1  warps 4..7   "dQ warps": thread m owns query m of the step; copy dQ
//                     from TMEM into an fp32 staging tile (128-byte swizzle)
//   WG2, WG3  warps 8..15  "dS warps": WG2 owns queries 0..63 of a step,
//                     WG3 queries 64..127; thread t owns key t.  Phase 1:
//                     P^T, packed to 16 bits over the first half of the
//                     warpgroup's own S^T columns for the dV MMA.  Phase 2:
//                     dS^T = P^T (dP^T - delta) to smem for the dK and dQ
//                     MMAs.  Epilogue: WG2 stores dV, WG3 stores dK.
// MMA issue order per step i: dV_i, S_{i+1}, dQ_i, dK_i, dP_{i+1}, so the dS
// warps compute P_{i+1} (the exp2-heavy phase) while dQ_i and dK_i run, and
// the dQ warps drain dQ_i from TMEM while dK_i runs.
// TMEM columns: dV [0,D) dK [D,2D) S^T/P^T [2D,2D+128) dP^T [2D+128,2D+256);
// dQ follows dP^T when it fits (D=64) and otherwise (D=128) reuses the dP^T
// columns, reclaimed by dP_{i+1} only after the dQ warps have read dQ_i.
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

template <int D>
struct BwdCfg {
  static constexpr int kTileBytes = kTileRows * D * 2;
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kTileBytes;
  static constexpr int kQOff = kVOff + kTileBytes;  // 2 stages
  static constexpr int kDOOff = kQOff + 2 * kTileBytes;
  static constexpr int kDSOff = kDOOff + kTileBytes;
  static constexpr int kDSBytes = kTileRows * kTileRows * 2;
  static constexpr int kDQOff = kDSOff + kDSBytes;  // fp32 staging: 2 boxes of 128 x 32
  static constexpr int kDQBytes = 2 * kTileRows * kSwizzleBytes;
  static constexpr int kLseOff = kDQOff + kDQBytes;        // float[2][128]
  static constexpr int kDeltaOff = kLseOff + 2 * 128 * 4;  // float[2][128]
  static constexpr int kBarOff = kDeltaOff + 2 * 128 * 4;
  // kv_full, q_full[2], q_empty[2], do_full, do_empty, ld_full[2], ld_empty[2],
  // s_full, dp_full, p_ready, ds_ready, ds_empty, dq_full, dq_empty,
  // stage_full[2], stage_free[2] (one per staging box), dkdv_done
  static constexpr int kNumBars = 1 + 4 + 2 + 4 + 12;
  static constexpr int kCtlOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kCtlOff + 64;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColDV = 0;
  static constexpr uint32_t kColDK = D;
  static constexpr uint32_t kColS = 2 * D;
  static constexpr uint32_t kColDP = 2 * D + 128;
  static constexpr bool kDqAliased = (2 * D + 256 + D) > 512;
  static constexpr uint32_t kColDQ = kDqAliased ? kColDP : 2 * D + 256;
  // dQ is reduced in passes of 64 head-dim columns (two 32-float boxes).
  static constexpr int kDqPasses = D / 64;
};

constexpr int kBwdThreads = 512;
// Launch allocation 128 registers x 512 threads = 65536; per warpgroup after
// setmaxnreg: WG0 56 + WG1 152 + WG2 152 + WG3 152 = 512 x 128 threads, which
// never exceeds the launch allocation (an inc beyond it would never return).
constexpr int kBwdLaunchRegs = 128;
constexpr int kRegsCtrl = 56;
constexpr int kRegsDq = 152;
constexpr int kRegsDs = 152;
static_assert(kRegsCtrl + kRegsDq + 2 * kRegsDs <= 4 * kBwdLaunchRegs, "register split exceeds the launch");

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, CtaControl* ctl,
                                          uint64_t timeout_ns, int* status, int site) {
  const bool ok = mbar_wait(bar, parity, ctl, timeout_ns, status, site);
  return __all_sync(0xffffffffu, ok);
}

// Stage one TMEM row (D fp32 values, times `mul`) as dtype into a swizzled
// 128-row tile in smem, row `r`.
template <int D, bool kBf16>
__device__ __forceinline__ void stage_row(uint32_t t_row, uint8_t* tile, int r, float mul) {
#pragma unroll
  for (int cb = 0; cb < D / 32; ++cb) {
    uint32_t v[32];
    tmem_ld32(t_row + cb * 32, v);
    tmem_wait_ld();
    reg_fence(v);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      uint4 w;
      w.x = pack2<kBf16>(__uint_as_float(v[ch * 8 + 0]) * mul, __uint_as_float(v[ch * 8 + 1]) * mul);
      w.y = pack2<kBf16>(__uint_as_float(v[ch * 8 + 2]) * mul, __uint_as_float(v[ch * 8 + 3]) * mul);
      w.z = pack2<kBf16>(__uint_as_float(v[ch * 8 + 4]) * mul, __uint_as_float(v[ch * 8 + 5]) * mul);
      w.w = pack2<kBf16>(__uint_as_float(v[ch * 8 + 6]) * mul, __uint_as_float(v[ch * 8 + 7]) * mul);
      *reinterpret_cast<uint4*>(tile + swz_offset(r, cb * 32 + ch * 8, kTileRows)) = w;
    }
  }
}

// P^T for 32 queries of one key row: p = exp2(s * scale*log2(e) - LSE2[q]).
// nlse_s holds the negated LSE values, read with 128-bit broadcast loads
// (every lane of the warp reads the same address), so each pair's argument
// is one packed fma.  kMasked adds the causal diagonal (query q0+e is dropped
// when it precedes this thread's key, diag_key) and the ragged key tail
// (key_ok false: the whole row is zero).
// Of the 16 exponential pairs of an unmasked 32-query chunk, the pairs of
// this many 4-query groups (two pairs each) run on the FMA pipe
// (exp2_fma_pair): with both dS warpgroups in their P phase the MUFU
// (16 exp2/clk/SM) would otherwise bound it.  2 of 8 measured best with the
// box-by-box dQ staging (1 and 3 were 1-2 % and 3-4 % slower end to end).
#ifndef TK_BWD_EMU_GROUPS_PER8
#define TK_BWD_EMU_GROUPS_PER8 2
#endif
constexpr int kBwdEmuGroupsPer8 = TK_BWD_EMU_GROUPS_PER8;

template <bool kMasked>
__device__ __forceinline__ void probs_chunk(const uint32_t (&sv)[32], const float* nlse_s, float scale_log2,
                                            int q0, int diag_key, bool key_ok, float (&p)[32]) {
  const float4* nlse4 = reinterpret_cast<const float4*>(nlse_s);
  const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    const float4 l = nlse4[e4];
    float x[4];
    const int e0 = e4 * 4;
    f2_unpack(ffma2(f2_pack(__uint_as_float(sv[e0]), __uint_as_float(sv[e0 + 1])), scale2, f2_pack(l.x, l.y)), x[0],
              x[1]);
    f2_unpack(ffma2(f2_pack(__uint_as_float(sv[e0 + 2]), __uint_as_float(sv[e0 + 3])), scale2, f2_pack(l.z, l.w)),
              x[2], x[3]);
    if (!kMasked && e4 >= 8 - kBwdEmuGroupsPer8) {
      // Unmasked: every argument is finite (LSE of a real row bounds it).
      exp2_fma_pair(x[0], x[1], p[e0], p[e0 + 1]);
      exp2_fma_pair(x[2], x[3], p[e0 + 2], p[e0 + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = e0 + j;
        float pv = ex2(x[j]);
        if constexpr (kMasked) {
          if (q0 + e < diag_key || !key_ok) pv = 0.0f;
        }
        p[e] = pv;
      }
    }
  }
}

// kWithDq false compiles the dQ path out (no dQ product, drain or
// reduction; tm_dq unused): the dK/dV half of the deterministic backward,
// whose dQ comes from attn_bwd_dq_kernel.
template <int D, bool kBf16, bool kWithDq>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                    const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse,
                    const float* __restrict__ delta, int S, int BH, int n_tiles, int causal, float scale,
                    float scale_log2, int d_real, unsigned long long timeout_ns, int* status) {
  using C = BwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  // Head-major order: the key tiles of one (batch, head) are adjacent in the
  // grid, so resident CTAs share a few heads' Q, dO and dQ-accumulator lines
  // in L2.  Within a head the key tiles with the most query steps (smallest
  // index under a causal mask) launch first.
  const int bh = static_cast<int>(blockIdx.x) / n_tiles;
  const int jn = static_cast<int>(blockIdx.x) % n_tiles;
  const int n0 = jn * kTileRows;
  const int i_start = causal ? jn : 0;
  const int n_steps = n_tiles - i_start;

  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sDO = smem + C::kDOOff;
  uint8_t* sDS = smem + C::kDSOff;
  uint8_t* sDQ = smem + C::kDQOff;
  float* sLse = reinterpret_cast<float*>(smem + C::kLseOff);
  float* sDelta = reinterpret_cast<float*>(smem + C::kDeltaOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + 2;
  uint64_t* do_full = q_empty + 2;
  uint64_t* do_empty = do_full + 1;
  uint64_t* ld_full = do_empty + 1;
  uint64_t* ld_empty = ld_full + 2;
  uint64_t* s_full = ld_empty + 2;
  uint64_t* dp_full = s_full + 1;
  uint64_t* p_ready = dp_full + 1;
  uint64_t* ds_ready = p_ready + 1;
  uint64_t* ds_empty = ds_ready + 1;
  uint64_t* dq_full = ds_empty + 1;
  uint64_t* dq_empty = dq_full + 1;
  uint64_t* stage_full = dq_empty + 1;  // [2]
  uint64_t* stage_free = stage_full + 2;  // [2]
  uint64_t* dkdv_done = stage_free + 2;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kCtlOff);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&ld_full[i], 32);
      mbar_init(&ld_empty[i], 8);
    }
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(ds_ready, 8);
    mbar_init(ds_empty, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&stage_full[i], 4);
      mbar_init(&stage_free[i], 1);
    }
    mbar_init(dkdv_done, 1);
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
    tma_prefetch_map(&tm_do);
    tma_prefetch_map(&tm_dk);
    tma_prefetch_map(&tm_dv);
    tma_prefetch_map(&tm_dq);
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const size_t row_base = static_cast<size_t>(bh) * S;

  if (wg == 0) {
    warpgroup_reg_dec<kRegsCtrl>();
    if (warp == 3) {
      // ---------------- Q producer (its own warp so a Q load never waits
      // behind the dO or LSE waits) ----------------
      for (int it = 0; it < n_steps; ++it) {
        const int m0 = (i_start + it) * kTileRows;
        const int st = it & 1;
        if (!warp_wait(&q_empty[st], ((it >> 1) & 1) ^ 1, ctl, timeout_ns, status, 1)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[st], C::kTileBytes);
#pragma unroll
          for (int b = 0; b < D / 64; ++b)
            tma_load_3d(sQ + st * C::kTileBytes + b * kBlockBytes, &tm_q, &q_full[st], b * 64, m0, bh);
        }
      }
    } else if (warp == 0) {
      // ---------------- K/V, dO and LSE/delta producer ----------------
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, 2 * C::kTileBytes);
#pragma unroll
        for (int b = 0; b < D / 64; ++b) {
          tma_load_3d(sK + b * kBlockBytes, &tm_k, kv_full, b * 64, n0, bh);
          tma_load_3d(sV + b * kBlockBytes, &tm_v, kv_full, b * 64, n0, bh);
        }
      }
      for (int it = 0; it < n_steps; ++it) {
        const int m0 = (i_start + it) * kTileRows;
        if (!warp_wait(do_empty, (it & 1) ^ 1, ctl, timeout_ns, status, 2)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(do_full, C::kTileBytes);
#pragma unroll
          for (int b = 0; b < D / 64; ++b) tma_load_3d(sDO + b * kBlockBytes, &tm_do, do_full, b * 64, m0, bh);
        }
        // -LSE / delta for this query step (LSE stored negated for the
        // packed P argument).  Padded queries get -LSE = -inf so their
        // probabilities are exactly zero.
        const int lb = it & 1;
        if (!warp_wait(&ld_empty[lb], ((it >> 1) & 1) ^ 1, ctl, timeout_ns, status, 3)) break;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int q = e * 32 + lane;
          const int mg = m0 + q;
          const bool valid = mg < S;
          sLse[lb * 128 + q] = valid ? -lse[row_base + mg] : -INFINITY;
          sDelta[lb * 128 + q] = valid ? delta[row_base + mg] : 0.0f;
        }
        mbar_arrive(&ld_full[lb]);
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      // The whole warp runs the loop (waits included) so that addresses and
      // descriptors stay warp-uniform; one elected lane issues each
      // tcgen05.mma / commit.  Descriptors are precomputed low words plus
      // compile-time offsets (one add per operand per MMA).
      const bool leader = elect_one();
      const uint32_t fmt = kBf16 ? 1u : 0u;
      const uint32_t idesc_s = idesc_f16(fmt, 128, 128, 0, 0);
      const uint32_t idesc_kv = idesc_f16(fmt, 128, D, 0, 1);
      const uint32_t idesc_dq = idesc_f16(fmt, 128, D, 1, 1);
      const uint32_t k_lo = sdesc_lo_kmajor(smem_u32(sK));
      const uint32_t k_mn_lo = sdesc_lo_mnmajor(smem_u32(sK), kTileRows);
      const uint32_t v_lo = sdesc_lo_kmajor(smem_u32(sV));
      const uint32_t ds_lo = sdesc_lo_kmajor(smem_u32(sDS));
      const uint32_t ds_mn_lo = sdesc_lo_mnmajor(smem_u32(sDS), kTileRows);
      const uint32_t do_lo = sdesc_lo_kmajor(smem_u32(sDO));
      const uint32_t do_mn_lo = sdesc_lo_mnmajor(smem_u32(sDO), kTileRows);
      const uint32_t q_lo0 = sdesc_lo_kmajor(smem_u32(sQ));
      const uint32_t q_mn_lo0 = sdesc_lo_mnmajor(smem_u32(sQ), kTileRows);
      constexpr uint32_t kTileLo = C::kTileBytes >> 4;  // low-word step between Q stages
      auto commit = [&](uint64_t* bar) {
        if (leader) umma_commit(bar);
        __syncwarp();
      };
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        if (!warp_wait(&q_full[st], (it >> 1) & 1, ctl, timeout_ns, status, 4)) return false;
        tc_fence_after();
        const uint32_t q_lo = q_lo0 + st * kTileLo;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss_w(tmem + C::kColS, k_lo + kmajor_koff(kTileRows, kk * 16), q_lo + kmajor_koff(kTileRows, kk * 16),
                      idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(s_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_dp = [&](int it) -> bool {
        if (!warp_wait(do_full, it & 1, ctl, timeout_ns, status, 5)) return false;
        if (kWithDq && C::kDqAliased && it > 0) {
          if (!warp_wait(dq_empty, (it - 1) & 1, ctl, timeout_ns, status, 6)) return false;
        }
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss_w(tmem + C::kColDP, v_lo + kmajor_koff(kTileRows, kk * 16), do_lo + kmajor_koff(kTileRows, kk * 16),
                      idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(dp_full);
        }
        __syncwarp();
        return true;
      };
      bool ok = warp_wait(kv_full, 0, ctl, timeout_ns, status, 7);
      if (ok && n_steps > 0) ok = issue_s(0) && issue_dp(0);
      for (int it = 0; ok && it < n_steps; ++it) {
        const int st = it & 1;
        const uint32_t q_mn_lo = q_mn_lo0 + st * kTileLo;
        // dV += P^T dO.  P^T of queries 64h..64h+63 sits packed in the
        // first 32 columns of warpgroup h's 64 S columns.
        if (!(ok = warp_wait(p_ready, it & 1, ctl, timeout_ns, status, 8))) break;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kTileRows / 16; ++kk)
            umma_ts_w(tmem + C::kColDV, tmem + C::kColS + (kk >> 2) * 64 + (kk & 3) * 8,
                      do_mn_lo + mnmajor_koff(kk * 16), idesc_kv, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit(do_empty);
        }
        __syncwarp();
        if (it + 1 < n_steps && !(ok = issue_s(it + 1))) break;
        // dQ = dS K  (dS in smem from the dS warps)
        if (!(ok = warp_wait(ds_ready, it & 1, ctl, timeout_ns, status, 9))) break;
        tc_fence_after();
        if constexpr (kWithDq) {
          if (!C::kDqAliased && it > 0) {
            if (!(ok = warp_wait(dq_empty, (it - 1) & 1, ctl, timeout_ns, status, 10))) break;
          }
          if (leader) {
#pragma unroll
            for (int kk = 0; kk < kTileRows / 16; ++kk)
              umma_ss_w(tmem + C::kColDQ, ds_mn_lo + mnmajor_koff(kk * 16), k_mn_lo + mnmajor_koff(kk * 16), idesc_dq,
                        kk > 0 ? 1u : 0u);
            umma_commit(dq_full);
          }
          __syncwarp();
        }
        // dK += dS^T Q; the smem dS tile is free after this one.
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kTileRows / 16; ++kk)
            umma_ss_w(tmem + C::kColDK, ds_lo + kmajor_koff(kTileRows, kk * 16), q_mn_lo + mnmajor_koff(kk * 16),
                      idesc_kv, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&q_empty[st]);
          umma_commit(ds_empty);
        }
        __syncwarp();
        if (it + 1 < n_steps && !(ok = issue_dp(it + 1))) break;
      }
      if (ok) commit(dkdv_done);
    } else if (warp == 2 && kWithDq) {
      // ---------------- dQ reduce issuer ----------------
      // Box by box: each 32-column box is reduced as soon as it is staged,
      // and released once the TMA has read it (checked one reduction later,
      // so that a box is being read while the other is being filled).
      bool ok = true;
      int prev = -1;
      for (int it = 0; ok && it < n_steps; ++it) {
        const int m0 = (i_start + it) * kTileRows;
#pragma unroll
        for (int pass = 0; pass < C::kDqPasses; ++pass) {
          const uint32_t cnt = static_cast<uint32_t>(it * C::kDqPasses + pass);
#pragma unroll
          for (int bx = 0; bx < 2; ++bx) {
            if (!(ok = warp_wait(&stage_full[bx], cnt & 1, ctl, timeout_ns, status, 18))) break;
            if (lane == 0) {
              // A head_dim below the kernel's width leaves whole boxes past
              // the tensor's last column: nothing to add there (the group
              // stays, empty, so that the count of groups in flight holds).
              if (pass * 64 + bx * 32 < d_real)
                tma_reduce_add_3d(&tm_dq, sDQ + bx * kTileRows * kSwizzleBytes, pass * 64 + bx * 32, m0, bh);
              tma_store_commit();
              tma_store_wait_read_le1();
              if (prev >= 0) mbar_arrive(&stage_free[prev]);
            }
            prev = bx;
            __syncwarp();
          }
          if (!ok) break;
        }
      }
      if (lane == 0) {
        tma_store_wait_read_all();
        if (ok && prev >= 0) mbar_arrive(&stage_free[prev]);
        tma_store_wait_all();
      }
    }
  } else if (wg == 1) {
    warpgroup_reg_inc<kRegsDq>();
    // ---------------- dQ warps: thread r owns query m0 + r ----------------
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    bool ok = true;
    for (int it = 0; kWithDq && ok && it < n_steps; ++it) {
      if (!(ok = warp_wait(dq_full, it & 1, ctl, timeout_ns, status, 16))) break;
      tc_fence_after();
      uint32_t v[D / 32][32];
#pragma unroll
      for (int cb = 0; cb < D / 32; ++cb) tmem_ld32(t_lane + C::kColDQ + cb * 32, v[cb]);
      tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < D / 32; ++cb) reg_fence(v[cb]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
#pragma unroll
      for (int pass = 0; pass < C::kDqPasses; ++pass) {
        const uint32_t cnt = static_cast<uint32_t>(it * C::kDqPasses + pass);
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          if (!(ok = warp_wait(&stage_free[bx], (cnt & 1) ^ 1, ctl, timeout_ns, status, 17))) break;
          uint8_t* box = sDQ + bx * kTileRows * kSwizzleBytes;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const float4 w = make_float4(__uint_as_float(v[pass * 2 + bx][ch * 4 + 0]) * scale,
                                         __uint_as_float(v[pass * 2 + bx][ch * 4 + 1]) * scale,
                                         __uint_as_float(v[pass * 2 + bx][ch * 4 + 2]) * scale,
                                         __uint_as_float(v[pass * 2 + bx][ch * 4 + 3]) * scale);
            *reinterpret_cast<float4*>(box + swz_offset_f32(r, ch * 4)) = w;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&stage_full[bx]);
        }
        if (!ok) break;
      }
    }
  } else {
    warpgroup_reg_inc<kRegsDs>();
    // ---------------- dS warps: thread t owns key n0 + t ----------------
    const int h = wg - 2;  // query half of the step owned by this warpgroup
    const int q4 = warp & 3;
    const int t = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t s_cols = t_lane + C::kColS + h * 64;
    const uint32_t dp_cols = t_lane + C::kColDP + h * 64;
    const bool key_ok = (n0 + t) < S;
    bool ok = true;
    for (int it = 0; it < n_steps; ++it) {
      const int i = i_start + it;
      const int lb = it & 1;
      if (!(ok = warp_wait(&ld_full[lb], (it >> 1) & 1, ctl, timeout_ns, status, 11))) break;
      if (!(ok = warp_wait(s_full, it & 1, ctl, timeout_ns, status, 12))) break;
      tc_fence_after();
      const bool diag = causal && (i == jn);
      const float* nlse_s = sLse + lb * 128 + h * 64;
      const float* del_s = sDelta + lb * 128 + h * 64;
      // Phase 1: P^T for this warpgroup's 64 queries -> registers and,
      // packed to 16 bits, back over the first 32 of its S columns (both
      // 32-column chunks are read before any packed half is written).
      float p[2][32];
      const bool masked = __any_sync(0xffffffffu, diag || !key_ok);
      {
        // Both 32-column loads are in flight together.
        uint32_t sv[2][32];
        tmem_ld32(s_cols, sv[0]);
        tmem_ld32(s_cols + 32, sv[1]);
        tmem_wait_ld();
        reg_fence(sv[0]);
        reg_fence(sv[1]);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (masked)
            probs_chunk<true>(sv[c], nlse_s + c * 32, scale_log2, h * 64 + c * 32, diag ? t : 0, key_ok, p[c]);
          else
            probs_chunk<false>(sv[c], nlse_s + c * 32, scale_log2, 0, 0, true, p[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pp[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pp[e] = pack2<kBf16>(p[c][2 * e], p[c][2 * e + 1]);
        tmem_st16(s_cols + c * 16, pp);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      // Phase 2: dS^T = P^T (dP^T - delta) -> smem for the dK and dQ MMAs.
      if (!(ok = warp_wait(dp_full, it & 1, ctl, timeout_ns, status, 13))) break;
      if (it > 0) {
        if (!(ok = warp_wait(ds_empty, (it - 1) & 1, ctl, timeout_ns, status, 14))) break;
      }
      tc_fence_after();
      uint32_t dpv2[2][32];
      tmem_ld32(dp_cols, dpv2[0]);
      tmem_ld32(dp_cols + 32, dpv2[1]);
      tmem_wait_ld();
      reg_fence(dpv2[0]);
      reg_fence(dpv2[1]);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t (&dpv)[32] = dpv2[c];
        uint32_t dd[16];
        const float4* del4 = reinterpret_cast<const float4*>(del_s + c * 32);
        const uint64_t neg1 = f2_pack(-1.0f, -1.0f);
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) {
          const float4 dl = del4[e4];  // one broadcast 128-bit load for 4 queries
          const int e = e4 * 4;
          // dS = P (dP - delta), two queries per packed instruction.
          float d0, d1, d2, d3;
          f2_unpack(fmul2(f2_pack(p[c][e], p[c][e + 1]),
                          ffma2(f2_pack(dl.x, dl.y), neg1,
                                f2_pack(__uint_as_float(dpv[e]), __uint_as_float(dpv[e + 1])))),
                    d0, d1);
          f2_unpack(fmul2(f2_pack(p[c][e + 2], p[c][e + 3]),
                          ffma2(f2_pack(dl.z, dl.w), neg1,
                                f2_pack(__uint_as_float(dpv[e + 2]), __uint_as_float(dpv[e + 3])))),
                    d2, d3);
          dd[e4 * 2] = pack2<kBf16>(d0, d1);
          dd[e4 * 2 + 1] = pack2<kBf16>(d2, d3);
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          uint4 v = make_uint4(dd[w * 4 + 0], dd[w * 4 + 1], dd[w * 4 + 2], dd[w * 4 + 3]);
          *reinterpret_cast<uint4*>(sDS + swz_offset(t, h * 64 + c * 32 + w * 8, kTileRows)) = v;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ld_empty[lb]);
        mbar_arrive(ds_ready);
      }
    }
    // Epilogue: WG2 stores dV (staged through Q stage 0), WG3 stores dK
    // (scaled, staged through the dO buffer).  Rows >= S are clipped by the
    // tensor map bounds.
    uint8_t* stage = (h == 0) ? sQ : sDO;
    if (ok) ok = warp_wait(dkdv_done, 0, ctl, timeout_ns, status, 15);
    if (ok) {
      tc_fence_after();
      if (h == 0)
        stage_row<D, kBf16>(t_lane + C::kColDV, stage, t, 1.0f);
      else
        stage_row<D, kBf16>(t_lane + C::kColDK, stage, t, scale);
      fence_proxy_async_smem();
    }
    named_barrier_sync(1 + h, 128);
    if ((warp & 3) == 0 && lane == 0 && !ctl->abort) {
      const CUtensorMap* map = (h == 0) ? &tm_dv : &tm_dk;
#pragma unroll
      for (int b = 0; b < D / 64; ++b) tma_store_3d(map, stage + b * kBlockBytes, b * 64, n0, bh);
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

template <int D, bool kBf16, bool kWithDq>
int launch_bwd_t(const BwdArgs& a) {
  using C = BwdCfg<D>;
  static_assert(C::kSmemBytes <= 232448, "backward shared memory exceeds the sm_100 limit");
  auto kern = attn_bwd_kernel<D, kBf16, kWithDq>;
  // The setmaxnreg split inside the kernel assumes exactly kBwdLaunchRegs
  // registers per thread at launch; a build that differs is refused.
  if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern), C::kSmemBytes, kBwdLaunchRegs, nullptr))
    return rc;
  const int n_tiles = static_cast<int>((a.S + kTileRows - 1) / kTileRows);
  const long long grid = static_cast<long long>(n_tiles) * a.BH;
  kern<<<static_cast<unsigned>(grid), kBwdThreads, C::kSmemBytes, a.stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_v, *a.tm_do, *a.tm_dk, *a.tm_dv, kWithDq ? *a.tm_dq : *a.tm_dk, a.lse, a.delta,
      static_cast<int>(a.S), static_cast<int>(a.BH), n_tiles, a.causal, a.scale, a.scale_log2,
      static_cast<int>(a.D), a.timeout_ns, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_attn_bwd(const BwdArgs& a) {
  // head_dim <= 64 runs the 64-column kernel, 64 < head_dim <= 128 the
  // 128-column one; the tensor maps carry the true width.
  if (a.D <= 64) return a.bf16 ? launch_bwd_t<64, true, true>(a) : launch_bwd_t<64, false, true>(a);
  if (a.D <= 128) return a.bf16 ? launch_bwd_t<128, true, true>(a) : launch_bwd_t<128, false, true>(a);
  return kErrUnsupported;
}

int launch_attn_bwd_dkdv(const BwdArgs& a) {
  if (a.D <= 64) return a.bf16 ? launch_bwd_t<64, true, false>(a) : launch_bwd_t<64, false, false>(a);
  if (a.D <= 128) return a.bf16 ? launch_bwd_t<128, true, false>(a) : launch_bwd_t<128, false, false>(a);
  return kErrUnsupported;
}

}  // namespace tk
