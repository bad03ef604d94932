// Flash-attention backward for head_dim 136..256 on sm_100a (B200): the
// fused recompute kernel of attn_bwd_sm100.cu re-shaped for wide heads.
//
// Semantics are those of the reference kernels `_attn_bwd_dkdv_kernel` and
// `_attn_bwd_dq_kernel` (src/tklab/kernels/flash_attention.py:398-533):
//   P  = exp2(scale*log2(e) * Q.K^T - LSE2)    dP = dO V^T
//   dV += P^T dO     dS = P (dP - delta)     dK += dS^T Q     dQ += dS K
// (dK and dQ scaled by the softmax scale), P and dS rounded to the input
// dtype for their products, causal blocks skipped and the diagonal / ragged
// tails masked.
//
// Why this shape.  Tensor memory holds 512 fp32 columns per SM.  A 128-key
// tile's dK and dV at head_dim 256 alone would fill it, so the head
// dimension of the three outputs is split between two CTAs: CTA `half` owns
// dK[:, 128*half .. +128), dV[...] and dQ[...] of one 128-key tile, while
// both recompute the full-width S^T = K Q^T and dP^T = V dO^T (contraction
// over all 256 columns).  Shared memory is the other limit: K (64 KB) stays
// resident for S^T and dQ, and V lives in tensor memory instead (packed
// 16-bit, the A operand of dP^T), which frees the room for two-stage rings
// of 64-query Q and dO tiles (4 x 32 KB).
//
// One CTA: 128 keys of one (batch, head), one head-dim half, walking 64-query
// steps (causal: from the first step that reaches the tile's first key).
// 16 warps:
//   WG0  warp 0   producer: K once, dO_i (2 stages), LSE/delta
//        warp 1   TMEM allocator and tcgen05.mma issuer (converged warp,
//                 one elected lane issues)
//        warp 2   issues the TMA reduce-add of each staged dQ box
//        warp 3   producer of the Q tiles (2 stages)
//   WG1  warps 4..7   dQ warps: thread r owns head-dim column 128*half + r;
//                     copy dQ^T from TMEM into fp32 staging boxes
//   WG2, WG3  warps 8..15  dS warps: thread t owns key n0 + t; WG2 queries
//                     0..31 of a step, WG3 32..63.  WG2 also loads V into
//                     TMEM before the first step.  Epilogue: WG2 stores dV,
//                     WG3 dK.
// TMEM columns: V packed [0,128), dV [128,256), dK [256,384), S^T/P^T
// [384,448), dP^T [448,512) shared with dQ^T (lane = head-dim column), which
// the dQ warps drain before the next dP^T is issued.
// MMA order per step i: dV_i, S_{i+1}, dQ_i, dK_i, dP_{i+1}.
#include "attn_launch.h"
#include "sm100_primitives.cuh"

namespace tk {
namespace {

struct WideBwdCfg {
  static constexpr int kW = 256;       // kernel width (head_dim padded with zero columns)
  static constexpr int kKeys = 128;    // keys per CTA (TMEM lanes)
  static constexpr int kQRows = 64;    // queries per step
  static constexpr int kHalf = 128;    // head-dim columns of the outputs per CTA
  static constexpr int kKBytes = kKeys * kW * 2;     // 64 KB, 4 column blocks of 128 rows
  static constexpr int kQBytes = kQRows * kW * 2;    // 32 KB, 4 column blocks of 64 rows
  static constexpr int kQBlock = kQRows * kSwizzleBytes;  // 8 KB
  static constexpr int kKOff = 0;
  static constexpr int kQOff = kKOff + kKBytes;       // 2 stages
  static constexpr int kDOOff = kQOff + 2 * kQBytes;  // 2 stages
  static constexpr int kDSOff = kDOOff + 2 * kQBytes;
  static constexpr int kDSBytes = kKeys * kQRows * 2;  // 16 KB, one column block
  static constexpr int kBoxBytes = kQRows * kSwizzleBytes;  // fp32 box: 64 rows x 32 floats
  static constexpr int kStageOff = kDSOff + kDSBytes;  // 2 boxes
  static constexpr int kLseOff = kStageOff + 2 * kBoxBytes;  // float[2][64]
  static constexpr int kDeltaOff = kLseOff + 2 * kQRows * 4;  // float[2][64]
  static constexpr int kBarOff = kDeltaOff + 2 * kQRows * 4;
  // kv_full, v_ready, q_full[2], q_empty[2], do_full[2], do_empty[2],
  // ld_full[2], ld_empty[2], s_full, dp_full, p_ready, ds_ready, ds_empty,
  // dq_full, dq_empty, stage_full[2], stage_free[2][2], dkdv_done
  static constexpr int kNumBars = 2 + 12 + 7 + 6 + 1;
  static constexpr int kCtlOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kCtlOff + 64;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColV = 0;
  static constexpr uint32_t kColDV = 128;
  static constexpr uint32_t kColDK = 256;
  static constexpr uint32_t kColS = 384;
  static constexpr uint32_t kColDP = 448;
  static constexpr uint32_t kColDQ = kColDP;
};

constexpr int kWideBwdThreads = 512;
// Launch allocation 128 registers x 512 threads; after setmaxnreg:
// WG0 56 + WG1 152 + WG2 152 + WG3 152 = 512 per 128 threads x 4 groups.
constexpr int kWideBwdLaunchRegs = 128;
constexpr int kWRegsCtrl = 56;
constexpr int kWRegsWork = 152;
static_assert(kWRegsCtrl + 3 * kWRegsWork <= 4 * kWideBwdLaunchRegs, "register split exceeds the launch");

__device__ __forceinline__ bool wwait(uint64_t* bar, uint32_t parity, CtaControl* ctl, uint64_t timeout_ns,
                                      int* status, int site) {
  const bool ok = mbar_wait(bar, parity, ctl, timeout_ns, status, site);
  return __all_sync(0xffffffffu, ok);
}

// P^T for 32 queries of one key row: p = exp2(s * scale*log2(e) - LSE2[q]).
// nlse holds the negated LSE values (padded queries: -inf, so p = 0).
// kMasked drops query q0 + e when it precedes this thread's key (q_rel and
// key_rel are positions relative to the tile's first key) and zeroes the
// whole row of a key past the sequence (key_ok false).  Unmasked chunks run
// 2 of every 8 exponential pairs on the FMA pipe.
template <bool kMasked>
__device__ __forceinline__ void wide_probs(const uint32_t (&sv)[32], const float* nlse, float scale_log2,
                                           int q_rel0, int key_rel, bool key_ok, float (&p)[32]) {
  const float4* nlse4 = reinterpret_cast<const float4*>(nlse);
  const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    const float4 l = nlse4[e4];
    float x[4];
    const int e0 = e4 * 4;
    f2_unpack(ffma2(f2_pack(__uint_as_float(sv[e0]), __uint_as_float(sv[e0 + 1])), scale2, f2_pack(l.x, l.y)),
              x[0], x[1]);
    f2_unpack(ffma2(f2_pack(__uint_as_float(sv[e0 + 2]), __uint_as_float(sv[e0 + 3])), scale2, f2_pack(l.z, l.w)),
              x[2], x[3]);
    if (!kMasked && e4 >= 6) {
      exp2_fma_pair(x[0], x[1], p[e0], p[e0 + 1]);
      exp2_fma_pair(x[2], x[3], p[e0 + 2], p[e0 + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = e0 + j;
        float pv = ex2(x[j]);
        if constexpr (kMasked) {
          if (q_rel0 + e < key_rel || !key_ok) pv = 0.0f;
        }
        p[e] = pv;
      }
    }
  }
}

// One TMEM row of 128 fp32 values (times `mul`) as dtype into a swizzled
// 128-row tile of two column blocks, row r.
template <bool kBf16>
__device__ __forceinline__ void wide_stage_row(uint32_t t_row, uint8_t* tile, int r, float mul) {
#pragma unroll
  for (int cb = 0; cb < 4; ++cb) {
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

template <bool kBf16>
__global__ void __launch_bounds__(kWideBwdThreads, 1)
    attn_bwd_d256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_dk,
                         const __grid_constant__ CUtensorMap tm_dv, const __grid_constant__ CUtensorMap tm_dq,
                         const uint16_t* __restrict__ v_raw, const float* __restrict__ lse,
                         const float* __restrict__ delta, int S, int n_ktiles, int causal, float scale,
                         float scale_log2, int d_real, unsigned long long timeout_ns, int* status) {
  using C = WideBwdCfg;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(status, kOk, kErrMisaligned);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  // Head-major; within a head the key tiles with the most steps first; the
  // two head-dim halves of a tile adjacent.
  const int half = static_cast<int>(blockIdx.x) & 1;
  const int tile = static_cast<int>(blockIdx.x) >> 1;
  const int bh = tile / n_ktiles;
  const int jn = tile % n_ktiles;
  const int n0 = jn * C::kKeys;
  const int n_qsteps = (S + C::kQRows - 1) / C::kQRows;
  const int i_start = causal ? n0 / C::kQRows : 0;
  const int n_steps = n_qsteps - i_start;
  const int col0 = half * C::kHalf;  // first head-dim column of this CTA's outputs

  uint8_t* sK = smem + C::kKOff;
  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sDO = smem + C::kDOOff;
  uint8_t* sDS = smem + C::kDSOff;
  uint8_t* sStage = smem + C::kStageOff;
  float* sLse = reinterpret_cast<float*>(smem + C::kLseOff);
  float* sDelta = reinterpret_cast<float*>(smem + C::kDeltaOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* v_ready = bars + 1;
  uint64_t* q_full = bars + 2;      // [2]
  uint64_t* q_empty = q_full + 2;   // [2]
  uint64_t* do_full = q_empty + 2;  // [2]
  uint64_t* do_empty = do_full + 2;  // [2]
  uint64_t* ld_full = do_empty + 2;  // [2]
  uint64_t* ld_empty = ld_full + 2;  // [2]
  uint64_t* s_full = ld_empty + 2;
  uint64_t* dp_full = s_full + 1;
  uint64_t* p_ready = dp_full + 1;
  uint64_t* ds_ready = p_ready + 1;
  uint64_t* ds_empty = ds_ready + 1;
  uint64_t* dq_full = ds_empty + 1;
  uint64_t* dq_empty = dq_full + 1;
  uint64_t* stage_full = dq_empty + 1;   // [2]: buffer b staged
  uint64_t* stage_free = stage_full + 2;  // [2][2]: buffer b free for producer p, at 2 * b + p
  uint64_t* dkdv_done = stage_free + 4;
  CtaControl* ctl = reinterpret_cast<CtaControl*>(smem + C::kCtlOff);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(v_ready, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&do_full[i], 1);
      mbar_init(&do_empty[i], 1);
      mbar_init(&ld_full[i], 32);
      mbar_init(&ld_empty[i], 8);
      mbar_init(&stage_full[i], 1);
      mbar_init(&stage_free[2 * i], 1);
      mbar_init(&stage_free[2 * i + 1], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(ds_ready, 8);
    mbar_init(ds_empty, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(dkdv_done, 1);
    ctl->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
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
    warpgroup_reg_dec<kWRegsCtrl>();
    if (warp == 3) {
      // ---------------- Q producer ----------------
      for (int it = 0; it < n_steps; ++it) {
        const int m0 = (i_start + it) * C::kQRows;
        const int st = it & 1;
        if (!wwait(&q_empty[st], ((it >> 1) & 1) ^ 1, ctl, timeout_ns, status, 31)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[st], C::kQBytes);
#pragma unroll
          for (int b = 0; b < 4; ++b)
            tma_load_3d(sQ + st * C::kQBytes + b * C::kQBlock, &tm_q, &q_full[st], b * 64, m0, bh);
        }
      }
    } else if (warp == 0) {
      // ---------------- K, dO and LSE/delta producer ----------------
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, C::kKBytes);
#pragma unroll
        for (int b = 0; b < 4; ++b) tma_load_3d(sK + b * kBlockBytes, &tm_k, kv_full, b * 64, n0, bh);
      }
      for (int it = 0; it < n_steps; ++it) {
        const int m0 = (i_start + it) * C::kQRows;
        const int st = it & 1;
        if (!wwait(&do_empty[st], ((it >> 1) & 1) ^ 1, ctl, timeout_ns, status, 32)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&do_full[st], C::kQBytes);
#pragma unroll
          for (int b = 0; b < 4; ++b)
            tma_load_3d(sDO + st * C::kQBytes + b * C::kQBlock, &tm_do, &do_full[st], b * 64, m0, bh);
        }
        if (!wwait(&ld_empty[st], ((it >> 1) & 1) ^ 1, ctl, timeout_ns, status, 33)) break;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int q = e * 32 + lane;
          const int mg = m0 + q;
          const bool valid = mg < S;
          sLse[st * C::kQRows + q] = valid ? -lse[row_base + mg] : -INFINITY;
          sDelta[st * C::kQRows + q] = valid ? delta[row_base + mg] : 0.0f;
        }
        mbar_arrive(&ld_full[st]);
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      const bool leader = elect_one();
      const uint32_t fmt = kBf16 ? 1u : 0u;
      const uint32_t idesc_s = idesc_f16(fmt, 128, C::kQRows, 0, 0);
      const uint32_t idesc_kv = idesc_f16(fmt, 128, C::kHalf, 0, 1);
      const uint32_t idesc_dq = idesc_f16(fmt, 128, C::kQRows, 1, 1);
      const uint32_t k_lo = sdesc_lo_kmajor(smem_u32(sK));
      // K^T of this CTA's head-dim half (M = 128 columns over two blocks).
      const uint32_t kt_lo = sdesc_lo_mnmajor(smem_u32(sK) + half * 2 * kBlockBytes, C::kKeys);
      const uint32_t ds_lo = sdesc_lo_kmajor(smem_u32(sDS));
      const uint32_t ds_mn_lo = sdesc_lo_mnmajor(smem_u32(sDS), C::kKeys);
      const uint32_t q_lo0 = sdesc_lo_kmajor(smem_u32(sQ));
      const uint32_t q_mn_lo0 = sdesc_lo_mnmajor(smem_u32(sQ) + half * 2 * C::kQBlock, C::kQRows);
      const uint32_t do_lo0 = sdesc_lo_kmajor(smem_u32(sDO));
      const uint32_t do_mn_lo0 = sdesc_lo_mnmajor(smem_u32(sDO) + half * 2 * C::kQBlock, C::kQRows);
      constexpr uint32_t kStageLo = C::kQBytes >> 4;
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        if (!wwait(&q_full[st], (it >> 1) & 1, ctl, timeout_ns, status, 34)) return false;
        tc_fence_after();
        const uint32_t q_lo = q_lo0 + st * kStageLo;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < C::kW / 16; ++kk)
            umma_ss_w(tmem + C::kColS, k_lo + kmajor_koff(C::kKeys, kk * 16),
                      q_lo + kmajor_koff(C::kQRows, kk * 16), idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(s_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_dp = [&](int it) -> bool {
        const int st = it & 1;
        if (!wwait(&do_full[st], (it >> 1) & 1, ctl, timeout_ns, status, 35)) return false;
        if (it > 0 && !wwait(dq_empty, (it - 1) & 1, ctl, timeout_ns, status, 36)) return false;
        tc_fence_after();
        const uint32_t do_lo = do_lo0 + st * kStageLo;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < C::kW / 16; ++kk)
            umma_ts_w(tmem + C::kColDP, tmem + C::kColV + kk * 8, do_lo + kmajor_koff(C::kQRows, kk * 16), idesc_s,
                      kk > 0 ? 1u : 0u);
          umma_commit(dp_full);
        }
        __syncwarp();
        return true;
      };
      bool ok = wwait(kv_full, 0, ctl, timeout_ns, status, 37) && wwait(v_ready, 0, ctl, timeout_ns, status, 38);
      if (ok) ok = issue_s(0) && issue_dp(0);
      for (int it = 0; ok && it < n_steps; ++it) {
        const int st = it & 1;
        // dV += P^T dO[:, half].  P^T of queries 32h..32h+31 sits packed in
        // the first 16 of dS warpgroup h's 32 S columns.
        if (!(ok = wwait(p_ready, it & 1, ctl, timeout_ns, status, 39))) break;
        tc_fence_after();
        if (leader) {
          const uint32_t do_mn_lo = do_mn_lo0 + st * kStageLo;
#pragma unroll
          for (int kk = 0; kk < C::kQRows / 16; ++kk)
            umma_ts_w(tmem + C::kColDV, tmem + C::kColS + (kk >> 1) * 32 + (kk & 1) * 8,
                      do_mn_lo + mnmajor_koff(kk * 16), idesc_kv, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&do_empty[st]);
        }
        __syncwarp();
        if (it + 1 < n_steps && !(ok = issue_s(it + 1))) break;
        if (!(ok = wwait(ds_ready, it & 1, ctl, timeout_ns, status, 40))) break;
        tc_fence_after();
        if (leader) {
          // dQ^T[half] = K^T[half] dS^T  (M = head-dim columns, N = queries)
#pragma unroll
          for (int kk = 0; kk < C::kKeys / 16; ++kk)
            umma_ss_w(tmem + C::kColDQ, kt_lo + mnmajor_koff(kk * 16), ds_mn_lo + mnmajor_koff(kk * 16), idesc_dq,
                      kk > 0 ? 1u : 0u);
          umma_commit(dq_full);
          // dK[:, half] += dS^T Q[:, half]; the dS tile and Q_i are free after it.
          const uint32_t q_mn_lo = q_mn_lo0 + st * kStageLo;
#pragma unroll
          for (int kk = 0; kk < C::kQRows / 16; ++kk)
            umma_ss_w(tmem + C::kColDK, ds_lo + kmajor_koff(C::kKeys, kk * 16), q_mn_lo + mnmajor_koff(kk * 16),
                      idesc_kv, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&q_empty[st]);
          umma_commit(ds_empty);
        }
        __syncwarp();
        if (it + 1 < n_steps && !(ok = issue_dp(it + 1))) break;
      }
      if (ok) {
        if (leader) umma_commit(dkdv_done);
        __syncwarp();
      }
    } else {
      // ---------------- dQ reduce issuer (warp 2) ----------------
      // Per step four boxes (32 head-dim columns x 64 queries) through two
      // buffers: box c of a step goes through buffer b = c & 1 and is staged
      // by producer p = c >> 1 (dQ warp c), so each buffer alternates between
      // two producers.  Each box is reduced as soon as it is staged; once the
      // TMA has read it (checked one reduction later) its buffer is handed to
      // the other producer of that buffer through that producer's own free
      // barrier (one barrier per producer, so no wait can see a phase two
      // uses old).
      bool ok = true;
      int prev = -1;  // 2 * buffer + producer of the previous box
      for (int it = 0; ok && it < n_steps; ++it) {
        const int m0 = (i_start + it) * C::kQRows;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int b = c & 1;
          const uint32_t use = static_cast<uint32_t>(2 * it + (c >> 1));
          if (!(ok = wwait(&stage_full[b], use & 1, ctl, timeout_ns, status, 41))) break;
          if (lane == 0) {
            const int c0 = col0 + c * 32;
            if (c0 < d_real) tma_reduce_add_3d(&tm_dq, sStage + b * C::kBoxBytes, c0, m0, bh);
            tma_store_commit();
            tma_store_wait_read_le1();
            if (prev >= 0) mbar_arrive(&stage_free[prev ^ 1]);  // the other producer of that buffer
          }
          prev = 2 * b + (c >> 1);
          __syncwarp();
        }
      }
      if (lane == 0) {
        tma_store_wait_read_all();
        if (ok && prev >= 0) mbar_arrive(&stage_free[prev ^ 1]);
        tma_store_wait_all();
      }
    }
  } else if (wg == 1) {
    warpgroup_reg_inc<kWRegsWork>();
    // ---------------- dQ warps: thread r owns head-dim column col0 + r ----------------
    const int q4 = warp & 3;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const int b = q4 & 1;   // staging buffer
    const int pr = q4 >> 1;  // producer slot of that buffer: 0 stages first in a step, 1 second
    bool ok = true;
    for (int it = 0; ok && it < n_steps; ++it) {
      if (!(ok = wwait(dq_full, it & 1, ctl, timeout_ns, status, 42))) break;
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld32(t_lane + C::kColDQ, v[0]);
      tmem_ld32(t_lane + C::kColDQ + 32, v[1]);
      tmem_wait_ld();
      reg_fence(v[0]);
      reg_fence(v[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
      // Producer 0's use in step it follows producer 1's use in step it - 1
      // (it completions of its free barrier, none needed at it = 0);
      // producer 1's follows producer 0's use in the same step (it + 1).
      const uint32_t parity = pr == 0 ? ((it & 1) ^ 1) : (it & 1);
      if (!(ok = wwait(&stage_free[2 * b + pr], parity, ctl, timeout_ns, status, 43))) break;
      uint8_t* box = sStage + b * C::kBoxBytes;
      // box[q][lane] = scale * dQ[q][col0 + 32 q4 + lane]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          *reinterpret_cast<float*>(box + swz_offset_f32(h * 32 + e, lane)) = __uint_as_float(v[h][e]) * scale;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&stage_full[b]);
    }
  } else {
    warpgroup_reg_inc<kWRegsWork>();
    // ---------------- dS warps: thread t owns key n0 + t ----------------
    const int h = wg - 2;  // query half of the step owned by this warpgroup
    const int q4 = warp & 3;
    const int t = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t s_cols = t_lane + C::kColS + h * 32;
    const uint32_t dp_cols = t_lane + C::kColDP + h * 32;
    const bool key_ok = (n0 + t) < S;
    if (h == 0) {
      // V row of key n0 + t, packed 16-bit pairs (the A operand layout of
      // dP^T = V dO^T), into TMEM columns [0, 128); zero past the sequence
      // and past head_dim.
      const uint4* src = reinterpret_cast<const uint4*>(v_raw + (row_base + n0 + t) * static_cast<size_t>(d_real));
      const int chunks = d_real / 8;  // 16-byte pieces of the row
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t w[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = j * 8 + u;
          uint4 x = make_uint4(0u, 0u, 0u, 0u);
          if (key_ok && c < chunks) x = src[c];
          w[4 * u] = x.x;
          w[4 * u + 1] = x.y;
          w[4 * u + 2] = x.z;
          w[4 * u + 3] = x.w;
        }
        tmem_st32(t_lane + C::kColV + j * 32, w);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(v_ready);
    }
    bool ok = true;
    for (int it = 0; it < n_steps; ++it) {
      const int m0 = (i_start + it) * C::kQRows;
      const int lb = it & 1;
      if (!(ok = wwait(&ld_full[lb], (it >> 1) & 1, ctl, timeout_ns, status, 44))) break;
      if (!(ok = wwait(s_full, it & 1, ctl, timeout_ns, status, 45))) break;
      tc_fence_after();
      const float* nlse_s = sLse + lb * C::kQRows + h * 32;
      const float* del_s = sDelta + lb * C::kQRows + h * 32;
      const int q_rel0 = m0 - n0 + h * 32;  // first query of this warpgroup, relative to key n0
      // Masked when some query of the step precedes some key of the tile
      // (causal), or the tile runs past the sequence.
      const bool masked = __any_sync(0xffffffffu, (causal && q_rel0 < t) || !key_ok);
      float p[32];
      {
        uint32_t sv[32];
        tmem_ld32(s_cols, sv);
        tmem_wait_ld();
        reg_fence(sv);
        if (masked)
          wide_probs<true>(sv, nlse_s, scale_log2, causal ? q_rel0 : (1 << 30), t, key_ok, p);
        else
          wide_probs<false>(sv, nlse_s, scale_log2, 0, 0, true, p);
      }
      {
        uint32_t pp[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pp[e] = pack2<kBf16>(p[2 * e], p[2 * e + 1]);
        tmem_st16(s_cols, pp);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      // dS^T = P^T (dP^T - delta) -> smem for the dK and dQ products.
      if (!(ok = wwait(dp_full, it & 1, ctl, timeout_ns, status, 46))) break;
      if (it > 0 && !(ok = wwait(ds_empty, (it - 1) & 1, ctl, timeout_ns, status, 47))) break;
      tc_fence_after();
      uint32_t dpv[32];
      tmem_ld32(dp_cols, dpv);
      tmem_wait_ld();
      reg_fence(dpv);
      uint32_t dd[16];
      const float4* del4 = reinterpret_cast<const float4*>(del_s);
      const uint64_t neg1 = f2_pack(-1.0f, -1.0f);
#pragma unroll
      for (int e4 = 0; e4 < 8; ++e4) {
        const float4 dl = del4[e4];
        const int e = e4 * 4;
        float d0, d1, d2, d3;
        f2_unpack(fmul2(f2_pack(p[e], p[e + 1]),
                        ffma2(f2_pack(dl.x, dl.y), neg1, f2_pack(__uint_as_float(dpv[e]), __uint_as_float(dpv[e + 1])))),
                  d0, d1);
        f2_unpack(fmul2(f2_pack(p[e + 2], p[e + 3]),
                        ffma2(f2_pack(dl.z, dl.w), neg1,
                              f2_pack(__uint_as_float(dpv[e + 2]), __uint_as_float(dpv[e + 3])))),
                  d2, d3);
        dd[e4 * 2] = pack2<kBf16>(d0, d1);
        dd[e4 * 2 + 1] = pack2<kBf16>(d2, d3);
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint4 x = make_uint4(dd[w * 4 + 0], dd[w * 4 + 1], dd[w * 4 + 2], dd[w * 4 + 3]);
        *reinterpret_cast<uint4*>(sDS + swz_offset(t, h * 32 + w * 8, C::kKeys)) = x;
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
    // (scaled, staged through Q stage 1).  Rows past the sequence are
    // clipped by the tensor map; column blocks past head_dim are skipped.
    uint8_t* stage = sQ + h * C::kQBytes;
    if (ok) ok = wwait(dkdv_done, 0, ctl, timeout_ns, status, 48);
    if (ok) {
      tc_fence_after();
      if (h == 0)
        wide_stage_row<kBf16>(t_lane + C::kColDV, stage, t, 1.0f);
      else
        wide_stage_row<kBf16>(t_lane + C::kColDK, stage, t, scale);
      fence_proxy_async_smem();
    }
    named_barrier_sync(1 + h, 128);
    if ((warp & 3) == 0 && lane == 0 && ok && !ctl->abort) {
      const CUtensorMap* map = (h == 0) ? &tm_dv : &tm_dk;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const int c0 = col0 + b * 64;
        if (c0 < d_real) tma_store_3d(map, stage + b * kBlockBytes, c0, n0, bh);
      }
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

}  // namespace

int launch_attn_bwd_d256(const BwdD256Args& a) {
  using C = WideBwdCfg;
  static_assert(C::kSmemBytes <= 232448, "wide-head backward shared memory exceeds the sm_100 limit");
  if (a.D <= 128 || a.D > C::kW || a.D % 8 != 0) return kErrUnsupported;
  const long long n_ktiles = (a.S + C::kKeys - 1) / C::kKeys;
  const long long grid = n_ktiles * a.BH * 2;
  if (grid > 0x7fffffffLL) return kErrTooLarge;
  auto kern = a.bf16 ? attn_bwd_d256_kernel<true> : attn_bwd_d256_kernel<false>;
  // The setmaxnreg split inside the kernel assumes exactly kWideBwdLaunchRegs
  // registers per thread at launch; a build that differs is refused.
  if (int rc = prepare_kernel(reinterpret_cast<const void*>(kern), C::kSmemBytes, kWideBwdLaunchRegs, nullptr))
    return rc;
  kern<<<static_cast<unsigned>(grid), kWideBwdThreads, C::kSmemBytes, a.stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_do, *a.tm_dk, *a.tm_dv, *a.tm_dq, static_cast<const uint16_t*>(a.v), a.lse, a.delta,
      static_cast<int>(a.S), static_cast<int>(n_ktiles), a.causal, a.scale, a.scale_log2, static_cast<int>(a.D),
      a.timeout_ns, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace tk
