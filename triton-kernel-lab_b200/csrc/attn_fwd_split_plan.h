// Key-split schedule of the forward (attn_fwd_sm100.cu), host and device
// side: which problems are cut into chunks of their key range, how long the
// chunks are, how many units that makes, and how a unit index maps back to
// (slab, query-tile group, chunk).  The test-only self-test library compiles
// this header too, so that CPU tests can check that the launcher's unit
// count and the kernel's decode walk enumerate the same chunks.
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <utility>
#include <vector>

namespace tk {

// Rows of a query tile and keys of a key tile of the 64/128-column forward.
constexpr int kSplitTileRows = 128;

// First query-tile group with a chunk `c` (key tiles [c L, c L + L)) under a
// causal mask, for kT query tiles per group: tile A of group ct sees
// kT ct + 1 key tiles.  Shared by the launcher's unit count and the kernel's
// decode so that both enumerate the same units.
__host__ __device__ __forceinline__ int split_ct_min(int c, int split_l, int kT, int causal) {
  return (!causal || c == 0) ? 0 : (c * split_l - 1) / kT + 1;
}

// Chunk-level walk of the split schedule: unit u -> (bh, ct, chunk) in
// out[0..2].  The kernel runs it once per CTA (one unit per CTA in that
// mode), by one thread.
__host__ __device__ __forceinline__ void fwd_split_decode(int u, int BH, int n_ctiles, int causal, int kT,
                                                          int split_l, int* out) {
  int rem = u, c = 0;
  // The launcher counts exactly the units this walk enumerates; the bound
  // only guards the loop.
  for (; c < 64; ++c) {
    const int per = n_ctiles - split_ct_min(c, split_l, kT, causal);
    if (per <= 0 || rem < BH * per) break;
    rem -= BH * per;
  }
  int per = n_ctiles - split_ct_min(c, split_l, kT, causal);
  if (per < 1) per = 1;
  out[0] = rem / per;
  out[1] = n_ctiles - 1 - rem % per;
  out[2] = c;
}

// Work-item shape of the 64/128-column forward kernels (FwdCfg in
// attn_fwd_sm100.cu, which checks that the two agree): head_dim <= 64 runs
// one query tile per item with two CTAs per SM, wider heads two tiles per
// item with one CTA per SM.
struct FwdKernelShape {
  int kT, min_blocks, width;
};
__host__ __device__ constexpr FwdKernelShape fwd_kernel_shape(int64_t head_dim) {
  return head_dim <= 64 ? FwdKernelShape{1, 2, 64} : FwdKernelShape{2, 1, 128};
}

struct FwdSplitPlan {
  int split_l = 0, cmax = 0, row0 = 0;
  long long units = 0;
  size_t part_bytes = 0, bytes = 0;
};

// A chunk's fixed cost in key-tile times: the CTA's prologue (TMEM and
// barrier set-up, Q load, pipeline fill), its fp32 partial store and its
// share of the merge.  Fitted to four measured split schedules (chunks of
// 16 and 28 key tiles at head_dim 128), which it reproduces within three
// tile times.
constexpr double kChunkOverheadTiles = 7.5;

// Estimated duration, in key-tile times, of the split schedule with chunks
// of L key tiles: its units in the kernel's launch order (chunk level, then
// slab, then query-tile group from the heaviest), each costing its tile-B
// key tiles plus kChunkOverheadTiles, handed to whichever of the `resident`
// CTA slots frees first, as the hardware does with a grid larger than the
// device.
inline double split_makespan(long long n_ctiles, long long n_ntiles, long long BH, int causal, int kT, long long L,
                             long long cmax, long long resident) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> slots;
  for (long long i = 0; i < resident; ++i) slots.push(0.0);
  double makespan = 0.0;
  for (long long c = 0; c < cmax; ++c) {
    const long long ct_lo = split_ct_min(static_cast<int>(c), static_cast<int>(L), kT, causal);
    for (long long bh = 0; bh < BH; ++bh) {
      for (long long ct = n_ctiles - 1; ct >= ct_lo; --ct) {
        const long long na = causal ? std::min<long long>(kT * ct + 1, n_ntiles) : n_ntiles;
        const long long nb = causal ? std::min<long long>(kT * ct + kT, n_ntiles) : n_ntiles;
        const long long j0 = c * L;
        const long long ea = std::min(j0 + L, na);
        const long long eb = (ea == na) ? nb : ea;
        const double t = slots.top() + static_cast<double>(eb - j0) + kChunkOverheadTiles;
        slots.pop();
        slots.push(t);
        makespan = std::max(makespan, t);
      }
    }
  }
  return makespan;
}

// The plan for a forward of BH slabs of length S on a kernel with kT query
// tiles per work item, min_blocks CTAs per SM and D columns, on a device
// with `sms` SMs.  Returns false when the problem is not split: when the
// regular schedule would be persistent, or its longest item has fewer than
// 48 key tiles or less than twice the average load of a resident CTA.
inline bool plan_fwd_split_impl(int kT, int min_blocks, int D, int64_t S, int64_t BH, int causal, int sms,
                                FwdSplitPlan& p) {
  constexpr int R = kSplitTileRows;
  if (sms <= 0 || S <= 0 || BH <= 0 || kT <= 0 || min_blocks <= 0) return false;
  const long long n_ctiles = (S + kT * R - 1) / (kT * R);
  const long long n_ntiles = (S + R - 1) / R;
  const long long resident = static_cast<long long>(min_blocks) * sms;
  const long long n_pair_units = ((n_ctiles + 1) / 2) * BH;
  const bool persist_shape = S <= 4 * R || (causal && (kT == 2 || S <= 16 * R));
  if (n_ctiles > 1 && n_pair_units >= 2LL * resident && persist_shape) return false;
  long long work = 0, na_max = 0;
  for (long long ct = 0; ct < n_ctiles; ++ct) {
    const long long na = causal ? std::min<long long>(kT * ct + 1, n_ntiles) : n_ntiles;
    work += na;
    na_max = std::max(na_max, na);
  }
  work *= BH;
  if (na_max < 48 || static_cast<double>(na_max) < 2.0 * static_cast<double>(work) / resident) return false;
  // Chunk length: the one whose simulated schedule ends first, among
  // lengths from 12 key tiles (shorter chunks pay their fixed cost too
  // often) to four times the average load per resident CTA, with at most
  // 32 chunks per item; ties go to the longer chunk (fewer partials).
  // Planned once per shape, kernel and device.
  static std::mutex mu;
  static std::map<std::tuple<int64_t, int64_t, int, int, int, int>, std::pair<long long, long long>> cache;
  long long L = 0, cmax = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(S, BH, causal, sms, kT, min_blocks);
    auto it = cache.find(key);
    if (it == cache.end()) {
      const long long hi = std::min<long long>(na_max - 1, std::max<long long>(12, 4 * work / resident + 1));
      double best = 0.0;
      for (long long l = hi; l >= 12; --l) {
        const long long cm = (na_max + l - 1) / l;
        if (cm > 32 || cm < 2) continue;
        const double t = split_makespan(n_ctiles, n_ntiles, BH, causal, kT, l, cm, resident);
        if (L == 0 || t < best) {
          best = t;
          L = l;
          cmax = cm;
        }
      }
      it = cache.emplace(key, std::make_pair(L, cmax)).first;
    }
    L = it->second.first;
    cmax = it->second.second;
  }
  if (L == 0 || cmax < 2) return false;
  long long units = 0;
  for (int c = 0; c < cmax; ++c) units += BH * (n_ctiles - split_ct_min(c, static_cast<int>(L), kT, causal));
  if (units > INT32_MAX || BH * cmax * S > INT32_MAX) return false;
  p.split_l = static_cast<int>(L);
  p.cmax = static_cast<int>(cmax);
  p.units = units;
  p.row0 = causal ? split_ct_min(1, p.split_l, kT, causal) * kT * R : 0;
  p.part_bytes = ((static_cast<size_t>(BH) * cmax * S * D * 4 + 255) / 256) * 256;
  p.bytes = p.part_bytes + static_cast<size_t>(BH) * cmax * S * 4;
  return true;
}

}  // namespace tk
