// Install-time planning of the pruned KV cache in native code (host, integer): the per-target
// segment tables and copy items of one layer's static slab schedule, and the strict budget
// schedule that decides which (source scale, head, layer) atoms are removed at each target.
//
// heatkv_slot_tables restates the derivations of _segmented_flat_build_static_slot_schedule
// (enable_real_pruning_fast.py:383-558) from a placement (heatkv_slot_schedule):
//   * target t's live segments are those with start_target <= t < end_target; per head they are
//     listed in source-scale order (:383-412);
//   * the activation copy of target t reads the dense cache of the old_len = scale_start[t] tokens
//     before it: for every live segment the part of its scale below old_len, from row
//     head * old_len + scale_start (:414-510);
//   * the append after scale s copies the whole scale into every segment (s, h) still live at
//     s + 1, from row head * n_s (:512-545);
//   copy items are sorted by destination slot, as the runs of :414-482 order them.
//
// heatkv_strict_budget restates the main loop of strict_pruning_schedule_for_budget_scale_specific
// (tools/utils.py:308-522): per target t the atoms to remove are the first prune_count[t + 1]
// entries of every source order s0..min(s1, t); walking the layer checkpoints l = 0..L-1, the
// atoms of layer l count as removed, the current scale's K/V of layer l enter the cache, and while
// the cache total exceeds budget * L * H * peak, atoms of later layers are activated early in
// priority order (last layer first, then larger source scale, then order rank). The cache total
// is kept as an integer; the comparisons with the threshold are the reference's (integer against
// double).
#include <algorithm>
#include <cstdint>
#include <tuple>
#include <vector>

#include "heatkv.h"

extern "C" int heatkv_slot_tables(int num_scales, int num_heads, const int64_t* scale_start,
                                  const int64_t* scale_end, const int64_t* offset,
                                  const int32_t* end_target, int32_t* meta_starts,
                                  int32_t* meta_ends, int32_t* meta_counts, int64_t* pack_items,
                                  int64_t* pack_index, int64_t* append_items,
                                  int64_t* append_index) {
  if (num_scales <= 0 || num_heads <= 0 || !scale_start || !scale_end || !offset || !end_target ||
      !meta_starts || !meta_ends || !meta_counts || !pack_items || !pack_index || !append_items ||
      !append_index)
    return HEATKV_ERR_INVALID_ARGUMENT;
  const int S = num_scales, H = num_heads;
  // per-target segment tables [S][H][S], sources in increasing order
  for (int64_t i = 0; i < int64_t(S) * H * S; ++i) meta_starts[i] = meta_ends[i] = 0;
  for (int64_t i = 0; i < int64_t(S) * H; ++i) meta_counts[i] = 0;
  for (int t = 1; t < S; ++t) {
    for (int s = 0; s < S; ++s) {
      for (int h = 0; h < H; ++h) {
        const int64_t k = int64_t(s) * H + h;
        if (offset[k] < 0 || !(s + 1 <= t && t < end_target[k])) continue;
        const int64_t len = scale_end[s] - scale_start[s];
        const int64_t row = int64_t(t) * H + h;
        const int c = meta_counts[row]++;
        meta_starts[row * S + c] = static_cast<int32_t>(offset[k]);
        meta_ends[row * S + c] = static_cast<int32_t>(offset[k] + len);
      }
    }
  }
  // activation copy items of every target, (dst, src, length) sorted by dst
  std::vector<std::tuple<int64_t, int64_t, int64_t>> items;
  int64_t n = 0;
  pack_index[0] = 0;
  pack_index[1] = 0;
  for (int t = 1; t < S; ++t) {
    items.clear();
    const int64_t old_len = scale_start[t];
    for (int s = 0; s < S; ++s) {
      for (int h = 0; h < H; ++h) {
        const int64_t k = int64_t(s) * H + h;
        if (offset[k] < 0 || !(s + 1 <= t && t < end_target[k])) continue;
        const int64_t hi = std::min(scale_end[s], old_len);
        if (scale_start[s] < hi)
          items.emplace_back(offset[k], int64_t(h) * old_len + scale_start[s], hi - scale_start[s]);
      }
    }
    std::sort(items.begin(), items.end());
    for (const auto& it : items) {
      pack_items[3 * n] = std::get<0>(it);
      pack_items[3 * n + 1] = std::get<1>(it);
      pack_items[3 * n + 2] = std::get<2>(it);
      ++n;
    }
    pack_index[t + 1] = n;
  }
  // append items after every scale s (into the segments live at s + 1)
  n = 0;
  append_index[0] = 0;
  for (int s = 0; s < S; ++s) {
    items.clear();
    const int64_t cur = scale_end[s] - scale_start[s];
    if (s + 1 < S && cur > 0) {
      for (int h = 0; h < H; ++h) {
        const int64_t k = int64_t(s) * H + h;
        if (offset[k] < 0 || !(s + 1 < end_target[k])) continue;
        items.emplace_back(offset[k], int64_t(h) * cur, cur);
      }
    }
    std::sort(items.begin(), items.end());
    for (const auto& it : items) {
      append_items[3 * n] = std::get<0>(it);
      append_items[3 * n + 1] = std::get<1>(it);
      append_items[3 * n + 2] = std::get<2>(it);
      ++n;
    }
    append_index[s + 1] = n;
  }
  return HEATKV_OK;
}

extern "C" int heatkv_strict_budget(const int32_t* orders, int num_sources, int num_layers,
                                    int num_heads, int num_scales, const int64_t* tokens,
                                    int source_start, int protected_prefix_scales, int budgeted,
                                    double threshold, const int64_t* prune_count,
                                    uint8_t* final_mask, int32_t* early, int64_t early_capacity,
                                    int64_t* early_count, int64_t* error_info) {
  if (!orders || !tokens || !prune_count || !final_mask || !early || !early_count || !error_info ||
      num_sources <= 0 || num_layers <= 0 || num_heads <= 0 || num_scales <= 0)
    return HEATKV_ERR_INVALID_ARGUMENT;
  const int S = num_scales, L = num_layers, H = num_heads, s0 = source_start;
  const int s1 = s0 + num_sources - 1;
  const int64_t LH = int64_t(L) * H;
  // rank of (head, layer) in the order of source s
  std::vector<int32_t> rank(size_t(num_sources) * LH, -1);
  for (int i = 0; i < num_sources; ++i)
    for (int64_t r = 0; r < LH; ++r) {
      const int h = orders[(i * LH + r) * 2], l = orders[(i * LH + r) * 2 + 1];
      if (h < 0 || h >= H || l < 0 || l >= L) return HEATKV_ERR_INVALID_ARGUMENT;
      rank[size_t(i) * LH + int64_t(l) * H + h] = static_cast<int32_t>(r);
    }
  auto at = [&](int s, int l, int h) { return (int64_t(s) * L + l) * H + h; };
  const int64_t per_t = int64_t(S) * L * H;
  for (int64_t i = 0; i < int64_t(S) * per_t; ++i) final_mask[i] = 0;
  std::vector<uint8_t> active(per_t, 0), target(per_t, 0), cur(per_t, 0);
  std::vector<int32_t> removed_sl(size_t(S) * L, 0);
  int64_t n_early = 0;
  error_info[0] = error_info[1] = error_info[2] = 0;
  for (int t = 0; t < S; ++t) {
    uint8_t* fin = final_mask + int64_t(t) * per_t;
    if (t >= budgeted) {
      std::copy(active.begin(), active.end(), fin);
      continue;
    }
    const int nxt = std::min(t + 1, S - 1);
    const int64_t count = prune_count[nxt];
    std::fill(target.begin(), target.end(), 0);
    for (int s = s0; s <= std::min(s1, t); ++s)
      for (int64_t r = 0; r < std::min<int64_t>(count, LH); ++r) {
        const int64_t e = ((s - s0) * LH + r) * 2;
        target[at(s, orders[e + 1], orders[e])] = 1;
      }
    // removed atoms per (source, layer) among the active set
    std::fill(removed_sl.begin(), removed_sl.end(), 0);
    for (int s = 0; s < S; ++s)
      for (int l = 0; l < L; ++l)
        for (int h = 0; h < H; ++h)
          if (active[at(s, l, h)]) ++removed_sl[size_t(s) * L + l];
    cur = active;
    // cache total with the current scale's K/V written for layers <= l
    int64_t protected_cached = 0;
    for (int s = 0; s < std::min(protected_prefix_scales, t); ++s) protected_cached += tokens[s];
    int64_t total = LH * protected_cached;
    for (int s = s0; s <= std::min(s1, t); ++s) {
      if (s == t) continue;
      for (int l = 0; l < L; ++l) total += (H - removed_sl[size_t(s) * L + l]) * tokens[s];
    }
    // early-activation candidates: later layer first, then larger source, then order rank
    std::vector<std::tuple<int, int, int32_t, int>> cand;  // (-layer, -source, rank, head)
    for (int s = s0; s <= std::min(s1, t); ++s) {
      if (s == t) continue;
      for (int l = 0; l < L; ++l)
        for (int h = 0; h < H; ++h)
          if (target[at(s, l, h)])
            cand.emplace_back(-l, -s, rank[size_t(s - s0) * LH + int64_t(l) * H + h], h);
    }
    std::sort(cand.begin(), cand.end());
    size_t cursor = 0;
    for (int l = 0; l < L; ++l) {
      for (int s = s0; s <= std::min(s1, t); ++s)
        for (int h = 0; h < H; ++h) {
          const int64_t k = at(s, l, h);
          if (target[k] && !cur[k]) {
            cur[k] = 1;
            ++removed_sl[size_t(s) * L + l];
            if (s != t) total -= tokens[s];
          }
        }
      if (s0 <= t && t <= s1) total += (H - removed_sl[size_t(t) * L + l]) * tokens[t];
      if (static_cast<double>(total) <= threshold) continue;
      while (cursor < cand.size()) {
        const int cl = -std::get<0>(cand[cursor]), cs = -std::get<1>(cand[cursor]);
        const int ch = std::get<3>(cand[cursor]);
        if (cl <= l) break;
        ++cursor;
        const int64_t k = at(cs, cl, ch);
        if (cur[k]) continue;
        cur[k] = 1;
        ++removed_sl[size_t(cs) * L + cl];
        if (n_early >= early_capacity) return HEATKV_ERR_INVALID_ARGUMENT;
        early[5 * n_early] = t;
        early[5 * n_early + 1] = l;
        early[5 * n_early + 2] = cs;
        early[5 * n_early + 3] = ch;
        early[5 * n_early + 4] = cl;
        ++n_early;
        total -= tokens[cs];
        if (static_cast<double>(total) <= threshold) break;
      }
      if (static_cast<double>(total) > threshold) {
        error_info[0] = 1;  // infeasible at (t, l)
        error_info[1] = t;
        error_info[2] = l;
        *early_count = n_early;
        return HEATKV_ERR_INVALID_ARGUMENT;
      }
    }
    if (static_cast<double>(total) > threshold) {
      error_info[0] = 2;  // infeasible at the end of t
      error_info[1] = t;
      *early_count = n_early;
      return HEATKV_ERR_INVALID_ARGUMENT;
    }
    if (cur != target) {
      error_info[0] = 3;  // end-of-scale removals not activated
      error_info[1] = t;
      *early_count = n_early;
      return HEATKV_ERR_INVALID_ARGUMENT;
    }
    active = target;
    std::copy(active.begin(), active.end(), fin);
  }
  *early_count = n_early;
  return HEATKV_OK;
}
