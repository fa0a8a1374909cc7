// Static flat-slab slot placement of one layer (host code, install time, integer).
//
// Restates the placement core of _segmented_flat_build_static_slot_schedule
// (enable_real_pruning_fast.py:260-370) and the capacity bound of
// _segmented_flat_cache_capacity_for_layer (:206-234), bit for bit:
//   * live interval of (source s, head h): [s + 1, end) with end the first target t > s whose
//     removed set holds h for s (else the number of scales); empty or zero-length ones dropped;
//   * intervals placed in (start, end, -length, source, head) order; before each placement the
//     intervals that ended by its start go back to the free list, which is sorted by offset and
//     coalesced (overlapping or touching blocks merge, zero-length blocks vanish); the segment
//     takes the free block with the least leftover, then the lowest offset, from its front, else
//     the high-water mark grows.
// The Python side (scheduler.py) derives the per-target metadata and copy descriptors from the
// placed offsets.
#include <algorithm>
#include <cstdint>
#include <tuple>
#include <vector>

#include "heatkv.h"

namespace {

struct Interval {
  int source, head, start_t, end_t;
  int64_t length;
  int64_t offset;
};

struct Block {
  int64_t off, len;
};

void coalesce(std::vector<Block>& free) {
  std::vector<Block> in;
  in.reserve(free.size());
  for (const Block& b : free)
    if (b.len > 0) in.push_back(b);
  std::sort(in.begin(), in.end(), [](const Block& a, const Block& b) {
    return a.off != b.off ? a.off < b.off : a.len < b.len;
  });
  free.clear();
  for (const Block& b : in) {
    if (!free.empty() && b.off <= free.back().off + free.back().len) {
      Block& last = free.back();
      last.len = std::max(last.off + last.len, b.off + b.len) - last.off;
    } else {
      free.push_back(b);
    }
  }
}

}  // namespace

extern "C" int heatkv_slot_schedule(const uint8_t* removed, int num_scales, int num_heads,
                                    const int64_t* scale_start, const int64_t* scale_end,
                                    int64_t* offset_out, int32_t* end_target_out,
                                    int64_t* capacity_out, int64_t* bound_out) {
  if (num_scales <= 0 || num_heads <= 0 || !removed || !scale_start || !scale_end ||
      !offset_out || !end_target_out || !capacity_out || !bound_out)
    return HEATKV_ERR_INVALID_ARGUMENT;
  const int S = num_scales, H = num_heads;
  auto rem = [&](int t, int s, int h) { return removed[(int64_t(t) * S + s) * H + h] != 0; };

  // capacity bound: max over targets of the retained tokens of the earlier sources
  int64_t bound = 0;
  for (int t = 1; t < S; ++t) {
    int64_t total = 0;
    for (int s = 0; s < t; ++s) {
      int64_t kept = H;
      for (int h = 0; h < H; ++h) kept -= rem(t, s, h) ? 1 : 0;
      total += kept * std::max<int64_t>(scale_end[s] - scale_start[s], 0);
    }
    bound = std::max(bound, total);
  }

  std::vector<Interval> intervals;
  for (int s = 0; s < S; ++s) {
    for (int h = 0; h < H; ++h) {
      offset_out[int64_t(s) * H + h] = -1;
      end_target_out[int64_t(s) * H + h] = -1;
    }
    const int start_t = s + 1;
    const int64_t length = scale_end[s] - scale_start[s];
    if (start_t >= S || length <= 0) continue;
    for (int h = 0; h < H; ++h) {
      int end_t = S;
      for (int t = start_t; t < S; ++t) {
        if (rem(t, s, h)) {
          end_t = t;
          break;
        }
      }
      if (end_t <= start_t) continue;
      intervals.push_back({s, h, start_t, end_t, length, -1});
    }
  }
  std::sort(intervals.begin(), intervals.end(), [](const Interval& a, const Interval& b) {
    return std::make_tuple(a.start_t, a.end_t, -a.length, a.source, a.head) <
           std::make_tuple(b.start_t, b.end_t, -b.length, b.source, b.head);
  });

  std::vector<Block> free;
  std::vector<const Interval*> active;
  int64_t high_water = 0;
  for (Interval& seg : intervals) {
    std::vector<const Interval*> still;
    for (const Interval* a : active) {
      if (a->end_t <= seg.start_t) free.push_back({a->offset, a->length});
      else still.push_back(a);
    }
    active.swap(still);
    coalesce(free);
    int best = -1;
    for (int i = 0; i < static_cast<int>(free.size()); ++i) {
      if (free[i].len < seg.length) continue;
      if (best < 0 || std::make_pair(free[i].len - seg.length, free[i].off) <
                          std::make_pair(free[best].len - seg.length, free[best].off))
        best = i;
    }
    if (best >= 0) {
      seg.offset = free[best].off;
      if (free[best].len == seg.length) {
        free.erase(free.begin() + best);
      } else {
        free[best].off += seg.length;
        free[best].len -= seg.length;
      }
    } else {
      seg.offset = high_water;
      high_water += seg.length;
    }
    active.push_back(&seg);
    offset_out[int64_t(seg.source) * H + seg.head] = seg.offset;
    end_target_out[int64_t(seg.source) * H + seg.head] = seg.end_t;
  }
  *capacity_out = high_water;
  *bound_out = bound;
  return HEATKV_OK;
}
