// Key-range split scratch shared by the tcgen05 attention kernels (attn_sm100_cs.cu,
// attn_sm100_cs64.cu): the workspace layout and its size for a call.
//
// A split block (one 128-row query block of one (b, h) whose key tiles are divided into `splits`
// contiguous ranges) needs a counter - how many of its splits have finished - and, per row of every
// split, the split's (running max, row sum) and its unnormalised fp32 O row. The counters live in
// a fixed region at the start of the workspace that nothing else writes: calls of different shapes
// and both kernels share one workspace, and a counter must find zero where an earlier call may
// have left partial results had the regions moved with the shape. The CTA that completes a block's
// last split resets its counter.
#include "attn.h"
#include "common.cuh"

#include <algorithm>

namespace heatkv {
namespace {

constexpr int kRowsPerBlock = 128;  // query rows per split block (both kernels)
constexpr int kD = 128;              // head dim

struct WsLayout {
  size_t counter_off, ml_off, o_off, total;
};

WsLayout ws_layout(int64_t blocks, int splits, int rows_per_block) {
  WsLayout w{};
  if (splits <= 1) return w;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  w.counter_off = 0;
  w.ml_off = size_t(kSplitCounterBlocks) * sizeof(uint32_t);
  const size_t rows = size_t(blocks) * size_t(splits) * size_t(rows_per_block);
  w.o_off = w.ml_off + up(rows * sizeof(float2));
  w.total = w.o_off + up(rows * kD * sizeof(float));
  return w;
}

}  // namespace

bool split_scratch(void* ws, size_t bytes, int64_t split_blocks, int splits, int rows_per_block,
                   SplitScratch* out) {
  const WsLayout wl = ws_layout(split_blocks, splits, rows_per_block);
  if (splits <= 1 || split_blocks > kSplitCounterBlocks || ws == nullptr || bytes < wl.total ||
      (reinterpret_cast<uintptr_t>(ws) & 255u))
    return false;
  uint8_t* base = static_cast<uint8_t*>(ws);
  out->counter = reinterpret_cast<uint32_t*>(base + wl.counter_off);
  out->ml = reinterpret_cast<float2*>(base + wl.ml_off);
  out->o = reinterpret_cast<float*>(base + wl.o_off);
  return true;
}

size_t attention_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int splits) {
  // kv_splits = 0: as many as either kernel would choose for these sizes
  if (splits <= 0)
    splits = std::max(attention_cs_auto_splits(batch, heads, q_len),
                      attention_cs64_auto_splits(batch, heads, q_len));
  splits = std::min(splits, kMaxKvSplits);
  const int64_t blocks = batch * heads * ((q_len + kRowsPerBlock - 1) / kRowsPerBlock);
  if (blocks > kSplitCounterBlocks) return 0;
  return ws_layout(blocks, splits, kRowsPerBlock).total;
}

}  // namespace heatkv
