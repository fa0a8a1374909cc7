// Launch interface shared by the attention kernels and the C entry points.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "heatkv.h"

namespace heatkv {

struct AttnArgs {
  const void* q;          // [B, H, Lq, D]
  const void* slab_k;     // [B, capacity, D] (may be null when capacity == 0)
  const void* slab_v;
  const int32_t* seg_starts;  // [H, max_segments]
  const int32_t* seg_ends;
  const int32_t* seg_counts;  // [H]
  const void* cur_k;      // [B, H, Lq, D]
  const void* cur_v;
  void* out;              // [B, Lq, H*D]
  int64_t batch;
  int64_t heads;
  int64_t q_len;
  int64_t capacity;
  int64_t max_segments;
  float scale;
  const int32_t* head_order = nullptr;  // [heads] permutation, longest first; null = natural
  int kv_splits = 1;                    // key-range splits per query block; 0 = automatic
  int64_t unsplit_blocks = 0;           // with kv_splits > 1: leading blocks left unsplit
  void* workspace = nullptr;            // split partials and counters (zeroed before first use)
  size_t workspace_bytes = 0;
  unsigned int* status = nullptr;       // device status word (device_status_ptr())
  bool static_meta = false;             // metadata not written by the preceding stream work
  bool current_in_segments = false;     // current keys end every non-empty head's segments
  // column-split kernel: CTA c of map_grid runs items item_map[c + k * map_grid] (-1 = none)
  const int32_t* item_map = nullptr;
  int64_t map_len = 0;
  int map_grid = 0;
  // scatter epilogue (tcgen05 kernel, unsplit): rows to n_out full outputs at mapped rows/heads
  void* const* out_ptrs = nullptr;      // [n_out] device array of base pointers
  const int32_t* out_rows = nullptr;    // [batch] -> row of the full output
  const int32_t* out_heads = nullptr;   // [heads] -> head of the full output
  int n_out = 0;
  int64_t out_batch = 0;
  int64_t out_heads_total = 0;
};

// Device address of the sticky status word on the current device (resolved once per device);
// null when it cannot be resolved.
unsigned int* device_status_ptr();

constexpr int kMaxSegments = 256;

cudaError_t launch_attention_simt(const AttnArgs& a, int q_dtype, int k_dtype, int v_dtype,
                                  cudaStream_t st);
// Column-split kernels (attn_sm100_cs.cu): one 128-row Q tile per CTA, the softmax of a tile
// split by columns over warpgroups, unsplit; cudaErrorNotSupported when they cannot take these
// arguments. _cs: q, k, v all bf16 or all f16 (scatter epilogue supported); _tf32: fp32 q and k
// with 16-bit v, kind::tf32 QK with Q in TMEM (no scatter).
cudaError_t launch_attention_sm100_cs(const AttnArgs& a, bool bf16, cudaStream_t st);
// 64-key tiles, two CTAs per SM (16-bit, scatter epilogue supported); cudaErrorNotSupported otherwise
cudaError_t launch_attention_sm100_cs64(const AttnArgs& a, bool bf16, cudaStream_t st);
// kv_splits = 0 for the 64-key kernel: enough splits of every 128-row block for two waves
int attention_cs64_auto_splits(int64_t batch, int64_t heads, int64_t q_len);
cudaError_t launch_attention_sm100_tf32(const AttnArgs& a, bool v_bf16, cudaStream_t st);
// Splits chosen by kv_splits = 0 and the workspace bytes a launch with `splits` needs.
// Key-range split scratch shared by the tcgen05 kernels: per split block a counter (zero between
// calls, in a fixed region at the start of the workspace), and per row of every split its (m, l)
// and unnormalised fp32 O row.
constexpr int kMaxKvSplits = 4;
constexpr int64_t kSplitCounterBlocks = 16384;
struct SplitScratch {
  uint32_t* counter;
  float2* ml;
  float* o;
};
// Carve the scratch of split_blocks blocks of rows_per_block query rows, split `splits` ways, out
// of the workspace; false when splits <= 1, the workspace is absent, small or misaligned, or there
// are more split blocks than counters.
bool split_scratch(void* ws, size_t bytes, int64_t split_blocks, int splits, int rows_per_block,
                   SplitScratch* out);

// kv_splits = 0 for the column-split kernel: enough splits of every 128-row block for two waves
int attention_cs_auto_splits(int64_t batch, int64_t heads, int64_t q_len);
size_t attention_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int splits);

cudaError_t launch_pack_kv(void* dst_k, void* dst_v, const void* src_k, const void* src_v,
                           int64_t row_bytes_k, int64_t row_bytes_v, int64_t batch,
                           int64_t src_rows, int64_t dst_rows, const int64_t* dst_starts,
                           const int64_t* src_starts, const int64_t* lengths, int64_t n_items,
                           int64_t max_length, unsigned int* status, cudaStream_t stream);

// Several packs in one launch (pack_kv.cu). max_vector_bytes: the widest vector (16, 8, 4, 2 or
// 1 bytes) that every job's pointers allow; the row sizes may narrow it further.
cudaError_t launch_pack_kv_batched(const heatkv_pack_job* jobs, int64_t n_jobs,
                                   const int32_t* item_job, const int64_t* dst_starts,
                                   const int64_t* src_starts, const int64_t* lengths,
                                   int64_t n_items, int64_t row_bytes_k, int64_t row_bytes_v,
                                   int64_t batch, int64_t max_length, int max_vector_bytes,
                                   unsigned int* status, cudaStream_t stream);

// One step of the cross-GPU barrier (peer_barrier.cu): publish this rank's next epoch into every
// rank's flag array, then wait (bounded) until every rank's epoch has arrived in its own.
cudaError_t launch_peer_barrier(uint32_t* const* flag_ptrs, uint32_t* counter, int world,
                                int rank, unsigned int* status, cudaStream_t stream);

// Head-shard reassembly (shard_gather.cu); sms = SMs of the device (grid sizing).
cudaError_t launch_shard_gather(void* dst, const void* src, const int32_t* row_map,
                                const int32_t* head_map, int64_t world, int64_t rows_per_rank,
                                int64_t q_len, int64_t heads_per_rank, int64_t batch,
                                int64_t heads, int64_t chunk_bytes, int sms,
                                unsigned int* status, cudaStream_t stream);

// S-CAS attention mass per (head, source scale) of one scale's queries (scas.cu).
cudaError_t launch_scas_mass(const void* q, const void* k, int dtype, int64_t heads, int64_t q_len,
                             int64_t k_len, float scale, const int32_t* bounds, int n_src,
                             double* mass_out, int64_t mass_stride, cudaStream_t st);

// The same on the tensor cores for fp32 q and k (scas_tc.cu: kind::tf32, three products a score);
// cudaErrorNotSupported outside its limits.
cudaError_t launch_scas_mass_tc(const float* q, const float* k, int64_t heads, int64_t q_len,
                                int64_t k_len, float scale, const int32_t* bounds, int n_src,
                                double* mass_out, int64_t mass_stride, unsigned int* status,
                                cudaStream_t st);

// q/k/v preparation after the QKV projection (qkv_prep.cu); sms = SMs of the device.
cudaError_t launch_qkv_project(const void* x, const void* w, const float* bias, void* q, void* k,
                               void* v, bool bf16, bool qk32, int64_t batch, int64_t seq_len, int64_t heads,
                               int64_t embed_dim, const float* scale_mul, float eps,
                               const float* rope_cos, const float* rope_sin,
                               int64_t rope_group_stride, void* cache_k, void* cache_v,
                               int64_t cache_rows, const int64_t* cache_offset,
                               unsigned int* status, cudaStream_t st);

cudaError_t launch_qkv_prepare(const void* qkv, void* q, void* k, void* v, int in_dtype,
                               int qk_dtype, int64_t batch, int64_t seq_len, int64_t heads,
                               const float* scale_mul, float eps, const float* rope_cos,
                               const float* rope_sin, int64_t rope_row_stride, void* slab_k,
                               void* slab_v, int64_t slab_rows, const int64_t* slab_offset,
                               int sms, unsigned int* status, cudaStream_t st);

}  // namespace heatkv
