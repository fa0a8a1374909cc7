// C entry points of libheatkv.so (declared in include/heatkv.h): argument validation, kernel
// selection, error strings and the sticky device status word.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "attn.h"
#include "common.cuh"

#include <atomic>
#include <mutex>

namespace heatkv {
__device__ unsigned int g_device_status = 0;

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("HEATKV_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// HEATKV_TCGEN05_VARIANT: "cs" (column-split kernel) or "cs64" (64-key kernel) for 16-bit calls
// that name neither (scattering calls included); unset: the 64-key kernel.
static int tcgen05_variant() {
  static const int v = [] {
    const char* e = getenv("HEATKV_TCGEN05_VARIANT");
    if (e && strcmp(e, "cs") == 0) return 2;
    if (e && strcmp(e, "cs64") == 0) return 3;
    return 0;
  }();
  return v;
}

unsigned int* device_status_ptr() {
  static std::atomic<unsigned int*> cache[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  unsigned int* p = cache[dev].load();
  if (p) return p;
  std::lock_guard<std::mutex> lock(mu);
  p = cache[dev].load();
  if (!p) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_device_status) != cudaSuccess) return nullptr;
    p = static_cast<unsigned int*>(addr);
    cache[dev].store(p);
  }
  return p;
}
}  // namespace heatkv

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(HEATKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool valid_dtype(int d) {
  return d == HEATKV_DTYPE_F32 || d == HEATKV_DTYPE_F16 || d == HEATKV_DTYPE_BF16;
}

int64_t dtype_size(int d) { return d == HEATKV_DTYPE_F32 ? 4 : 2; }

}  // namespace

extern "C" {

const char* heatkv_last_error_string(void) { return g_last_error.c_str(); }

const char* heatkv_version(void) { return "heatkv-b200 0.1 (sm_100a)"; }

int heatkv_pack_kv(void* dst_k, void* dst_v, const void* src_k, const void* src_v, int k_dtype,
                   int v_dtype, int64_t batch, int64_t src_rows, int64_t dst_rows,
                   int64_t head_dim, const int64_t* dst_starts, const int64_t* src_starts,
                   const int64_t* lengths, int64_t n_items, int64_t max_length, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(k_dtype) || !valid_dtype(v_dtype))
    return fail(HEATKV_ERR_UNSUPPORTED, "pack_flat_segments_kv: unsupported dtype code");
  if (batch < 0 || src_rows < 0 || dst_rows < 0 || head_dim <= 0 || n_items < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "pack_flat_segments_kv: negative size");
  if (n_items == 0 || batch == 0 || max_length <= 0) return HEATKV_OK;
  if (!dst_k || !dst_v || !src_k || !src_v || !dst_starts || !src_starts || !lengths)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "pack_flat_segments_kv: null pointer");
  if (n_items > 65535 || batch > 65535)
    return fail(HEATKV_ERR_UNSUPPORTED,
                "pack_flat_segments_kv supports at most 65535 items and 65535 batch rows per call");
  if ((max_length + 31) / 32 > 0x7fffffffLL)
    return fail(HEATKV_ERR_UNSUPPORTED, "pack_flat_segments_kv: max_length too large");
  cudaError_t e = heatkv::launch_pack_kv(
      dst_k, dst_v, src_k, src_v, head_dim * dtype_size(k_dtype), head_dim * dtype_size(v_dtype),
      batch, src_rows, dst_rows, dst_starts, src_starts, lengths, n_items, max_length,
      heatkv::device_status_ptr(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pack_flat_segments_kv launch");
  return HEATKV_OK;
}

int heatkv_pack_kv_batched(const heatkv_pack_job* jobs, int64_t n_jobs, const int32_t* item_job,
                           const int64_t* dst_starts, const int64_t* src_starts,
                           const int64_t* lengths, int64_t n_items, int k_dtype, int v_dtype,
                           int64_t batch, int64_t head_dim, int64_t max_length,
                           int max_vector_bytes, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(k_dtype) || !valid_dtype(v_dtype))
    return fail(HEATKV_ERR_UNSUPPORTED, "heatkv_pack_kv_batched: unsupported dtype code");
  if (n_jobs < 0 || n_items < 0 || batch < 0 || head_dim <= 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_pack_kv_batched: negative size");
  if (max_vector_bytes != 16 && max_vector_bytes != 8 && max_vector_bytes != 4 &&
      max_vector_bytes != 2 && max_vector_bytes != 1)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_pack_kv_batched: max_vector_bytes must be 16, 8, 4, 2 or 1");
  if (n_items == 0 || batch == 0 || n_jobs == 0 || max_length <= 0) return HEATKV_OK;
  if (!jobs || !item_job || !dst_starts || !src_starts || !lengths)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_pack_kv_batched: null pointer");
  if (n_items > 65535 || batch > 65535)
    return fail(HEATKV_ERR_UNSUPPORTED,
                "heatkv_pack_kv_batched supports at most 65535 items and 65535 batch rows per call");
  if ((max_length + 31) / 32 > 0x7fffffffLL)
    return fail(HEATKV_ERR_UNSUPPORTED, "heatkv_pack_kv_batched: max_length too large");
  cudaError_t e = heatkv::launch_pack_kv_batched(
      jobs, n_jobs, item_job, dst_starts, src_starts, lengths, n_items,
      head_dim * dtype_size(k_dtype), head_dim * dtype_size(v_dtype), batch, max_length,
      max_vector_bytes, heatkv::device_status_ptr(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_pack_kv_batched launch");
  return HEATKV_OK;
}

struct Scatter {
  void* const* out_ptrs;
  const int32_t* out_rows;
  const int32_t* out_heads;
  int n_out;
  int64_t out_batch, out_heads_total;
};

struct AttnPlan {
  int run;      // heatkv_attn_run
  bool strict;  // a tensor-core kernel was asked for: no fallback to the exact kernel
};

// The kernel an attention call runs, from its dtypes, sizes and selector (the launch itself may
// still find its shape outside a tensor-core kernel's limits; see attention_impl).
static int plan_attention(int q_dtype, int k_dtype, int v_dtype, int64_t batch, int64_t heads,
                          int64_t q_len, int kernel, int kv_splits, bool has_workspace,
                          int64_t unsplit_blocks, bool scatter, AttnPlan* out) {
  kernel &= ~(HEATKV_ATTN_STATIC_META | HEATKV_ATTN_CURRENT_IN_SEGMENTS);
  // 3 (the retired two-tile kernel) is no longer a selector
  if (kernel < HEATKV_ATTN_AUTO || kernel > HEATKV_ATTN_TCGEN05_CS64 || kernel == 3)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "real_scale_fused_segmented: unknown kernel selector");
  // the column-split or 64-key variant asked for by name; otherwise HEATKV_TCGEN05_VARIANT
  const int variant = kernel == HEATKV_ATTN_TCGEN05_CS     ? 2
                    : kernel == HEATKV_ATTN_TCGEN05_CS64   ? 3
                                                           : heatkv::tcgen05_variant();
  const bool named_cs64 = kernel == HEATKV_ATTN_TCGEN05_CS64;
  if (kernel == HEATKV_ATTN_TCGEN05_CS || kernel == HEATKV_ATTN_TCGEN05_CS64)
    kernel = HEATKV_ATTN_TCGEN05;
  const bool same16 = (q_dtype == k_dtype && k_dtype == v_dtype && q_dtype != HEATKV_DTYPE_F32);
  // fp32 q and k with 16-bit v (the real model's dtypes): tf32 QK, P rounded to v's dtype
  const bool qk32 = (q_dtype == HEATKV_DTYPE_F32 && k_dtype == HEATKV_DTYPE_F32 &&
                     v_dtype != HEATKV_DTYPE_F32);
  if (named_cs64 && !same16)
    return fail(HEATKV_ERR_UNSUPPORTED,
                "the 64-key tcgen05 kernel needs q, k and v all bfloat16 or all float16");
  if (kernel == HEATKV_ATTN_TCGEN05 && !same16 && !(qk32 && !scatter))
    return fail(HEATKV_ERR_UNSUPPORTED,
                "tcgen05 segmented attention needs q, k and v all bfloat16 or all float16, or q "
                "and k float32 with 16-bit v");
  out->strict = kernel == HEATKV_ATTN_TCGEN05;
  if (kernel != HEATKV_ATTN_EXACT && qk32 && !scatter) {
    out->run = HEATKV_RUN_TCGEN05_TF32;
  } else if (kernel != HEATKV_ATTN_EXACT && same16) {
    // Default: the 64-key kernel (two CTAs per SM), faster at every launch size measured, with
    // or without key-range splits (unsplit_blocks counts 128-row blocks for both kernels) and
    // for scattering calls (unsplit) too.
    (void)kv_splits;
    (void)has_workspace;
    (void)unsplit_blocks;
    (void)batch;
    (void)heads;
    (void)q_len;
    out->run = variant != 2 ? HEATKV_RUN_TCGEN05_CS64 : HEATKV_RUN_TCGEN05_CS;
  } else {
    if (scatter)
      return fail(HEATKV_ERR_UNSUPPORTED,
                  "heatkv_segmented_attention_scatter needs q, k and v all bfloat16 or all float16");
    out->run = HEATKV_RUN_EXACT;
  }
  return HEATKV_OK;
}

static int attention_impl(const void* q, const void* slab_k, const void* slab_v,
                          const int32_t* seg_starts, const int32_t* seg_ends,
                          const int32_t* seg_counts, const void* cur_k, const void* cur_v, void* out,
                          int q_dtype, int k_dtype, int v_dtype, int64_t batch, int64_t heads,
                          int64_t q_len, int64_t capacity, int64_t head_dim, int64_t max_segments,
                          float softmax_scale, int kernel, const int32_t* head_order,
                          int kv_splits, void* workspace, size_t workspace_bytes, void* stream,
                          const Scatter* scatter = nullptr, int64_t unsplit_blocks = 0,
                          const int32_t* item_map = nullptr, int64_t map_len = 0,
                          int map_grid = 0) {
  g_last_error.clear();
  if (!valid_dtype(q_dtype) || !valid_dtype(k_dtype) || !valid_dtype(v_dtype))
    return fail(HEATKV_ERR_UNSUPPORTED,
                "real_scale_fused_segmented supports only float16, bfloat16, or float32 tensors");
  if (head_dim != 128)
    return fail(HEATKV_ERR_UNSUPPORTED, "real_scale_fused_segmented v1 only supports head_dim=128");
  if (q_len <= 0)
    return fail(HEATKV_ERR_UNSUPPORTED, "real_scale_fused_segmented requires current_len > 0");
  if (batch < 0 || heads <= 0 || capacity < 0 || max_segments < 0 || kv_splits < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "real_scale_fused_segmented: invalid sizes");
  if (batch == 0) return HEATKV_OK;
  if (!q || !cur_k || !cur_v || (!out && !scatter) || !seg_counts ||
      (max_segments > 0 && (!seg_starts || !seg_ends)))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "real_scale_fused_segmented: null pointer");
  if (capacity > 0 && (!slab_k || !slab_v))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "real_scale_fused_segmented: null slab with capacity > 0");
  if (max_segments > heatkv::kMaxSegments)
    return fail(HEATKV_ERR_UNSUPPORTED, "real_scale_fused_segmented supports at most %d segments per head",
                heatkv::kMaxSegments);
  if (heads > 65535 || batch > 65535 || (q_len + 63) / 64 > 0x7fffffffLL)
    return fail(HEATKV_ERR_UNSUPPORTED, "real_scale_fused_segmented: grid too large");
  const bool static_meta = (kernel & HEATKV_ATTN_STATIC_META) != 0;
  const bool current_in_segments = (kernel & HEATKV_ATTN_CURRENT_IN_SEGMENTS) != 0;
  AttnPlan plan;
  int rc = plan_attention(q_dtype, k_dtype, v_dtype, batch, heads, q_len, kernel, kv_splits,
                          workspace != nullptr, unsplit_blocks, scatter != nullptr, &plan);
  if (rc != HEATKV_OK) return rc;

  heatkv::AttnArgs a{q,     slab_k,        slab_v, seg_starts, seg_ends, seg_counts, cur_k,
                     cur_v, out,           batch,  heads,      q_len,    capacity,   max_segments,
                     softmax_scale};
  a.head_order = head_order;
  a.kv_splits = kv_splits;
  a.unsplit_blocks = unsplit_blocks;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.status = heatkv::device_status_ptr();
  a.static_meta = static_meta;
  a.current_in_segments = current_in_segments;
  a.item_map = item_map;
  a.map_len = map_len;
  a.map_grid = map_grid;
  if (scatter) {
    a.out_ptrs = scatter->out_ptrs;
    a.out_rows = scatter->out_rows;
    a.out_heads = scatter->out_heads;
    a.n_out = scatter->n_out;
    a.out_batch = scatter->out_batch;
    a.out_heads_total = scatter->out_heads_total;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (plan.run == HEATKV_RUN_TCGEN05_TF32) {
    cudaError_t e = heatkv::launch_attention_sm100_tf32(a, v_dtype == HEATKV_DTYPE_BF16, st);
    if (e == cudaSuccess) return HEATKV_OK;
    if (e != cudaErrorNotSupported || plan.strict)
      return cuda_fail(e, "tcgen05 tf32 segmented attention launch");
  } else if (plan.run == HEATKV_RUN_TCGEN05_CS || plan.run == HEATKV_RUN_TCGEN05_CS64) {
    const bool bf16 = q_dtype == HEATKV_DTYPE_BF16;
    cudaError_t e = cudaErrorNotSupported;
    if (plan.run == HEATKV_RUN_TCGEN05_CS64) {
      // outside the 64-key kernel's limits (segment table, splits asked with a map): column split
      e = heatkv::launch_attention_sm100_cs64(a, bf16, st);
      if (e == cudaErrorNotSupported) {
        a.item_map = nullptr;  // a map planned for the 64-key kernel numbers different items
        e = heatkv::launch_attention_sm100_cs(a, bf16, st);
      }
    } else {
      e = heatkv::launch_attention_sm100_cs(a, bf16, st);
    }
    if (e == cudaSuccess) return HEATKV_OK;
    if (e == cudaErrorNotSupported && scatter)
      return fail(HEATKV_ERR_UNSUPPORTED,
                  "heatkv_segmented_attention_scatter: these sizes need the split or exact path");
    if (e != cudaErrorNotSupported || plan.strict)
      return cuda_fail(e, "tcgen05 segmented attention launch");
  }
  // the exact kernel: asked for, or the fallback of an automatic choice
  cudaError_t e = heatkv::launch_attention_simt(a, q_dtype, k_dtype, v_dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "segmented attention launch");
  return HEATKV_OK;
}

int heatkv_attention_kernel_for(int q_dtype, int k_dtype, int v_dtype, int64_t batch,
                                int64_t heads, int64_t q_len, int kernel, int kv_splits,
                                int has_workspace, int64_t unsplit_blocks) {
  g_last_error.clear();
  if (!valid_dtype(q_dtype) || !valid_dtype(k_dtype) || !valid_dtype(v_dtype))
    return fail(HEATKV_ERR_UNSUPPORTED,
                "real_scale_fused_segmented supports only float16, bfloat16, or float32 tensors");
  if (batch < 0 || heads <= 0 || q_len <= 0 || kv_splits < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_attention_kernel_for: invalid sizes");
  AttnPlan plan;
  const int rc = plan_attention(q_dtype, k_dtype, v_dtype, batch, heads, q_len, kernel, kv_splits,
                                has_workspace != 0, unsplit_blocks, false, &plan);
  return rc != HEATKV_OK ? rc : plan.run;
}

int heatkv_segmented_attention(const void* q, const void* slab_k, const void* slab_v,
                               const int32_t* seg_starts, const int32_t* seg_ends,
                               const int32_t* seg_counts, const void* cur_k, const void* cur_v,
                               void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch,
                               int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
                               int64_t max_segments, float softmax_scale, int use_exp2,
                               int kernel, void* stream) {
  (void)use_exp2;  // exp and exp2 modes compute the same softmax
  return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, out,
                        q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                        max_segments, softmax_scale, kernel, nullptr, 1, nullptr, 0, stream);
}

int heatkv_segmented_attention_ws(const void* q, const void* slab_k, const void* slab_v,
                                  const int32_t* seg_starts, const int32_t* seg_ends,
                                  const int32_t* seg_counts, const void* cur_k, const void* cur_v,
                                  void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch,
                                  int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
                                  int64_t max_segments, float softmax_scale, int use_exp2,
                                  int kernel, const int32_t* head_order, int kv_splits,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  (void)use_exp2;
  if (kv_splits != 1 && workspace != nullptr) {
    const size_t need = heatkv::attention_workspace_bytes(batch, heads, q_len, kv_splits);
    if (workspace_bytes < need)
      return fail(HEATKV_ERR_INVALID_ARGUMENT,
                  "heatkv_segmented_attention_ws: workspace of %zu bytes, %zu needed",
                  workspace_bytes, need);
  }
  return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, out,
                        q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                        max_segments, softmax_scale, kernel, head_order, kv_splits, workspace,
                        workspace_bytes, stream);
}

static int scatter_impl(const char* name, const void* q, const void* slab_k, const void* slab_v,
                        const int32_t* seg_starts, const int32_t* seg_ends,
                        const int32_t* seg_counts, const void* cur_k, const void* cur_v,
                        void* const* out_ptrs, int n_out, const int32_t* out_rows,
                        const int32_t* out_heads, int64_t out_batch, int64_t out_heads_total,
                        int q_dtype, int k_dtype, int v_dtype, int64_t batch, int64_t heads,
                        int64_t q_len, int64_t capacity, int64_t head_dim, int64_t max_segments,
                        float softmax_scale, const int32_t* head_order, const int32_t* item_map,
                        int64_t map_len, int map_grid, void* stream) {
  g_last_error.clear();
  if (n_out <= 0 || n_out > 64 || !out_ptrs || !out_rows || !out_heads)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: 1..64 destinations and both maps are required",
                name);
  if (out_batch < batch || out_heads_total < heads || out_batch > 0x7fffffff ||
      out_heads_total > 0x7fffffff)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: the full output is smaller than this shard",
                name);
  const Scatter sc{out_ptrs, out_rows, out_heads, n_out, out_batch, out_heads_total};
  return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, nullptr,
                        q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                        max_segments, softmax_scale, HEATKV_ATTN_TCGEN05, head_order, 1, nullptr, 0,
                        stream, &sc, 0, item_map, map_len, map_grid);
}

int heatkv_segmented_attention_scatter(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* const* out_ptrs, int n_out, const int32_t* out_rows, const int32_t* out_heads,
    int64_t out_batch, int64_t out_heads_total, int q_dtype, int k_dtype, int v_dtype,
    int64_t batch, int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
    int64_t max_segments, float softmax_scale, const int32_t* head_order, void* stream) {
  return scatter_impl("heatkv_segmented_attention_scatter", q, slab_k, slab_v, seg_starts,
                      seg_ends, seg_counts, cur_k, cur_v, out_ptrs, n_out, out_rows, out_heads,
                      out_batch, out_heads_total, q_dtype, k_dtype, v_dtype, batch, heads, q_len,
                      capacity, head_dim, max_segments, softmax_scale, head_order, nullptr, 0, 0,
                      stream);
}

int heatkv_segmented_attention_scatter_mapped(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* const* out_ptrs, int n_out, const int32_t* out_rows, const int32_t* out_heads,
    int64_t out_batch, int64_t out_heads_total, int q_dtype, int k_dtype, int v_dtype,
    int64_t batch, int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
    int64_t max_segments, float softmax_scale, const int32_t* head_order, const int32_t* item_map,
    int64_t map_len, int map_grid, void* stream) {
  if (!item_map || map_len <= 0 || map_len >= (int64_t(1) << 31) || map_grid <= 0 ||
      map_grid > 65535 || map_len % map_grid != 0) {
    g_last_error.clear();
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "heatkv_segmented_attention_scatter_mapped: item_map of rounds x map_grid slots "
                "required");
  }
  return scatter_impl("heatkv_segmented_attention_scatter_mapped", q, slab_k, slab_v, seg_starts,
                      seg_ends, seg_counts, cur_k, cur_v, out_ptrs, n_out, out_rows, out_heads,
                      out_batch, out_heads_total, q_dtype, k_dtype, v_dtype, batch, heads, q_len,
                      capacity, head_dim, max_segments, softmax_scale, head_order, item_map,
                      map_len, map_grid, stream);
}

int heatkv_peer_barrier(uint32_t* const* flag_ptrs, uint32_t* counter, int world, int rank,
                        void* stream) {
  g_last_error.clear();
  if (world <= 0 || world > 32 || rank < 0 || rank >= world || !flag_ptrs || !counter)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_peer_barrier: invalid world, rank or pointer");
  cudaError_t e = heatkv::launch_peer_barrier(flag_ptrs, counter, world, rank,
                                              heatkv::device_status_ptr(),
                                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_peer_barrier launch");
  return HEATKV_OK;
}

int heatkv_peer_alloc(size_t bytes, void** ptr, void* handle) {
  g_last_error.clear();
  if (!ptr || !handle || bytes == 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_peer_alloc: null pointer or zero size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_peer_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "heatkv_peer_alloc: cudaIpcGetMemHandle");
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return HEATKV_OK;
}

int heatkv_peer_open(const void* handle, void** ptr) {
  g_last_error.clear();
  if (!ptr || !handle) return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_peer_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_peer_open: cudaIpcOpenMemHandle");
  return HEATKV_OK;
}

int heatkv_peer_close(void* ptr) {
  g_last_error.clear();
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_peer_close");
  return HEATKV_OK;
}

int heatkv_peer_free(void* ptr) {
  g_last_error.clear();
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_peer_free");
  return HEATKV_OK;
}

int heatkv_enable_peer_access(int peer_device) {
  g_last_error.clear();
  int dev = 0, can = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceCanAccessPeer(&can, dev, peer_device);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_enable_peer_access: query");
  if (!can)
    return fail(HEATKV_ERR_UNSUPPORTED, "device %d cannot access device %d directly", dev,
                peer_device);
  e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    e = cudaSuccess;
  }
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_enable_peer_access");
  return HEATKV_OK;
}

int heatkv_segmented_attention_sched(const void* q, const void* slab_k, const void* slab_v,
                                     const int32_t* seg_starts, const int32_t* seg_ends,
                                     const int32_t* seg_counts, const void* cur_k,
                                     const void* cur_v, void* out, int q_dtype, int k_dtype,
                                     int v_dtype, int64_t batch, int64_t heads, int64_t q_len,
                                     int64_t capacity, int64_t head_dim, int64_t max_segments,
                                     float softmax_scale, int kernel, const int32_t* head_order,
                                     int kv_splits, int64_t unsplit_blocks, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (kv_splits < 1 || unsplit_blocks < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "heatkv_segmented_attention_sched: kv_splits >= 1 and unsplit_blocks >= 0 required");
  if (kv_splits != 1 && workspace != nullptr) {
    const size_t need = heatkv::attention_workspace_bytes(batch, heads, q_len, kv_splits);
    if (workspace_bytes < need)
      return fail(HEATKV_ERR_INVALID_ARGUMENT,
                  "heatkv_segmented_attention_sched: workspace of %zu bytes, %zu needed",
                  workspace_bytes, need);
  }
  return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, out,
                        q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                        max_segments, softmax_scale, kernel, head_order, kv_splits, workspace,
                        workspace_bytes, stream, nullptr, unsplit_blocks);
}

int heatkv_segmented_attention_mapped(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch, int64_t heads, int64_t q_len,
    int64_t capacity, int64_t head_dim, int64_t max_segments, float softmax_scale, int kernel,
    const int32_t* head_order, int kv_splits, int64_t unsplit_blocks, const int32_t* item_map,
    int64_t map_len, int map_grid, void* workspace, size_t workspace_bytes, void* stream) {
  if (kv_splits < 1 || unsplit_blocks < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "heatkv_segmented_attention_mapped: kv_splits >= 1 and unsplit_blocks >= 0 required");
  if (!item_map || map_len <= 0 || map_len >= (int64_t(1) << 31) || map_grid <= 0 ||
      map_grid > 65535 || map_len % map_grid != 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "heatkv_segmented_attention_mapped: item_map of rounds x map_grid slots required");
  if (kv_splits != 1 && workspace != nullptr) {
    const size_t need = heatkv::attention_workspace_bytes(batch, heads, q_len, kv_splits);
    if (workspace_bytes < need)
      return fail(HEATKV_ERR_INVALID_ARGUMENT,
                  "heatkv_segmented_attention_mapped: workspace of %zu bytes, %zu needed",
                  workspace_bytes, need);
  }
  return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, out,
                        q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                        max_segments, softmax_scale, kernel, head_order, kv_splits, workspace,
                        workspace_bytes, stream, nullptr, unsplit_blocks, item_map, map_len,
                        map_grid);
}

size_t heatkv_attention_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len,
                                        int kv_splits) {
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_splits < 0) return 0;
  return heatkv::attention_workspace_bytes(batch, heads, q_len, kv_splits);
}

int heatkv_gather_head_shards(void* dst, const void* src, int dtype, int64_t world,
                              int64_t rows_per_rank, int64_t q_len, int64_t heads_per_rank,
                              int64_t batch, int64_t heads, int64_t head_dim,
                              const int32_t* row_map, const int32_t* head_map, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype))
    return fail(HEATKV_ERR_UNSUPPORTED, "heatkv_gather_head_shards: unsupported dtype code");
  if (world < 0 || rows_per_rank < 0 || q_len < 0 || heads_per_rank < 0 || batch < 0 ||
      heads < 0 || head_dim <= 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_gather_head_shards: negative size");
  if (world * rows_per_rank * q_len * heads_per_rank == 0) return HEATKV_OK;
  if (!dst || !src || !row_map || !head_map)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_gather_head_shards: null pointer");
  if (world * rows_per_rank * heads_per_rank > batch * heads)
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "heatkv_gather_head_shards: %lld shard units for a [%lld rows x %lld heads] output",
                static_cast<long long>(world * rows_per_rank * heads_per_rank),
                static_cast<long long>(batch), static_cast<long long>(heads));
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_gather_head_shards: device query");
  e = heatkv::launch_shard_gather(dst, src, row_map, head_map, world, rows_per_rank, q_len,
                                  heads_per_rank, batch, heads, head_dim * dtype_size(dtype), sms,
                                  heatkv::device_status_ptr(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_gather_head_shards launch");
  return HEATKV_OK;
}

int heatkv_scas_mass(const void* q, const void* k, int dtype, int64_t heads, int64_t q_len,
                     int64_t k_len, int64_t head_dim, float scale, const int32_t* bounds,
                     int n_src, double* mass_out, int64_t mass_stride, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype))
    return fail(HEATKV_ERR_UNSUPPORTED, "heatkv_scas_mass: unsupported dtype code");
  if (head_dim != 128)
    return fail(HEATKV_ERR_UNSUPPORTED, "heatkv_scas_mass only supports head_dim=128");
  if (heads <= 0 || q_len < 0 || k_len < 0 || n_src < 0 || n_src > 32 ||
      mass_stride < n_src || heads > 65535 || (q_len + 63) / 64 > 0x7fffffffLL)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_scas_mass: invalid sizes");
  if (q_len == 0 || k_len == 0 || n_src == 0) return HEATKV_OK;
  if (!q || !k || !bounds || !mass_out)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_scas_mass: null pointer");
  const uintptr_t need = dtype == HEATKV_DTYPE_F32 ? 15u : 7u;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & need)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_scas_mass: misaligned q or k");
  // fp32: the tensor-core kernel (three tf32 products a score) unless HEATKV_SCAS_KERNEL=cuda_cores
  // (read per call); 16-bit inputs, and fp32 calls outside its limits, the CUDA-core kernel
  cudaError_t e = cudaErrorNotSupported;
  const char* sel = getenv("HEATKV_SCAS_KERNEL");
  if (dtype == HEATKV_DTYPE_F32 && !(sel && strcmp(sel, "cuda_cores") == 0))
    e = heatkv::launch_scas_mass_tc(static_cast<const float*>(q), static_cast<const float*>(k),
                                    heads, q_len, k_len, scale, bounds, n_src, mass_out,
                                    mass_stride, heatkv::device_status_ptr(),
                                    static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)
    e = heatkv::launch_scas_mass(q, k, dtype, heads, q_len, k_len, scale, bounds, n_src, mass_out,
                                 mass_stride, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_scas_mass launch");
  return HEATKV_OK;
}

}  // extern "C"

namespace {

int qkv_prepare_impl(const char* name, const void* qkv, void* q, void* k, void* v, int in_dtype,
                     int qk_dtype, int64_t batch, int64_t seq_len, int64_t heads, int64_t head_dim,
                     const float* scale_mul, float eps, const float* rope_cos,
                     const float* rope_sin, int64_t rope_row_stride, void* slab_k, void* slab_v,
                     int64_t slab_rows, const int64_t* slab_offset, void* stream) {
  g_last_error.clear();
  if ((in_dtype != HEATKV_DTYPE_BF16 && in_dtype != HEATKV_DTYPE_F16) || !valid_dtype(qk_dtype))
    return fail(HEATKV_ERR_UNSUPPORTED,
                "%s: qkv must be bfloat16 or float16, q/k float32, bfloat16 or float16",
                name);
  if (head_dim != 128)
    return fail(HEATKV_ERR_UNSUPPORTED, "%s only supports head_dim=128", name);
  if (batch < 0 || seq_len < 0 || heads < 0 || slab_rows < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: negative size", name);
  if (batch * seq_len * heads == 0) return HEATKV_OK;
  if (!qkv || !q || !k || !v || (rope_cos && !rope_sin) || (!rope_cos && rope_sin))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (slab_offset && (!slab_k || !slab_v))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: slab offsets given without slab_k/slab_v",
                name);
  if (rope_cos && (rope_row_stride < head_dim / 2 || (rope_row_stride & 1)))
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "%s: rope_row_stride must be even and at least head_dim / 2", name);
  if (!(eps >= 0.f)) return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: eps must be >= 0", name);
  const uintptr_t a8 = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(v) |
                       reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin) |
                       reinterpret_cast<uintptr_t>(slab_v) |
                       reinterpret_cast<uintptr_t>(slab_offset);
  const uintptr_t aqk = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(slab_k);
  if ((a8 & 7u) || (aqk & (qk_dtype == HEATKV_DTYPE_F32 ? 15u : 7u)))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: misaligned pointer", name);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, name);
  e = heatkv::launch_qkv_prepare(qkv, q, k, v, in_dtype, qk_dtype, batch, seq_len, heads,
                                 scale_mul, eps, rope_cos, rope_sin, rope_row_stride,
                                 slab_offset ? slab_k : nullptr, slab_offset ? slab_v : nullptr,
                                 slab_rows, slab_offset, sms, heatkv::device_status_ptr(),
                                 static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  return HEATKV_OK;
}

}  // namespace

extern "C" {

int heatkv_qkv_prepare(const void* qkv, void* q, void* k, void* v, int in_dtype, int qk_dtype,
                       int64_t batch, int64_t seq_len, int64_t heads, int64_t head_dim,
                       const float* scale_mul, float eps, const float* rope_cos,
                       const float* rope_sin, int64_t rope_row_stride, void* stream) {
  return qkv_prepare_impl("heatkv_qkv_prepare", qkv, q, k, v, in_dtype, qk_dtype, batch, seq_len,
                          heads, head_dim, scale_mul, eps, rope_cos, rope_sin, rope_row_stride,
                          nullptr, nullptr, 0, nullptr, stream);
}

int heatkv_qkv_prepare_append(const void* qkv, void* q, void* k, void* v, int in_dtype,
                              int qk_dtype, int64_t batch, int64_t seq_len, int64_t heads,
                              int64_t head_dim, const float* scale_mul, float eps,
                              const float* rope_cos, const float* rope_sin,
                              int64_t rope_row_stride, void* slab_k, void* slab_v,
                              int64_t slab_rows, const int64_t* slab_offset, void* stream) {
  if (!slab_offset) {
    g_last_error.clear();
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_qkv_prepare_append: null slab_offset");
  }
  return qkv_prepare_impl("heatkv_qkv_prepare_append", qkv, q, k, v, in_dtype, qk_dtype, batch,
                          seq_len, heads, head_dim, scale_mul, eps, rope_cos, rope_sin,
                          rope_row_stride, slab_k, slab_v, slab_rows, slab_offset, stream);
}

int heatkv_qkv_project(const void* x, const void* w, const float* bias, void* q, void* k, void* v,
                       int dtype, int qk_dtype,
                       int64_t batch, int64_t seq_len, int64_t heads, int64_t embed_dim,
                       const float* scale_mul, float eps, const float* rope_cos,
                       const float* rope_sin, int64_t rope_group_stride, void* cache_k,
                       void* cache_v, int64_t cache_rows, const int64_t* cache_offset,
                       void* stream) {
  static const char* name = "heatkv_qkv_project";
  g_last_error.clear();
  if (dtype != HEATKV_DTYPE_BF16 && dtype != HEATKV_DTYPE_F16)
    return fail(HEATKV_ERR_UNSUPPORTED, "%s: x and W must be bfloat16 or float16", name);
  if (qk_dtype != dtype && qk_dtype != HEATKV_DTYPE_F32)
    return fail(HEATKV_ERR_UNSUPPORTED, "%s: q and k must be float32 or the dtype of x", name);
  if (batch < 0 || seq_len < 0 || heads < 0 || embed_dim < 0 || cache_rows < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: negative size", name);
  if (heads % 2 != 0)
    return fail(HEATKV_ERR_UNSUPPORTED, "%s: the number of heads must be even", name);
  if (embed_dim % 64 != 0 || embed_dim == 0)
    return fail(HEATKV_ERR_UNSUPPORTED, "%s: embed_dim must be a positive multiple of 64", name);
  if (batch * seq_len * heads == 0) return HEATKV_OK;
  if ((batch * seq_len + 127) / 128 * (3 * heads / 2) > INT32_MAX)
    return fail(HEATKV_ERR_UNSUPPORTED, "%s: too many tiles", name);
  if (!x || !w || !q || !k || !v || (rope_cos && !rope_sin) || (!rope_cos && rope_sin))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (cache_offset && (!cache_k || !cache_v))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: cache offsets given without caches", name);
  if (rope_cos && (rope_group_stride < 4 * seq_len || (rope_group_stride & 3)))
    return fail(HEATKV_ERR_INVALID_ARGUMENT,
                "%s: rope_group_stride must be a multiple of 4 and at least 4 * seq_len", name);
  if (!(eps >= 0.f)) return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: eps must be >= 0", name);
  const uintptr_t a16 = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                        reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(rope_cos) |
                        reinterpret_cast<uintptr_t>(rope_sin) |
                        reinterpret_cast<uintptr_t>(cache_offset ? cache_k : nullptr) |
                        reinterpret_cast<uintptr_t>(cache_offset ? cache_v : nullptr);
  if ((a16 & 15u) || (reinterpret_cast<uintptr_t>(cache_offset) & 7u))
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "%s: misaligned pointer", name);
  cudaError_t e = heatkv::launch_qkv_project(
      x, w, bias, q, k, v, dtype == HEATKV_DTYPE_BF16, qk_dtype == HEATKV_DTYPE_F32, batch, seq_len, heads, embed_dim, scale_mul, eps,
      rope_cos, rope_sin, rope_group_stride, cache_offset ? cache_k : nullptr,
      cache_offset ? cache_v : nullptr, cache_rows, cache_offset, heatkv::device_status_ptr(),
      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  return HEATKV_OK;
}

int heatkv_device_status(uint32_t* flags, int clear, void* stream) {
  g_last_error.clear();
  if (!flags) return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_device_status: null flags");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, heatkv::g_device_status, sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_device_status read");
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(heatkv::g_device_status, &zero, sizeof(zero), 0,
                                cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "heatkv_device_status clear");
  }
  *flags = v;
  return HEATKV_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Attention without any allocation (see heatkv_segmented_attention_noalloc in include/heatkv.h).
//
// Some callers cannot allocate device memory at the moment they call the attention: code running
// under an allocator that is frozen or owned by someone else (a memory pool that must not grow
// while a serving step is in flight), and library hosts with no CUDA allocator of their own. For
// them the split-KV scratch lives in this fixed array, which every GPU that loads the library
// keeps until the process exits. Its device address is looked up once per device.
// ------------------------------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;      // 32 MiB per device
constexpr size_t kStaticCounterBytes = size_t(16384) * sizeof(uint32_t);  // split counters
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device, resolved on the first call made
// with each device current (host code cannot use the symbol itself as a device pointer).
int static_scratch_ptr(void** out) {
  static std::atomic<void*> cache[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "heatkv_segmented_attention_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64)
    return fail(HEATKV_ERR_UNSUPPORTED, "heatkv_segmented_attention_noalloc: device index %d", dev);
  void* p = cache[dev].load();
  if (!p) {
    std::lock_guard<std::mutex> lock(mu);
    p = cache[dev].load();
    if (!p) {
      e = cudaGetSymbolAddress(&p, g_static_scratch);
      if (e != cudaSuccess || p == nullptr)
        return cuda_fail(e, "heatkv_segmented_attention_noalloc: cudaGetSymbolAddress");
      cache[dev].store(p);
    }
  }
  *out = p;
  return HEATKV_OK;
}

}  // namespace

extern "C" int heatkv_segmented_attention_noalloc(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch, int64_t heads, int64_t q_len,
    int64_t capacity, int64_t head_dim, int64_t max_segments, float softmax_scale, int use_exp2,
    int kernel, const int32_t* head_order, int kv_splits, void* stream) {
  (void)use_exp2;
  g_last_error.clear();
  if (kv_splits < 0)
    return fail(HEATKV_ERR_INVALID_ARGUMENT, "heatkv_segmented_attention_noalloc: kv_splits < 0");
  if (batch <= 0 || heads <= 0 || q_len <= 0)
    return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, out,
                          q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                          max_segments, softmax_scale, kernel, head_order, 1, nullptr, 0, stream);
  const size_t need = heatkv::attention_workspace_bytes(batch, heads, q_len, kv_splits);
  if (need > kStaticScratchBytes)
    return fail(HEATKV_ERR_UNSUPPORTED,
                "heatkv_segmented_attention_noalloc: these sizes need %zu bytes of scratch, more "
                "than the fixed %zu; use kv_splits=1 or heatkv_segmented_attention_ws",
                need, kStaticScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    int rc = static_scratch_ptr(&scratch);
    if (rc != HEATKV_OK) return rc;
    // the split counters must read zero when the kernel starts
    cudaError_t e = cudaMemsetAsync(scratch, 0, kStaticCounterBytes,
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "heatkv_segmented_attention_noalloc: clear counters");
  }
  return attention_impl(q, slab_k, slab_v, seg_starts, seg_ends, seg_counts, cur_k, cur_v, out,
                        q_dtype, k_dtype, v_dtype, batch, heads, q_len, capacity, head_dim,
                        max_segments, softmax_scale, kernel, head_order, need > 0 ? kv_splits : 1,
                        scratch, need > 0 ? kStaticScratchBytes : 0, stream);
}
