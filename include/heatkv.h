/*
 * heatkv.h - C ABI of libheatkv.so, the B200 (sm_100a) kernels of the HeatKV hot path.
 *
 * The library replaces the two device operations of the reference's kernel module
 * (real_pruning_fused_attention.py):
 *   - heatkv_pack_kv            <- pack_flat_segments_kv (:365-441) and its Triton kernel
 *                                  _pack_flat_segments_kv_kernel (:33-73)
 *   - heatkv_segmented_attention <- fused_real_pruning_flat_segmented_attention (:445-591) and its
 *                                  Triton kernel _fused_real_pruning_segmented_attention_kernel
 *                                  (:76-267)
 * and, on the caller's side of the attention, the PyTorch chain that prepares q, k, v after the
 * QKV projection (enable_real_pruning_fast.py:2040-2072):
 *   - heatkv_qkv_prepare         <- unbind/permute, F.normalize * scale_mul, apply_rotary_emb
 *                                  (infinity/models/basic.py:97-117)
 *   - heatkv_qkv_prepare_append  <- the same, plus the slab append of the scale
 *                                  (enable_real_pruning_fast.py:2218-2225) for hazard-free heads
 *   - heatkv_qkv_project         <- the QKV projection (F.linear, :2040-2043) with the two above
 *                                  in its epilogue
 *
 * Conventions
 *   - Every pointer argument is a device pointer unless stated otherwise; tensors are dense,
 *     row-major (C-contiguous) and the caller owns them.
 *   - Every call is asynchronous on `stream` (a cudaStream_t passed as void*; NULL = legacy
 *     default stream) and performs no host<->device synchronisation and no allocation.
 *   - Every call returns a heatkv_status; on failure heatkv_last_error_string() holds a message
 *     for the calling thread. No C++ exception crosses this interface.
 *   - Errors that can only be seen on the device (a copy descriptor outside its tensor, a bounded
 *     wait that expired) never fault: the offending work is skipped and a sticky flag is raised,
 *     read with heatkv_device_status().
 */
#ifndef HEATKV_H_
#define HEATKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. The Python layer maps INVALID_ARGUMENT to ValueError and the others to
 * RuntimeError, matching the exception types of the reference wrappers. */
typedef enum {
  HEATKV_OK = 0,
  HEATKV_ERR_INVALID_ARGUMENT = -1, /* shape / pointer / size mismatch */
  HEATKV_ERR_UNSUPPORTED = -2,      /* dtype, head_dim or sequence length not supported */
  HEATKV_ERR_CUDA = -3,             /* CUDA runtime or driver error while launching */
} heatkv_status;

/* Element types of tensors crossing the interface. */
typedef enum {
  HEATKV_DTYPE_F32 = 0,
  HEATKV_DTYPE_F16 = 1,
  HEATKV_DTYPE_BF16 = 2,
} heatkv_dtype;

/* Bits of the sticky device status word (heatkv_device_status). */
#define HEATKV_DEVICE_PACK_OUT_OF_RANGE 0x1u  /* a pack descriptor left its tensor; item skipped */
#define HEATKV_DEVICE_WAIT_TIMEOUT 0x2u       /* a bounded pipeline wait expired; tile skipped */
#define HEATKV_DEVICE_BAD_SEGMENT 0x4u        /* a segment lay outside the slab; it was clipped */
#define HEATKV_DEVICE_GATHER_OUT_OF_RANGE 0x8u /* a shard map entry left dst; chunk skipped */
#define HEATKV_DEVICE_BAD_ITEM_MAP 0x10u      /* an item map entry outside the launch; skipped */

/* Attention kernel selection for heatkv_segmented_attention. */
typedef enum {
  HEATKV_ATTN_AUTO = 0,   /* tensor-core kernel when q/k/v are all bf16 or all f16, or q and k
                             are f32 with bf16/f16 v (tf32 QK, P in v's dtype), else exact */
  HEATKV_ATTN_EXACT = 1,  /* CUDA-core kernel: fp32 products and accumulation for every dtype */
  HEATKV_ATTN_TCGEN05 = 2, /* tcgen05/TMEM kernel; requires q/k/v all bf16 or all f16, or q and
                              k f32 with bf16/f16 v. 16-bit calls take the 64-key kernel
                              (scattering calls included); f32 q/k the column-split kernel's
                              tf32 mode */
  /* 3 is retired (a two-tile kernel of 256 query rows per CTA) and rejected */
  HEATKV_ATTN_TCGEN05_CS = 4,   /* the column-split tcgen05 kernel (128 query rows per CTA) */
  HEATKV_ATTN_TCGEN05_CS64 = 5  /* 64-key tiles, two CTAs per SM (128 query rows each); q/k/v all
                                   bf16 or all f16 */
} heatkv_attn_kernel;

/* The kernel an attention call runs (heatkv_attention_kernel_for). */
typedef enum {
  HEATKV_RUN_EXACT = 1,         /* attn_simt_kernel: CUDA cores, fp32 products */
  /* 2 is retired (the two-tile kernel) */
  HEATKV_RUN_TCGEN05_CS = 3,    /* attn_sm100_cs_kernel, 16-bit mode */
  HEATKV_RUN_TCGEN05_TF32 = 4,  /* attn_sm100_cs_kernel, tf32 mode (fp32 q/k, 16-bit v) */
  HEATKV_RUN_TCGEN05_CS64 = 5   /* attn_sm100_cs64_kernel: 64-key tiles, two CTAs per SM */
} heatkv_attn_run;

/* OR into the kernel selector: the segment metadata (starts, ends, counts) and the head order are
 * not written by the work that precedes the call in the stream (e.g. uploaded once at install),
 * so the column-split kernel may stage them while the preceding kernel is still running. */
#define HEATKV_ATTN_STATIC_META 0x100

/* OR into the kernel selector: the current scale's keys are already the last rows of the last
 * segment of every head that has a segment (e.g. a dense cache the scale was appended to before
 * its attention), so the kernel reads no separate current tiles for those heads; heads without a
 * segment still attend the current K/V. Same keys in the same order, one tile fewer wherever the
 * cached prefix and the scale together fit fewer 128-key tiles. */
#define HEATKV_ATTN_CURRENT_IN_SEGMENTS 0x200

/* Message describing the last failing call made by this thread ("" if none). */
const char* heatkv_last_error_string(void);

/* Library version string. */
const char* heatkv_version(void);

/*
 * heatkv_pack_kv - copy token runs of K and V into the flat slab.
 * Replaces pack_flat_segments_kv (real_pruning_fused_attention.py:365-441).
 *
 * For item i in [0, n_items) and batch row b in [0, batch):
 *     dst_k[b, dst_starts[i] + t, :] = src_k[b, src_starts[i] + t, :]   for t < lengths[i]
 * and the same for V. src_* are [batch, src_rows, head_dim] (the flat [B, H*S, D] view of a
 * [B, H, S, D] tensor), dst_* are [batch, dst_rows, head_dim]. K and V may have different dtypes
 * (k_dtype for src_k/dst_k, v_dtype for src_v/dst_v); bytes are copied unchanged.
 * dst_starts / src_starts / lengths are int64 device arrays of n_items entries.
 * max_length must be >= every lengths[i] (rows beyond max_length are not copied).
 * Items with a negative start or length, or reaching past src_rows / dst_rows, are skipped and
 * raise HEATKV_DEVICE_PACK_OUT_OF_RANGE.
 */
int heatkv_pack_kv(void* dst_k, void* dst_v, const void* src_k, const void* src_v,
                   int k_dtype, int v_dtype, int64_t batch, int64_t src_rows, int64_t dst_rows,
                   int64_t head_dim, const int64_t* dst_starts, const int64_t* src_starts,
                   const int64_t* lengths, int64_t n_items, int64_t max_length, void* stream);

/*
 * heatkv_pack_kv_batched - several heatkv_pack_kv copies (jobs) in one launch.
 * No counterpart in the reference, which packs once per layer call; a caller that holds the K/V
 * of every layer of a scale (a pre-planned step, a graph) issues all of that scale's appends at
 * once instead of one launch per layer.
 *
 * jobs      : device array of n_jobs heatkv_pack_job; job j copies like heatkv_pack_kv with its
 *             own tensors and row counts (all jobs share k_dtype, v_dtype, batch and head_dim).
 * item_job  : int32 device array [n_items], the job of each item.
 * dst_starts / src_starts / lengths : int64 device arrays [n_items], as in heatkv_pack_kv, relative
 *             to the item's job. max_length >= every lengths[i].
 * max_vector_bytes : 16, 8, 4, 2 or 1 - the widest access every job's four base pointers allow
 *             (all aligned to it); row sizes narrow it further.
 * Items of different jobs must not write the same rows. Out-of-range items or job indices are
 * skipped and raise HEATKV_DEVICE_PACK_OUT_OF_RANGE.
 */
typedef struct {
  void* dst_k;
  void* dst_v;
  const void* src_k;
  const void* src_v;
  int64_t src_rows; /* rows of src_* per batch row */
  int64_t dst_rows; /* rows of dst_* per batch row */
} heatkv_pack_job;

int heatkv_pack_kv_batched(const heatkv_pack_job* jobs, int64_t n_jobs, const int32_t* item_job,
                           const int64_t* dst_starts, const int64_t* src_starts,
                           const int64_t* lengths, int64_t n_items, int k_dtype, int v_dtype,
                           int64_t batch, int64_t head_dim, int64_t max_length,
                           int max_vector_bytes, void* stream);

/*
 * heatkv_segmented_attention - block-causal attention of the current scale's queries over the
 * head's slab segments plus the current scale's K/V.
 * Replaces fused_real_pruning_flat_segmented_attention (real_pruning_fused_attention.py:445-591).
 *
 *   q, cur_k, cur_v : [batch, heads, q_len, head_dim], dtypes q_dtype / k_dtype / v_dtype
 *   slab_k, slab_v  : [batch, capacity, head_dim], dtypes k_dtype / v_dtype; may be NULL when
 *                     capacity == 0 (the reference's persisted_k=None)
 *   seg_starts, seg_ends : int32 [heads, max_segments]; seg_counts : int32 [heads]
 *                     head h attends slab rows [seg_starts[h,i], seg_ends[h,i]) for
 *                     i < seg_counts[h]; entries with start >= end are skipped; ranges are
 *                     clipped to [0, capacity) (HEATKV_DEVICE_BAD_SEGMENT when clipping occurs)
 *   out             : [batch, q_len, heads * head_dim] in q_dtype
 *   softmax_scale   : multiplies q.k before the softmax; use_exp2 selects the reference's
 *                     "exp2" mode, which computes the same softmax (it only rescales the
 *                     exponent base), so it is accepted and has no numerical effect here.
 * head_dim must be 128 and q_len > 0. max_segments <= 256.
 */
int heatkv_segmented_attention(const void* q, const void* slab_k, const void* slab_v,
                               const int32_t* seg_starts, const int32_t* seg_ends,
                               const int32_t* seg_counts, const void* cur_k, const void* cur_v,
                               void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch,
                               int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
                               int64_t max_segments, float softmax_scale, int use_exp2,
                               int kernel, void* stream);

/*
 * heatkv_segmented_attention_ws - heatkv_segmented_attention with the length-aware scheduler's
 * options. Same computation and arguments, plus:
 *   head_order      : int32 [heads] device array, a permutation of the heads, longest key range
 *                     first (NULL = natural order). Work is issued in this order over a persistent
 *                     grid of at most one CTA per SM, which balances uneven slab lengths.
 *   kv_splits       : split every 256-row query block's key tiles into this many ranges processed
 *                     by different CTAs and merged by the last one (0 = choose from the shapes,
 *                     1 = no split). Applies to the tcgen05 kernel.
 *   workspace       : device scratch of workspace_bytes >= heatkv_attention_workspace_bytes(...)
 *                     for kv_splits > 1, 256-byte aligned, zero-filled once before its first use
 *                     (every call leaves it zeroed again). Concurrent calls need separate
 *                     workspaces. NULL runs unsplit. A call whose CTAs gave up on a bounded
 *                     wait (heatkv_device_status reports HEATKV_DEVICE_WAIT_TIMEOUT) can leave
 *                     split counters non-zero: zero the workspace again before reusing it.
 * Extends fused_real_pruning_flat_segmented_attention (real_pruning_fused_attention.py:445-591);
 * the reference's Triton grid has no scheduler options.
 */
int heatkv_segmented_attention_ws(const void* q, const void* slab_k, const void* slab_v,
                                  const int32_t* seg_starts, const int32_t* seg_ends,
                                  const int32_t* seg_counts, const void* cur_k, const void* cur_v,
                                  void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch,
                                  int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
                                  int64_t max_segments, float softmax_scale, int use_exp2,
                                  int kernel, const int32_t* head_order, int kv_splits,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * heatkv_segmented_attention_scatter - the attention of one GPU's share of a (batch row x head)
 * sharded call, storing every output row straight into n_out full output tensors - typically every
 * rank's copy, through peer (NVLink) pointers - instead of a local block that an all-gather would
 * then have to move and reorder. No counterpart in the reference, which runs on one GPU.
 *   out_ptrs        : device array of n_out (1..64) base pointers of [out_batch, q_len,
 *                     out_heads_total * head_dim] tensors in q's dtype (local or peer memory)
 *   out_rows        : int32 [batch] device array, the full-output row of each local batch row
 *   out_heads       : int32 [heads] device array, the full-output head of each local head
 * Other arguments as heatkv_segmented_attention_ws, always on a 16-bit tcgen05 kernel unsplit (q,
 * k, v all bf16 or all f16; the 64-key kernel unless HEATKV_TCGEN05_VARIANT=cs). Each destination
 * must be 16-byte aligned. A mapped row or head outside the full output is skipped and raises
 * HEATKV_DEVICE_GATHER_OUT_OF_RANGE. The stores are complete and visible system-wide when the
 * kernel completes; readers on other GPUs must still synchronise with it (heatkv_peer_barrier).
 */
int heatkv_segmented_attention_scatter(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* const* out_ptrs, int n_out, const int32_t* out_rows, const int32_t* out_heads,
    int64_t out_batch, int64_t out_heads_total, int q_dtype, int k_dtype, int v_dtype,
    int64_t batch, int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
    int64_t max_segments, float softmax_scale, const int32_t* head_order, void* stream);

/*
 * heatkv_segmented_attention_scatter_mapped - heatkv_segmented_attention_scatter with an explicit
 * assignment of its items (128-row query blocks, schedule order) to map_grid CTAs, as
 * heatkv_segmented_attention_mapped with kv_splits = 1: the peer-to-peer exchange passes the
 * longest-first map its planner made for the same launch. No reference counterpart.
 */
int heatkv_segmented_attention_scatter_mapped(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* const* out_ptrs, int n_out, const int32_t* out_rows, const int32_t* out_heads,
    int64_t out_batch, int64_t out_heads_total, int q_dtype, int k_dtype, int v_dtype,
    int64_t batch, int64_t heads, int64_t q_len, int64_t capacity, int64_t head_dim,
    int64_t max_segments, float softmax_scale, const int32_t* head_order, const int32_t* item_map,
    int64_t map_len, int map_grid, void* stream);

/*
 * heatkv_peer_barrier - one step of a barrier across the `world` GPUs of a sharded call, run by
 * every rank on its own GPU after its scatter. flag_ptrs: device array of `world` pointers, entry i
 * being rank i's array of `world` uint32 flags (peer-accessible memory, zero before the first step);
 * counter: a uint32 in this GPU's memory (zero before the first step), advanced by one per call.
 * The kernel publishes this rank's step into every rank's array and waits until every rank's step
 * has arrived in its own; afterwards every peer's rows stored before its barrier are visible here.
 * The wait is bounded (~2 s): on expiry HEATKV_DEVICE_WAIT_TIMEOUT is raised and it returns.
 * Every rank must call it the same number of times. No counterpart in the reference.
 */
int heatkv_peer_barrier(uint32_t* const* flag_ptrs, uint32_t* counter, int world, int rank,
                        void* stream);

/*
 * Device memory shared between the processes of one node (one process per GPU), for the
 * peer-to-peer exchange of a sharded call. No counterpart in the reference.
 *   heatkv_peer_alloc         : cudaMalloc `bytes` on the current device, zero them, and write the
 *                               64-byte CUDA IPC handle of the allocation to `handle`.
 *   heatkv_peer_open          : map another process's allocation (its handle) into this process for
 *                               kernels on the current device (peer access is enabled for it).
 *   heatkv_peer_close         : unmap a pointer returned by heatkv_peer_open.
 *   heatkv_peer_free          : free a pointer returned by heatkv_peer_alloc (after every peer has
 *                               closed its mapping).
 *   heatkv_enable_peer_access : let kernels on the current device access `peer_device`'s memory.
 */
int heatkv_peer_alloc(size_t bytes, void** ptr, void* handle);
int heatkv_peer_open(const void* handle, void** ptr);
int heatkv_peer_close(void* ptr);
int heatkv_peer_free(void* ptr);
int heatkv_enable_peer_access(int peer_device);

/*
 * heatkv_segmented_attention_sched - heatkv_segmented_attention_ws with the split applied to the
 * tail of the schedule only: the first `unsplit_blocks` query blocks of the schedule order (head
 * rank major, then batch row, then 128-row query block) run whole, every later block is divided into kv_splits (>= 1) key ranges that different CTAs
 * process and the last one merges. A planner that knows the key tiles of every head chooses
 * unsplit_blocks so that the last wave of blocks over the SMs is filled with half-size work
 * instead of leaving SMs idle. The workspace needs at most
 * heatkv_attention_workspace_bytes(batch, heads, q_len, kv_splits). No reference counterpart
 * (the reference's Triton grid has no scheduler).
 */
int heatkv_segmented_attention_sched(const void* q, const void* slab_k, const void* slab_v,
                                     const int32_t* seg_starts, const int32_t* seg_ends,
                                     const int32_t* seg_counts, const void* cur_k,
                                     const void* cur_v, void* out, int q_dtype, int k_dtype,
                                     int v_dtype, int64_t batch, int64_t heads, int64_t q_len,
                                     int64_t capacity, int64_t head_dim, int64_t max_segments,
                                     float softmax_scale, int kernel, const int32_t* head_order,
                                     int kv_splits, int64_t unsplit_blocks, void* workspace,
                                     size_t workspace_bytes, void* stream);

/*
 * heatkv_segmented_attention_mapped - heatkv_segmented_attention_sched with an explicit
 * assignment of the tcgen05 kernels' items to their CTAs: the launch has map_grid CTAs and CTA
 * c runs, in order, the items item_map[c], item_map[c + map_grid], ... (-1 = empty slot); map_len
 * (a multiple of map_grid) is the number of slots. Items are numbered as the kernel numbers them:
 * the first unsplit_blocks blocks of 128 query rows (schedule order), then kv_splits items per
 * later block. Every item must appear exactly once; an entry outside the item space is skipped
 * and raises HEATKV_DEVICE_BAD_ITEM_MAP. A planner that knows every block's key tiles fills the
 * map (e.g. longest first to the least-loaded CTA) so that no CTA runs long while others idle.
 * The map is a schedule only: the output is the same with or without it, and launches that run
 * the exact kernel or another split layout (a workspace too small for the splits) ignore it. No reference counterpart.
 */
int heatkv_segmented_attention_mapped(
    const void* q, const void* slab_k, const void* slab_v, const int32_t* seg_starts,
    const int32_t* seg_ends, const int32_t* seg_counts, const void* cur_k, const void* cur_v,
    void* out, int q_dtype, int k_dtype, int v_dtype, int64_t batch, int64_t heads, int64_t q_len,
    int64_t capacity, int64_t head_dim, int64_t max_segments, float softmax_scale, int kernel,
    const int32_t* head_order, int kv_splits, int64_t unsplit_blocks, const int32_t* item_map,
    int64_t map_len, int map_grid, void* workspace, size_t workspace_bytes, void* stream);

/*
 * heatkv_attention_workspace_bytes - scratch bytes heatkv_segmented_attention_ws needs for these
 * sizes and kv_splits (0 = the automatic choice); 0 when no scratch is needed.
 */
size_t heatkv_attention_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len,
                                        int kv_splits);

/*
 * heatkv_segmented_attention_noalloc - heatkv_segmented_attention_ws for callers that cannot
 * allocate device memory: code running under a memory pool that must not grow while a serving
 * step is in flight, or a host without a CUDA allocator of its own. It takes no workspace; the
 * split-KV scratch is a fixed 32 MiB array inside the library that every GPU which loads the
 * library keeps until the process exits. No counterpart exists in the reference (its Triton
 * kernel needs no scratch).
 *   - Allocates nothing: no cudaMalloc/cudaFree and no allocating library routine. The first call
 *     made with a device current looks up that device's scratch address (cudaGetSymbolAddress);
 *     make that first call before any stream capture. The address is kept per device index for
 *     the life of the process: it is not valid across cudaDeviceReset (or any other teardown of
 *     the device's primary context), after which this entry point must not be called again.
 *   - kv_splits whose scratch would exceed 32 MiB (heatkv_attention_workspace_bytes(...) >
 *     33554432) are rejected with HEATKV_ERR_UNSUPPORTED; kv_splits = 1 needs no scratch.
 *   - Every call shares the one array and leaves its last contents there; the split counters are
 *     cleared on `stream` before each launch. Calls that overlap on the GPU (different streams
 *     without ordering) race on the array.
 * Other arguments as heatkv_segmented_attention_ws.
 */
int heatkv_segmented_attention_noalloc(const void* q, const void* slab_k, const void* slab_v,
                                       const int32_t* seg_starts, const int32_t* seg_ends,
                                       const int32_t* seg_counts, const void* cur_k,
                                       const void* cur_v, void* out, int q_dtype, int k_dtype,
                                       int v_dtype, int64_t batch, int64_t heads, int64_t q_len,
                                       int64_t capacity, int64_t head_dim, int64_t max_segments,
                                       float softmax_scale, int use_exp2, int kernel,
                                       const int32_t* head_order, int kv_splits, void* stream);

/*
 * heatkv_gather_head_shards - place head-sharded attention outputs, after their all-gather across
 * GPUs, into the single-GPU output layout. No counterpart in the reference, which runs on one GPU.
 *
 * When a layer's (batch row, head) units are split over `world` GPUs, rank r computes the output
 * of its rows_per_rank rows x heads_per_rank heads as [rows_per_rank, q_len, heads_per_rank *
 * head_dim]; an all-gather stacks these rank after rank into
 *   src : [world, rows_per_rank, q_len, heads_per_rank * head_dim]   (dtype `dtype`)
 * and this call writes
 *   dst[row_map[r * rows_per_rank + i], t, head_map[r * heads_per_rank + j] * head_dim + d]
 *       = src[r, i, t, j * head_dim + d]
 * with dst : [batch, q_len, heads * head_dim]. row_map / head_map are int32 device arrays of
 * world * rows_per_rank and world * heads_per_rank entries. A chunk whose mapped row or head lies
 * outside dst is skipped and raises HEATKV_DEVICE_GATHER_OUT_OF_RANGE.
 */
int heatkv_gather_head_shards(void* dst, const void* src, int dtype, int64_t world,
                              int64_t rows_per_rank, int64_t q_len, int64_t heads_per_rank,
                              int64_t batch, int64_t heads, int64_t head_dim,
                              const int32_t* row_map, const int32_t* head_map, void* stream);

/*
 * heatkv_attention_kernel_for - the kernel (heatkv_attn_run, > 0) that heatkv_segmented_attention
 * _ws / _sched would run with these dtypes, sizes, selector (HEATKV_ATTN_STATIC_META allowed),
 * kv_splits, workspace presence (has_workspace != 0) and unsplit_blocks; a negative
 * heatkv_status for arguments such a call rejects. It assumes 16-byte aligned tensors and shapes
 * within the tensor-core kernels' limits (heads <= 128, heads * max_segments <= 2048, fewer than
 * 2^31 rows); under HEATKV_ATTN_AUTO a call outside them runs the exact kernel instead. No device
 * is needed.
 */
int heatkv_attention_kernel_for(int q_dtype, int k_dtype, int v_dtype, int64_t batch,
                                int64_t heads, int64_t q_len, int kernel, int kv_splits,
                                int has_workspace, int64_t unsplit_blocks);

/*
 * heatkv_scas_mass - the S-CAS accumulation of tools/compute_scas.py:114-128 for one layer and one
 * scale, without materialising the attention probabilities. For the queries q [heads, q_len,
 * head_dim] of batch row 0 and every key so far k [heads, k_len, head_dim] (the cached scales,
 * then the current one; dtype: f32, bf16 or f16, read as fp32), with probs = softmax(q k^T *
 * scale) in fp32, adds
 *   mass_out[h * mass_stride + s] += mean over the queries of sum_{bounds[s] <= key < bounds[s+1]} probs
 * for every source s < n_src (<= 32). bounds: int32 device array of n_src + 1 increasing key
 * offsets; mass_out: float64 device array (the reference's accumulator row of this layer, from
 * its first source scale). head_dim must be 128; q and k 16-byte aligned for f32, 8 for 16-bit.
 * f32 inputs run on the tensor cores: kind::tf32 MMAs with each operand split into a tf32 head
 * and its fp32 remainder, three products a score (fp32-level scores; HEATKV_SCAS_KERNEL=cuda_cores
 * selects the CUDA-core kernel instead); 16-bit inputs on CUDA cores with fp32 products.
 */
int heatkv_scas_mass(const void* q, const void* k, int dtype, int64_t heads, int64_t q_len,
                     int64_t k_len, int64_t head_dim, float scale, const int32_t* bounds,
                     int n_src, double* mass_out, int64_t mass_stride, void* stream);

/*
 * heatkv_qkv_prepare - the q/k/v preparation of the patched attention forward between the QKV
 * projection and the attention call (enable_real_pruning_fast.py:2040-2072), in one pass:
 *   qkv : [batch, seq_len, 3, heads, head_dim] (in_dtype: bf16 or f16), the projection output
 *   q, k: [batch, heads, seq_len, head_dim] (qk_dtype: f32, bf16 or f16)
 *   v   : [batch, heads, seq_len, head_dim] (in_dtype), a copy
 * With scale_mul != null (cos-attention, [heads] fp32 device array of the exp'd, clamped
 * scale_mul_1H11): q = q / max(||q||, eps) * scale_mul[h], k = k / max(||k||, eps) (norm and
 * quotient in fp32, as F.normalize under autocast). With rope_cos != null: the 2-D rotary
 * embedding of infinity/models/basic.py:97-117 in fp32, pair (x[2i], x[2i+1]) of token l turned by
 * (rope_cos[l * rope_row_stride + i], rope_sin[...]): the rope cache rows of this scale
 * (rope2d_freqs_grid[...][0/1, 0, 0, 0, start:start+seq_len, :]). head_dim must be 128; qkv, v and
 * the rope rows 8-byte aligned, q and k 16-byte aligned when fp32.
 */
int heatkv_qkv_prepare(const void* qkv, void* q, void* k, void* v, int in_dtype, int qk_dtype,
                       int64_t batch, int64_t seq_len, int64_t heads, int64_t head_dim,
                       const float* scale_mul, float eps, const float* rope_cos,
                       const float* rope_sin, int64_t rope_row_stride, void* stream);

/*
 * heatkv_qkv_prepare_append - heatkv_qkv_prepare that also writes the slab append of this scale
 * (enable_real_pruning_fast.py:2218-2225 -> _segmented_flat_static_append_current :969-1024) for
 * the heads given an offset: slab_k[b, slab_offset[h] + l, :] = k[b, h, l, :] and the same for v,
 * for every b and l, with slab_offset an int64 [heads] device array (-1 = head not written here).
 *   slab_k : [batch, slab_rows, head_dim] (qk_dtype); slab_v : [batch, slab_rows, head_dim]
 *            (in_dtype) - the layer's flat slab.
 * Only heads whose segment shares no slot with the segments the same scale's attention reads may
 * be given here (the attention runs after this call); the rest stay with heatkv_pack_kv after the
 * attention. A head whose segment leaves the slab is skipped and raises
 * HEATKV_DEVICE_PACK_OUT_OF_RANGE. slab_k is aligned like q, slab_v and slab_offset 8-byte aligned.
 */
int heatkv_qkv_prepare_append(const void* qkv, void* q, void* k, void* v, int in_dtype,
                              int qk_dtype, int64_t batch, int64_t seq_len, int64_t heads,
                              int64_t head_dim, const float* scale_mul, float eps,
                              const float* rope_cos, const float* rope_sin,
                              int64_t rope_row_stride, void* slab_k, void* slab_v,
                              int64_t slab_rows, const int64_t* slab_offset, void* stream);

/*
 * heatkv_qkv_project - the QKV projection of the patched attention forward with the q/k/v
 * preparation and the cache append in its epilogue, on the tensor cores: replaces
 * F.linear(x, mat_qkv.weight, cat(q_bias, zero_k_bias, v_bias)) (enable_real_pruning_fast.py:
 * 2040-2043) followed by
 * heatkv_qkv_prepare_append (the chain of :2044-2072 and the append of :2218-2225).
 *   x       : [batch * seq_len, embed_dim] (dtype: bf16 or f16), the layer input of one scale
 *   w       : [3 * heads * 128, embed_dim] (dtype), the nn.Linear weight rows of the q, k and v
 *             heads
 *   bias    : fp32 [3 * heads * 128] (the concatenated q, zero k and v biases, in the values the
 *             reference's F.linear sees, e.g. rounded to dtype under autocast), or NULL for none;
 *             added to the fp32 accumulator before the rounding to dtype
 *   q, k, v : [batch, heads, seq_len, 128]; v in dtype, q and k in qk_dtype (dtype, or f32 as the
 *             reference's chain gives them under autocast). The projection is rounded to dtype, then
 *             prepared as heatkv_qkv_prepare does (scale_mul: cos-attention; rope: the rotary
 *             angles of the scale's tokens in pair-group-major order - the cos (sin) of pairs
 *             4g .. 4g+3 of token l at rope_cos[(g * rope_group_stride) + 4 * l + 0..3], g < 16,
 *             i.e. a [16, tokens, 4] table with rope_group_stride = 4 * its tokens, from the
 *             scale's first token; rope_group_stride >= 4 * seq_len, a multiple of 4)
 *   cache_* : as heatkv_qkv_prepare_append's slab (cache_offset -1 = head not written; cache_k
 *             rows in qk_dtype, cache_v rows in dtype); rows of the heads given an offset are
 *             written from the same registers
 * heads must be even, embed_dim a multiple of 64; x, w, bias, q, k, v, the rope rows and the
 * caches 16-byte aligned. Results equal heatkv_qkv_prepare_append applied to the rounded projection up
 * to the summation order of the projection and of the row norms.
 */
int heatkv_qkv_project(const void* x, const void* w, const float* bias, void* q, void* k, void* v,
                       int dtype, int qk_dtype,
                       int64_t batch, int64_t seq_len, int64_t heads, int64_t embed_dim,
                       const float* scale_mul, float eps, const float* rope_cos,
                       const float* rope_sin, int64_t rope_group_stride, void* cache_k,
                       void* cache_v, int64_t cache_rows, const int64_t* cache_offset,
                       void* stream);

/*
 * heatkv_slot_schedule - host-side slab placement of one layer's static schedule, replacing the
 * placement core of _segmented_flat_build_static_slot_schedule (enable_real_pruning_fast.py:
 * 260-370) and _segmented_flat_cache_capacity_for_layer (:206-234), bit for bit.
 *   removed      : uint8 [num_scales (target), num_scales (source), num_heads], 1 where the head
 *                  of that source scale is removed at that target (host memory)
 *   scale_start/_end : int64 [num_scales] token range of every scale (host)
 *   offset_out   : int64 [num_scales * num_heads] slab offset of (source, head), -1 if never live
 *   end_target_out : int32 [num_scales * num_heads] first target without it (exclusive), -1
 *   capacity_out : the high-water mark; bound_out : the capacity bound
 * No device is touched.
 */
int heatkv_slot_schedule(const uint8_t* removed, int num_scales, int num_heads,
                         const int64_t* scale_start, const int64_t* scale_end, int64_t* offset_out,
                         int32_t* end_target_out, int64_t* capacity_out, int64_t* bound_out);

/*
 * heatkv_slot_tables - the per-target segment tables and copy items of one layer's static slab
 * schedule, from a placement made by heatkv_slot_schedule; replaces the derivations of
 * _segmented_flat_build_static_slot_schedule (enable_real_pruning_fast.py:383-558). Host memory.
 *   offset, end_target : heatkv_slot_schedule's outputs ([num_scales * num_heads])
 *   meta_starts/meta_ends : int32 [num_scales (target), num_heads, num_scales] slab ranges of the
 *                  segments live at each target, per head in source-scale order; meta_counts :
 *                  int32 [num_scales, num_heads] (target 0 has none)
 *   pack_items   : int64 [n, 3] (dst slot, src row, length) of every target's activation copy from
 *                  the dense cache of the tokens before it (src = head * tokens_before + start),
 *                  sorted by dst; target t's items are rows pack_index[t] .. pack_index[t + 1]
 *                  (pack_index: int64 [num_scales + 1]); at most num_scales * num_heads per target
 *   append_items : int64 [n, 3] of the append after each scale s (src = head * n_s), rows
 *                  append_index[s] .. append_index[s + 1]; at most num_heads per scale
 */
int heatkv_slot_tables(int num_scales, int num_heads, const int64_t* scale_start,
                       const int64_t* scale_end, const int64_t* offset, const int32_t* end_target,
                       int32_t* meta_starts, int32_t* meta_ends, int32_t* meta_counts,
                       int64_t* pack_items, int64_t* pack_index, int64_t* append_items,
                       int64_t* append_index);

/*
 * heatkv_strict_budget - the main loop of strict_pruning_schedule_for_budget_scale_specific
 * (tools/utils.py:308-522): which (source scale, head, layer) atoms are removed after each target
 * and which are activated early inside it so every layer checkpoint's cache stays at or under
 * `threshold` (= budget * num_layers * num_heads * peak tokens). Host memory.
 *   orders        : int32 [num_sources, num_layers * num_heads, 2] (head, layer) removal order of
 *                   source scales source_start .. source_start + num_sources - 1 (validated)
 *   tokens        : int64 [num_scales] tokens per scale; budgeted = scales under the budget
 *                   (num_scales - 1 when the last scale is not cached)
 *   prune_count   : int64 [num_scales] pruned_heads_for_budget's counts
 *   final_mask    : uint8 [num_scales (target), num_scales (source), num_layers, num_heads], 1 for
 *                   atoms removed after the target
 *   early         : int32 [early_capacity, 5] (target, checkpoint layer, source, head, layer) of
 *                   every early activation in activation order; early_count receives their number
 *   error_info    : int64 [3]: on HEATKV_ERR_INVALID_ARGUMENT from an infeasible budget,
 *                   (1, target, layer) - over budget at that layer checkpoint, (2, target, 0) -
 *                   over budget at the end of the target, or (3, target, 0) - the end-of-scale
 *                   removals were not all activated; (0, 0, 0) otherwise
 */
int heatkv_strict_budget(const int32_t* orders, int num_sources, int num_layers, int num_heads,
                         int num_scales, const int64_t* tokens, int source_start,
                         int protected_prefix_scales, int budgeted, double threshold,
                         const int64_t* prune_count, uint8_t* final_mask, int32_t* early,
                         int64_t early_capacity, int64_t* early_count, int64_t* error_info);

/*
 * heatkv_device_status - read (and with clear != 0, reset) the sticky HEATKV_DEVICE_* flags of
 * the current CUDA device. This call synchronises `stream`. Not part of the reference interface:
 * the reference's Triton kernels do not check descriptors on the device.
 */
int heatkv_device_status(uint32_t* flags, int clear, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HEATKV_H_ */
