// Slab compaction: copy (src_start, dst_start, length) token runs of K and V into the flat slab.
//
// Same copy as the reference's _pack_flat_segments_kv_kernel (real_pruning_fused_attention.py:33-73):
//   dst[b, dst_start + t, :] = src[b, src_start + t, :]   for every item, t < length, K and V.
// The reference launches a (batch, item, 32-token chunk) grid of masked scalar element copies.
// Here the copy is pure bytes: each block moves chunks of rows of one item for one batch row,
// K then V, with 16-byte vector loads/stores when the rows allow it (256-byte bf16 rows, 512-byte
// fp32 rows), all loads of a thread issued before its stores. The kernel is HBM-bound: every byte
// is read once and written once. Descriptors are bounds-checked on the device; an item reaching
// outside its tensor is skipped and flagged instead of corrupting memory.
#include <algorithm>

#include "attn.h"
#include "common.cuh"

namespace heatkv {

constexpr int kPackThreads = 256;
constexpr int kPackRowsPerBlock = 32;   // rows of K (and of V) per block
constexpr int kPackUnroll = 4;          // vectors in flight per thread

template <typename V>
__device__ __forceinline__ void copy_rows(char* __restrict__ dst, const char* __restrict__ src,
                                          int64_t nbytes) {
  // nbytes and both pointers are multiples of sizeof(V)
  const int64_t nvec = nbytes / static_cast<int64_t>(sizeof(V));
  const V* s = reinterpret_cast<const V*>(src);
  V* d = reinterpret_cast<V*>(dst);
  for (int64_t base = threadIdx.x; base < nvec; base += int64_t(kPackThreads) * kPackUnroll) {
    V regs[kPackUnroll];
#pragma unroll
    for (int u = 0; u < kPackUnroll; ++u) {
      const int64_t i = base + int64_t(u) * kPackThreads;
      if (i < nvec) regs[u] = __ldg(s + i);
    }
#pragma unroll
    for (int u = 0; u < kPackUnroll; ++u) {
      const int64_t i = base + int64_t(u) * kPackThreads;
      if (i < nvec) d[i] = regs[u];
    }
  }
}

struct PackArgs {
  char* dst_k;
  char* dst_v;
  const char* src_k;
  const char* src_v;
  int64_t row_bytes_k;
  int64_t row_bytes_v;
  int64_t src_rows;
  int64_t dst_rows;
  const int64_t* dst_starts;
  const int64_t* src_starts;
  const int64_t* lengths;
  unsigned int* status;
};

// grid = (chunk slots, items, batch rows): block x copies row chunks x, x + gridDim.x, ... of its
// item, so the launcher sizes gridDim.x to the work (many items: one block per item and batch
// row, none idle on short items; few items: the chunks of long ones spread over many blocks)
template <typename VK, typename VV>
__global__ void __launch_bounds__(kPackThreads) pack_kv_kernel(PackArgs a) {
  pdl_trigger();
  pdl_wait();
  const int64_t item = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t len = a.lengths[item];
  if (int64_t(blockIdx.x) * kPackRowsPerBlock >= len) return;
  const int64_t d0 = a.dst_starts[item];
  const int64_t s0 = a.src_starts[item];
  if (len < 0 || d0 < 0 || s0 < 0 || d0 + len > a.dst_rows || s0 + len > a.src_rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) raise_status(a.status, HEATKV_DEVICE_PACK_OUT_OF_RANGE);
    return;
  }
  for (int64_t row0 = int64_t(blockIdx.x) * kPackRowsPerBlock; row0 < len;
       row0 += int64_t(gridDim.x) * kPackRowsPerBlock) {
    const int64_t rows = min(int64_t(kPackRowsPerBlock), len - row0);
    {
      const int64_t rb = a.row_bytes_k;
      copy_rows<VK>(a.dst_k + ((b * a.dst_rows) + d0 + row0) * rb,
                    a.src_k + ((b * a.src_rows) + s0 + row0) * rb, rows * rb);
    }
    {
      const int64_t rb = a.row_bytes_v;
      copy_rows<VV>(a.dst_v + ((b * a.dst_rows) + d0 + row0) * rb,
                    a.src_v + ((b * a.src_rows) + s0 + row0) * rb, rows * rb);
    }
  }
}

// Several packs in one launch: item i belongs to job item_job[i], whose tensors and row counts
// come from jobs[]. Used to issue the appends of every layer of one scale together.
template <typename VK, typename VV>
__global__ void __launch_bounds__(kPackThreads) pack_kv_batched_kernel(
    const heatkv_pack_job* __restrict__ jobs, const int32_t* __restrict__ item_job,
    const int64_t* __restrict__ dst_starts, const int64_t* __restrict__ src_starts,
    const int64_t* __restrict__ lengths, int64_t n_jobs, int64_t row_bytes_k,
    int64_t row_bytes_v, unsigned int* status) {
  pdl_trigger();
  pdl_wait();
  const int64_t item = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t len = lengths[item];
  if (int64_t(blockIdx.x) * kPackRowsPerBlock >= len) return;
  const int64_t jid = item_job[item];
  if (jid < 0 || jid >= n_jobs) {
    if (blockIdx.x == 0 && threadIdx.x == 0) raise_status(status, HEATKV_DEVICE_PACK_OUT_OF_RANGE);
    return;
  }
  const heatkv_pack_job& jb = jobs[jid];
  const int64_t d0 = dst_starts[item];
  const int64_t s0 = src_starts[item];
  if (len < 0 || d0 < 0 || s0 < 0 || d0 + len > jb.dst_rows || s0 + len > jb.src_rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) raise_status(status, HEATKV_DEVICE_PACK_OUT_OF_RANGE);
    return;
  }
  for (int64_t row0 = int64_t(blockIdx.x) * kPackRowsPerBlock; row0 < len;
       row0 += int64_t(gridDim.x) * kPackRowsPerBlock) {
    const int64_t rows = min(int64_t(kPackRowsPerBlock), len - row0);
    copy_rows<VK>(static_cast<char*>(jb.dst_k) + ((b * jb.dst_rows) + d0 + row0) * row_bytes_k,
                  static_cast<const char*>(jb.src_k) + ((b * jb.src_rows) + s0 + row0) * row_bytes_k,
                  rows * row_bytes_k);
    copy_rows<VV>(static_cast<char*>(jb.dst_v) + ((b * jb.dst_rows) + d0 + row0) * row_bytes_v,
                  static_cast<const char*>(jb.src_v) + ((b * jb.src_rows) + s0 + row0) * row_bytes_v,
                  rows * row_bytes_v);
  }
}

// Blocks per (item, batch row): enough that the launch has ~32 blocks per SM when the items are
// few, one when there are many (each block then loops over its item's chunks).
static unsigned chunk_slots(int64_t max_length, int64_t n_items, int64_t batch) {
  const int64_t chunks = (max_length + kPackRowsPerBlock - 1) / kPackRowsPerBlock;
  const int64_t want = int64_t(148) * 32;
  const int64_t per = (want + n_items * batch - 1) / (n_items * batch);
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(chunks, per)));
}

static int vec_width(const void* p0, const void* p1, int64_t row_bytes) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1) |
                         static_cast<uintptr_t>(row_bytes);
  if ((bits & 15u) == 0) return 16;
  if ((bits & 7u) == 0) return 8;
  if ((bits & 3u) == 0) return 4;
  if ((bits & 1u) == 0) return 2;
  return 1;
}

template <typename VK>
static cudaError_t launch_v(int wv, dim3 grid, cudaStream_t st, const PackArgs& a) {
  switch (wv) {
    case 16: return launch_pdl(pack_kv_kernel<VK, uint4>, grid, dim3(kPackThreads), 0, st, a);
    case 8: return launch_pdl(pack_kv_kernel<VK, uint2>, grid, dim3(kPackThreads), 0, st, a);
    case 4: return launch_pdl(pack_kv_kernel<VK, uint32_t>, grid, dim3(kPackThreads), 0, st, a);
    case 2: return launch_pdl(pack_kv_kernel<VK, uint16_t>, grid, dim3(kPackThreads), 0, st, a);
    default: return launch_pdl(pack_kv_kernel<VK, uint8_t>, grid, dim3(kPackThreads), 0, st, a);
  }
}

cudaError_t launch_pack_kv(void* dst_k, void* dst_v, const void* src_k, const void* src_v,
                           int64_t row_bytes_k, int64_t row_bytes_v, int64_t batch,
                           int64_t src_rows, int64_t dst_rows, const int64_t* dst_starts,
                           const int64_t* src_starts, const int64_t* lengths, int64_t n_items,
                           int64_t max_length, unsigned int* status, cudaStream_t stream) {
  PackArgs a{static_cast<char*>(dst_k), static_cast<char*>(dst_v),
             static_cast<const char*>(src_k), static_cast<const char*>(src_v),
             row_bytes_k, row_bytes_v, src_rows, dst_rows, dst_starts, src_starts, lengths, status};
  dim3 grid(chunk_slots(max_length, n_items, batch), static_cast<unsigned>(n_items),
            static_cast<unsigned>(batch));
  const int wk = vec_width(dst_k, src_k, row_bytes_k);
  const int wv = vec_width(dst_v, src_v, row_bytes_v);
  switch (wk) {
    case 16: return launch_v<uint4>(wv, grid, stream, a);
    case 8: return launch_v<uint2>(wv, grid, stream, a);
    case 4: return launch_v<uint32_t>(wv, grid, stream, a);
    case 2: return launch_v<uint16_t>(wv, grid, stream, a);
    default: return launch_v<uint8_t>(wv, grid, stream, a);
  }
}

static int width_of(int64_t row_bytes, int max_width) {
  int w = max_width;
  while (w > 1 && (row_bytes % w) != 0) w /= 2;
  return w;
}

template <typename VK>
static void launch_batched_v(int wv, dim3 grid, cudaStream_t st, const heatkv_pack_job* jobs,
                             const int32_t* item_job, const int64_t* dst_starts,
                             const int64_t* src_starts, const int64_t* lengths, int64_t n_jobs,
                             int64_t rbk, int64_t rbv, unsigned int* status) {
#define HEATKV_PACK_B(VV) \
  (void)launch_pdl(pack_kv_batched_kernel<VK, VV>, grid, dim3(kPackThreads), 0, st, jobs, \
                   item_job, dst_starts, src_starts, lengths, n_jobs, rbk, rbv, status)
  switch (wv) {
    case 16: HEATKV_PACK_B(uint4); break;
    case 8: HEATKV_PACK_B(uint2); break;
    case 4: HEATKV_PACK_B(uint32_t); break;
    case 2: HEATKV_PACK_B(uint16_t); break;
    default: HEATKV_PACK_B(uint8_t); break;
  }
#undef HEATKV_PACK_B
}

cudaError_t launch_pack_kv_batched(const heatkv_pack_job* jobs, int64_t n_jobs,
                                   const int32_t* item_job, const int64_t* dst_starts,
                                   const int64_t* src_starts, const int64_t* lengths,
                                   int64_t n_items, int64_t row_bytes_k, int64_t row_bytes_v,
                                   int64_t batch, int64_t max_length, int max_vector_bytes,
                                   unsigned int* status, cudaStream_t stream) {
  dim3 grid(chunk_slots(max_length, n_items, batch), static_cast<unsigned>(n_items),
            static_cast<unsigned>(batch));
  const int wk = width_of(row_bytes_k, max_vector_bytes);
  const int wv = width_of(row_bytes_v, max_vector_bytes);
  switch (wk) {
    case 16: launch_batched_v<uint4>(wv, grid, stream, jobs, item_job, dst_starts, src_starts, lengths, n_jobs, row_bytes_k, row_bytes_v, status); break;
    case 8: launch_batched_v<uint2>(wv, grid, stream, jobs, item_job, dst_starts, src_starts, lengths, n_jobs, row_bytes_k, row_bytes_v, status); break;
    case 4: launch_batched_v<uint32_t>(wv, grid, stream, jobs, item_job, dst_starts, src_starts, lengths, n_jobs, row_bytes_k, row_bytes_v, status); break;
    case 2: launch_batched_v<uint16_t>(wv, grid, stream, jobs, item_job, dst_starts, src_starts, lengths, n_jobs, row_bytes_k, row_bytes_v, status); break;
    default: launch_batched_v<uint8_t>(wv, grid, stream, jobs, item_job, dst_starts, src_starts, lengths, n_jobs, row_bytes_k, row_bytes_v, status); break;
  }
  return cudaGetLastError();
}

}  // namespace heatkv
