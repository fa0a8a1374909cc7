// Reassembly of head-sharded attention outputs after the all-gather across GPUs.
//
// When the (batch row, head) units of a layer are split over GPUs, rank r computes the attention
// output of its rows x heads as a dense [rows_per_rank, Lq, heads_per_rank * D] block. An NCCL
// all-gather concatenates these blocks rank after rank into src [world, rows_per_rank, Lq,
// heads_per_rank * D]; this kernel scatters every (rank, row, token, head) chunk of D elements to
// its place in the model's layout dst [B, Lq, H * D] (heads innermost, as the single-GPU kernel
// writes it). It is a byte copy bound by HBM bandwidth: 16-byte vectors, one vector per thread
// per step, chunks of one token row of a rank read contiguously. The maps are bounds-checked;
// a chunk whose row or head lies outside dst is skipped and flagged.
#include "common.cuh"

namespace heatkv {

constexpr int kGatherThreads = 256;

struct GatherArgs {
  char* dst;
  const char* src;
  const int32_t* row_map;   // [world * rows_per_rank] -> global batch row
  const int32_t* head_map;  // [world * heads_per_rank] -> global head
  int64_t world, rows_per_rank, q_len, heads_per_rank, batch, heads;
  int64_t chunk_bytes;      // head_dim * element size
  unsigned int* status;
};

// IT: index type; 32-bit arithmetic whenever the vector count fits, since this loop is a handful
// of integer divisions per 16-byte move.
template <typename V, typename IT>
__global__ void __launch_bounds__(kGatherThreads) shard_gather_kernel(GatherArgs a) {
  const IT vpc = static_cast<IT>(a.chunk_bytes / static_cast<int64_t>(sizeof(V)));  // per chunk
  const IT hpr = static_cast<IT>(a.heads_per_rank);
  const IT q_len = static_cast<IT>(a.q_len);
  const IT rpr = static_cast<IT>(a.rows_per_rank);
  const IT total = static_cast<IT>(a.world * a.rows_per_rank * a.q_len * a.heads_per_rank) * vpc;
  const V* src = reinterpret_cast<const V*>(a.src);
  V* dst = reinterpret_cast<V*>(a.dst);
  for (IT g = IT(blockIdx.x) * kGatherThreads + threadIdx.x; g < total;
       g += IT(gridDim.x) * kGatherThreads) {
    const IT c = g / vpc;
    const IT v = g - c * vpc;
    // c enumerates (rank, local row, token, local head) in src order
    const IT rt = c / hpr;               // (rank, local row, token)
    const IT j = c - rt * hpr;
    const IT ri = rt / q_len;            // (rank, local row)
    const IT t = rt - ri * q_len;
    const IT r = ri / rpr;
    const int64_t row = a.row_map[ri];
    const int64_t head = a.head_map[r * hpr + j];
    if (row < 0 || row >= a.batch || head < 0 || head >= a.heads) {
      if (v == 0) raise_status(a.status, HEATKV_DEVICE_GATHER_OUT_OF_RANGE);
      continue;
    }
    const int64_t d = ((row * a.q_len + int64_t(t)) * a.heads + head) * int64_t(vpc) + int64_t(v);
    dst[d] = src[g];
  }
}

template <typename V>
static void launch_v(unsigned grid, bool narrow, const GatherArgs& a, cudaStream_t stream) {
  if (narrow)
    shard_gather_kernel<V, uint32_t><<<grid, kGatherThreads, 0, stream>>>(a);
  else
    shard_gather_kernel<V, int64_t><<<grid, kGatherThreads, 0, stream>>>(a);
}

cudaError_t launch_shard_gather(void* dst, const void* src, const int32_t* row_map,
                                const int32_t* head_map, int64_t world, int64_t rows_per_rank,
                                int64_t q_len, int64_t heads_per_rank, int64_t batch,
                                int64_t heads, int64_t chunk_bytes, int sms,
                                unsigned int* status, cudaStream_t stream) {
  GatherArgs a{static_cast<char*>(dst), static_cast<const char*>(src), row_map, head_map,
               world, rows_per_rank, q_len, heads_per_rank, batch, heads, chunk_bytes, status};
  const uintptr_t bits = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                         static_cast<uintptr_t>(chunk_bytes);
  const int64_t chunks = world * rows_per_rank * q_len * heads_per_rank;
  auto grid_for = [&](int64_t vec) {
    const int64_t threads = chunks * (chunk_bytes / vec);
    const int64_t blocks = (threads + kGatherThreads - 1) / kGatherThreads;
    const int64_t cap = int64_t(sms > 0 ? sms : 148) * 8;   // 8 resident CTAs of 256 per SM
    return static_cast<unsigned>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
  };
  const int64_t vec = (bits & 15u) == 0 ? 16 : (bits & 7u) == 0 ? 8 : (bits & 3u) == 0 ? 4 : 2;
  // the loop index also reaches total + grid * threads before it stops
  const bool narrow = chunks * (chunk_bytes / vec) + int64_t(grid_for(vec)) * kGatherThreads <
                      (int64_t(1) << 32);
  switch (vec) {
    case 16: launch_v<uint4>(grid_for(16), narrow, a, stream); break;
    case 8: launch_v<uint2>(grid_for(8), narrow, a, stream); break;
    case 4: launch_v<uint32_t>(grid_for(4), narrow, a, stream); break;
    default: launch_v<uint16_t>(grid_for(2), narrow, a, stream); break;
  }
  return cudaGetLastError();
}

}  // namespace heatkv
