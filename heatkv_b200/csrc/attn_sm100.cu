// Segmented flat-slab attention on Blackwell tensor cores (sm_100a): TMA + tcgen05 + TMEM, with a
// persistent length-aware scheduler and split-KV.
//
// Computes what _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// computes with its default bf16 dot modes: for batch row b and head h, the keys are the head's
// slab segments [start, end) in segment order followed by the current scale's K/V, softmax(q k^T *
// scale) with fp32 scores and fp32 row sums, P rounded to the value dtype for the PV product, fp32
// accumulation, output [B, Lq, H*D] in q's dtype.
//
// Work decomposition. A query block is 256 rows (two 128-row Q tiles) of one (b, h). Its key
// tiles are the head's segments in 128-row steps followed by the current scale's tiles; pruned
// scales have no segment and cost nothing. An item is (head, b, query block, split): with
// kv_splits = S > 1 the block's key tiles are divided into S contiguous ranges whose partial
// results (unnormalised O, running max m, row sum l) go to the workspace; the CTA that finishes a
// block's last split (an atomic counter per block) merges the S partials into the output. Items
// are ordered longest head first (head_order, computed by the host from the segment lengths) and
// CTA c of a persistent grid of at most one CTA per SM runs items c, c + grid, c + 2*grid, ...
// which balances the uneven slab lengths across the SMs. No CTA ever waits on another.
//
// CTA roles (384 threads, 168 registers each, 1 CTA per SM, 211 KB shared memory):
//   * warp 8       : TMA producer of Q and K. Per item the two Q tiles (after the previous item's
//                    last QK), then K tiles into a 2-stage ring. Rows past a segment's end are
//                    loaded and masked; rows past the tensor end are zero-filled by TMA.
//   * warp 11      : TMA producer of V tiles, into their own 2-stage ring (a K tile never waits
//                    for a V slot, which frees later, after the second Q tile's PV).
//   * warp 9       : TMEM allocator and single-thread tcgen05.mma issuer.
//                    S_t = Q_t K^T (M=128, N=128, K=128, both operands K-major SW128 in smem),
//                    O_t += P_t V (A = P_t read from TMEM, B = V as an MN-major SW128 operand).
//                    Issue order per key tile j: PV_0(j-1), QK_0(j), PV_1(j-1), QK_1(j), so one Q
//                    tile's MMAs run while the other tile's softmax runs.
//   * warps 0-3, 4-7 : softmax warpgroups of Q tiles 0 and 1, one TMEM lane (query row) per
//                    thread. Scores come from TMEM in one 128-column load, P = exp2(s*scale*log2e
//                    - m) is written back over them as bf16/f16 pairs. The running max is only
//                    raised when a tile exceeds it by more than 8 (factor 256); O in TMEM is then
//                    rescaled in place. The epilogue writes O / l (or a partial) from TMEM.
//   * warp 10      : clears the rows past the valid keys of partial V tiles (see below).
//   TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// Every wait is bounded (common.cuh); on expiry the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains
// its in-flight copies and MMAs, frees TMEM and returns.
#include "attn.h"
#include "common.cuh"
#include "sm100_util.cuh"

#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <algorithm>
#include <mutex>

namespace heatkv {

namespace sm100 {

constexpr int kBM = 128;        // query rows per Q tile
constexpr int kNQ = 2;          // Q tiles per query block
constexpr int kBN = kKeyTile;   // keys per K/V tile
constexpr int kD = 128;         // head dim
constexpr int kStages = 2;      // K/V ring depth
constexpr int kThreads = 384;   // 12 warps = 3 warpgroups
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kVFixWarp = 10;
constexpr int kVLoadWarp = 11;
constexpr uint32_t kHalfBytes = kBM * 64 * 2;    // one 128-row x 64-column 16-bit box: 16 KiB
constexpr uint32_t kTileBytes = 2 * kHalfBytes;  // 128 x 128 x 2 bytes
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxHeads = 128;
constexpr int kMaxSegTable = 2048;               // heads x segments kept in shared memory
constexpr int kMaxSplits = kMaxKvSplits;  // key-range splits per query block

struct __align__(1024) Smem {
  uint8_t q[kNQ][kTileBytes];
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint64_t q_full, q_empty;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_ready[kStages];   // V tile landed and, if partial, its tail rows cleared
  uint64_t v_empty[kStages];
  uint64_t s_full[kNQ];
  uint64_t p_full[kNQ];
  uint64_t o_final[kNQ];
  uint64_t o_free[kNQ];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int last_flag;
  int head_order[kMaxHeads];
  int head_nseg[kMaxHeads];     // compacted segments of each head
  int head_tiles[kMaxHeads];    // key tiles of each head (segments + current scale)
  int seg_start[kMaxSegTable];  // [head * seg_stride + i]
  int seg_end[kMaxSegTable];
};

struct Params {
  int64_t batch, heads, q_len, capacity, max_segments;
  const int32_t* seg_starts;
  const int32_t* seg_ends;
  const int32_t* seg_counts;
  const int32_t* head_order;  // [heads] or null (natural order)
  void* out;
  uint32_t* ws_counter;       // [blocks] (zero between calls) when splits > 1
  float2* ws_ml;              // [blocks * splits * 256]
  float* ws_o;                // [blocks * splits * 256 * 128]
  unsigned int* status;       // device status word
  float scale_log2;           // softmax_scale * log2(e)
  int qpairs;                 // query blocks per (b, h): ceil(Lq / 256)
  int splits;                 // key-range splits of each split query block
  int unsplit;                // leading query blocks (schedule order) that are not split
  int n_items;                // unsplit + (heads * batch * qpairs - unsplit) * splits
  int seg_stride;             // segment-table row length (max_segments)
  int current_in_segments;    // the current keys end every non-empty head's segments
  // scatter epilogue (n_out > 0): every output row goes to n_out full [out_batch, Lq,
  // out_heads_total * D] tensors (e.g. every rank's copy, over NVLink) at row out_rows[b] and head
  // out_heads[h]; otherwise to `out` in the local [batch, Lq, heads * D] layout
  void* const* out_ptrs;
  const int32_t* out_rows;
  const int32_t* out_heads;
  int n_out;
  int out_batch;
  int out_heads_total;
};

struct Item {
  int h, b, qp, split, block;  // block = (rank * batch + b) * qpairs + qp
  int nsplit, sblock;          // splits of this block (1 = unsplit), index among split blocks
  int q0, nq;                  // first query row, Q tiles (1 or 2)
  int j0, n;                   // first key tile of the split, number of key tiles
};

__device__ __forceinline__ Item decode_item(const Smem& sm, const Params& p, int item) {
  Item it;
  if (item < p.unsplit) {
    it.block = item;
    it.split = 0;
    it.nsplit = 1;
  } else {
    const int k = item - p.unsplit;
    it.block = p.unsplit + k / p.splits;
    it.split = k % p.splits;
    it.nsplit = p.splits;
  }
  it.sblock = it.block - p.unsplit;
  it.qp = it.block % p.qpairs;
  const int rb = it.block / p.qpairs;
  it.b = rb % static_cast<int>(p.batch);
  const int rank = rb / static_cast<int>(p.batch);
  it.h = sm.head_order[rank];
  it.q0 = it.qp * (kNQ * kBM);
  it.nq = (static_cast<int>(p.q_len) - it.q0) > kBM ? 2 : 1;
  const int tiles = sm.head_tiles[it.h];
  it.j0 = static_cast<int>((int64_t(tiles) * it.split) / it.nsplit);
  it.n = static_cast<int>((int64_t(tiles) * (it.split + 1)) / it.nsplit) - it.j0;
  return it;
}

template <bool kBF16, int kPolyCount>
__global__ void __launch_bounds__(kThreads, 1)
    attn_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_ck,
                      const __grid_constant__ CUtensorMap tm_cv,
                      const __grid_constant__ CUtensorMap tm_sk,
                      const __grid_constant__ CUtensorMap tm_sv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int Lq = static_cast<int>(p.q_len);
  const int H = static_cast<int>(p.heads);
  const int stride = p.seg_stride;

  // ---------------------------------------------------------------- setup
  // Shared memory and TMEM are set up while the previous kernel of the stream may still run
  // (programmatic dependent launch); no global memory is touched before pdl_wait().
  pdl_trigger();
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_ready[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < kNQ; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], 4);   // one arrive per softmax warp
      mbar_init(&sm.o_final[t], 1);
      mbar_init(&sm.o_free[t], 4);
    }
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
  }
  pdl_wait();
  if (warp == kProducerWarp) {
    // stage the [H, S] metadata, then compact every head's non-empty segments in place, clipped
    // to the slab, and count its key tiles
    const int S = static_cast<int>(p.max_segments);
    for (int i = lane; i < H * S; i += 32) {
      sm.seg_start[i] = p.seg_starts[i];
      sm.seg_end[i] = p.seg_ends[i];
    }
    bool bad = false;
    for (int r = lane; r < H; r += 32) {
      int h = p.head_order ? p.head_order[r] : r;
      if (h < 0 || h >= H) {
        bad = true;
        h = r;
      }
      sm.head_order[r] = h;
      sm.head_nseg[r] = p.seg_counts[r];
    }
    __syncwarp();
    for (int h = lane; h < H; h += 32) {
      const int cnt = max(0, min(sm.head_nseg[h], S));
      int n = 0, tiles = 0;
      for (int i = 0; i < cnt; ++i) {
        int s0 = sm.seg_start[h * S + i];
        int e0 = sm.seg_end[h * S + i];
        if (s0 >= e0) continue;
        if (s0 < 0 || e0 > p.capacity) bad = true;
        s0 = max(s0, 0);
        e0 = static_cast<int>(min64(e0, p.capacity));
        if (s0 >= e0) continue;
        sm.seg_start[h * S + n] = s0;  // n <= i: compaction in place
        sm.seg_end[h * S + n] = e0;
        ++n;
        tiles += (e0 - s0 + kBN - 1) / kBN;
      }
      sm.head_nseg[h] = n;
      sm.head_tiles[h] = tiles + ((p.current_in_segments && n > 0) ? 0 : (Lq + kBN - 1) / kBN);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0 && blockIdx.x == 0)
      raise_status(p.status, HEATKV_DEVICE_BAD_SEGMENT);
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_ck);
      tma_prefetch_desc(&tm_cv);
      tma_prefetch_desc(&tm_sk);
      tma_prefetch_desc(&tm_sv);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;


  if (warp == kProducerWarp || warp == kVLoadWarp) {
    // ---------------------------------------------------------------- TMA producers
    // Warp 8 loads Q and K, warp 11 loads V, each into its own ring: a K tile is requested as
    // soon as its slot is free (QK of both Q tiles done), without queueing behind the V slot,
    // which frees only when the later PV of the second Q tile completes.
    const bool loads_k = warp == kProducerWarp;
    if (lane == 0) {
      uint32_t gx = 0, qcnt = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const Item it = decode_item(sm, p, item);
        if (it.n == 0) continue;
        const int bh = it.b * H + it.h;
        if (loads_k) {
          if (qcnt > 0 && !(ok = mbar_wait(&sm.q_empty, (qcnt - 1) & 1, abort_flag, p.status))) break;
          const int qrow = bh * Lq + it.q0;
          mbar_arrive_expect_tx(&sm.q_full, it.nq * kTileBytes);
          for (int t = 0; t < it.nq; ++t) {
            tma_load_2d(sm.q[t], &tm_q, 0, qrow + t * kBM, &sm.q_full);
            tma_load_2d(sm.q[t] + kHalfBytes, &tm_q, 64, qrow + t * kBM, &sm.q_full);
          }
          ++qcnt;
        }
        const int cur_row0 = bh * Lq;
        const int slab_row0 = static_cast<int>(int64_t(it.b) * p.capacity);
        TileCursor cur;
        cur.begin(sm, it.h, stride, it.j0);
        for (int j = 0; j < it.n; ++j, ++gx) {
          const CUtensorMap* m = loads_k ? (cur.current ? &tm_ck : &tm_sk)
                                         : (cur.current ? &tm_cv : &tm_sv);
          const int row = cur.current ? cur_row0 + cur.pos : slab_row0 + cur.pos;
          const int s = gx % kStages;
          uint64_t* full = loads_k ? &sm.k_full[s] : &sm.v_full[s];
          uint64_t* empty = loads_k ? &sm.k_empty[s] : &sm.v_empty[s];
          uint8_t* dst = loads_k ? sm.k[s] : sm.v[s];
          if (gx >= kStages && !(ok = mbar_wait(empty, ((gx / kStages) - 1) & 1, abort_flag, p.status)))
            break;
          mbar_arrive_expect_tx(full, kTileBytes);
          tma_load_2d(dst, m, 0, row, full);
          tma_load_2d(dst + kHalfBytes, m, 64, row, full);
          cur.next();
        }
      }
      if (!ok || *abort_flag) {
        // let every copy already issued land before the CTA's shared memory goes away
        if (loads_k && qcnt > 0) mbar_drain(&sm.q_full, (qcnt - 1) & 1, p.status);
        for (uint32_t g = gx > kStages ? gx - kStages : 0; g < gx; ++g)
          mbar_drain(loads_k ? &sm.k_full[g % kStages] : &sm.v_full[g % kStages],
                     (g / kStages) & 1, p.status);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kBF16, kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(kBF16, kBM, kD, false, true);
      auto issue_pv = [&](int t, uint32_t g, bool accumulate) {
        const uint32_t vbase = smem_u32(sm.v[g % kStages]);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // B = V rows [16kk, 16kk+16): 16 keys x 128 columns, MN-major; 8-key groups 1 KiB
          // apart (SBO), the two 64-column halves 16 KiB apart (LBO)
          const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, kHalfBytes, 1024);
          umma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, bdesc, idesc_pv,
                  (accumulate || kk > 0) ? 1u : 0u);
        }
      };
      auto issue_qk = [&](int t, uint32_t g) {
        const uint32_t qbase = smem_u32(sm.q[t]);
        const uint32_t kbase = smem_u32(sm.k[g % kStages]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk / 4) * kHalfBytes + (kk % 4) * 32;
          const uint64_t adesc = smem_desc_sw128(qbase + off, 16, 1024);
          const uint64_t bdesc = smem_desc_sw128(kbase + off, 16, 1024);
          umma_ss(tmem + t * 128, adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      uint32_t g = 0, qcnt = 0;
      uint32_t pcnt[kNQ] = {0, 0}, ocnt[kNQ] = {0, 0};
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const Item it = decode_item(sm, p, item);
        if (it.n == 0) continue;
        if (!(ok = mbar_wait(&sm.q_full, qcnt & 1, abort_flag, p.status))) break;
        ++qcnt;
        tc_fence_after();
        for (int j = 0; ok && j < it.n; ++j) {
          const uint32_t gj = g + j;
          for (int t = 0; t < it.nq; ++t) {
            if (j > 0) {
              if (t == 0 && !(ok = mbar_wait(&sm.v_ready[(gj - 1) % kStages], ((gj - 1) / kStages) & 1,
                                              abort_flag, p.status)))
                break;
              if (!(ok = mbar_wait(&sm.p_full[t], (pcnt[t] + j - 1) & 1, abort_flag, p.status))) break;
              if (j == 1 && ocnt[t] > 0 &&
                  !(ok = mbar_wait(&sm.o_free[t], (ocnt[t] - 1) & 1, abort_flag, p.status)))
                break;
              tc_fence_after();
              issue_pv(t, gj - 1, j > 1);
              if (t == it.nq - 1) tc_commit(&sm.v_empty[(gj - 1) % kStages]);
            }
            if (t == 0) {
              if (!(ok = mbar_wait(&sm.k_full[gj % kStages], (gj / kStages) & 1, abort_flag, p.status))) break;
              tc_fence_after();
            }
            issue_qk(t, gj);
            tc_commit(&sm.s_full[t]);
          }
          if (!ok) break;
          tc_commit(&sm.k_empty[gj % kStages]);
          if (j == it.n - 1) tc_commit(&sm.q_empty);
        }
        if (!ok) break;
        const uint32_t gl = g + it.n - 1;
        if (!(ok = mbar_wait(&sm.v_ready[gl % kStages], (gl / kStages) & 1, abort_flag, p.status))) break;
        for (int t = 0; t < it.nq; ++t) {
          if (!(ok = mbar_wait(&sm.p_full[t], (pcnt[t] + it.n - 1) & 1, abort_flag, p.status))) break;
          if (it.n == 1 && ocnt[t] > 0 &&
              !(ok = mbar_wait(&sm.o_free[t], (ocnt[t] - 1) & 1, abort_flag, p.status)))
            break;
          tc_fence_after();
          issue_pv(t, gl, it.n > 1);
          tc_commit(&sm.o_final[t]);
        }
        if (!ok) break;
        tc_commit(&sm.v_empty[gl % kStages]);
        g += it.n;
        for (int t = 0; t < it.nq; ++t) {
          pcnt[t] += it.n;
          ocnt[t] += 1;
        }
      }
      // every MMA issued by this thread has completed once `drain` fires
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else if (warp == kVFixWarp) {
    // ---------------------------------------------------------------- V tail clearing
    // A V tile is 128 slab rows; past the end of a segment (or of the current scale) they hold
    // whatever the slab holds there. P is exactly 0 for those keys, but 0 x NaN (uninitialised
    // slab slots) would still poison O, so this warp clears the tail rows of every partial tile
    // after it lands and before the MMA issuer may read it (v_ready). A 128-byte swizzled row keeps
    // all of its bytes inside its own 128-byte line, so whole lines are cleared.
    uint32_t g = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      const Item it = decode_item(sm, p, item);
      if (it.n == 0) continue;
      TileCursor cur;
      cur.begin(sm, it.h, stride, it.j0);
      for (int j = 0; j < it.n; ++j, ++g) {
        const int s = g % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.v_full[s], (g / kStages) & 1, abort_flag, p.status));
        if (!ok) break;
        const int valid = cur.valid(Lq);
        if (valid < kBN) {
          uint8_t* base = sm.v[s];
          const int chunks = (kBN - valid) * 2 * 8;  // rows x halves x 16-byte chunks
          for (int i = lane; i < chunks; i += 32) {
            const int line = i / 8;
            const int row = valid + line / 2, half = line % 2;
            *reinterpret_cast<uint4*>(base + half * kHalfBytes + row * 128 + (i % 8) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.v_ready[s]);
        cur.next();
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- softmax warpgroups
    const int t = warp / 4;
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // TMEM lane == query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + 256 + t * 128;
    const float c = p.scale_log2;
    using OutT = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
    uint32_t cnt = 0, ocnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x) {
      const Item it = decode_item(sm, p, item);
      const bool active = ok && (t < it.nq) && (it.n > 0);
      float m_run = -INFINITY;
      float l_run = 0.f;
      const bool row_live = it.q0 + t * kBM + row < Lq;
      if (active) {
        TileCursor cur;
        cur.begin(sm, it.h, stride, it.j0);
        for (int j = 0; j < it.n; ++j) {
          const int valid = cur.valid(Lq);
          ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], (cnt + j) & 1, abort_flag, p.status));
          if (!ok) break;
          tc_fence_after();
          float x[128];
          tmem_ld_row128(tS, x);
          mask_tail(x, valid);
          const float mx2 = row_max128(x) * c;
          // Lazy max: keep the running max unless this tile exceeds it by more than 8 (a factor
          // of 256 in P); raising it requires rescaling this row of O, done below once the scores
          // are dead (PV(j-1) has completed: the commit that signalled S(j) covers it).
          float alpha = 1.f;
          bool rescale = false;
          if (j == 0) {
            m_run = mx2;
          } else if (__any_sync(0xffffffffu, row_live && mx2 > m_run + 8.0f)) {
            const float m_new = fmaxf(m_run, mx2);
            alpha = ex2(m_run - m_new);
            l_run *= alpha;
            m_run = m_new;
            rescale = true;
          }
          {
            // P = exp2(s * c - m) in pairs, stored over the scores in 16-column steps
            const uint64_t c2 = f2pack(c, c);
            const uint64_t nm2 = f2pack(-m_run, -m_run);
            uint64_t acc[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[k] = f2pack(0.f, 0.f);
#pragma unroll
            for (int quarter = 0; quarter < 4; ++quarter) {
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int pi = quarter * 16 + i;  // pair index: columns 2pi, 2pi+1
                const uint64_t y = fma2(f2pack(x[2 * pi], x[2 * pi + 1]), c2, nm2);
                float p0, p1;
                if (kPolyCount == 3) {  // packed half-precision exp2 for every pair
                  float y0, y1;
                  f2unpack(y, y0, y1);
                  exp2_half_x2(y0, y1, p0, p1);
                } else if ((pi % kPolyMod) >= kPolyMod - kPolyCount) {
                  exp2_poly_x2(y, p0, p1);
                  if (valid < kBN) {
                    p0 = (2 * pi < valid) ? p0 : 0.f;
                    p1 = (2 * pi + 1 < valid) ? p1 : 0.f;
                  }
                } else {
                  float y0, y1;
                  f2unpack(y, y0, y1);
                  p0 = ex2(y0);
                  p1 = ex2(y1);
                }
                acc[pi & 3] = add2(acc[pi & 3], f2pack(p0, p1));
                pk[i] = pack2<kBF16>(p0, p1);
              }
              tmem_st16(tS + 16 * quarter, pk);
            }
            const uint64_t s01 = add2(acc[0], acc[1]);
            const uint64_t s23 = add2(acc[2], acc[3]);
            float u0, u1;
            f2unpack(add2(s01, s23), u0, u1);
            l_run += u0 + u1;
          }
          if (rescale) {  // warp-uniform
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              float o[16];
              tmem_ld16_sync(tO + cc * 16, o);
              uint32_t w[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(o[i] * alpha);
              tmem_st16(tO + cc * 16, w);
            }
          }
          // every lane's TMEM stores are complete and ordered before the warp's single arrive
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_full[t]);
          cur.next();
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.o_final[t], ocnt & 1, abort_flag, p.status));
        cnt += it.n;
      }
      const bool have_o = active && ok;
      if (have_o) tc_fence_after();
      const int qrow = it.q0 + t * kBM + row;
      if (it.nsplit == 1) {
        if (have_o) {
          const float inv = 1.f / l_run;
          int64_t off = ((int64_t(it.b) * p.q_len + qrow) * p.heads + it.h) * kD;
          int n_dst = 1;
          bool in_range = true;
          if (p.n_out > 0) {
            const int grow = __ldg(p.out_rows + it.b), ghead = __ldg(p.out_heads + it.h);
            in_range = grow >= 0 && grow < p.out_batch && ghead >= 0 && ghead < p.out_heads_total;
            if (!in_range && row == 0) raise_status(p.status, HEATKV_DEVICE_GATHER_OUT_OF_RANGE);
            off = ((int64_t(grow) * p.q_len + qrow) * p.out_heads_total + ghead) * kD;
            n_dst = p.n_out;
          }
#pragma unroll 1
          for (int cc = 0; cc < 8; ++cc) {
            float o[16];
            tmem_ld16_sync(tO + cc * 16, o);
            if (qrow < Lq && in_range) {
              uint32_t w[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) w[i] = pack2<kBF16>(o[2 * i] * inv, o[2 * i + 1] * inv);
#pragma unroll 1
              for (int r = 0; r < n_dst; ++r) {
                OutT* base = p.n_out > 0 ? static_cast<OutT*>(p.out_ptrs[r]) : static_cast<OutT*>(p.out);
                uint4* dst = reinterpret_cast<uint4*>(base + off + cc * 16);
                dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
              }
            }
          }
          // stores to other GPUs are visible system-wide before this kernel's completion is
          if (p.n_out > 0) __threadfence_system();
        }
      } else {
        // partial result of this split: (m, l) and the unnormalised O row
        const int64_t slot = (int64_t(it.sblock) * it.nsplit + it.split) * (kNQ * kBM) + t * kBM + row;
        if (have_o) {
          float4* dst = reinterpret_cast<float4*>(p.ws_o + slot * kD);
#pragma unroll 1
          for (int cc = 0; cc < 8; ++cc) {
            float o[16];
            tmem_ld16_sync(tO + cc * 16, o);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              __stcg(dst + cc * 4 + i, make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]));
          }
          __stcg(p.ws_ml + slot, make_float2(m_run, l_run));
        } else {
          __stcg(p.ws_ml + slot, make_float2(-INFINITY, 0.f));
        }
        if (have_o) {
          // O_t has been read: the MMA may start the next item's first PV into it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.o_free[t]);
          ++ocnt;
        }
        // grid-sync pattern: CTA barrier, then one thread publishes with a gpu-scope fence
        named_bar_softmax();
        if (threadIdx.x == 0) {
          __threadfence();
          const unsigned old = atomicAdd(p.ws_counter + it.sblock, 1u);
          const int last = (old == static_cast<unsigned>(it.nsplit - 1)) ? 1 : 0;
          if (last) {
            p.ws_counter[it.sblock] = 0;  // every split has arrived: reset for the next call
            __threadfence();
          }
          sm.last_flag = last;
        }
        named_bar_softmax();
        if (sm.last_flag && t < it.nq && qrow < Lq) {
          // merge the splits of this row: O = sum_k 2^(m_k - M) O_k / sum_k 2^(m_k - M) l_k
          const int64_t base = int64_t(it.sblock) * it.nsplit * (kNQ * kBM) + t * kBM + row;
          float2 ml[kMaxSplits];
          float M = -INFINITY;
#pragma unroll
          for (int k = 0; k < kMaxSplits; ++k) {
            ml[k] = k < it.nsplit ? __ldcg(p.ws_ml + base + int64_t(k) * (kNQ * kBM))
                                 : make_float2(-INFINITY, 0.f);
            if (ml[k].y > 0.f) M = fmaxf(M, ml[k].x);
          }
          float w[kMaxSplits];
          float L = 0.f;
#pragma unroll
          for (int k = 0; k < kMaxSplits; ++k) {
            w[k] = ml[k].y > 0.f ? ex2(ml[k].x - M) : 0.f;
            L = fmaf(w[k], ml[k].y, L);
          }
          const float inv = 1.f / L;
#pragma unroll
          for (int k = 0; k < kMaxSplits; ++k) w[k] *= inv;
          OutT* orow = static_cast<OutT*>(p.out) + ((int64_t(it.b) * p.q_len + qrow) * p.heads + it.h) * kD;
#pragma unroll 1
          for (int cc = 0; cc < 8; ++cc) {  // 16 columns per step, every split's loads in flight
            float4 v[kMaxSplits][4];
#pragma unroll
            for (int k = 0; k < kMaxSplits; ++k) {
              const float4* src = reinterpret_cast<const float4*>(
                                      p.ws_o + (base + int64_t(k) * (kNQ * kBM)) * kD) + cc * 4;
#pragma unroll
              for (int i = 0; i < 4; ++i)
                v[k][i] = (w[k] != 0.f) ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
              for (int k = 0; k < kMaxSplits; ++k) {
                a.x = fmaf(w[k], v[k][i].x, a.x);
                a.y = fmaf(w[k], v[k][i].y, a.y);
                a.z = fmaf(w[k], v[k][i].z, a.z);
                a.w = fmaf(w[k], v[k][i].w, a.w);
              }
              pk[2 * i] = pack2<kBF16>(a.x, a.y);
              pk[2 * i + 1] = pack2<kBF16>(a.z, a.w);
            }
            uint4* dst = reinterpret_cast<uint4*>(orow + cc * 16);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
      if (it.nsplit == 1 && have_o) {
        // O_t has been read: the MMA may start the next item's first PV into it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_free[t]);
        ++ocnt;
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
struct WsLayout {
  size_t counter_off, ml_off, o_off, total;
};

// The per-block counters live in a fixed region at the start of the workspace that nothing else
// ever writes: calls of different shapes (and both tcgen05 kernels) share one workspace, and a
// counter must find zero where an earlier call may have left partial results had the regions
// moved with the shape.
static WsLayout ws_layout(int64_t blocks, int splits, int rows_per_block) {
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

}  // namespace sm100

bool split_scratch(void* ws, size_t bytes, int64_t split_blocks, int splits, int rows_per_block,
                   SplitScratch* out) {
  const sm100::WsLayout wl = sm100::ws_layout(split_blocks, splits, rows_per_block);
  if (splits <= 1 || split_blocks > kSplitCounterBlocks || ws == nullptr || bytes < wl.total ||
      (reinterpret_cast<uintptr_t>(ws) & 255u))
    return false;
  uint8_t* base = static_cast<uint8_t*>(ws);
  out->counter = reinterpret_cast<uint32_t*>(base + wl.counter_off);
  out->ml = reinterpret_cast<float2*>(base + wl.ml_off);
  out->o = reinterpret_cast<float*>(base + wl.o_off);
  return true;
}

int attention_auto_splits(int64_t batch, int64_t heads, int64_t q_len) {
  using namespace sm100;
  const int64_t blocks = batch * heads * ((q_len + kNQ * kBM - 1) / (kNQ * kBM));
  const int64_t target = 2 * int64_t(sm_count());
  if (blocks >= target) return 1;
  return static_cast<int>(std::min<int64_t>(kMaxSplits, (target + blocks - 1) / blocks));
}

size_t attention_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int splits) {
  using namespace sm100;
  if (splits <= 0) splits = attention_auto_splits(batch, heads, q_len);
  splits = std::min(splits, kMaxKvSplits);
  // enough for either kernel: 256-row blocks (two-tile) or 128-row blocks (column split)
  const int64_t pair_blocks = batch * heads * ((q_len + kNQ * kBM - 1) / (kNQ * kBM));
  const int64_t cs_blocks = batch * heads * ((q_len + kBM - 1) / kBM);
  size_t need = 0;
  if (pair_blocks <= kSplitCounterBlocks) need = ws_layout(pair_blocks, splits, kNQ * kBM).total;
  if (cs_blocks <= kSplitCounterBlocks)
    need = std::max(need, ws_layout(cs_blocks, splits, kBM).total);
  return need;
}

cudaError_t launch_attention_sm100(const AttnArgs& a, bool bf16, cudaStream_t st) {
  using namespace sm100;
  const int64_t cur_rows = a.batch * a.heads * a.q_len;
  const int64_t slab_rows = a.batch * a.capacity;
  if (cur_rows >= (int64_t(1) << 31) || slab_rows >= (int64_t(1) << 31) ||
      a.heads > kMaxHeads || a.heads * std::max<int64_t>(a.max_segments, 1) > kMaxSegTable ||
      !(a.scale > 0.f))
    return cudaErrorNotSupported;
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.cur_k) |
                          reinterpret_cast<uintptr_t>(a.cur_v) |
                          reinterpret_cast<uintptr_t>(a.slab_k) |
                          reinterpret_cast<uintptr_t>(a.slab_v) | reinterpret_cast<uintptr_t>(a.out);
  if (align & 15u) return cudaErrorNotSupported;
  const int qpairs = static_cast<int>((a.q_len + kNQ * kBM - 1) / (kNQ * kBM));
  const int64_t blocks = a.batch * a.heads * qpairs;
  int splits = a.kv_splits <= 0 ? attention_auto_splits(a.batch, a.heads, a.q_len) : a.kv_splits;
  if (splits > kMaxSplits) splits = kMaxSplits;
  int64_t unsplit = splits > 1 ? std::min<int64_t>(std::max<int64_t>(a.unsplit_blocks, 0), blocks)
                               : blocks;
  if (unsplit == blocks) splits = 1;
  SplitScratch scratch{};
  if (splits > 1 && !split_scratch(a.workspace, a.workspace_bytes, blocks - unsplit, splits,
                                   kNQ * kBM, &scratch)) {
    splits = 1;  // no (or too small) workspace: run unsplit
    unsplit = blocks;
  }
  const int64_t n_items = unsplit + (blocks - unsplit) * splits;
  if (n_items >= (int64_t(1) << 31)) return cudaErrorNotSupported;
  CUtensorMap tq, tck, tcv, tsk, tsv;
  const void* sk = a.capacity > 0 ? a.slab_k : a.cur_k;
  const void* sv = a.capacity > 0 ? a.slab_v : a.cur_v;
  if (!encode_rows(&tq, a.q, cur_rows, bf16) || !encode_rows(&tck, a.cur_k, cur_rows, bf16) ||
      !encode_rows(&tcv, a.cur_v, cur_rows, bf16) ||
      !encode_rows(&tsk, sk, a.capacity > 0 ? slab_rows : cur_rows, bf16) ||
      !encode_rows(&tsv, sv, a.capacity > 0 ? slab_rows : cur_rows, bf16))
    return cudaErrorInvalidValue;
  Params p;
  p.batch = a.batch;
  p.heads = a.heads;
  p.q_len = a.q_len;
  p.capacity = a.capacity;
  p.max_segments = a.max_segments;
  p.seg_starts = a.seg_starts;
  p.seg_ends = a.seg_ends;
  p.seg_counts = a.seg_counts;
  p.head_order = a.head_order;
  p.out = a.out;
  p.out_ptrs = a.out_ptrs;
  p.out_rows = a.out_rows;
  p.out_heads = a.out_heads;
  p.n_out = a.n_out;
  p.out_batch = static_cast<int>(a.out_batch);
  p.out_heads_total = static_cast<int>(a.out_heads_total);
  if (a.n_out > 0 && splits != 1) return cudaErrorNotSupported;
  p.status = a.status;
  p.ws_counter = splits > 1 ? scratch.counter : nullptr;
  p.ws_ml = splits > 1 ? scratch.ml : nullptr;
  p.ws_o = splits > 1 ? scratch.o : nullptr;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.qpairs = qpairs;
  p.splits = splits;
  p.unsplit = static_cast<int>(unsplit);
  p.n_items = static_cast<int>(n_items);
  p.seg_stride = static_cast<int>(std::max<int64_t>(a.max_segments, 1));
  p.current_in_segments = a.current_in_segments ? 1 : 0;
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  // exp2 variant: HEATKV_EXP2_POLY = 0 (fp32 MUFU), 1-2 (quarters of the pairs on the FMA
  // pipe), 3 (packed half-precision MUFU for every pair); default 0
  static const int poly = [] {
    const char* e = getenv("HEATKV_EXP2_POLY");
    const int v = e ? atoi(e) : 0;
    return (v >= 0 && v <= 3) ? v : 0;
  }();
  using Kern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, Params);
  static const Kern table[2][4] = {
      {attn_sm100_kernel<false, 0>, attn_sm100_kernel<false, 1>, attn_sm100_kernel<false, 2>,
       attn_sm100_kernel<false, 3>},
      {attn_sm100_kernel<true, 0>, attn_sm100_kernel<true, 1>, attn_sm100_kernel<true, 2>,
       attn_sm100_kernel<true, 3>}};
  const Kern kern = table[bf16 ? 1 : 0][poly];
  // opt in to >48 KiB dynamic shared memory once per device (never inside a graph capture)
  static std::atomic<uint64_t> configured[2] = {{0}, {0}};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured[bf16].load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[bf16].fetch_or(bit);
  }
  const int grid = static_cast<int>(std::min<int64_t>(n_items, sm_count()));
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), static_cast<size_t>(smem), st, tq, tck, tcv,
                 tsk, tsv, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace heatkv
