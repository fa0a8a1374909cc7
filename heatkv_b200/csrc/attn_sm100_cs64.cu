// Segmented flat-slab attention on Blackwell tensor cores with 64-key tiles and two CTAs per SM.
//
// Computes what _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// computes with its default dot modes for 16-bit q, k and v (all bf16 or all f16): for batch row
// b and head h the keys are the head's slab segments [start, end) in segment order followed by
// the current scale's K/V; fp32 scores and row statistics, P rounded to the value dtype before the
// PV product (:179-180, :241-242), fp32 accumulation, output [B, Lq, H*D] in q's dtype.
//
// One 128-row query tile per CTA, as attn_sm100_cs.cu, but each CTA needs only 256 TMEM columns
// (S_0 | S_1 of 64 keys each, then O) and ~109 KiB of shared memory, so two CTAs share every SM.
// Within a CTA the chain QK(g) -> softmax(g) -> PV(g) -> QK(g + 2) serialises the tensor pipe and
// the exponentials of one S buffer; with two CTAs on the SM one CTA's exponentials run while the
// other's MMAs do, without any protocol between them. A 64-key tile also wastes less of the last
// tile of a short segment. An N = 64 QK reads A (4 KiB) and B (2 KiB) from shared memory per 32
// tensor cycles, so QK runs at ~2/3 of the tensor rate; PV (P from TMEM) does not.
//
// CTA roles (256 threads, __launch_bounds__(256, 2)):
//   * warps 0-3: softmax, one TMEM lane (query row) per thread, all 64 columns of a tile; the lazy
//                running max (moved only when a tile exceeds it by more than 8), P = exp2(s*scale*
//                log2e - m) stored as 16-bit pairs over the first 32 columns of the S buffer, the
//                row sum, O rescaled in TMEM when the max moves; epilogue O / l.
//   * warp 4   : TMA producer of Q and K tiles (Q after the previous item's last QK completed).
//   * warp 5   : TMEM allocator and QK issuer: QK(g) into S buffer g % 2 once K(g) has landed and
//                PV(g - 2), the last reader of that buffer, has completed.
//   * warp 6   : clears V rows past a partial tile's valid keys (0 x NaN from uninitialised slab
//                slots would poison O; P is 0 there), then issues PV(g) once P(g) is stored.
//   * warp 7   : TMA producer of V tiles.
// Items are (head rank, batch row, 128-row query block); CTA c runs items c, c + grid, ... or, with
// an item map, item_map[c], item_map[c + grid], ... (-1 = empty slot). Key-range splits as in
// attn_sm100_cs.cu: the blocks after the first `unsplit` are cut into `splits` ranges of their key
// tiles; a split writes (m, l) and its unnormalised O rows to the workspace, and the CTA that
// completes a block's last split (an atomic counter per block) merges them; a split without key
// tiles only publishes (-inf, 0). The scatter epilogue (its own instantiation, unsplit calls
// only) stores every output row into n_out full outputs - every rank's copy, through peer
// pointers - at the mapped row and head, as attn_sm100_cs.cu's does. Every wait is bounded; on expiry the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains its copies and
// MMAs, frees TMEM and returns.
#include "attn.h"
#include "common.cuh"
#include "sm100_util.cuh"

#include <cmath>

namespace heatkv {
namespace sm100 {
namespace cs64 {

constexpr int kBM = 128;                   // query rows per item
constexpr int kBN = 64;                    // keys per tile
constexpr int kD = kHeadDim;
constexpr uint32_t kQBox = 128 * 128;      // Q box: 128 rows x 128 bytes (64 columns), 16 KiB
constexpr uint32_t kKVBox = kBN * 128;     // K/V box: 64 rows x 128 bytes, 8 KiB
constexpr uint32_t kKVTile = 2 * kKVBox;   // 64 keys x 128 columns
constexpr uint32_t kTmemCols = 256;        // S_0 [0, 64), S_1 [64, 128), O [128, 256)
constexpr uint32_t kColO = 128;
constexpr int kMaxHeads = 128;
constexpr int kMaxSegTable = 1024;
constexpr int kMapRounds = 64;
constexpr int kThreads = 256;
constexpr int kSoftmaxWarps = 4;
constexpr int kKWarp = 4;
constexpr int kQkWarp = 5;
constexpr int kPvWarp = 6;
constexpr int kVWarp = 7;

using Cursor = TileCursorT<kBN>;

struct __align__(1024) Smem {
  uint8_t q[2 * kQBox];
  uint8_t k[2][kKVTile];
  uint8_t v[2][kKVTile];
  uint64_t q_full;      // Q of the item landed
  uint64_t q_empty;     // the item's last QK completed (Q may be overwritten)
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t s_full[2];   // QK(g) done: scores in S buffer g % 2 (and K stage g % 2 free)
  uint64_t p_full[2];   // P(g) stored by every softmax warp
  uint64_t pv_done[2];  // PV(g) done: V stage and S buffer g % 2 free
  uint64_t o_final;     // the item's last PV completed
  uint64_t o_free;      // every softmax warp has read the item's O
  uint64_t drain;       // both issuers' products have completed
  uint32_t tmem_base;
  int abort_flag;
  int last_flag;        // this CTA completed the last split of its block
  int head_order[kMaxHeads];
  int head_nseg[kMaxHeads];
  int head_tiles[kMaxHeads];
  int seg_start[kMaxSegTable];
  int seg_end[kMaxSegTable];
  int slot_items[kMapRounds];
};

struct Params {
  int64_t batch, heads, q_len, capacity, max_segments;
  const int32_t* seg_starts;
  const int32_t* seg_ends;
  const int32_t* seg_counts;
  const int32_t* head_order;
  void* out;
  unsigned int* status;
  float scale_log2;
  int qblocks;
  int n_items;          // unsplit + (blocks - unsplit) * splits
  int splits;           // key-range splits of each split block (1 = none)
  int unsplit;          // leading blocks (schedule order) that are not split
  uint32_t* ws_counter; // [split blocks], zero between calls
  float2* ws_ml;        // [split blocks * splits * 128]
  float* ws_o;          // [split blocks * splits * 128 * 128]
  const int32_t* item_map;
  int n_slots;
  int seg_stride;
  int static_meta;
  int current_in_segments;
  int out_align32;      // out is 32-byte aligned: 32-byte stores in the epilogue
  // scatter epilogue (kScatter, unsplit): every output row goes to n_out full [out_batch, Lq,
  // out_heads_total * D] tensors at row out_rows[b] and head out_heads[h]
  void* const* out_ptrs;
  const int32_t* out_rows;
  const int32_t* out_heads;
  int n_out;
  int out_batch;
  int out_heads_total;
};

struct Item {
  int h, b, q0;       // head, batch row, first query row
  int j0, n;          // first key tile of the item, key tiles
  int split, nsplit;  // split index, splits of the block (1 = unsplit)
  int sblock;         // index of the block among the split blocks
};

__device__ __forceinline__ Item decode_item(const Smem& sm, const Params& p, int item) {
  Item it;
  int block;
  if (item < p.unsplit) {
    block = item;
    it.split = 0;
    it.nsplit = 1;
  } else {
    const int k = item - p.unsplit;
    block = p.unsplit + k / p.splits;
    it.split = k % p.splits;
    it.nsplit = p.splits;
  }
  it.sblock = block - p.unsplit;
  const int qb = block % p.qblocks;
  const int rb = block / p.qblocks;
  it.b = rb % static_cast<int>(p.batch);
  it.h = sm.head_order[rb / static_cast<int>(p.batch)];
  it.q0 = qb * kBM;
  const int tiles = sm.head_tiles[it.h];
  if (it.nsplit == 1) {  // unsplit (the common case): no 64-bit divisions on the item's path
    it.j0 = 0;
    it.n = tiles;
  } else {
    it.j0 = static_cast<int>((int64_t(tiles) * it.split) / it.nsplit);
    it.n = static_cast<int>((int64_t(tiles) * (it.split + 1)) / it.nsplit) - it.j0;
  }
  return it;
}

__device__ __forceinline__ int checked_item(const Params& p, int item) {
  if (item >= p.n_items || item < -1) {
    raise_status(p.status, HEATKV_DEVICE_BAD_ITEM_MAP);
    return -1;
  }
  return item;
}

__device__ __forceinline__ int slot_item(const Smem& sm, const Params& p, int slot) {
  if (p.item_map == nullptr) return slot;
  const int k = (slot - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x);
  if (k < kMapRounds) return sm.slot_items[k];
  const int item = __ldg(p.item_map + slot);
  return (item >= p.n_items || item < -1) ? -1 : item;
}

template <bool kBF16, bool kScatter>
__global__ void __launch_bounds__(kThreads, 2)
    attn_sm100_cs64_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_ck,
                           const __grid_constant__ CUtensorMap tm_cv,
                           const __grid_constant__ CUtensorMap tm_sk,
                           const __grid_constant__ CUtensorMap tm_sv, const Params p) {
  using OutT = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int Lq = static_cast<int>(p.q_len);
  const int H = static_cast<int>(p.heads);
  const int stride = p.seg_stride;

  // ---------------------------------------------------------------- setup
  pdl_trigger();
  if (warp == kQkWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.k_full[b], 1);
      mbar_init(&sm.v_full[b], 1);
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b], kSoftmaxWarps);
      mbar_init(&sm.pv_done[b], 1);
    }
    mbar_init(&sm.o_final, 1);
    mbar_init(&sm.o_free, kSoftmaxWarps);
    mbar_init(&sm.drain, 2);
    fence_mbar_init();
  }
  if (!p.static_meta) pdl_wait();
  if (warp == kKWarp) {
    // stage the [H, S] metadata, compact every head's non-empty segments in place (clipped to
    // the slab) and count its 64-key tiles; stage this CTA's item map slots
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
        sm.seg_start[h * S + n] = s0;
        sm.seg_end[h * S + n] = e0;
        ++n;
        tiles += (e0 - s0 + kBN - 1) / kBN;
      }
      sm.head_nseg[h] = n;
      sm.head_tiles[h] = tiles + ((p.current_in_segments && n > 0) ? 0 : (Lq + kBN - 1) / kBN);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0 && blockIdx.x == 0)
      raise_status(p.status, HEATKV_DEVICE_BAD_SEGMENT);
    if (p.item_map != nullptr) {
      for (int k = lane; k < kMapRounds; k += 32) {
        const int slot = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
        sm.slot_items[k] = slot < p.n_slots ? checked_item(p, __ldg(p.item_map + slot)) : -1;
      }
      for (int slot = static_cast<int>(blockIdx.x) + (kMapRounds + lane) * static_cast<int>(gridDim.x);
           slot < p.n_slots; slot += 32 * static_cast<int>(gridDim.x))
        checked_item(p, __ldg(p.item_map + slot));
    }
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_ck);
      tma_prefetch_desc(&tm_cv);
      tma_prefetch_desc(&tm_sk);
      tma_prefetch_desc(&tm_sv);
    }
  }
  if (p.static_meta) pdl_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == kKWarp || warp == kVWarp) {
    // ---------------------------------------------------------------- TMA producers
    const bool loads_k = warp == kKWarp;
    if (lane == 0) {
      uint32_t gx = 0, qcnt = 0;
      bool ok = true;
      for (int slot = blockIdx.x; ok && slot < p.n_slots; slot += gridDim.x) {
        const int item = slot_item(sm, p, slot);
        if (item < 0) continue;
        const Item it = decode_item(sm, p, item);
        if (it.n == 0) continue;  // an empty split: no Q, no tiles
        const int bh = it.b * H + it.h;
        if (loads_k) {
          // Q rows of the item once the previous item's last QK has completed; rows past the
          // tensor are zero-filled, rows past Lq of this head are never written out
          if (qcnt > 0 && !(ok = mbar_wait(&sm.q_empty, (qcnt - 1) & 1, abort_flag, p.status))) break;
          mbar_arrive_expect_tx(&sm.q_full, 2 * kQBox);
          tma_load_2d(sm.q, &tm_q, 0, bh * Lq + it.q0, &sm.q_full);
          tma_load_2d(sm.q + kQBox, &tm_q, 64, bh * Lq + it.q0, &sm.q_full);
          ++qcnt;
        }
        const int cur_row0 = bh * Lq;
        const int slab_row0 = static_cast<int>(int64_t(it.b) * p.capacity);
        Cursor cur;
        cur.begin(sm, it.h, stride, it.j0);
        for (int j = 0; j < it.n; ++j, ++gx) {
          const int s = gx % 2;
          // the stage's previous tile (gx - 2) is done with: its QK (K) or its PV (V)
          if (gx >= 2) {
            const uint32_t pg = gx - 2;
            uint64_t* done = loads_k ? &sm.s_full[pg % 2] : &sm.pv_done[pg % 2];
            if (!(ok = mbar_wait(done, (pg / 2) & 1, abort_flag, p.status))) break;
          }
          const int row = cur.current ? cur_row0 + cur.pos : slab_row0 + cur.pos;
          const CUtensorMap* m = loads_k ? (cur.current ? &tm_ck : &tm_sk)
                                         : (cur.current ? &tm_cv : &tm_sv);
          uint64_t* full = loads_k ? &sm.k_full[s] : &sm.v_full[s];
          uint8_t* dst = loads_k ? sm.k[s] : sm.v[s];
          mbar_arrive_expect_tx(full, kKVTile);
          tma_load_2d(dst, m, 0, row, full);
          tma_load_2d(dst + kKVBox, m, 64, row, full);
          cur.next();
        }
      }
      if (!ok || *abort_flag) {
        // let every copy already issued land before the CTA's shared memory goes away
        if (loads_k && qcnt > 0) mbar_drain(&sm.q_full, (qcnt - 1) & 1, p.status);
        for (uint32_t g = gx > 2 ? gx - 2 : 0; g < gx; ++g)
          mbar_drain(loads_k ? &sm.k_full[g % 2] : &sm.v_full[g % 2], (g / 2) & 1, p.status);
      }
    }
  } else if (warp == kQkWarp) {
    // ---------------------------------------------------------------- QK issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kBF16, kBM, kBN, false, false);
      uint32_t g = 0, qcnt = 0;
      bool ok = true;
      for (int slot = blockIdx.x; ok && slot < p.n_slots; slot += gridDim.x) {
        const int item = slot_item(sm, p, slot);
        if (item < 0) continue;
        const Item it = decode_item(sm, p, item);
        if (it.n == 0) continue;
        if (!(ok = mbar_wait(&sm.q_full, qcnt & 1, abort_flag, p.status))) break;
        ++qcnt;
        for (int j = 0; j < it.n; ++j, ++g) {
          const uint32_t b = g % 2;
          if (!(ok = mbar_wait(&sm.k_full[b], (g / 2) & 1, abort_flag, p.status))) break;
          // S buffer b last held P(g - 2): its PV must have completed
          if (g >= 2 && !(ok = mbar_wait(&sm.pv_done[b], ((g / 2) - 1) & 1, abort_flag, p.status)))
            break;
          tc_fence_after();
          // S_b = Q K^T, both K-major SW128: a K step is 32 bytes into the 128-byte rows of the
          // 64-column box it falls in
          const uint32_t qbase = smem_u32(sm.q);
          const uint32_t kbase = smem_u32(sm.k[b]);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t col = (kk % 4) * 32;
            umma_ss(tmem + b * kBN, smem_desc_sw128(qbase + (kk / 4) * kQBox + col, 16, 1024),
                    smem_desc_sw128(kbase + (kk / 4) * kKVBox + col, 16, 1024), idesc_qk,
                    kk > 0 ? 1u : 0u);
          }
          tc_commit(&sm.s_full[b]);
          if (j == it.n - 1) tc_commit(&sm.q_empty);
        }
      }
      // every MMA issued by this thread has completed once `drain` fires (with the PV issuer's)
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else if (warp == kPvWarp) {
    // ---------------------------------------------------------------- V tail clearing, PV issuer
    constexpr uint32_t idesc_pv = idesc_f16(kBF16, kBM, kD, false, true);
    uint32_t g = 0, ocnt = 0;
    bool ok = true;
    for (int slot = blockIdx.x; ok && slot < p.n_slots; slot += gridDim.x) {
      const int item = slot_item(sm, p, slot);
      if (item < 0) continue;
      const Item it = decode_item(sm, p, item);
      if (it.n == 0) continue;
      Cursor cur;
      cur.begin(sm, it.h, stride, it.j0);
      for (int j = 0; j < it.n; ++j, ++g) {
        const uint32_t b = g % 2;
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.v_full[b], (g / 2) & 1, abort_flag, p.status));
        if (!ok) break;
        const int valid = cur.valid(Lq);
        if (valid < kBN) {
          // rows x halves x 16-byte chunks; a 128-byte swizzled row keeps its bytes in its line
          uint8_t* base = sm.v[b];
          const int chunks = (kBN - valid) * 2 * 8;
          for (int i = lane; i < chunks; i += 32) {
            const int line = i / 8;
            const int row = valid + line / 2, half = line % 2;
            *reinterpret_cast<uint4*>(base + half * kKVBox + row * 128 + (i % 8) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncwarp();
        if (lane == 0) {
          ok = mbar_wait(&sm.p_full[b], (g / 2) & 1, abort_flag, p.status);
          if (ok && j == 0 && ocnt > 0) ok = mbar_wait(&sm.o_free, (ocnt - 1) & 1, abort_flag, p.status);
          if (ok) {
            tc_fence_after();
            // O += P V: A = P (16-bit pairs in the first 32 columns of S_b), B = V, MN-major
            // SW128: 8-key groups 1 KiB apart (SBO), the two 64-column halves 8 KiB apart (LBO)
            const uint32_t vbase = smem_u32(sm.v[b]);
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, kKVBox, 1024);
              umma_ts(tmem + kColO, tmem + b * kBN + kk * 8, bdesc, idesc_pv,
                      (j > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&sm.pv_done[b]);
            if (j == it.n - 1) tc_commit(&sm.o_final);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        cur.next();
      }
      ++ocnt;
    }
    if (lane == 0) {
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else if (warp < kSoftmaxWarps) {
    // ---------------------------------------------------------------- softmax warps
    const int row = warp * 32 + lane;  // TMEM lane == query row
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tO = tmem + lane_off + kColO;
    const float c = p.scale_log2;
    // workspace row of this thread's query row in split `split` of the item's block
    auto split_slot = [&](const Item& it, int split) {
      return (int64_t(it.sblock) * it.nsplit + split) * kBM + row;
    };
    // After every softmax thread has published its split's partial row: count the split in, and
    // if it was the block's last, merge the partials of this thread's row into the output. All
    // four softmax warps take both barriers.
    auto split_finish = [&](const Item& it) {
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
      if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(p.ws_counter + it.sblock, 1u);
        const int last = old == static_cast<unsigned>(it.nsplit - 1) ? 1 : 0;
        if (last) {
          p.ws_counter[it.sblock] = 0;  // every split has arrived: reset for the next call
          __threadfence();
        }
        sm.last_flag = last;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
      const int qrow = it.q0 + row;
      if (!sm.last_flag || qrow >= Lq) return;
      float2 ml[kMaxKvSplits];
      float mmax = -INFINITY;
#pragma unroll
      for (int k = 0; k < kMaxKvSplits; ++k) {
        ml[k] = k < it.nsplit ? __ldcg(p.ws_ml + split_slot(it, k)) : make_float2(-INFINITY, 0.f);
        if (ml[k].y > 0.f) mmax = fmaxf(mmax, ml[k].x);
      }
      float wk[kMaxKvSplits];
      float lsum = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxKvSplits; ++k) {
        wk[k] = ml[k].y > 0.f ? ex2(ml[k].x - mmax) : 0.f;
        lsum = fmaf(wk[k], ml[k].y, lsum);
      }
      const float inv = 1.f / lsum;
#pragma unroll
      for (int k = 0; k < kMaxKvSplits; ++k) wk[k] *= inv;
      OutT* orow = static_cast<OutT*>(p.out) + ((int64_t(it.b) * Lq + qrow) * H + it.h) * kD;
#pragma unroll 1
      for (int cc = 0; cc < kD / 16; ++cc) {  // 16 columns a step, every split's loads in flight
        float4 v[kMaxKvSplits][4];
#pragma unroll
        for (int k = 0; k < kMaxKvSplits; ++k) {
          const float4* src = reinterpret_cast<const float4*>(p.ws_o + split_slot(it, k) * kD) + cc * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            v[k][i] = wk[k] != 0.f ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        uint32_t wv[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int k = 0; k < kMaxKvSplits; ++k) {
            acc.x = fmaf(wk[k], v[k][i].x, acc.x);
            acc.y = fmaf(wk[k], v[k][i].y, acc.y);
            acc.z = fmaf(wk[k], v[k][i].z, acc.z);
            acc.w = fmaf(wk[k], v[k][i].w, acc.w);
          }
          wv[2 * i] = pack2<kBF16>(acc.x, acc.y);
          wv[2 * i + 1] = pack2<kBF16>(acc.z, acc.w);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 16);
        dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
      }
    };
    uint32_t g = 0, ocnt = 0;
    bool ok = true;
    for (int slot = blockIdx.x; slot < p.n_slots; slot += gridDim.x) {
      const int item = slot_item(sm, p, slot);
      if (item < 0) continue;
      const Item it = decode_item(sm, p, item);
      if (it.n == 0) {
        // a split without key tiles: it contributes nothing to its block
        if (it.q0 + row < Lq) __stcg(p.ws_ml + split_slot(it, it.split), make_float2(-INFINITY, 0.f));
        split_finish(it);
        continue;
      }
      float m_run = -INFINITY;
      float l_run = 0.f;
      const bool row_live = it.q0 + row < Lq;
      Cursor cur;
      cur.begin(sm, it.h, stride, it.j0);
      for (int j = 0; j < it.n; ++j, ++g) {
        const uint32_t b = g % 2;
        const uint32_t tS = tmem + lane_off + b * kBN;
        const int valid = cur.valid(Lq);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[b], (g / 2) & 1, abort_flag, p.status));
        if (ok) {
          tc_fence_after();
          float x[kBN];
          tmem_ld_row64(tS, x);
          if (valid < kBN) {
#pragma unroll
            for (int i = 0; i < kBN; ++i) x[i] = i < valid ? x[i] : -INFINITY;
          }
          // key 0 of every tile is valid, so the max is finite
          const float mx = row_max<kBN>(x) * c;
          float alpha = 1.f;
          bool rescale = false;
          if (j == 0) {
            m_run = mx;
          } else if (__any_sync(0xffffffffu, row_live && mx > m_run + 8.0f)) {
            const float m_new = fmaxf(m_run, mx);
            alpha = ex2(m_run - m_new);
            l_run *= alpha;
            m_run = m_new;
            rescale = true;
          }
          const uint64_t c2 = f2pack(c, c);
          const uint64_t nm2 = f2pack(-m_run, -m_run);
          uint64_t acc[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[k] = f2pack(0.f, 0.f);
#pragma unroll
          for (int part = 0; part < kBN / 32; ++part) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int pi = part * 16 + i;  // keys 2pi, 2pi + 1
              const uint64_t y = fma2(f2pack(x[2 * pi], x[2 * pi + 1]), c2, nm2);
              float y0, y1;
              f2unpack(y, y0, y1);
              const float p0 = ex2(y0);
              const float p1 = ex2(y1);
              acc[pi & 3] = add2(acc[pi & 3], f2pack(p0, p1));
              pk[i] = pack2<kBF16>(p0, p1);
            }
            // P of keys [32 part, +32) -> 16-bit pair columns [16 part, +16) of S_b
            tmem_st16(tS + 16 * part, pk);
          }
          float u0, u1;
          f2unpack(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])), u0, u1);
          l_run += u0 + u1;
          if (rescale) {  // warp-uniform; O must hold PV(g - 1) first
            ok = __all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(g - 1) % 2], ((g - 1) / 2) & 1,
                                                   abort_flag, p.status));
            if (ok) {
              tc_fence_after();
#pragma unroll 1
              for (int cc = 0; cc < kD / 16; ++cc) {
                float o[16];
                tmem_ld16_sync(tO + cc * 16, o);
                uint32_t wv[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) wv[i] = __float_as_uint(o[i] * alpha);
                tmem_st16(tO + cc * 16, wv);
              }
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          // P is in TMEM (tcgen05.wait::st): as for o_free, a relaxed arrive, which does not wait
          // for the previous item's output stores
          if (lane == 0) mbar_arrive_relaxed(&sm.p_full[b]);
        }
        cur.next();
      }
      const bool split = !kScatter && it.nsplit > 1;  // a scattering launch runs unsplit
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.o_final, ocnt & 1, abort_flag, p.status));
      if (split && it.q0 + row < Lq)
        __stcg(p.ws_ml + split_slot(it, it.split),
               ok ? make_float2(m_run, l_run) : make_float2(-INFINITY, 0.f));
      if (ok) {
        tc_fence_after();
        const int qrow = it.q0 + row;
        const float inv = 1.f / l_run;
        OutT* orow = kScatter ? nullptr
                              : static_cast<OutT*>(p.out) + ((int64_t(it.b) * Lq + qrow) * H + it.h) * kD;
        float* prow = split ? p.ws_o + split_slot(it, it.split) * kD : nullptr;
        // scatter: the row's place in every full output (the same offset in each)
        int64_t soff = 0;
        bool in_range = true;
        if constexpr (kScatter) {
          const int grow = __ldg(p.out_rows + it.b), ghead = __ldg(p.out_heads + it.h);
          in_range = grow >= 0 && grow < p.out_batch && ghead >= 0 && ghead < p.out_heads_total;
          if (!in_range && row == 0) raise_status(p.status, HEATKV_DEVICE_GATHER_OUT_OF_RANGE);
          soff = ((int64_t(grow) * Lq + qrow) * p.out_heads_total + ghead) * kD;
        }
#pragma unroll 1
        for (int half = 0; half < 4; ++half) {
          float o[32];
          tmem_ld32_sync(tO + 32 * half, o);
          if (split) {
            // a split's partial row, unnormalised (the merge divides by the combined sum)
            if (qrow < Lq) {
              float4* d4 = reinterpret_cast<float4*>(prow + 32 * half);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                __stcg(d4 + i, make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]));
            }
          } else if (qrow < Lq) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              uint32_t wv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i)
                wv[i] = pack2<kBF16>(o[cc * 16 + 2 * i] * inv, o[cc * 16 + 2 * i + 1] * inv);
              if constexpr (kScatter) {
                if (in_range) {
#pragma unroll 1
                  for (int r = 0; r < p.n_out; ++r) {
                    OutT* dst = static_cast<OutT*>(p.out_ptrs[r]) + soff + 32 * half + 16 * cc;
                    if ((reinterpret_cast<uintptr_t>(dst) & 31u) == 0) {
                      st_global_v8(dst, wv);
                    } else {
                      uint4* d4 = reinterpret_cast<uint4*>(dst);
                      d4[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                      d4[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
                    }
                  }
                }
              } else if (p.out_align32) {
                // one full 32-byte sector per store: half the store instructions of 16-byte
                // vectors, and no partial-sector writes (each thread writes its own row)
                st_global_v8(orow + 32 * half + 16 * cc, wv);
              } else {
                uint4* dst = reinterpret_cast<uint4*>(orow + 32 * half + 16 * cc);
                dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
              }
            }
          }
        }
        // stores to other GPUs are visible system-wide before this kernel's completion is
        if constexpr (kScatter) __threadfence_system();
        tc_fence_before();
        __syncwarp();
        // O has been read into registers (tcgen05.wait::ld): the hand-off to the next item's PV
        // orders nothing else, so the arrive does not wait for the output stores to drain
        if (lane == 0) mbar_arrive_relaxed(&sm.o_free);
      }
      ++ocnt;
      if (split) split_finish(it);
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kQkWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool kBF16, bool kScatter>
static cudaError_t launch_t(const CUtensorMap& tq, const CUtensorMap& tck, const CUtensorMap& tcv,
                            const CUtensorMap& tsk, const CUtensorMap& tsv, const Params& p,
                            int grid, cudaStream_t st) {
  auto kern = attn_sm100_cs64_kernel<kBF16, kScatter>;
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  static_assert(2 * (sizeof(Smem) + 1024 + 1024) <= 228 * 1024, "two CTAs per SM");
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), static_cast<size_t>(smem), st, tq, tck, tcv,
                 tsk, tsv, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace cs64
}  // namespace sm100

int attention_cs64_auto_splits(int64_t batch, int64_t heads, int64_t q_len) {
  // enough splits of every 128-row block for two waves of the kernel's two CTAs per SM
  const int64_t blocks = batch * heads * ((q_len + sm100::cs64::kBM - 1) / sm100::cs64::kBM);
  const int64_t target = 4 * int64_t(sm100::sm_count());
  if (blocks <= 0 || blocks >= target) return 1;
  return static_cast<int>(std::min<int64_t>(kMaxKvSplits, (target + blocks - 1) / blocks));
}

cudaError_t launch_attention_sm100_cs64(const AttnArgs& a, bool bf16, cudaStream_t st) {
  using namespace sm100::cs64;
  const int64_t cur_rows = a.batch * a.heads * a.q_len;
  const int64_t slab_rows = a.batch * a.capacity;
  if (cur_rows >= (int64_t(1) << 31) || slab_rows >= (int64_t(1) << 31) ||
      a.heads > kMaxHeads || a.heads * std::max<int64_t>(a.max_segments, 1) > kMaxSegTable ||
      !(a.scale > 0.f) || a.q_len <= 0 || a.n_out < 0 || a.n_out > 64)
    return cudaErrorNotSupported;
  const bool scatter = a.n_out > 0;
  if (scatter && (!a.out_ptrs || !a.out_rows || !a.out_heads || a.out_batch > 0x7fffffff ||
                  a.out_heads_total > 0x7fffffff))
    return cudaErrorInvalidValue;
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.cur_k) |
                          reinterpret_cast<uintptr_t>(a.cur_v) |
                          reinterpret_cast<uintptr_t>(a.slab_k) |
                          reinterpret_cast<uintptr_t>(a.slab_v) | reinterpret_cast<uintptr_t>(a.out);
  if (align & 15u) return cudaErrorNotSupported;
  const int qblocks = static_cast<int>((a.q_len + kBM - 1) / kBM);
  const int64_t blocks = a.batch * a.heads * qblocks;
  // key-range splits of the blocks after the first unsplit_blocks (128-row blocks)
  int splits = a.kv_splits <= 0 ? attention_cs64_auto_splits(a.batch, a.heads, a.q_len)
                                : a.kv_splits;
  splits = std::min(splits, kMaxKvSplits);
  if (scatter) splits = 1;  // the scatter epilogue stores finished rows only
  int64_t unsplit = splits > 1 ? std::min<int64_t>(std::max<int64_t>(a.unsplit_blocks, 0), blocks)
                               : blocks;
  if (unsplit == blocks) splits = 1;
  const int requested = splits;
  SplitScratch scratch{};
  if (splits > 1 &&
      !split_scratch(a.workspace, a.workspace_bytes, blocks - unsplit, splits, kBM, &scratch)) {
    splits = 1;  // no (or too small) workspace: run unsplit
    unsplit = blocks;
  }
  const int64_t n_items = unsplit + (blocks - unsplit) * splits;
  if (n_items >= (int64_t(1) << 31)) return cudaErrorNotSupported;
  // an item map numbers the items of the requested split layout: kept only when that layout runs
  // and the map has a slot for every item
  const bool use_map = a.item_map != nullptr && a.map_grid > 0 && splits == requested &&
                       a.map_len >= n_items && a.map_len < (int64_t(1) << 31);
  const bool slab = a.capacity > 0;
  const void* sk = slab ? a.slab_k : a.cur_k;
  const void* sv = slab ? a.slab_v : a.cur_v;
  const int64_t srows = slab ? slab_rows : cur_rows;
  CUtensorMap tq, tck, tcv, tsk, tsv;
  if (!sm100::encode_rows(&tq, a.q, cur_rows, bf16, kBM) ||
      !sm100::encode_rows(&tck, a.cur_k, cur_rows, bf16, kBN) ||
      !sm100::encode_rows(&tcv, a.cur_v, cur_rows, bf16, kBN) ||
      !sm100::encode_rows(&tsk, sk, srows, bf16, kBN) ||
      !sm100::encode_rows(&tsv, sv, srows, bf16, kBN))
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
  p.status = a.status;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.qblocks = qblocks;
  p.n_items = static_cast<int>(n_items);
  p.splits = splits;
  p.unsplit = static_cast<int>(unsplit);
  p.ws_counter = splits > 1 ? scratch.counter : nullptr;
  p.ws_ml = splits > 1 ? scratch.ml : nullptr;
  p.ws_o = splits > 1 ? scratch.o : nullptr;
  p.item_map = use_map ? a.item_map : nullptr;
  p.n_slots = static_cast<int>(use_map ? a.map_len : n_items);
  p.seg_stride = static_cast<int>(std::max<int64_t>(a.max_segments, 1));
  p.static_meta = a.static_meta ? 1 : 0;
  p.current_in_segments = a.current_in_segments ? 1 : 0;
  p.out_align32 = (reinterpret_cast<uintptr_t>(a.out) & 31u) == 0 ? 1 : 0;
  p.out_ptrs = a.out_ptrs;
  p.out_rows = a.out_rows;
  p.out_heads = a.out_heads;
  p.n_out = a.n_out;
  p.out_batch = static_cast<int>(a.out_batch);
  p.out_heads_total = static_cast<int>(a.out_heads_total);
  const int grid = use_map ? a.map_grid
                           : static_cast<int>(std::min<int64_t>(n_items, 2 * sm100::sm_count()));
  if (scatter)
    return bf16 ? launch_t<true, true>(tq, tck, tcv, tsk, tsv, p, grid, st)
                : launch_t<false, true>(tq, tck, tcv, tsk, tsv, p, grid, st);
  return bf16 ? launch_t<true, false>(tq, tck, tcv, tsk, tsv, p, grid, st)
              : launch_t<false, false>(tq, tck, tcv, tsk, tsv, p, grid, st);
}

}  // namespace heatkv
