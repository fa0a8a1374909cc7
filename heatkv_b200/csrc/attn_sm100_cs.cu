// Segmented flat-slab attention on Blackwell tensor cores, one 128-row query tile per CTA with the
// softmax of every key tile split by columns over several warpgroups ("column split").
//
// Computes what _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// computes with its default dot modes: for batch row b and head h the keys are the head's slab
// segments [start, end) in segment order followed by the current scale's K/V; fp32 scores and row
// statistics, P rounded to the value dtype before the PV product (:179-180, :241-242), fp32
// accumulation, output [B, Lq, H*D] in q's dtype. Two input modes:
//   * 16-bit: q, k, v all bf16 or all f16; QK is kind::f16 with Q and K from shared memory.
//   * tf32: q and k fp32 with bf16/f16 v, the real model's dtypes (its cos-attention normalises q
//     and k in fp32 under autocast); tl.dot on fp32 operands is a tf32 product (:141-142), so QK
//     is kind::tf32. An fp32 Q tile (64 KiB) does not fit shared memory beside an fp32 K ring, so
//     Q is the A operand from TMEM, staged (fp32 -> tf32, round to nearest) by the softmax warps.
//
// TMEM (512 columns): tf32: Q | S_0 S_1 | O (one O shared by the warpgroups); 16-bit: the
// independent halves below. Key tile g uses S buffer g % kNumS and K/V stage g % 2. P of tile g
// is stored as 16-bit pairs over the first 64 columns of its S buffer once every warpgroup holds
// its scores in registers. (The kernel is written for kWG warpgroups and a shared O in 16-bit mode
// too - S_0 S_1 S_2 | O -, but the library instantiates two warpgroups, the shared O for tf32 and
// the independent halves for 16-bit, the fastest measured.)
//
// Per key tile, warpgroup w of kWG takes the keys [w*128/kWG, (w+1)*128/kWG) of every query row
// (one TMEM lane per thread); the part-row maxima meet in shared memory behind a named barrier;
// each warpgroup keeps its part's row sum, rescales its columns of O and writes them out. The
// running max is lazy: it only moves when a tile exceeds it by more than 8 (a factor 256 in P),
// and every warpgroup takes the same decision for every row. QK and PV are issued by two threads:
// QK(g) as soon as K(g) has landed and PV(g - kNumS), the last reader of its S buffer, has
// completed; PV(g) as soon as P(g) is stored. With three S buffers (16-bit mode) the dependency
// chain QK -> softmax -> PV of one buffer spans three tiles, so the tensor pipe is fed from the
// other buffers meanwhile.
//
// Independent halves (kIndep, 16-bit mode, two warpgroups): TMEM = S_0 | S_1 | O_0 | O_1 and
// warpgroup w runs its own online softmax over the keys [64w, 64w+64) of every tile - its own
// running max and row sum, its P stored inside its own score columns, its own PV (K = 64, the
// tile's V rows [64w, 64w+64)) into O_w - so the two warpgroups never wait on each other within
// an item; the halves are merged once per item in the epilogue,
//   O = (2^(m0-M) O_0 + 2^(m1-M) O_1) / (2^(m0-M) l_0 + 2^(m1-M) l_1),  M = max(m0, m1).
//
// CTA roles (kWG * 128 + 128 threads, 1 CTA per SM):
//   * warps 0 .. 4kWG-1 : softmax warpgroups (and, tf32 mode, Q staging into TMEM); epilogue
//                          (optionally scattering every row into several full outputs).
//   * warp 4kWG         : TMA producer of Q (16-bit mode) and K tiles.
//   * warp 4kWG+1       : TMEM allocator, QK issuer (lane 0).
//   * warp 4kWG+2       : clears V rows past the valid keys of a partial V tile, then issues PV.
//   * warp 4kWG+3       : TMA producer of V tiles.
// Items are (head, batch row, 128-row query block) in longest-head-first order (head_order); CTA c
// of a persistent grid runs items c, c + grid, ... Every wait is bounded (common.cuh); on expiry
// the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains its copies and MMAs, frees TMEM and returns.
//
// Key-range splits (16-bit mode): the blocks after the first `unsplit` (schedule order) are cut
// into `splits` contiguous ranges of their key tiles, one item each. A split writes its row
// maxima and sums (m, l) and its unnormalised O rows (fp32) to the workspace; the CTA that
// completes a block's last split (an atomic counter per block) merges them,
//   O = sum_k 2^(m_k - M) O_k / sum_k 2^(m_k - M) l_k,  M = max over splits with l_k > 0,
// and writes the block's output. A split without key tiles (a block with fewer tiles than splits)
// only publishes (m, l) = (-inf, 0).
//
// Item map (optional, planned on the host from the static segment tables): CTA c runs the items
// item_map[c], item_map[c + grid], ... instead of c, c + grid, ...; -1 marks an empty slot. The
// pre-planned hot path assigns items greedily, longest first, to the least-loaded CTA, which a
// fixed round-robin order cannot do. Entries outside the item space are skipped and raise
// HEATKV_DEVICE_BAD_ITEM_MAP.
#include "attn.h"
#include "common.cuh"
#include "sm100_util.cuh"

#include <cmath>
#include <cstdlib>

namespace heatkv {
namespace sm100 {
namespace cs {

constexpr int kBM = 128;          // query rows per item
constexpr int kBN = kKeyTile;     // keys per tile
constexpr int kD = kHeadDim;
constexpr uint32_t kBox = 128 * 128;         // one TMA box: 128 rows x 128 bytes = 16 KiB
constexpr uint32_t kVTileBytes = 2 * kBox;   // 128 keys x 128 16-bit columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 384;
constexpr int kMaxHeads = 128;
constexpr int kMaxSegTable = 2048;
constexpr int kMapRounds = 64;    // item map slots of a CTA staged in shared memory

template <bool kTf32, bool kIndep = false>
struct Mode {
  static constexpr int kNumS = (kTf32 || kIndep) ? 2 : 3;  // S buffers in TMEM
  static constexpr uint32_t kColS = kTf32 ? 128 : 0;     // first S buffer (Q at 0 in tf32 mode)
  static constexpr uint32_t kColO0 = kIndep ? 256 : 384;  // O (O_0 and O_1 = +128 if kIndep)
  static constexpr int kKBoxes = kTf32 ? 4 : 2;          // 32 fp32 or 64 16-bit columns a box
  static constexpr uint32_t kKTileBytes = kKBoxes * kBox;
  static constexpr uint32_t kQBytes = kTf32 ? 1024 : 2 * kBox;  // Q in shared memory (16-bit)
};

template <bool kTf32, int kWG, bool kIndep = false>
struct __align__(1024) Smem {
  uint8_t k[2][Mode<kTf32>::kKTileBytes];
  uint8_t v[2][kVTileBytes];
  uint8_t q[Mode<kTf32>::kQBytes];
  uint64_t q_full;     // Q of the item is in place (TMA bytes, or every softmax warp's TMEM stores)
  uint64_t q_empty;    // 16-bit mode: the item's last QK has completed (Q may be overwritten)
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t s_full[Mode<kTf32, kIndep>::kNumS];     // QK(g) done: scores in S buffer g % kNumS
  uint64_t p_full[Mode<kTf32, kIndep>::kNumS][2];  // P(g) stored (kIndep: per warpgroup)
  uint64_t pv_done[Mode<kTf32, kIndep>::kNumS];    // PV(g) done: V stage g % 2, S buffer free
  uint64_t o_final;    // the item's last PV has completed
  uint64_t o_free;     // every softmax warp has read the item's O
  uint64_t drain;      // both issuers' products have completed
  uint32_t tmem_base;
  int abort_flag;
  int last_flag;       // this CTA completed the last split of its block
  float red_max[2][kWG][kBM];  // [tile parity][warpgroup][row]: part-row maxima
  float red_sum[kWG][kBM];     // [warpgroup][row]: part-row sums of an item
  float2 red_ml[2][2][kBM];    // kIndep: [item parity][warpgroup][row] (running max, row sum)
  int head_order[kMaxHeads];
  int head_nseg[kMaxHeads];
  int head_tiles[kMaxHeads];
  int seg_start[kMaxSegTable];
  int seg_end[kMaxSegTable];
  int slot_items[kMapRounds];  // item map: this CTA's first kMapRounds slots, checked
};

struct Params {
  int64_t batch, heads, q_len, capacity, max_segments;
  const float* q;               // tf32 mode: [B, H, Lq, D] fp32 (16-bit mode: through tm_q)
  const int32_t* seg_starts;
  const int32_t* seg_ends;
  const int32_t* seg_counts;
  const int32_t* head_order;    // [heads] or null
  void* out;                    // [B, Lq, H * D] in q's dtype
  unsigned int* status;
  float scale_log2;             // softmax_scale * log2(e)
  int qblocks;                  // ceil(Lq / 128)
  int n_items;                  // unsplit + (heads * batch * qblocks - unsplit) * splits
  int splits;                   // key-range splits of each split block (1 = none)
  const int32_t* item_map;      // [n_slots] item of every slot, -1 = none; null = slot i is item i
  int n_slots;                  // slots the CTAs walk (n_items without a map)
  int unsplit;                  // leading blocks (schedule order) that are not split
  uint32_t* ws_counter;         // [split blocks], zero between calls
  float2* ws_ml;                // [split blocks * splits * 128]
  float* ws_o;                  // [split blocks * splits * 128 * 128]
  int seg_stride;
  int static_meta;              // stage the metadata before the dependency wait
  int current_in_segments;      // the current keys end every non-empty head's segments
  // scatter epilogue (16-bit mode, n_out > 0): every output row goes to n_out full [out_batch,
  // Lq, out_heads_total * D] tensors at row out_rows[b] and head out_heads[h]
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

// The item of a map entry (-1: none); an entry outside the item space is skipped and reported.
__device__ __forceinline__ int checked_item(const Params& p, int item) {
  if (item >= p.n_items || item < -1) {
    raise_status(p.status, HEATKV_DEVICE_BAD_ITEM_MAP);
    return -1;
  }
  return item;
}

// The item of one of this CTA's slots (-1: none): the slot itself without a map, else the map
// entry, staged in shared memory for the first kMapRounds slots of the CTA.
template <class SmemT>
__device__ __forceinline__ int slot_item(const SmemT& sm, const Params& p, int slot) {
  if (p.item_map == nullptr) return slot;
  const int k = (slot - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x);
  if (k < kMapRounds) return sm.slot_items[k];
  const int item = __ldg(p.item_map + slot);
  return (item >= p.n_items || item < -1) ? -1 : item;
}

template <class SmemT>
__device__ __forceinline__ Item decode_item(const SmemT& sm, const Params& p, int item) {
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

// fp32 -> tf32, round to nearest (ties away from zero); the low 13 bits of the result are zero.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

template <int kWG>
__device__ __forceinline__ void named_bar_softmax_wg() {
  asm volatile("bar.sync 1, %0;" ::"n"(kWG * 128) : "memory");
}

template <bool kTf32, bool kBF16, int kWG, bool kIndep>
__global__ void __launch_bounds__(kWG * 128 + 128, 1)
    attn_sm100_cs_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_ck,
                         const __grid_constant__ CUtensorMap tm_cv,
                         const __grid_constant__ CUtensorMap tm_sk,
                         const __grid_constant__ CUtensorMap tm_sv, const Params p) {
  static_assert(!kIndep || (!kTf32 && kWG == 2), "independent halves: 16-bit, two warpgroups");
  using M = Mode<kTf32, kIndep>;
  using SmemT = Smem<kTf32, kWG, kIndep>;
  constexpr int kNumS = M::kNumS;
  constexpr uint32_t kColS = M::kColS;
  constexpr int kCols = kBN / kWG;        // score (and O) columns of one warpgroup
  constexpr int kSoftmaxWarps = 4 * kWG;
  constexpr int kKWarp = kSoftmaxWarps;
  constexpr int kQkWarp = kSoftmaxWarps + 1;
  constexpr int kPvWarp = kSoftmaxWarps + 2;
  constexpr int kVWarp = kSoftmaxWarps + 3;
  using OutT = typename std::conditional<kTf32, float,
               typename std::conditional<kBF16, __nv_bfloat16, __half>::type>::type;

  extern __shared__ uint8_t smem_raw[];
  SmemT& sm = *reinterpret_cast<SmemT*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
    mbar_init(&sm.q_full, kTf32 ? kSoftmaxWarps : 1);
    mbar_init(&sm.q_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.k_full[b], 1);
      mbar_init(&sm.v_full[b], 1);
    }
    for (int b = 0; b < kNumS; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b][0], kIndep ? 4 : kSoftmaxWarps);
      mbar_init(&sm.p_full[b][1], 4);
      mbar_init(&sm.pv_done[b], 1);
    }
    mbar_init(&sm.o_final, 1);
    mbar_init(&sm.o_free, kSoftmaxWarps);
    mbar_init(&sm.drain, 2);
    fence_mbar_init();
  }
  // The metadata is staged before the dependency wait when the caller guarantees that the
  // preceding work does not write it (HEATKV_ATTN_STATIC_META), else after it.
  if (!p.static_meta) pdl_wait();
  if (warp == kKWarp) {
    // stage the [H, S] metadata, compact every head's non-empty segments in place (clipped to
    // the slab) and count its key tiles
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
    // this CTA's item map slots (static like the metadata: read before the dependency wait
    // under HEATKV_ATTN_STATIC_META, so the first item is known as soon as the wait ends); slots
    // past the first kMapRounds are read and checked from global memory when reached
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
      if (!kTf32) tma_prefetch_desc(&tm_q);
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
        if constexpr (!kTf32) {
          if (loads_k) {
            // Q rows of the item once the previous item's last QK has completed; rows past the
            // tensor are zero-filled, rows past Lq of this head are never written out
            if (qcnt > 0 && !(ok = mbar_wait(&sm.q_empty, (qcnt - 1) & 1, abort_flag, p.status))) break;
            mbar_arrive_expect_tx(&sm.q_full, 2 * kBox);
            tma_load_2d(sm.q, &tm_q, 0, bh * Lq + it.q0, &sm.q_full);
            tma_load_2d(sm.q + kBox, &tm_q, 64, bh * Lq + it.q0, &sm.q_full);
            ++qcnt;
          }
        }
        const int cur_row0 = bh * Lq;
        const int slab_row0 = static_cast<int>(int64_t(it.b) * p.capacity);
        TileCursor cur;
        cur.begin(sm, it.h, stride, it.j0);
        for (int j = 0; j < it.n; ++j, ++gx) {
          const int s = gx % 2;
          // the stage's previous tile (gx - 2) is done with: its QK (K) or its PV (V)
          if (gx >= 2) {
            const uint32_t pg = gx - 2;
            uint64_t* done = loads_k ? &sm.s_full[pg % kNumS] : &sm.pv_done[pg % kNumS];
            if (!(ok = mbar_wait(done, (pg / kNumS) & 1, abort_flag, p.status))) break;
          }
          const int row = cur.current ? cur_row0 + cur.pos : slab_row0 + cur.pos;
          if (loads_k) {
            const CUtensorMap* m = cur.current ? &tm_ck : &tm_sk;
            mbar_arrive_expect_tx(&sm.k_full[s], M::kKTileBytes);
#pragma unroll
            for (int box = 0; box < M::kKBoxes; ++box)
              tma_load_2d(sm.k[s] + box * kBox, m, box * (128 / M::kKBoxes), row, &sm.k_full[s]);
          } else {
            const CUtensorMap* m = cur.current ? &tm_cv : &tm_sv;
            mbar_arrive_expect_tx(&sm.v_full[s], kVTileBytes);
            tma_load_2d(sm.v[s], m, 0, row, &sm.v_full[s]);
            tma_load_2d(sm.v[s] + kBox, m, 64, row, &sm.v_full[s]);
          }
          cur.next();
        }
      }
      if (!ok || *abort_flag) {
        // let every copy already issued land before the CTA's shared memory goes away
        if (!kTf32 && loads_k && qcnt > 0) mbar_drain(&sm.q_full, (qcnt - 1) & 1, p.status);
        for (uint32_t g = gx > 2 ? gx - 2 : 0; g < gx; ++g)
          mbar_drain(loads_k ? &sm.k_full[g % 2] : &sm.v_full[g % 2], (g / 2) & 1, p.status);
      }
    }
  } else if (warp == kQkWarp) {
    // ---------------------------------------------------------------- QK issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = kTf32 ? idesc_tf32(kBM, kBN) : idesc_f16(kBF16, kBM, kBN, false, false);
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
          const uint32_t b = g % kNumS;
          const uint32_t ks = g % 2;
          if (!(ok = mbar_wait(&sm.k_full[ks], (g / 2) & 1, abort_flag, p.status))) break;
          // S buffer b last held P(g - kNumS): its PV must have completed
          if (g >= static_cast<uint32_t>(kNumS) &&
              !(ok = mbar_wait(&sm.pv_done[b], ((g / kNumS) - 1) & 1, abort_flag, p.status)))
            break;
          tc_fence_after();
          // S_b = Q K^T. B = K tile, K-major SW128: a K step is 32 bytes into the 128-byte row
          // of its box. tf32: A = Q from TMEM, 8 tf32 columns a step; 16-bit: A = Q in shared
          // memory with the K tile's layout
          const uint32_t kbase = smem_u32(sm.k[ks]);
          const uint32_t d = tmem + kColS + b * 128;
          if constexpr (kTf32) {
#pragma unroll
            for (int kk = 0; kk < kD / 8; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(kbase + (kk / 4) * kBox + (kk % 4) * 32, 16, 1024);
              umma_tf32_ts(d, tmem + kk * 8, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
            }
          } else {
            const uint32_t qbase = smem_u32(sm.q);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t off = (kk / 4) * kBox + (kk % 4) * 32;
              umma_ss(d, smem_desc_sw128(qbase + off, 16, 1024),
                      smem_desc_sw128(kbase + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
            }
          }
          tc_commit(&sm.s_full[b]);
          if (!kTf32 && j == it.n - 1) tc_commit(&sm.q_empty);
        }
      }
      // every MMA issued by this thread has completed once `drain` fires (with the PV issuer's)
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else if (warp == kPvWarp) {
    // ---------------------------------------------------------------- V tail clearing, PV issuer
    // Past the end of a segment (or of the current scale) a V tile holds whatever the slab holds
    // there; P is 0 for those keys but 0 x NaN would poison O, so the tail rows are cleared (a
    // 128-byte swizzled row keeps its bytes inside its own 128-byte line) before lane 0 issues
    // the tile's PV.
    constexpr uint32_t idesc_pv = idesc_f16(kBF16, kBM, kD, false, true);
    uint32_t g = 0, ocnt = 0;
    bool ok = true;
    for (int slot = blockIdx.x; ok && slot < p.n_slots; slot += gridDim.x) {
      const int item = slot_item(sm, p, slot);
      if (item < 0) continue;
      const Item it = decode_item(sm, p, item);
      if (it.n == 0) continue;
      TileCursor cur;
      cur.begin(sm, it.h, stride, it.j0);
      for (int j = 0; j < it.n; ++j, ++g) {
        const uint32_t vs = g % 2;
        const uint32_t b = g % kNumS;
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.v_full[vs], (g / 2) & 1, abort_flag, p.status));
        if (!ok) break;
        const int valid = cur.valid(Lq);
        if (valid < kBN) {
          uint8_t* base = sm.v[vs];
          const int chunks = (kBN - valid) * 2 * 8;  // rows x halves x 16-byte chunks
          for (int i = lane; i < chunks; i += 32) {
            const int line = i / 8;
            const int row = valid + line / 2, half = line % 2;
            *reinterpret_cast<uint4*>(base + half * kBox + row * 128 + (i % 8) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          // the cleared rows are visible to the tensor core (async proxy)
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncwarp();
        if (lane == 0) {
          // O += P V: A = P (16-bit pairs in TMEM), B = V tile, MN-major SW128: 8-key groups
          // 1 KiB apart (SBO), the two 64-column halves 16 KiB apart (LBO); 16 keys a step
          const uint32_t vbase = smem_u32(sm.v[vs]);
          const uint32_t a = tmem + kColS + b * 128;
          if constexpr (kIndep) {
            // each half as soon as its warpgroup has stored it: keys [64w, 64w+64) (P in pair
            // columns [64w, 64w+32) of S_b) into O_w
#pragma unroll
            for (int w = 0; w < 2 && ok; ++w) {
              ok = mbar_wait(&sm.p_full[b][w], (g / kNumS) & 1, abort_flag, p.status);
              if (ok && w == 0 && j == 0 && ocnt > 0)
                ok = mbar_wait(&sm.o_free, (ocnt - 1) & 1, abort_flag, p.status);
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int kk = 4 * w; kk < 4 * w + 4; ++kk) {
                const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, kBox, 1024);
                umma_ts(tmem + M::kColO0 + 128 * w, a + 64 * w + (kk - 4 * w) * 8, bdesc,
                        idesc_pv, (j > 0 || kk > 4 * w) ? 1u : 0u);
              }
            }
          } else {
            ok = mbar_wait(&sm.p_full[b][0], (g / kNumS) & 1, abort_flag, p.status);
            if (ok && j == 0 && ocnt > 0) ok = mbar_wait(&sm.o_free, (ocnt - 1) & 1, abort_flag, p.status);
            if (ok) {
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk) {
                const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, kBox, 1024);
                umma_ts(tmem + kColO, a + kk * 8, bdesc, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
              }
            }
          }
          if (ok) {
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
    // ---------------------------------------------------------------- softmax warpgroups
    const int w = warp / 4;            // columns [w * kCols, (w + 1) * kCols) of S and of O
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // TMEM lane == query row
    const int c0 = w * kCols;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    // O columns this thread rescales: its warpgroup's share of O, or (kIndep) all of O_w
    const uint32_t tO = kIndep ? tmem + lane_off + M::kColO0 + 128 * w : tmem + lane_off + kColO + c0;
    constexpr int kOCols = kIndep ? 128 : kCols;
    const float c = p.scale_log2;
    // tf32 mode: Q rows of an item -> TMEM (this warpgroup's columns), zero past Lq
    auto load_q = [&](int item) {
      if constexpr (kTf32) {
        const Item it = decode_item(sm, p, item);
        const int qr = it.q0 + row;
#pragma unroll
        for (int part = 0; part < kCols / 32; ++part) {
          uint32_t r[32];
          if (qr < Lq) {
            const float4* src = reinterpret_cast<const float4*>(
                p.q + ((int64_t(it.b) * H + it.h) * Lq + qr) * kD + c0 + 32 * part);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 v = __ldg(src + i);
              r[4 * i] = to_tf32(v.x);
              r[4 * i + 1] = to_tf32(v.y);
              r[4 * i + 2] = to_tf32(v.z);
              r[4 * i + 3] = to_tf32(v.w);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          tmem_st32(tmem + lane_off + c0 + 32 * part, r);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.q_full);
      }
    };
    // workspace row of this thread's query row in split `split` of split block `sblock`
    auto split_slot = [&](const Item& it, int split) {
      return (int64_t(it.sblock) * it.nsplit + split) * kBM + row;
    };
    // After every softmax thread has published its split's partial rows: count the split in, and
    // if it was the block's last, merge the partials of this thread's row and columns
    // [c0, c0 + kCols) into the output. Every softmax thread takes both barriers.
    auto split_finish = [&](const Item& it) {
      named_bar_softmax_wg<kWG>();
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
      named_bar_softmax_wg<kWG>();
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
      OutT* orow = static_cast<OutT*>(p.out) + ((int64_t(it.b) * Lq + qrow) * H + it.h) * kD + c0;
#pragma unroll 1
      for (int cc = 0; cc < kCols / 16; ++cc) {  // 16 columns a step, every split's loads in flight
        float4 v[kMaxKvSplits][4];
#pragma unroll
        for (int k = 0; k < kMaxKvSplits; ++k) {
          const float4* src =
              reinterpret_cast<const float4*>(p.ws_o + split_slot(it, k) * kD + c0) + cc * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            v[k][i] = wk[k] != 0.f ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float a[16];
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
          a[4 * i] = acc.x;
          a[4 * i + 1] = acc.y;
          a[4 * i + 2] = acc.z;
          a[4 * i + 3] = acc.w;
        }
        if constexpr (kTf32) {
          float4* d4 = reinterpret_cast<float4*>(orow + cc * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_float4(a[4 * i], a[4 * i + 1], a[4 * i + 2], a[4 * i + 3]);
        } else {
          uint32_t wv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) wv[i] = pack2<kBF16>(a[2 * i], a[2 * i + 1]);
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 16);
          dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
        }
      }
    };
    uint32_t g = 0, ocnt = 0;
    bool ok = true;
    // tf32 mode: the next item of this CTA after slot `slot` (-1: none)
    auto next_item = [&](int slot) {
      for (slot += gridDim.x; slot < p.n_slots; slot += gridDim.x) {
        const int item = slot_item(sm, p, slot);
        if (item >= 0) return item;
      }
      return -1;
    };
    if constexpr (kTf32) {
      const int first = next_item(static_cast<int>(blockIdx.x) - static_cast<int>(gridDim.x));
      if (first >= 0) load_q(first);
    }
    for (int slot = blockIdx.x; slot < p.n_slots; slot += gridDim.x) {
      const int item = slot_item(sm, p, slot);
      if (item < 0) continue;
      const Item it = decode_item(sm, p, item);
      if (it.n == 0) {
        // a split without key tiles (16-bit mode only): it contributes nothing to its block
        if (w == 0 && it.q0 + row < Lq)
          __stcg(p.ws_ml + split_slot(it, it.split), make_float2(-INFINITY, 0.f));
        split_finish(it);
        continue;
      }
      float m_run = -INFINITY;
      float l_run = 0.f;
      const bool row_live = it.q0 + row < Lq;
      TileCursor cur;
      cur.begin(sm, it.h, stride, it.j0);
      // Every softmax warp takes the same named barriers in the same order, including after an
      // abort (the work is skipped, the barriers are not).
      for (int j = 0; j < it.n; ++j, ++g) {
        const uint32_t b = g % kNumS;
        const uint32_t tS = tmem + lane_off + kColS + b * 128;
        const int valid = cur.valid(Lq);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[b], (g / kNumS) & 1, abort_flag, p.status));
        float x[kCols];
        float mx = -INFINITY;
        if (ok) {
          tc_fence_after();
          tmem_ld_cols<kCols>(tS + c0, x);
          if (valid < kBN) {
#pragma unroll
            for (int i = 0; i < kCols; ++i) x[i] = (c0 + i < valid) ? x[i] : -INFINITY;
          }
          mx = row_max<kCols>(x) * c;
        }
        if constexpr (!kIndep) {
          sm.red_max[g & 1][w][row] = mx;
          // every warpgroup's scores are in its registers before P is stored over them
          tc_fence_before();
          named_bar_softmax_wg<kWG>();
          tc_fence_after();
          mx = sm.red_max[g & 1][0][row];
#pragma unroll
          for (int v = 1; v < kWG; ++v) mx = fmaxf(mx, sm.red_max[g & 1][v][row]);
        }
        if (ok) {
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
          // kIndep: a warpgroup whose keys of the item so far are all masked has m = -inf; its
          // P must be 0, not 2^(-inf + inf)
          const float msub = (kIndep && m_run == -INFINITY) ? 0.f : m_run;
          const uint64_t nm2 = f2pack(-msub, -msub);
          uint64_t acc[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[k] = f2pack(0.f, 0.f);
#pragma unroll
          for (int part = 0; part < kCols / 32; ++part) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int pi = part * 16 + i;  // columns c0 + 2pi, c0 + 2pi + 1
              const uint64_t y = fma2(f2pack(x[2 * pi], x[2 * pi + 1]), c2, nm2);
              float y0, y1;
              f2unpack(y, y0, y1);
              const float p0 = ex2(y0);
              const float p1 = ex2(y1);
              acc[pi & 3] = add2(acc[pi & 3], f2pack(p0, p1));
              pk[i] = pack2<kBF16>(p0, p1);
            }
            // P of keys [c0 + 32 part, +32) -> 16-bit pair columns [c0/2 + 16 part, +16), or
            // (kIndep) inside this warpgroup's own score columns, [c0 + 16 part, +16)
            tmem_st16(tS + (kIndep ? c0 : c0 / 2) + 16 * part, pk);
          }
          const uint64_t s01 = add2(acc[0], acc[1]);
          const uint64_t s23 = add2(acc[2], acc[3]);
          float u0, u1;
          f2unpack(add2(s01, s23), u0, u1);
          l_run += u0 + u1;
          if (rescale) {  // warp-uniform; O must hold PV(g - 1) first
            ok = __all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(g - 1) % kNumS],
                                                   ((g - 1) / kNumS) & 1, abort_flag, p.status));
            if (ok) {
              tc_fence_after();
#pragma unroll
              for (int cc = 0; cc < kOCols / 16; ++cc) {
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
          if (lane == 0) mbar_arrive(&sm.p_full[b][kIndep ? w : 0]);
        }
        cur.next();
      }
      // tf32 mode: the item's last QK has completed (its scores were read): stage the next
      // item's Q now, so its first QK overlaps this item's last PV and the epilogue
      if constexpr (kTf32) {
        const int next = next_item(slot);
        if (ok && next >= 0) load_q(next);
      }
      float l_tot, a0 = 1.f, a1 = 0.f;
      float m_fin = m_run;  // the row's max over the item's keys (scaled, log2 units)
      if constexpr (kIndep) {
        // merge weights of the two halves; WG0's max is finite (key 0 of every tile is valid)
        sm.red_ml[ocnt & 1][w][row] = make_float2(m_run, l_run);
        named_bar_softmax_wg<kWG>();
        const float2 h0 = sm.red_ml[ocnt & 1][0][row], h1 = sm.red_ml[ocnt & 1][1][row];
        const float mm = fmaxf(h0.x, h1.x);
        m_fin = mm;
        a0 = h0.x == -INFINITY ? 0.f : ex2(h0.x - mm);
        a1 = h1.x == -INFINITY ? 0.f : ex2(h1.x - mm);
        l_tot = h0.y * a0 + h1.y * a1;
      } else {
        sm.red_sum[w][row] = l_run;
        named_bar_softmax_wg<kWG>();
        l_tot = sm.red_sum[0][row];
#pragma unroll
        for (int v = 1; v < kWG; ++v) l_tot += sm.red_sum[v][row];
      }
      const bool split = it.nsplit > 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.o_final, ocnt & 1, abort_flag, p.status));
      if (split && w == 0 && it.q0 + row < Lq)
        __stcg(p.ws_ml + split_slot(it, it.split),
               ok ? make_float2(m_fin, l_tot) : make_float2(-INFINITY, 0.f));
      if (ok) {
        tc_fence_after();
        const int qrow = it.q0 + row;
        // a split writes its O rows unnormalised (the merge divides by the combined sum)
        const float inv = split ? 1.f : 1.f / l_tot;
        int64_t off = ((int64_t(it.b) * Lq + qrow) * H + it.h) * kD + c0;
        int n_dst = 1;
        bool in_range = true;
        if (!kTf32 && p.n_out > 0) {
          const int grow = __ldg(p.out_rows + it.b), ghead = __ldg(p.out_heads + it.h);
          in_range = grow >= 0 && grow < p.out_batch && ghead >= 0 && ghead < p.out_heads_total;
          if (!in_range && row == 0 && w == 0) raise_status(p.status, HEATKV_DEVICE_GATHER_OUT_OF_RANGE);
          off = ((int64_t(grow) * Lq + qrow) * p.out_heads_total + ghead) * kD + c0;
          n_dst = p.n_out;
        }
        const bool write = qrow < Lq && in_range;
        float* ws_row = split ? p.ws_o + split_slot(it, it.split) * kD + c0 : nullptr;
        // 16 output columns [col, col + 16) of this row (already normalised), or of a split's
        // partial row
        auto store16 = [&](int col, const float* v) {
          if (split) {
            float4* d4 = reinterpret_cast<float4*>(ws_row + col);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              __stcg(d4 + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
          } else if constexpr (kTf32) {
            float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off + col);
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            uint32_t wv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[i] = pack2<kBF16>(v[2 * i], v[2 * i + 1]);
#pragma unroll 1
            for (int r = 0; r < n_dst; ++r) {
              OutT* base = p.n_out > 0 ? static_cast<OutT*>(p.out_ptrs[r]) : static_cast<OutT*>(p.out);
              uint4* dst = reinterpret_cast<uint4*>(base + off + col);
              dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
              dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
            }
          }
        };
        if constexpr (kIndep) {
          // output columns [c0, c0 + 64) = the merge of O_0 and O_1 there
          const float w0 = a0 * inv, w1 = a1 * inv;
          const uint32_t tA = tmem + lane_off + M::kColO0 + c0;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            float o0[32], o1[32];
            tmem_ld32_sync(tA + 32 * half, o0);
            tmem_ld32_sync(tA + 128 + 32 * half, o1);
            if (write) {
#pragma unroll
              for (int cc = 0; cc < 2; ++cc) {
                float v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = fmaf(o0[cc * 16 + i], w0, o1[cc * 16 + i] * w1);
                store16(32 * half + 16 * cc, v);
              }
            }
          }
        } else {
          float o[kCols];
          tmem_ld_cols<kCols>(tO, o);  // this warpgroup's O columns in one load
          if (write) {
#pragma unroll
            for (int cc = 0; cc < kCols / 16; ++cc) {
              float v[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = o[cc * 16 + i] * inv;
              store16(16 * cc, v);
            }
          }
        }
        // stores to other GPUs are visible system-wide before this kernel's completion is
        if (!kTf32 && p.n_out > 0) __threadfence_system();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_free);
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

// rows x 128 fp32 matrix, box 32 x 128 (128 bytes per row) with 128-byte swizzle
static bool encode_rows_f32(CUtensorMap* map, const void* base, int64_t rows) {
  auto enc = get_encode();
  if (!enc) return false;
  if (rows <= 0) rows = 1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD * 4)};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(kBN)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                   strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool kTf32, bool kBF16, int kWG, bool kIndep = false>
static cudaError_t launch_t(const CUtensorMap& tq, const CUtensorMap& tck, const CUtensorMap& tcv,
                            const CUtensorMap& tsk, const CUtensorMap& tsv, const Params& p,
                            int map_grid, cudaStream_t st) {
  auto kern = attn_sm100_cs_kernel<kTf32, kBF16, kWG, kIndep>;
  const int smem = static_cast<int>(sizeof(Smem<kTf32, kWG, kIndep>)) + 1024;
  static_assert(sizeof(Smem<kTf32, kWG, kIndep>) + 1024 <= 227 * 1024, "shared memory of one CTA");
  // opt in to >48 KiB dynamic shared memory once per device (never inside a graph capture)
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
  // a map fixes the grid it was planned for; otherwise at most one CTA per SM
  const int grid = p.item_map ? map_grid : static_cast<int>(std::min<int>(p.n_items, sm_count()));
  e = launch_pdl(kern, dim3(grid), dim3(kWG * 128 + 128), static_cast<size_t>(smem), st, tq, tck,
                 tcv, tsk, tsv, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <bool kTf32, bool kBF16>
static cudaError_t launch_mode(const AttnArgs& a, cudaStream_t st) {
  const int64_t cur_rows = a.batch * a.heads * a.q_len;
  const int64_t slab_rows = a.batch * a.capacity;
  if (cur_rows >= (int64_t(1) << 31) || slab_rows >= (int64_t(1) << 31) ||
      a.heads > kMaxHeads || a.heads * std::max<int64_t>(a.max_segments, 1) > kMaxSegTable ||
      !(a.scale > 0.f) || a.q_len <= 0 || (kTf32 && a.n_out > 0))
    return cudaErrorNotSupported;
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.cur_k) |
                          reinterpret_cast<uintptr_t>(a.cur_v) |
                          reinterpret_cast<uintptr_t>(a.slab_k) |
                          reinterpret_cast<uintptr_t>(a.slab_v) | reinterpret_cast<uintptr_t>(a.out);
  if (align & 15u) return cudaErrorNotSupported;
  const int qblocks = static_cast<int>((a.q_len + kBM - 1) / kBM);
  const int64_t blocks = a.batch * a.heads * qblocks;
  // key-range splits: 16-bit mode with the plain epilogue only
  int splits = a.kv_splits <= 0 ? attention_cs_auto_splits(a.batch, a.heads, a.q_len) : a.kv_splits;
  splits = std::min(splits, kMaxKvSplits);
  if (kTf32 || a.n_out > 0) splits = 1;
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
  bool ok;
  if constexpr (kTf32) {
    ok = encode_rows(&tq, a.cur_v, cur_rows, kBF16) &&  // unused in tf32 mode; well-formed
         encode_rows_f32(&tck, a.cur_k, cur_rows) && encode_rows_f32(&tsk, sk, srows);
  } else {
    ok = encode_rows(&tq, a.q, cur_rows, kBF16) && encode_rows(&tck, a.cur_k, cur_rows, kBF16) &&
         encode_rows(&tsk, sk, srows, kBF16);
  }
  ok = ok && encode_rows(&tcv, a.cur_v, cur_rows, kBF16) && encode_rows(&tsv, sv, srows, kBF16);
  if (!ok) return cudaErrorInvalidValue;
  Params p;
  p.batch = a.batch;
  p.heads = a.heads;
  p.q_len = a.q_len;
  p.capacity = a.capacity;
  p.max_segments = a.max_segments;
  p.q = static_cast<const float*>(a.q);
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
  p.item_map = use_map ? a.item_map : nullptr;
  p.n_slots = static_cast<int>(use_map ? a.map_len : n_items);
  p.ws_counter = splits > 1 ? scratch.counter : nullptr;
  p.ws_ml = splits > 1 ? scratch.ml : nullptr;
  p.ws_o = splits > 1 ? scratch.o : nullptr;
  p.seg_stride = static_cast<int>(std::max<int64_t>(a.max_segments, 1));
  p.static_meta = a.static_meta ? 1 : 0;
  p.current_in_segments = a.current_in_segments ? 1 : 0;
  p.out_ptrs = a.out_ptrs;
  p.out_rows = a.out_rows;
  p.out_heads = a.out_heads;
  p.n_out = a.n_out;
  p.out_batch = static_cast<int>(a.out_batch);
  p.out_heads_total = static_cast<int>(a.out_heads_total);
  const int mg = a.map_grid;
  // two softmax warpgroups; 16-bit mode with independent halves (each warpgroup its own keys and
  // its own O), tf32 mode with one O shared by the warpgroups
  if constexpr (!kTf32) return launch_t<false, kBF16, 2, true>(tq, tck, tcv, tsk, tsv, p, mg, st);
  return launch_t<kTf32, kBF16, 2>(tq, tck, tcv, tsk, tsv, p, mg, st);
}

}  // namespace cs
}  // namespace sm100

int attention_cs_auto_splits(int64_t batch, int64_t heads, int64_t q_len) {
  const int64_t blocks = batch * heads * ((q_len + sm100::cs::kBM - 1) / sm100::cs::kBM);
  const int64_t target = 2 * int64_t(sm100::sm_count());
  if (blocks <= 0 || blocks >= target) return 1;
  return static_cast<int>(std::min<int64_t>(kMaxKvSplits, (target + blocks - 1) / blocks));
}

cudaError_t launch_attention_sm100_tf32(const AttnArgs& a, bool v_bf16, cudaStream_t st) {
  return v_bf16 ? sm100::cs::launch_mode<true, true>(a, st)
                : sm100::cs::launch_mode<true, false>(a, st);
}

cudaError_t launch_attention_sm100_cs(const AttnArgs& a, bool bf16, cudaStream_t st) {
  return bf16 ? sm100::cs::launch_mode<false, true>(a, st)
              : sm100::cs::launch_mode<false, false>(a, st);
}

}  // namespace heatkv
