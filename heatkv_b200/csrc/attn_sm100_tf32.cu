// Segmented flat-slab attention on Blackwell tensor cores for fp32 queries and keys with 16-bit
// values: the dtypes of the real model, whose cos-attention normalises q and k in fp32 under
// autocast while v stays bf16.
//
// Computes what _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// computes with its default dot modes on these dtypes: scores = tl.dot(q, k) on fp32 operands is a
// tf32 tensor-core product (:141-142, :203-204), P is rounded to the value dtype for the PV
// product (:179-180, :241-242), fp32 row statistics and accumulation, output [B, Lq, H*D] in q's
// dtype (fp32). The keys of batch row b and head h are the head's slab segments [start, end) in
// segment order followed by the current scale's K/V.
//
// Why a second kernel: an fp32 Q tile (64 KiB) plus a 2-stage ring of fp32 K tiles (128 KiB) and
// a ring of 16-bit V tiles (64 KiB) does not fit shared memory, so Q lives in TMEM as the A
// operand of kind::tf32 (A from TMEM, K from shared memory), one 128-row Q tile per CTA:
//   TMEM columns: Q [0,128) (tf32), S_0 [128,256), S_1 [256,384) (double-buffered scores, P
//   stored over the first 64 columns as 16-bit pairs), O [384,512).
// With a single Q tile the two softmax warpgroups split each tile's columns: warpgroup w takes
// keys [64w, 64w+64) of every row, the two half-row maxima meet in shared memory behind a named
// barrier, each warpgroup keeps the row sum of its half and rescales its half of O. The MMA
// thread runs one score tile ahead: QK(j+1) is issued before PV(j), so the softmax of tile j
// overlaps QK(j+1). QK and PV are issued by two threads: a single issuer blocks ~85 cycles on
// every tcgen05.mma, so with both products on one thread PV(j) waited behind the whole of
// QK(j+1); with two, the tensor pipe takes whichever is ready.
//
// CTA roles (384 threads, 1 CTA per SM):
//   * warps 0-7 : softmax (two warpgroups, one TMEM lane = query row per thread); they also stage
//                 the next item's Q rows (fp32 -> tf32, round to nearest) into TMEM as soon as the
//                 current item's last QK has completed, and write the output.
//   * warp 8    : TMA producer of K tiles (four 32-column fp32 boxes, 128-byte swizzle).
//   * warp 9    : TMEM allocator; lane 0 issues QK(j) once K(j) has landed and PV(j-2), the
//                 last reader of the S buffer, has completed.
//   * warp 10   : clears the V rows past the valid keys of a partial V tile, then lane 0 issues
//                 PV(j) once P(j) is stored.
//   * warp 11   : TMA producer of V tiles.
// Items are (head, batch row, 128-row query block) in longest-head-first order (head_order), CTA
// c of a persistent grid runs items c, c + grid, ... Every wait is bounded (common.cuh); on expiry
// the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains its copies and MMAs, frees TMEM and returns.
#include "attn.h"
#include "common.cuh"
#include "sm100_util.cuh"

namespace heatkv {
namespace sm100 {
namespace tf32 {

constexpr int kBM = 128;          // query rows per item
constexpr int kBN = kKeyTile;     // keys per tile
constexpr int kD = kHeadDim;
constexpr int kStages = 2;
constexpr int kThreads = 384;
constexpr int kKWarp = 8;
constexpr int kQkWarp = 9;
constexpr int kPvWarp = 10;
constexpr int kVWarp = 11;
constexpr uint32_t kKBox = kBN * 128;         // 128 keys x 32 fp32 columns: 16 KiB
constexpr uint32_t kKTileBytes = 4 * kKBox;   // 128 x 128 x 4 bytes
constexpr uint32_t kVHalf = kBN * 128;        // 128 keys x 64 16-bit columns: 16 KiB
constexpr uint32_t kVTileBytes = 2 * kVHalf;  // 128 x 128 x 2 bytes
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColQ = 0;
constexpr uint32_t kColS = 128;  // + 128 * buffer
constexpr uint32_t kColO = 384;
constexpr int kMaxHeads = 128;
constexpr int kMaxSegTable = 2048;

struct __align__(1024) Smem {
  uint8_t k[kStages][kKTileBytes];
  uint8_t v[kStages][kVTileBytes];
  uint64_t q_full;              // the 8 softmax warps stored the item's Q into TMEM
  uint64_t k_full[kStages];
  uint64_t v_full[kStages];
  // K stage, S buffer and V stage of tile g are all index g % 2 (kStages == 2):
  uint64_t s_full[2];           // QK(g) done: scores in S buffer g % 2, K stage g % 2 free
  uint64_t p_full[2];           // the 8 softmax warps stored P of tile g over S buffer g % 2
  uint64_t pv_done[2];          // PV(g) done: V stage and S buffer g % 2 free, O includes tile g
  uint64_t o_final;             // the item's last PV product has completed
  uint64_t o_free;              // the 8 softmax warps have read the item's O
  uint64_t drain;               // both issuers' products have completed
  uint32_t tmem_base;
  int abort_flag;
  float red_max[2][2][kBM];     // [tile parity][warpgroup][row]: half-row maxima
  float red_sum[2][kBM];        // [warpgroup][row]: half-row sums of an item
  int head_order[kMaxHeads];
  int head_nseg[kMaxHeads];
  int head_tiles[kMaxHeads];
  int seg_start[kMaxSegTable];
  int seg_end[kMaxSegTable];
};
static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory of one CTA");
static_assert(kStages == 2, "K/V stages share the index of the two S buffers");

struct Params {
  int64_t batch, heads, q_len, capacity, max_segments;
  const float* q;               // [B, H, Lq, D] fp32
  const int32_t* seg_starts;
  const int32_t* seg_ends;
  const int32_t* seg_counts;
  const int32_t* head_order;    // [heads] or null
  float* out;                   // [B, Lq, H * D] fp32
  unsigned int* status;
  float scale_log2;             // softmax_scale * log2(e)
  int qblocks;                  // ceil(Lq / 128)
  int n_items;                  // heads * batch * qblocks
  int seg_stride;
};

struct Item {
  int h, b, q0, n;  // head, batch row, first query row, key tiles
};

__device__ __forceinline__ Item decode_item(const Smem& sm, const Params& p, int item) {
  Item it;
  const int qb = item % p.qblocks;
  const int rb = item / p.qblocks;
  it.b = rb % static_cast<int>(p.batch);
  it.h = sm.head_order[rb / static_cast<int>(p.batch)];
  it.q0 = qb * kBM;
  it.n = sm.head_tiles[it.h];
  return it;
}

// 64 consecutive TMEM columns of this thread's lane, waited on inside the same asm.
__device__ __forceinline__ void tmem_ld_row64(uint32_t taddr, float (&x)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,"
      "%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,"
      "%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]),
        "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]),
        "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]),
        "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]),
        "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(r[i]);
}

// Row max of 64 scores: 8 independent chains of 3-input max.
__device__ __forceinline__ float row_max64(const float (&x)[64]) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = fmaxf(x[k], x[k + 8]);
#pragma unroll
  for (int i = 2; i < 8; i += 2) {
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = max3f(a[k], x[k + 8 * i], x[k + 8 * i + 8]);
  }
  return max3f(max3f(a[0], a[1], a[2]), max3f(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}

// fp32 -> tf32, round to nearest (ties away from zero); the low 13 bits of the result are zero.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_sm100_tf32_kernel(const __grid_constant__ CUtensorMap tm_ck,
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
  pdl_trigger();
  if (warp == kQkWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 8);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.k_full[b], 1);
      mbar_init(&sm.v_full[b], 1);
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b], 8);
      mbar_init(&sm.pv_done[b], 1);
    }
    mbar_init(&sm.o_final, 1);
    mbar_init(&sm.o_free, 8);
    mbar_init(&sm.drain, 2);
    fence_mbar_init();
  }
  pdl_wait();
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
      sm.head_tiles[h] = tiles + (Lq + kBN - 1) / kBN;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0 && blockIdx.x == 0)
      raise_status(p.status, HEATKV_DEVICE_BAD_SEGMENT);
    if (lane == 0) {
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

  if (warp == kKWarp || warp == kVWarp) {
    // ---------------------------------------------------------------- TMA producers
    const bool loads_k = warp == kKWarp;
    if (lane == 0) {
      uint32_t gx = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const Item it = decode_item(sm, p, item);
        const int bh = it.b * H + it.h;
        const int cur_row0 = bh * Lq;
        const int slab_row0 = static_cast<int>(int64_t(it.b) * p.capacity);
        TileCursor cur;
        cur.begin(sm, it.h, stride, 0);
        for (int j = 0; j < it.n; ++j, ++gx) {
          const int s = gx % kStages;
          uint64_t* full = loads_k ? &sm.k_full[s] : &sm.v_full[s];
          // the stage's previous tile (gx - 2) is done with: its QK (K) or its PV (V)
          uint64_t* empty = loads_k ? &sm.s_full[s] : &sm.pv_done[s];
          if (gx >= kStages &&
              !(ok = mbar_wait(empty, ((gx / kStages) - 1) & 1, abort_flag, p.status)))
            break;
          const int row = cur.current ? cur_row0 + cur.pos : slab_row0 + cur.pos;
          if (loads_k) {
            const CUtensorMap* m = cur.current ? &tm_ck : &tm_sk;
            mbar_arrive_expect_tx(full, kKTileBytes);
#pragma unroll
            for (int box = 0; box < 4; ++box)
              tma_load_2d(sm.k[s] + box * kKBox, m, box * 32, row, full);
          } else {
            const CUtensorMap* m = cur.current ? &tm_cv : &tm_sv;
            mbar_arrive_expect_tx(full, kVTileBytes);
            tma_load_2d(sm.v[s], m, 0, row, full);
            tma_load_2d(sm.v[s] + kVHalf, m, 64, row, full);
          }
          cur.next();
        }
      }
      if (!ok || *abort_flag) {
        // let every copy already issued land before the CTA's shared memory goes away
        for (uint32_t g = gx > kStages ? gx - kStages : 0; g < gx; ++g)
          mbar_drain(loads_k ? &sm.k_full[g % kStages] : &sm.v_full[g % kStages],
                     (g / kStages) & 1, p.status);
      }
    }
  } else if (warp == kQkWarp) {
    // ---------------------------------------------------------------- QK issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_tf32(kBM, kBN);
      uint32_t g = 0, qcnt = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const Item it = decode_item(sm, p, item);
        if (!(ok = mbar_wait(&sm.q_full, qcnt & 1, abort_flag, p.status))) break;
        ++qcnt;
        for (int j = 0; j < it.n; ++j, ++g) {
          const uint32_t b = g & 1u;
          if (!(ok = mbar_wait(&sm.k_full[b], (g >> 1) & 1, abort_flag, p.status))) break;
          // S buffer b last held P(g - 2): its PV must have completed
          if (g >= 2 && !(ok = mbar_wait(&sm.pv_done[b], ((g >> 1) - 1) & 1, abort_flag, p.status)))
            break;
          tc_fence_after();
          // S_b = Q K^T: A = Q from TMEM (8 tf32 columns per instruction), B = K tile, K-major
          // SW128: K step kk is 32 bytes into the 128-byte row of box kk / 4
          const uint32_t kbase = smem_u32(sm.k[b]);
          const uint32_t d = tmem + kColS + b * 128;
#pragma unroll
          for (int kk = 0; kk < kD / 8; ++kk) {
            const uint64_t bdesc = smem_desc_sw128(kbase + (kk / 4) * kKBox + (kk % 4) * 32, 16, 1024);
            umma_tf32_ts(d, tmem + kColQ + kk * 8, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&sm.s_full[b]);
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
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      const Item it = decode_item(sm, p, item);
      TileCursor cur;
      cur.begin(sm, it.h, stride, 0);
      for (int j = 0; j < it.n; ++j, ++g) {
        const uint32_t b = g & 1u;
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.v_full[b], (g >> 1) & 1, abort_flag, p.status));
        if (!ok) break;
        const int valid = cur.valid(Lq);
        if (valid < kBN) {
          uint8_t* base = sm.v[b];
          const int chunks = (kBN - valid) * 2 * 8;  // rows x halves x 16-byte chunks
          for (int i = lane; i < chunks; i += 32) {
            const int line = i / 8;
            const int row = valid + line / 2, half = line % 2;
            *reinterpret_cast<uint4*>(base + half * kVHalf + row * 128 + (i % 8) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          // the cleared rows are visible to the tensor core (async proxy)
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncwarp();
        if (lane == 0) {
          ok = mbar_wait(&sm.p_full[b], (g >> 1) & 1, abort_flag, p.status);
          if (ok && j == 0 && ocnt > 0) ok = mbar_wait(&sm.o_free, (ocnt - 1) & 1, abort_flag, p.status);
          if (ok) {
            tc_fence_after();
            // O += P V: A = P (16-bit pairs over S_b), B = V tile, MN-major SW128: 8-key groups
            // 1 KiB apart (SBO), the two 64-column halves 16 KiB apart (LBO)
            const uint32_t vbase = smem_u32(sm.v[b]);
            const uint32_t a = tmem + kColS + b * 128;
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, kVHalf, 1024);
              umma_ts(tmem + kColO, a + kk * 8, bdesc, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
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
  } else {
    // ---------------------------------------------------------------- softmax warpgroups
    const int w = warp / 4;            // key half [64w, 64w + 64) of every tile
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // TMEM lane == query row
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tQ = tmem + lane_off + kColQ + 64 * w;
    const uint32_t tO = tmem + lane_off + kColO + 64 * w;
    const float c = p.scale_log2;
    // Q rows of an item -> TMEM (tf32), zero past Lq; then one arrive per warp
    auto load_q = [&](int item) {
      const Item it = decode_item(sm, p, item);
      const int qr = it.q0 + row;
      uint32_t lo[32], hi[32];
      if (qr < Lq) {
        const float4* src = reinterpret_cast<const float4*>(
            p.q + ((int64_t(it.b) * H + it.h) * Lq + qr) * kD + 64 * w);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 v = __ldg(src + i);
          uint32_t* d = i < 8 ? lo + 4 * i : hi + 4 * (i - 8);
          d[0] = to_tf32(v.x);
          d[1] = to_tf32(v.y);
          d[2] = to_tf32(v.z);
          d[3] = to_tf32(v.w);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) lo[i] = hi[i] = 0u;
      }
      tmem_st32(tQ, lo);
      tmem_st32(tQ + 32, hi);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_full);
    };
    uint32_t g = 0, ocnt = 0;
    bool ok = true;
    if (static_cast<int>(blockIdx.x) < p.n_items) load_q(blockIdx.x);
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x) {
      const Item it = decode_item(sm, p, item);
      float m_run = -INFINITY;
      float l_run = 0.f;
      const bool row_live = it.q0 + row < Lq;
      TileCursor cur;
      cur.begin(sm, it.h, stride, 0);
      // Every warp of both warpgroups takes the same named barriers in the same order, including
      // after an abort (the work is skipped, the barriers are not).
      for (int j = 0; j < it.n; ++j) {
        const uint32_t gj = g + j;
        const uint32_t buf = gj & 1u;
        const uint32_t tS = tmem + lane_off + kColS + buf * 128;
        const int valid = cur.valid(Lq);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[buf], (gj >> 1) & 1, abort_flag, p.status));
        float x[64];
        float mx = -INFINITY;
        if (ok) {
          tc_fence_after();
          tmem_ld_row64(tS + 64 * w, x);
          if (valid < kBN) {
#pragma unroll
            for (int i = 0; i < 64; ++i) x[i] = (64 * w + i < valid) ? x[i] : -INFINITY;
          }
          mx = row_max64(x) * c;
        }
        sm.red_max[buf][w][row] = mx;
        // the other warpgroup's scores are in its registers before P is stored over them
        tc_fence_before();
        named_bar_softmax();
        tc_fence_after();
        mx = fmaxf(mx, sm.red_max[buf][w ^ 1][row]);
        if (ok) {
          // Lazy max, as in the 16-bit kernel: the running max only moves when a tile exceeds it
          // by more than 8 (a factor 256 in P); both warpgroups see the same maxima and take the
          // same decision for every row.
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
          for (int half = 0; half < 2; ++half) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int pi = half * 16 + i;  // pair of columns 2pi, 2pi+1 of this half
              const uint64_t y = fma2(f2pack(x[2 * pi], x[2 * pi + 1]), c2, nm2);
              float y0, y1;
              f2unpack(y, y0, y1);
              const float p0 = ex2(y0);
              const float p1 = ex2(y1);
              acc[pi & 3] = add2(acc[pi & 3], f2pack(p0, p1));
              pk[i] = pack2<kBF16>(p0, p1);
            }
            // P of keys [64w, 64w + 64) -> 16-bit pair columns [32w, 32w + 32) of the buffer
            tmem_st16(tS + 32 * w + 16 * half, pk);
          }
          const uint64_t s01 = add2(acc[0], acc[1]);
          const uint64_t s23 = add2(acc[2], acc[3]);
          float u0, u1;
          f2unpack(add2(s01, s23), u0, u1);
          l_run += u0 + u1;
          if (rescale) {  // warp-uniform; O must hold PV(j-1) first
            ok = __all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(gj - 1) & 1u], ((gj - 1) >> 1) & 1,
                                                   abort_flag, p.status));
            if (ok) {
              tc_fence_after();
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
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
          if (lane == 0) mbar_arrive(&sm.p_full[buf]);
        }
        cur.next();
      }
      g += it.n;
      // the item's last QK has completed (its scores were read): stage the next item's Q now, so
      // its first QK overlaps this item's last PV and the epilogue
      const int next = item + gridDim.x;
      if (ok && next < p.n_items) load_q(next);
      sm.red_sum[w][row] = l_run;
      named_bar_softmax();
      const float l_tot = sm.red_sum[0][row] + sm.red_sum[1][row];
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.o_final, ocnt & 1, abort_flag, p.status));
      if (ok) {
        tc_fence_after();
        const int qrow = it.q0 + row;
        const float inv = 1.f / l_tot;
        float* dst = p.out + ((int64_t(it.b) * Lq + qrow) * H + it.h) * kD + 64 * w;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          float o[16];
          tmem_ld16_sync(tO + cc * 16, o);
          if (qrow < Lq) {
            float4* d4 = reinterpret_cast<float4*>(dst + cc * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              d4[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv,
                                  o[4 * i + 3] * inv);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_free);
      }
      ++ocnt;
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

}  // namespace tf32
}  // namespace sm100

cudaError_t launch_attention_sm100_tf32(const AttnArgs& a, bool v_bf16, cudaStream_t st) {
  using namespace sm100;
  using namespace sm100::tf32;
  const int64_t cur_rows = a.batch * a.heads * a.q_len;
  const int64_t slab_rows = a.batch * a.capacity;
  if (cur_rows >= (int64_t(1) << 31) || slab_rows >= (int64_t(1) << 31) ||
      a.heads > kMaxHeads || a.heads * std::max<int64_t>(a.max_segments, 1) > kMaxSegTable ||
      !(a.scale > 0.f) || a.n_out > 0)
    return cudaErrorNotSupported;
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.cur_k) |
                          reinterpret_cast<uintptr_t>(a.cur_v) |
                          reinterpret_cast<uintptr_t>(a.slab_k) |
                          reinterpret_cast<uintptr_t>(a.slab_v) | reinterpret_cast<uintptr_t>(a.out);
  if (align & 15u) return cudaErrorNotSupported;
  const int qblocks = static_cast<int>((a.q_len + kBM - 1) / kBM);
  const int64_t n_items = a.batch * a.heads * qblocks;
  if (n_items >= (int64_t(1) << 31)) return cudaErrorNotSupported;
  CUtensorMap tck, tcv, tsk, tsv;
  const bool slab = a.capacity > 0;
  if (!encode_rows_f32(&tck, a.cur_k, cur_rows) || !encode_rows(&tcv, a.cur_v, cur_rows, v_bf16) ||
      !encode_rows_f32(&tsk, slab ? a.slab_k : a.cur_k, slab ? slab_rows : cur_rows) ||
      !encode_rows(&tsv, slab ? a.slab_v : a.cur_v, slab ? slab_rows : cur_rows, v_bf16))
    return cudaErrorInvalidValue;
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
  p.out = static_cast<float*>(a.out);
  p.status = a.status;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.qblocks = qblocks;
  p.n_items = static_cast<int>(n_items);
  p.seg_stride = static_cast<int>(std::max<int64_t>(a.max_segments, 1));
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  using Kern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, Params);
  const Kern kern = v_bf16 ? attn_sm100_tf32_kernel<true> : attn_sm100_tf32_kernel<false>;
  // opt in to >48 KiB dynamic shared memory once per device (never inside a graph capture)
  static std::atomic<uint64_t> configured[2] = {{0}, {0}};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured[v_bf16].load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[v_bf16].fetch_or(bit);
  }
  const int grid = static_cast<int>(std::min<int64_t>(n_items, sm_count()));
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), static_cast<size_t>(smem), st, tck, tcv, tsk,
                 tsv, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace heatkv
