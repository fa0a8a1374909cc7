// The QKV projection with the q/k/v preparation and the cache append in its epilogue, on
// Blackwell tensor cores.
//
// The patched attention forward computes, per call (enable_real_pruning_fast.py:2040-2072 and the
// append of :2218-2225):
//   qkv = x @ W^T + bias              x [M = batch * seq_len, C], W [3 * H * 128, C] (nn.Linear),
//                                     bias = cat(q_bias, 0, v_bias) or none
//   q, k, v = qkv.view(B, L, 3, H, 128) permuted to [B, H, L, 128]
//   q = normalize(q) * scale_mul[h], k = normalize(k)          (cos-attention, fp32)
//   q, k = 2-D rotary embedding (infinity/models/basic.py:97-117, fp32)
// then appends k and v of the scale into the layer's cache. This kernel does all of it in one
// pass: the GEMM accumulates in TMEM, and the epilogue turns each accumulator row into the
// prepared q/k/v rows, written once, plus the cache rows of the heads given an offset (the dense
// cache before a layer's first pruned target, or the slab heads whose segment no live segment of
// the scale overlaps). The projection output is rounded to x's 16-bit type first, as the unfused
// path stores it, and the preparation then follows heatkv_qkv_prepare's arithmetic (fp32 norm,
// separately rounded rotary products) except that x / max(norm, eps) is taken as x times the
// correctly rounded reciprocal (one fp32 rounding step at most). Those and the summation order of
// the GEMM and of the row norm are the only differences from the unfused path.
//
// Tiles are 256 rows x 256 columns (two heads of one of q, k, v) over K steps of 64, each computed
// by a cluster of two CTAs on two SMs with tcgen05.mma.cta_group::2 (the protocol is described
// above qkv_project_pair_kernel); a persistent grid of pairs walks the tiles row panel by row panel
// (the 24 column tiles of a panel run on neighbouring pairs, so the x panel is read from HBM once
// and the weight stays in L2). CTA (384 threads, 1 per SM): warp 0 issues the TMA loads of a
// 6-stage ring (this CTA's 128 rows of x and of W per stage, 128-byte swizzle); warp 1 allocates
// TMEM (two 256-column accumulators) and, in the leader, issues the MMAs; warps 4-11 are the
// epilogue, one TMEM lane (accumulator row) and one head block per thread, two warps per SM
// sub-partition, working on one accumulator while the MMAs fill the other. Every wait is bounded;
// on expiry the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains its copies and MMAs, frees TMEM and
// returns.
#include "attn.h"
#include "common.cuh"
#include "sm100_util.cuh"

namespace heatkv {
namespace sm100 {
namespace qkvproj {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kThreads = 384;
constexpr int kLoadWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 4;    // warps 4-11: epilogue; warp 4 + 4 j + q reads TMEM lanes
constexpr int kEpiWarps = 8;    // [32 q, +32) of head block j (two warps per SM sub-partition)
constexpr uint32_t kTmemCols = 512;           // two 256-column accumulators

struct Params {
  int64_t rows;          // M = batch * seq_len
  int64_t seq_len;
  int64_t heads;         // local heads H (output columns 3 * H * 128)
  int k_blocks;          // C / 64
  int n_tiles;           // 3 * H * 128 / 256
  int tiles;             // ceil(M / 128) * n_tiles
  void* q;
  void* k;
  void* v;
  const float* bias;     // [3 * H * 128] fp32, or null
  const float* scale_mul;
  float eps;
  const float* rope_cos;  // pair-group-major: pairs 4g..4g+3 of token l at (g * stride + l) * 4
  const float* rope_sin;
  int64_t rope_stride;    // floats between consecutive pair groups
  void* cache_k;
  void* cache_v;
  int64_t cache_rows;
  const int64_t* cache_offset;
  unsigned int* status;
  int align32;           // q, k, v and the caches 32-byte aligned: 32-byte stores
};

// x[i] += bias[i] for 64 columns (fp32 add, as the GEMM's bias epilogue does before rounding)
__device__ __forceinline__ void add_bias64(const float4* bias, float (&x)[64]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float4 b = __ldg(bias + j);
    x[4 * j] += b.x;
    x[4 * j + 1] += b.y;
    x[4 * j + 2] += b.z;
    x[4 * j + 3] += b.w;
  }
}

template <bool kBF16>
__device__ __forceinline__ float round16(float x) {
  if constexpr (kBF16) return __bfloat162float(__float2bfloat16_rn(x));
  else return __half2float(__float2half_rn(x));
}

// The epilogue of one 128-column head block of this thread's accumulator row: add the bias, round
// to the projection dtype, prepare (q/k), store the row and the cache row. The row is read from TMEM in
// two 64-column halves (twice for q/k with cos-attention: once for the norm, once to write), which
// keeps the live registers of the epilogue warps low. tcgen05.ld is warp-collective, so rows past
// the end still load and only skip their stores.
template <bool kBF16, bool kCos, bool kRope, bool kQK32>
__device__ __forceinline__ void head_block(const Params& p, uint32_t taddr, int64_t m, int col0) {
  const bool live = m < p.rows;
  const int64_t mm = live ? m : 0;
  const int64_t H = p.heads;
  const int64_t C = H * 128;
  const int sec = static_cast<int>(col0 / C);          // 0 q, 1 k, 2 v
  const int64_t h = (col0 % C) / 128;
  const int64_t b = mm / p.seq_len, l = mm % p.seq_len;
  const bool prep = sec < 2;
  const float4* bias = p.bias != nullptr ? reinterpret_cast<const float4*>(p.bias + col0) : nullptr;
  float inv_scale = 1.f, n = 1.f;
  if (kCos && prep) {
    float ss = 0.f;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      float x[64];
      tmem_ld_row64(taddr + half * 64, x);
      if (bias != nullptr) add_bias64(bias + half * 16, x);
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float r = round16<kBF16>(x[i]);
        ss = fmaf(r, r, ss);
      }
    }
    n = fmaxf(sqrtf(ss), p.eps);
    // one correctly rounded reciprocal per row, then products: within one fp32 rounding of
    // x / n, far below the 16-bit rounding of the result
    n = __frcp_rn(n);
    inv_scale = sec == 0 ? __ldg(p.scale_mul + h) : 1.f;
  }
  // q and k as fp32 (the reference's chain under autocast normalises and rotates in fp32) or in
  // the 16-bit dtype; v always in the 16-bit dtype. Row bytes: 128 elements of esz bytes.
  const bool f32out = kQK32 && prep;
  const int64_t esz = f32out ? 4 : 2;
  uint8_t* outb = static_cast<uint8_t*>(sec == 0 ? p.q : sec == 1 ? p.k : p.v);
  uint8_t* dstb = outb + ((b * H + h) * p.seq_len + l) * 128 * esz;
  uint8_t* cdb = nullptr;
  if (live && sec >= 1 && p.cache_offset != nullptr) {
    const int64_t off = __ldg(p.cache_offset + h);
    if (off >= 0) {
      if (off > p.cache_rows - p.seq_len) {
        if (l == 0) raise_status(p.status, HEATKV_DEVICE_PACK_OUT_OF_RANGE);
      } else {
        uint8_t* cache = static_cast<uint8_t*>(sec == 1 ? p.cache_k : p.cache_v);
        cdb = cache + (b * p.cache_rows + off + l) * 128 * esz;
      }
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(dstb);
  uint4* cd = reinterpret_cast<uint4*>(cdb);
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float x[64];
    tmem_ld_row64(taddr + half * 64, x);
    if (bias != nullptr) add_bias64(bias + half * 16, x);
#pragma unroll
    for (int i = 0; i < 64; ++i) x[i] = round16<kBF16>(x[i]);
    if (kCos && prep) {
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        x[i] = __fmul_rn(x[i], n);
        if (sec == 0) x[i] = __fmul_rn(x[i], inv_scale);
      }
    }
    if (kRope && prep) {
      // pair-group-major tables: the 32 lanes (consecutive tokens) of a warp load 512 contiguous
      // bytes per group, where a token-major table made every load touch 32 cache lines
      const float* cbase = p.rope_cos + l * 4 + int64_t(half) * 8 * p.rope_stride;
      const float* sbase = p.rope_sin + l * 4 + int64_t(half) * 8 * p.rope_stride;
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // pairs 4j .. 4j + 3 of this half
        const float4 c = __ldg(reinterpret_cast<const float4*>(cbase + j * p.rope_stride));
        const float4 s = __ldg(reinterpret_cast<const float4*>(sbase + j * p.rope_stride));
        const float cc[4] = {c.x, c.y, c.z, c.w}, sc[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 4 * j + e;
          const float a0 = x[2 * i], a1 = x[2 * i + 1];
          x[2 * i] = __fsub_rn(__fmul_rn(cc[e], a0), __fmul_rn(sc[e], a1));
          x[2 * i + 1] = __fadd_rn(__fmul_rn(sc[e], a0), __fmul_rn(cc[e], a1));
        }
      }
    }
    if (live && f32out) {
      // 64 fp32 values = 256 bytes of this half's row
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = __float_as_uint(x[8 * j + e]);
        if (p.align32) {
          st_global_v8(dstb + half * 256 + j * 32, w);
          if (cdb != nullptr) st_global_v8(cdb + half * 256 + j * 32, w);
        } else {
          dst[half * 16 + 2 * j] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[half * 16 + 2 * j + 1] = make_uint4(w[4], w[5], w[6], w[7]);
          if (cd != nullptr) {
            cd[half * 16 + 2 * j] = make_uint4(w[0], w[1], w[2], w[3]);
            cd[half * 16 + 2 * j + 1] = make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
      }
    } else if (live && p.align32) {
      // one full 32-byte sector per store (each thread writes its own row)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = pack2<kBF16>(x[16 * j + 2 * e], x[16 * j + 2 * e + 1]);
        st_global_v8(dst + half * 8 + 2 * j, w);
        if (cdb != nullptr) st_global_v8(cd + half * 8 + 2 * j, w);
      }
    } else if (live) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 w = make_uint4(pack2<kBF16>(x[8 * j], x[8 * j + 1]),
                                   pack2<kBF16>(x[8 * j + 2], x[8 * j + 3]),
                                   pack2<kBF16>(x[8 * j + 4], x[8 * j + 5]),
                                   pack2<kBF16>(x[8 * j + 6], x[8 * j + 7]));
        dst[half * 8 + j] = w;
        if (cdb != nullptr) cd[half * 8 + j] = w;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs on two SMs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 M=256 N=256 K=16. Each CTA loads its own 128 rows of x and its own 128
// rows of W per K step (every load copies this GPU's memory into the loading CTA's own shared
// memory), so an SM receives 32 KiB of operands per 512 tensor cycles instead of 48 KiB:
// one CTA alone with a 128 x 256 tile needs 96 B per cycle from L2, more than it gets, and ran at
// ~70 % of the tensor rate. The even CTA of the pair (the leader) issues the MMAs, which read both
// CTAs' shared memory and write each CTA's 128 accumulator rows into its own TMEM. Protocol:
//   * both CTAs' TMA loads of a stage complete on the leader's full[s] barrier (the leader posts
//     the transaction bytes of both); the MMA's stage release is committed to empty[s] of both
//     CTAs (tcgen05.commit multicast), so each producer reuses its own stage;
//   * the accumulator completion is committed to acc_full[a] of both CTAs; each CTA's epilogue
//     warps arrive on the leader's acc_empty[a] (8 arrivals) when they have read it;
//   * TMEM is allocated and freed with cta_group::2 by one warp of each CTA; cluster barriers
//     after the set-up and before the exit keep either CTA from running ahead of its peer's
//     barriers or freeing memory its peer still uses.
// ------------------------------------------------------------------------------------------------
constexpr int kPairStages = 6;
constexpr uint32_t kPairABytes = 128 * kBK * 2;   // this CTA's 128 rows of x, 16 KiB
constexpr uint32_t kPairBBytes = 128 * kBK * 2;   // this CTA's 128 rows of W, 16 KiB

struct __align__(1024) PairSmem {
  uint8_t a[kPairStages][kPairABytes];
  uint8_t b[kPairStages][kPairBBytes];
  uint64_t full[kPairStages];
  uint64_t empty[kPairStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion counts on the mbarrier at
// `bar_cluster_addr`, which may be the peer CTA's (cta_group::2).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int c0,
                                                 int c1, uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster_addr)
      : "memory");
}
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at this shared offset in both CTAs once the issued MMAs complete
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)), "h"(static_cast<uint16_t>(3))
      : "memory");
}

template <bool kBF16, bool kCos, bool kRope, bool kQK32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    qkv_project_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                            const __grid_constant__ CUtensorMap tm_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  PairSmem& sm = *reinterpret_cast<PairSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x / 2), npairs = static_cast<int>(gridDim.x / 2);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 2 * kEpiWarps);   // the epilogue warps of both CTAs
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (warp == kLoadWarp && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  pdl_trigger();
  tc_fence_before();
  cluster_sync_all();   // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  pdl_wait();
  const uint32_t tmem = sm.tmem_base;
  const int KB = p.k_blocks;
  const int m_tiles = static_cast<int>((p.rows + 255) / 256);
  const int tiles = m_tiles * p.n_tiles;

  if (warp == kLoadWarp) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += npairs) {
        const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % kPairStages;
          if (it >= kPairStages &&
              !(ok = mbar_wait(&sm.empty[s], ((it / kPairStages) - 1) & 1, abort_flag, p.status)))
            break;
          if (leader) mbar_arrive_expect_tx(&sm.full[s], 2 * (kPairABytes + kPairBBytes));
          const uint32_t bar = peer_addr(&sm.full[s], 0);
          tma_load_2d_pair(sm.a[s], &tm_x, kb * kBK, mt * 256 + static_cast<int>(rank) * 128, bar);
          tma_load_2d_pair(sm.b[s], &tm_w, kb * kBK, nt * kBN + static_cast<int>(rank) * 128, bar);
        }
      }
      if (leader && (!ok || *abort_flag)) {
        // the leader's full barriers count both CTAs' copies: wait for all issued ones to land
        for (uint32_t g = it > kPairStages ? it - kPairStages : 0; g < it; ++g)
          mbar_drain(&sm.full[g % kPairStages], (g / kPairStages) & 1, p.status);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16(kBF16, 256, kBN, false, false);
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += npairs, ++tcount) {
        const uint32_t acc = tcount % 2;
        if (tcount >= 2 &&
            !(ok = mbar_wait(&sm.acc_empty[acc], ((tcount / 2) - 1) & 1, abort_flag, p.status)))
          break;
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % kPairStages;
          if (!(ok = mbar_wait(&sm.full[s], (it / kPairStages) & 1, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t abase = smem_u32(sm.a[s]);
          const uint32_t bbase = smem_u32(sm.b[s]);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_ss_pair(tmem + acc * kBN, smem_desc_sw128(abase + kk * 32, 16, 1024),
                         smem_desc_sw128(bbase + kk * 32, 16, 1024), idesc,
                         (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit_pair(&sm.empty[s]);
        }
        if (ok) tc_commit_pair(&sm.acc_full[acc]);
      }
      // every MMA issued here has completed once `drain` fires (a cta_group::2 commit: the kernel
      // uses one CTA-group width for all its tcgen05 operations)
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   ::"r"(smem_u32(&sm.drain)) : "memory");
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else if (warp >= kEpiWarp0) {
    const int quarter = (warp - kEpiWarp0) % 4;
    const int hb = (warp - kEpiWarp0) / 4;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t tcount = 0;
    bool ok = true;
    for (int tile = pair; tile < tiles; tile += npairs, ++tcount) {
      const uint32_t acc = tcount % 2;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&sm.acc_full[acc], (tcount / 2) & 1, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
      const int64_t m = int64_t(mt) * 256 + rank * 128 + quarter * 32 + lane;
      head_block<kBF16, kCos, kRope, kQK32>(p, tmem + lane_off + acc * kBN + hb * 128, m,
                                     nt * kBN + hb * 128);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(peer_addr(&sm.acc_empty[acc], 0));
    }
  }
  tc_fence_before();
  cluster_sync_all();   // the peer is done with this CTA's memory and TMEM
  tc_fence_after();
  if (warp == kMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
}

// rows x cols 16-bit matrix, box 64 columns x box_rows rows, 128-byte swizzle
bool encode_matrix(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, bool bf16,
                   int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool kBF16, bool kCos, bool kRope, bool kQK32>
cudaError_t launch_pair_t(const CUtensorMap& tx, const CUtensorMap& tw, const Params& p, int grid,
                          cudaStream_t st) {
  auto kern = qkv_project_pair_kernel<kBF16, kCos, kRope, kQK32>;
  const size_t smem = sizeof(PairSmem) + 1024;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, st, tx, tw, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace qkvproj
}  // namespace sm100

cudaError_t launch_qkv_project(const void* x, const void* w, const float* bias, void* q, void* k,
                               void* v, bool bf16, bool qk32, int64_t batch, int64_t seq_len, int64_t heads,
                               int64_t embed_dim, const float* scale_mul, float eps,
                               const float* rope_cos, const float* rope_sin,
                               int64_t rope_group_stride, void* cache_k, void* cache_v,
                               int64_t cache_rows, const int64_t* cache_offset,
                               unsigned int* status, cudaStream_t st) {
  using namespace sm100::qkvproj;
  CUtensorMap tx, tw;
  const int64_t M = batch * seq_len;
  // each CTA of a pair loads 128 rows of x and 128 rows of W per K step
  if (!encode_matrix(&tx, x, M, embed_dim, bf16, kBM) ||
      !encode_matrix(&tw, w, 3 * heads * 128, embed_dim, bf16, 128))
    return cudaErrorInvalidValue;
  Params p{};
  p.rows = M;
  p.seq_len = seq_len;
  p.heads = heads;
  p.k_blocks = static_cast<int>(embed_dim / kBK);
  p.n_tiles = static_cast<int>(3 * heads * 128 / kBN);
  p.tiles = static_cast<int>((M + kBM - 1) / kBM) * p.n_tiles;
  p.q = q;
  p.k = k;
  p.v = v;
  p.bias = bias;
  p.scale_mul = scale_mul;
  p.eps = eps;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.rope_stride = rope_group_stride;
  p.cache_k = cache_k;
  p.cache_v = cache_v;
  p.cache_rows = cache_rows;
  p.cache_offset = cache_offset;
  p.status = status;
  p.align32 = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(cache_k) |
                reinterpret_cast<uintptr_t>(cache_v)) & 31u) == 0 ? 1 : 0;
  const bool cos = scale_mul != nullptr, rope = rope_cos != nullptr;
  const int64_t pair_tiles = (M + 255) / 256 * p.n_tiles;
  const int grid = 2 * static_cast<int>(std::min<int64_t>(pair_tiles, sm100::sm_count() / 2));
#define HEATKV_QKV_PROJ_PAIR(B, Q)                                                   \
  (cos && rope ? launch_pair_t<B, true, true, Q>(tx, tw, p, grid, st)                \
   : cos       ? launch_pair_t<B, true, false, Q>(tx, tw, p, grid, st)               \
   : rope      ? launch_pair_t<B, false, true, Q>(tx, tw, p, grid, st)               \
               : launch_pair_t<B, false, false, Q>(tx, tw, p, grid, st))
  if (qk32)
    return bf16 ? HEATKV_QKV_PROJ_PAIR(true, true) : HEATKV_QKV_PROJ_PAIR(false, true);
  return bf16 ? HEATKV_QKV_PROJ_PAIR(true, false) : HEATKV_QKV_PROJ_PAIR(false, false);
#undef HEATKV_QKV_PROJ_PAIR
}

}  // namespace heatkv
