// S-CAS accumulation on the tensor cores: per-(head, source scale) attention mass of one scale's
// queries with fp32-accurate scores from three tf32 products.
//
// tools/compute_scas.py:217-218 computes scores = q.float() @ k.float()^T * scale in fp32 and
// probs = softmax(scores); ScasAccumulator.update (:114-128) adds, for each source scale s,
//   mass[h][s] = mean over the queries of sum over the keys of scale s of probs.
// scas.cu does this on CUDA cores with fp32 products. Here the products run as kind::tf32 MMAs
// with each operand split into a tf32 head and an fp32 remainder (x = hi + lo, hi = x rounded to
// tf32, lo = x - hi exactly):
//   S = Q_lo K_hi^T + Q_hi K_lo^T + Q_hi K_hi^T
// (the smaller products first); the dropped Q_lo K_lo^T term and the tf32 reading of the
// remainders are below 2^-21 of each product, the size of fp32 rounding itself.
//
// Item = (head, 128-row query block); a persistent grid of one CTA per SM runs items c, c + grid,
// ... Per item the statistics warps stage Q_hi | Q_lo into TMEM (the MMAs' A operand); per 64-key
// tile the TMA warp loads fp32 K into shared memory, the split warps leave K_hi in place and write
// K_lo beside it, the MMA thread issues the 48 MMAs into one of two S buffers, and the statistics
// warps (one TMEM lane = query row per thread) run the online softmax with one running partial
// sum per source scale (rescaled with the row sum whenever the row max rises, as scas.cu). At the
// end of the item every row's partials are divided by its row sum, summed over each warp's rows in
// float64 and added to mass_out[h * mass_stride + s] (float64 atomics) divided by q_len.
//
// CTA (320 threads, 1 per SM): warps 0-3 statistics, warps 4-7 K split, warp 8 TMA, warp 9 TMEM
// allocation and MMA issue. TMEM: Q_hi [0, 128), Q_lo [128, 256), S_0 [256, 320), S_1 [320, 384).
// Every wait is bounded; on expiry the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains its copies
// and MMAs, frees TMEM and returns.
#include "attn.h"
#include "common.cuh"
#include "sm100_util.cuh"

#include <cmath>

namespace heatkv {
namespace sm100 {
namespace scastc {

constexpr int kBM = 128;                 // query rows per item
constexpr int kBN = 64;                  // keys per tile
constexpr int kD = 128;
constexpr uint32_t kBox = kBN * 128;     // one 32-column fp32 box of a K tile: 64 rows x 128 B
constexpr uint32_t kTile = 4 * kBox;     // 64 keys x 128 fp32 = 32 KiB
constexpr int kStages = 2;
constexpr int kNumS = 2;
constexpr uint32_t kColQh = 0, kColQl = 128, kColS = 256;
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxSrc = 32;
constexpr int kPartStride = kMaxSrc + 1;  // odd stride: a warp's rows fall in different banks
constexpr int kThreads = 320;
constexpr int kStatWarps = 4;
constexpr int kSplitWarp0 = 4;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;

struct __align__(1024) Smem {
  uint8_t khi[kStages][kTile];  // TMA lands fp32 K here; the split leaves tf32(K) in place
  uint8_t klo[kStages][kTile];  // K - tf32(K), same swizzled layout
  float part[kBM][kPartStride];
  int bounds[kMaxSrc + 1];
  uint64_t k_full[kStages];     // K tile landed
  uint64_t k_split[kStages];    // hi / lo written (4 split warps)
  uint64_t k_empty[kStages];    // MMAs of the stage completed
  uint64_t s_full[kNumS];       // scores of tile g in S buffer g % 2
  uint64_t s_free[kNumS];       // the statistics warps have read them (4 warps)
  uint64_t q_full;              // Q_hi | Q_lo in TMEM (4 warps)
  uint64_t q_empty;             // the item's last MMAs completed
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct Params {
  const float* q;        // [heads, q_len, 128]
  int64_t heads, q_len, k_len;
  float scale;
  int n_src;
  int qblocks;
  int n_items;
  int ntiles;
  double* mass_out;
  int64_t mass_stride;
  unsigned int* status;
};

// x rounded to tf32 (10-bit mantissa), as an fp32 value whose low 13 bits are zero
__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ uint64_t kdesc(uint32_t base, int kk) {
  // K-major SW128: a K step of 8 tf32 is 32 bytes into the 128-byte rows of its 32-column box
  return smem_desc_sw128(base + (kk / 4) * kBox + (kk % 4) * 32, 16, 1024);
}

__global__ void __launch_bounds__(kThreads, 1)
    scas_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const Params p,
                   const int32_t* __restrict__ bounds) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  volatile int* abort_flag = &sm.abort_flag;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_split[s], 4);
      mbar_init(&sm.k_empty[s], 1);
    }
    for (int b = 0; b < kNumS; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.s_free[b], kStatWarps);
    }
    mbar_init(&sm.q_full, kStatWarps);
    mbar_init(&sm.q_empty, 1);
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) tma_prefetch_desc(&tm_k);
  pdl_wait();
  for (int i = threadIdx.x; i <= p.n_src; i += kThreads) sm.bounds[i] = bounds[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int ntiles = p.ntiles;

  if (warp == kTmaWarp) {
    // ---------------------------------------------------------------- TMA of fp32 K tiles
    if (lane == 0) {
      uint32_t gx = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const int h = item / p.qblocks;
        for (int j = 0; j < ntiles; ++j, ++gx) {
          const int s = gx % kStages;
          if (gx >= kStages &&
              !(ok = mbar_wait(&sm.k_empty[s], ((gx / kStages) - 1) & 1, abort_flag, p.status)))
            break;
          // rows past this head's keys belong to the next head (masked by the statistics) or
          // lie past the tensor (zero-filled)
          const int row = static_cast<int>(h * p.k_len) + j * kBN;
          mbar_arrive_expect_tx(&sm.k_full[s], kTile);
#pragma unroll
          for (int bx = 0; bx < 4; ++bx)
            tma_load_2d(sm.khi[s] + bx * kBox, &tm_k, bx * 32, row, &sm.k_full[s]);
        }
      }
      if (!ok || *abort_flag) {
        for (uint32_t g = gx > kStages ? gx - kStages : 0; g < gx; ++g)
          mbar_drain(&sm.k_full[g % kStages], (g / kStages) & 1, p.status);
      }
    }
  } else if (warp >= kSplitWarp0 && warp < kSplitWarp0 + 4) {
    // ---------------------------------------------------------------- K = hi + lo
    const int t = threadIdx.x - kSplitWarp0 * 32;
    uint32_t g = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      for (int j = 0; j < ntiles; ++j, ++g) {
        const int s = g % kStages;
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&sm.k_full[s], (g / kStages) & 1, abort_flag, p.status));
        if (!ok) break;
        // element-wise, so the swizzled layout carries over to the remainder unchanged
        float4* hi = reinterpret_cast<float4*>(sm.khi[s]);
        float4* lo = reinterpret_cast<float4*>(sm.klo[s]);
#pragma unroll 4
        for (int i = t; i < static_cast<int>(kTile / 16); i += 128) {
          const float4 v = hi[i];
          const float4 a = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
          hi[i] = a;
          lo[i] = make_float4(v.x - a.x, v.y - a.y, v.z - a.z, v.w - a.w);
        }
        // generic-proxy writes, read by the tensor core through the async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.k_split[s]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, kBN);
      uint32_t g = 0, qcnt = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        if (!(ok = mbar_wait(&sm.q_full, qcnt & 1, abort_flag, p.status))) break;
        ++qcnt;
        for (int j = 0; j < ntiles; ++j, ++g) {
          const int s = g % kStages;
          const uint32_t b = g % kNumS;
          if (!(ok = mbar_wait(&sm.k_split[s], (g / kStages) & 1, abort_flag, p.status))) break;
          if (g >= static_cast<uint32_t>(kNumS) &&
              !(ok = mbar_wait(&sm.s_free[b], ((g / kNumS) - 1) & 1, abort_flag, p.status)))
            break;
          tc_fence_after();
          const uint32_t d = tmem + kColS + b * kBN;
          const uint32_t hb = smem_u32(sm.khi[s]), lb = smem_u32(sm.klo[s]);
#pragma unroll
          for (int kk = 0; kk < kD / 8; ++kk)
            umma_tf32_ts(d, tmem + kColQl + kk * 8, kdesc(hb, kk), idesc, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < kD / 8; ++kk)
            umma_tf32_ts(d, tmem + kColQh + kk * 8, kdesc(lb, kk), idesc, 1u);
#pragma unroll
          for (int kk = 0; kk < kD / 8; ++kk)
            umma_tf32_ts(d, tmem + kColQh + kk * 8, kdesc(hb, kk), idesc, 1u);
          tc_commit(&sm.s_full[b]);
          tc_commit(&sm.k_empty[s]);
          if (j == ntiles - 1) tc_commit(&sm.q_empty);
        }
      }
      // every MMA issued has completed once `drain` fires
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else if (warp < kStatWarps) {
    // ---------------------------------------------------------------- statistics
    const int row = warp * 32 + lane;  // TMEM lane == query row
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    float* part = sm.part[row];
    uint32_t g = 0, qcnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      const int h = item / p.qblocks;
      const int64_t qr = int64_t(item % p.qblocks) * kBM + row;
      const bool live = qr < p.q_len;
      // Q_hi | Q_lo of this row into TMEM once the previous item's MMAs are done with Q
      if (qcnt > 0)
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&sm.q_empty, (qcnt - 1) & 1, abort_flag, p.status));
      if (!ok) break;
      ++qcnt;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t rh[32], rl[32];
        if (live) {
          const float4* src =
              reinterpret_cast<const float4*>(p.q + (int64_t(h) * p.q_len + qr) * kD + 32 * c);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 v = __ldg(src + i);
            const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a = tf32_hi(x[e]);
              rh[4 * i + e] = __float_as_uint(a);
              rl[4 * i + e] = __float_as_uint(x[e] - a);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) rh[i] = rl[i] = 0u;
        }
        tmem_st32(tmem + lane_off + kColQh + 32 * c, rh);
        tmem_st32(tmem + lane_off + kColQl + 32 * c, rl);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_full);
      for (int s = 0; s < p.n_src; ++s) part[s] = 0.f;
      float m_run = -INFINITY, l_run = 0.f;
      int src0 = 0;  // first source that can still meet a tile (tiles walk the keys in order)
      for (int j = 0; j < ntiles; ++j, ++g) {
        const uint32_t b = g % kNumS;
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&sm.s_full[b], (g / kNumS) & 1, abort_flag, p.status));
        if (!ok) break;
        tc_fence_after();
        float x[kBN];
        tmem_ld_row64(tmem + lane_off + kColS + b * kBN, x);
        // the scores are in registers: the S buffer is free for tile g + 2
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[b]);
        const int t0 = j * kBN;
        const int nvalid = static_cast<int>(min64(kBN, p.k_len - t0));
        // scores in base-2 units: exp(s * scale - m) = 2^(s * scale * log2(e) - m')
        const float c = p.scale * 1.4426950408889634f;
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          x[i] = i < nvalid ? x[i] * c : -INFINITY;
          mx = fmaxf(mx, x[i]);
        }
        // key 0 of every tile is valid, so mx is finite
        if (mx > m_run) {
          const float alpha = ex2(m_run - mx);  // 0 on the first tile
          l_run *= alpha;
          for (int s = 0; s < p.n_src; ++s) part[s] *= alpha;
          m_run = mx;
        }
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          x[i] = ex2(x[i] - m_run);
          sum += x[i];
        }
        l_run += sum;
        // this tile's share of every source it meets (sources are ascending key ranges)
        while (src0 < p.n_src && sm.bounds[src0 + 1] <= t0) ++src0;
        for (int s = src0; s < p.n_src && sm.bounds[s] < t0 + nvalid; ++s) {
          const int lo = sm.bounds[s] - t0, hi = sm.bounds[s + 1] - t0;
          float share = 0.f;
#pragma unroll
          for (int i = 0; i < kBN; ++i) share += (i >= lo && i < hi) ? x[i] : 0.f;
          part[s] += share;
        }
      }
      if (!ok) break;
      // masses: partial / row sum, summed over the warp's rows in float64, one atomic per
      // (warp, source)
      const double inv = live ? 1.0 / double(l_run) : 0.0;
      for (int s = 0; s < p.n_src; ++s) {
        double v = double(part[s]) * inv;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) atomicAdd(p.mass_out + int64_t(h) * p.mass_stride + s, v / double(p.q_len));
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

}  // namespace scastc
}  // namespace sm100

// The tensor-core S-CAS launch for fp32 q and k; cudaErrorNotSupported when these arguments are
// outside its limits (the caller then runs scas.cu).
cudaError_t launch_scas_mass_tc(const float* q, const float* k, int64_t heads, int64_t q_len,
                                int64_t k_len, float scale, const int32_t* bounds, int n_src,
                                double* mass_out, int64_t mass_stride, unsigned int* status,
                                cudaStream_t st) {
  using namespace sm100::scastc;
  if (n_src < 0 || n_src > kMaxSrc || heads <= 0 || q_len <= 0 || k_len <= 0 ||
      heads * k_len + kBN >= (int64_t(1) << 31) || heads * ((q_len + kBM - 1) / kBM) >= (1 << 30) ||
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & 15u))
    return cudaErrorNotSupported;
  auto enc = sm100::get_encode();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(heads * k_len)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD * 4)};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(kBN)};
  cuuint32_t elem[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(k), dims, strides, box, elem,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  Params p{};
  p.q = q;
  p.heads = heads;
  p.q_len = q_len;
  p.k_len = k_len;
  p.scale = scale;
  p.n_src = n_src;
  p.qblocks = static_cast<int>((q_len + kBM - 1) / kBM);
  p.n_items = static_cast<int>(heads * p.qblocks);
  p.ntiles = static_cast<int>((k_len + kBN - 1) / kBN);
  p.mass_out = mass_out;
  p.mass_stride = mass_stride;
  p.status = status;
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory of one CTA");
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    e = cudaFuncSetAttribute(scas_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  const int grid = static_cast<int>(std::min<int64_t>(p.n_items, sm100::sm_count()));
  e = launch_pdl(scas_tc_kernel, dim3(grid), dim3(kThreads), static_cast<size_t>(smem), st, tm, p,
                 bounds);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace heatkv
