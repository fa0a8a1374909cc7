// Segmented flat-slab attention on Blackwell tensor cores (sm_100a): TMA + tcgen05 + TMEM.
//
// Computes what _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// computes with its default bf16 dot modes: for batch row b and head h, the keys are the head's
// slab segments [start, end) in segment order followed by the current scale's K/V, softmax(q k^T *
// scale) with fp32 scores and fp32 row sums, P rounded to the value dtype for the PV product, fp32
// accumulation, output [B, Lq, H*D] in q's dtype.
//
// Design (one CTA per (b, h, 256 query rows), 1 CTA per SM):
//   * warp 8      : TMA producer. Q (two 128-row tiles) once, then K and V tiles of 128 keys into
//                   a 2-stage ring. A tile is 128 rows of one segment (or of the current scale);
//                   pruned scales have no segment and cost nothing. Rows past a segment's end are
//                   loaded but masked; rows past the tensor end are zero-filled by TMA.
//   * warp 9      : TMEM allocator and single-thread tcgen05.mma issuer.
//                   S_t = Q_t K^T (M=128, N=128, K=128, SS operands, K-major SW128) into TMEM,
//                   O_t += P_t V (A = P_t read from TMEM, B = V as an MN-major SW128 operand).
//                   Issue order per key tile j: PV_0(j-1), QK_0(j), PV_1(j-1), QK_1(j), so one Q
//                   tile's MMAs run while the other tile's softmax runs.
//   * warps 0-3, 4-7 : softmax warpgroups of Q tiles 0 and 1, one TMEM lane (query row) per
//                   thread. Scores are read from TMEM, masked past the tile's valid keys, and
//                   turned into P = exp2(s*scale*log2e - m) which is written back into TMEM over
//                   the scores (bf16/f16 pairs). The running max m is only raised when a tile's
//                   max exceeds it by more than 8 (factor 256); O in TMEM is then rescaled in
//                   place. The final O / l is written straight to global memory.
//   TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// Every wait is bounded (common.cuh); on expiry the CTA raises HEATKV_DEVICE_WAIT_TIMEOUT, drains
// its in-flight copies and MMAs, frees TMEM and returns.
#include "attn.h"
#include "common.cuh"

#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

namespace heatkv {

namespace sm100 {

constexpr int kBM = 128;        // query rows per Q tile
constexpr int kNQ = 2;          // Q tiles per CTA
constexpr int kBN = 128;        // keys per K/V tile
constexpr int kD = 128;         // head dim
constexpr int kStages = 2;      // K/V ring depth
constexpr int kThreads = 320;   // 10 warps
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kHalfBytes = kBM * 64 * 2;    // one 128-row x 64-column 16-bit box: 16 KiB
constexpr uint32_t kTileBytes = 2 * kHalfBytes;  // 128 x 128 x 2 bytes
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) Smem {
  uint8_t q[kNQ][kTileBytes];
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[kNQ];
  uint64_t p_full[kNQ];
  uint64_t o_final[kNQ];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int nseg;
  int ntiles;
  int seg_start[kMaxSegments];
  int seg_end[kMaxSegments];
};

struct Params {
  int64_t batch, heads, q_len, capacity, max_segments;
  const int32_t* seg_starts;
  const int32_t* seg_ends;
  const int32_t* seg_counts;
  void* out;
  float scale_log2;  // softmax_scale * log2(e)
  int qpairs;        // ceil(Lq / 256)
};

// Walks the key tiles of one head: each segment in 128-row steps, then the current scale.
struct TileCursor {
  int seg;
  int pos;
  bool current;
  __device__ void begin(const Smem& sm) {
    seg = 0;
    current = sm.nseg == 0;
    pos = current ? 0 : sm.seg_start[0];
  }
  __device__ int valid(const Smem& sm, int q_len) const {
    return current ? min(kBN, q_len - pos) : min(kBN, sm.seg_end[seg] - pos);
  }
  __device__ void next(const Smem& sm, int q_len) {
    pos += kBN;
    if (!current && pos >= sm.seg_end[seg]) {
      ++seg;
      if (seg < sm.nseg) {
        pos = sm.seg_start[seg];
      } else {
        current = true;
        pos = 0;
      }
    }
  }
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// 128 consecutive TMEM columns of this warp's 32 lanes, waited on inside the same asm so no use
// of the registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld128_sync(uint32_t taddr, float (&x)[128]) {
  uint32_t r[32];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr + c * 32)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(r[i]);
  }
}

__device__ __forceinline__ void tmem_ld32_sync(uint32_t taddr, float (&x)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(r[i]);
}

// A drain wait for the error path: bounded, ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles / 4) {
      raise_status(HEATKV_DEVICE_WAIT_TIMEOUT);
      return;
    }
  }
}

template <bool kBF16>
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
  // work item: blockIdx.x = (h * batch + b) * qpairs + qp
  const int qp = blockIdx.x % p.qpairs;
  const int bh_lin = blockIdx.x / p.qpairs;
  const int b = bh_lin % p.batch;
  const int h = bh_lin / p.batch;
  const int Lq = static_cast<int>(p.q_len);
  const int q0 = qp * (kNQ * kBM);
  const int nq = (Lq - q0) > kBM ? 2 : 1;

  // ---------------------------------------------------------------- setup
  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < kNQ; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], kBM);
      mbar_init(&sm.o_final[t], 1);
    }
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    // this head's non-empty segments, clipped to the slab, compacted in order
    const int cnt = max(0, min(p.seg_counts[h], static_cast<int>(p.max_segments)));
    int total = 0;
    bool clipped = false;
    for (int base = 0; base < cnt; base += 32) {
      const int i = base + lane;
      int s = 0, e = 0;
      if (i < cnt) {
        s = p.seg_starts[int64_t(h) * p.max_segments + i];
        e = p.seg_ends[int64_t(h) * p.max_segments + i];
        if (s < e && (s < 0 || e > p.capacity)) clipped = true;
        s = max(s, 0);
        e = static_cast<int>(min64(e, p.capacity));
      }
      const bool keep = (i < cnt) && (s < e);
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const int slot = total + __popc(m & ((1u << lane) - 1u));
        sm.seg_start[slot] = s;
        sm.seg_end[slot] = e;
      }
      total += __popc(m);
    }
    if (__any_sync(0xffffffffu, clipped) && lane == 0 && b == 0 && qp == 0)
      raise_status(HEATKV_DEVICE_BAD_SEGMENT);
    __syncwarp();
    if (lane == 0) {
      int nt = 0;
      for (int i = 0; i < total; ++i) nt += (sm.seg_end[i] - sm.seg_start[i] + kBN - 1) / kBN;
      nt += (Lq + kBN - 1) / kBN;
      sm.nseg = total;
      sm.ntiles = nt;
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_ck);
      tma_prefetch_desc(&tm_cv);
      tma_prefetch_desc(&tm_sk);
      tma_prefetch_desc(&tm_sv);
    }
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int ntiles = sm.ntiles;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const int qrow = static_cast<int>((int64_t(b) * p.heads + h) * p.q_len) + q0;
      mbar_arrive_expect_tx(&sm.q_full, nq * kTileBytes);
      for (int t = 0; t < nq; ++t) {
        tma_load_2d(sm.q[t], &tm_q, 0, qrow + t * kBM, &sm.q_full);
        tma_load_2d(sm.q[t] + kHalfBytes, &tm_q, 64, qrow + t * kBM, &sm.q_full);
      }
      const int cur_row0 = static_cast<int>((int64_t(b) * p.heads + h) * p.q_len);
      const int slab_row0 = static_cast<int>(int64_t(b) * p.capacity);
      TileCursor cur;
      cur.begin(sm);
      int j = 0;
      for (; j < ntiles; ++j) {
        const int s = j % kStages;
        const uint32_t use = j / kStages;
        const CUtensorMap* mk = cur.current ? &tm_ck : &tm_sk;
        const CUtensorMap* mv = cur.current ? &tm_cv : &tm_sv;
        const int row = cur.current ? cur_row0 + cur.pos : slab_row0 + cur.pos;
        if (j >= kStages && !mbar_wait(&sm.k_empty[s], (use - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&sm.k_full[s], kTileBytes);
        tma_load_2d(sm.k[s], mk, 0, row, &sm.k_full[s]);
        tma_load_2d(sm.k[s] + kHalfBytes, mk, 64, row, &sm.k_full[s]);
        if (j >= kStages && !mbar_wait(&sm.v_empty[s], (use - 1) & 1, abort_flag)) {
          ++j;  // the K half of this tile is in flight
          break;
        }
        mbar_arrive_expect_tx(&sm.v_full[s], kTileBytes);
        tma_load_2d(sm.v[s], mv, 0, row, &sm.v_full[s]);
        tma_load_2d(sm.v[s] + kHalfBytes, mv, 64, row, &sm.v_full[s]);
        cur.next(sm, Lq);
      }
      if (*abort_flag) {
        // let every copy already issued land before the CTA's shared memory goes away
        mbar_drain(&sm.q_full, 0);
        for (int jj = max(0, j - kStages); jj < j; ++jj) {
          mbar_drain(&sm.k_full[jj % kStages], (jj / kStages) & 1);
          mbar_drain(&sm.v_full[jj % kStages], (jj / kStages) & 1);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kBF16, kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(kBF16, kBM, kD, false, true);
      const uint32_t tm_s[2] = {tmem + 0, tmem + 128};
      const uint32_t tm_o[2] = {tmem + 256, tmem + 384};
      bool ok = mbar_wait(&sm.q_full, 0, abort_flag);
      if (ok) tc_fence_after();
      auto issue_pv = [&](int t, int jj) {
        const uint32_t vbase = smem_u32(sm.v[jj % kStages]);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // B = V rows [16kk, 16kk+16): 16 keys x 128 columns, MN-major; 8-key groups 1 KiB
          // apart (SBO), the two 64-column halves 16 KiB apart (LBO)
          const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, kHalfBytes, 1024);
          umma_ts(tm_o[t], tm_s[t] + kk * 8, bdesc, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
        }
      };
      auto issue_qk = [&](int t, int jj) {
        const uint32_t qbase = smem_u32(sm.q[t]);
        const uint32_t kbase = smem_u32(sm.k[jj % kStages]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk / 4) * kHalfBytes + (kk % 4) * 32;
          const uint64_t adesc = smem_desc_sw128(qbase + off, 16, 1024);
          const uint64_t bdesc = smem_desc_sw128(kbase + off, 16, 1024);
          umma_ss(tm_s[t], adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j % kStages;
        if (!(ok = mbar_wait(&sm.k_full[s], (j / kStages) & 1, abort_flag))) break;
        tc_fence_after();
        for (int t = 0; t < nq && ok; ++t) {
          if (j > 0) {
            if (t == 0) {
              if (!(ok = mbar_wait(&sm.v_full[(j - 1) % kStages], ((j - 1) / kStages) & 1,
                                   abort_flag)))
                break;
            }
            if (!(ok = mbar_wait(&sm.p_full[t], (j - 1) & 1, abort_flag))) break;
            tc_fence_after();
            issue_pv(t, j - 1);
            if (t == nq - 1) tc_commit(&sm.v_empty[(j - 1) % kStages]);
          }
          issue_qk(t, j);
          tc_commit(&sm.s_full[t]);
        }
        if (ok) tc_commit(&sm.k_empty[s]);
      }
      if (ok) {
        const int j = ntiles - 1;
        ok = mbar_wait(&sm.v_full[j % kStages], (j / kStages) & 1, abort_flag);
        for (int t = 0; t < nq && ok; ++t) {
          if (!(ok = mbar_wait(&sm.p_full[t], j & 1, abort_flag))) break;
          tc_fence_after();
          issue_pv(t, j);
          tc_commit(&sm.o_final[t]);
        }
      }
      // every MMA issued by this thread has completed once `drain` fires
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax warpgroups
    const int t = warp / 4;
    const int quad = warp % 4;
    if (t < nq) {
      const int row = quad * 32 + lane;  // TMEM lane == query row within the tile
      const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
      const uint32_t tS = tmem + lane_off + t * 128;
      const uint32_t tO = tmem + lane_off + 256 + t * 128;
      const float c = p.scale_log2;
      float m_run = -INFINITY;
      float l_run = 0.f;
      bool ok = true;
      TileCursor cur;
      cur.begin(sm);
      for (int j = 0; j < ntiles; ++j) {
        const int valid = cur.valid(sm, Lq);
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        float x[128];
        tmem_ld128_sync(tS, x);
        float mx = -INFINITY;
        if (valid >= kBN) {
#pragma unroll
          for (int i = 0; i < 128; ++i) mx = fmaxf(mx, x[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            x[i] = (i < valid) ? x[i] : -INFINITY;
            mx = fmaxf(mx, x[i]);
          }
        }
        const float mx2 = mx * c;
        if (j == 0) {
          m_run = mx2;
        } else if (__any_sync(0xffffffffu, mx2 > m_run + 8.0f)) {
          // raise the running max; rescale this row of O (PV(j-1) has completed: the commit
          // that signalled S(j) covers every earlier MMA)
          const float m_new = fmaxf(m_run, mx2);
          const float alpha = ex2(m_run - m_new);
          l_run *= alpha;
          m_run = m_new;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            float o[32];
            tmem_ld32_sync(tO + cc * 32, o);
            uint32_t w[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(o[i] * alpha);
            tmem_st32(tO + cc * 32, w);
          }
        }
        const float neg_m = -m_run;
        float sum = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float p0 = ex2(fmaf(x[64 * half + 2 * i], c, neg_m));
            const float p1 = ex2(fmaf(x[64 * half + 2 * i + 1], c, neg_m));
            sum += p0 + p1;
            pk[i] = pack2<kBF16>(p0, p1);
          }
          tmem_st32(tS + 32 * half, pk);
        }
        l_run += sum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.p_full[t]);
        cur.next(sm, Lq);
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.o_final[t], 0, abort_flag));
      if (ok) {
        tc_fence_after();
        const int qrow = q0 + t * kBM + row;
        const float inv = 1.f / l_run;
        using OutT = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
        OutT* orow = static_cast<OutT*>(p.out) +
                     ((int64_t(b) * p.q_len + qrow) * p.heads + h) * kD;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float o[32];
          tmem_ld32_sync(tO + cc * 32, o);
          if (qrow < Lq) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = pack2<kBF16>(o[2 * i] * inv, o[2 * i + 1] * inv);
            uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
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
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// rows x 128 16-bit matrix, box 64 x 128 with 128-byte swizzle
static bool encode_rows(CUtensorMap* map, const void* base, int64_t rows, bool bf16) {
  auto enc = get_encode();
  if (!enc) return false;
  if (rows <= 0) rows = 1;  // an empty tensor is never read; keep the map well-formed
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kBM)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace sm100

cudaError_t launch_attention_sm100(const AttnArgs& a, bool bf16, cudaStream_t st) {
  using namespace sm100;
  const int64_t cur_rows = a.batch * a.heads * a.q_len;
  const int64_t slab_rows = a.batch * a.capacity;
  if (cur_rows >= (int64_t(1) << 31) || slab_rows >= (int64_t(1) << 31) ||
      a.max_segments > kMaxSegments || !(a.scale > 0.f))
    return cudaErrorNotSupported;
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.cur_k) |
                          reinterpret_cast<uintptr_t>(a.cur_v) |
                          reinterpret_cast<uintptr_t>(a.slab_k) |
                          reinterpret_cast<uintptr_t>(a.slab_v) | reinterpret_cast<uintptr_t>(a.out);
  if (align & 15u) return cudaErrorNotSupported;
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
  p.out = a.out;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.qpairs = static_cast<int>((a.q_len + kNQ * kBM - 1) / (kNQ * kBM));
  const int64_t blocks = a.batch * a.heads * p.qpairs;
  if (blocks >= (int64_t(1) << 31)) return cudaErrorNotSupported;
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  auto kern = bf16 ? attn_sm100_kernel<true> : attn_sm100_kernel<false>;
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
  kern<<<static_cast<unsigned>(blocks), kThreads, smem, st>>>(tq, tck, tcv, tsk, tsv, p);
  return cudaGetLastError();
}

}  // namespace heatkv
