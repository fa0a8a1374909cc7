// Exact segmented attention on CUDA cores: fp32 products, fp32 accumulation, expf softmax.
//
// Semantics of _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// with its fp32 dot modes (QK_DOT_MODE "fp32"/"ieee", VALUE_DOT_MODE "fp32"): for batch row b and
// head h the keys are the head's slab segments [start, end) in segment order, then the current
// scale's K/V; online softmax over key tiles; output [B, Lq, H*D] in q's dtype. This kernel
// serves every dtype combination the tensor-core kernels do not (inputs are widened to fp32 on
// load) and is the path of the fp32 configuration, whose tolerance (1e-5) rules out tf32/bf16
// products.
//
// Block = 256 threads computes 64 query rows of one (b, h); two blocks per SM. Key tiles are 64
// consecutive keys of the head's key sequence (segments concatenated, then the current scale), so
// short segments share a tile; the first 64 threads resolve each tile key's source row. Q and the
// K tile are staged transposed in shared memory, so per head-dim step a thread reads two float4
// and does 16 FMAs of its 4 rows x 4 keys; the row statistics reduce over the 16 threads of a
// half-warp; P goes back to shared memory over the K tile, and O += P V with each thread owning
// 4 rows x 8 columns (columns 4t..4t+3 and 64+4t..64+4t+3, conflict-free float4 reads of V).
#include <atomic>

#include "attn.h"
#include "common.cuh"

namespace heatkv {

namespace {

constexpr int kM = 64;          // query rows per block
constexpr int kN = 64;          // keys per tile
constexpr int kD = 128;         // head dim
constexpr int kThreads = 256;
constexpr int kTS = kM + 4;     // row stride (floats) of the transposed tiles and of P
constexpr int kVS = kD + 4;     // row stride (floats) of the V tile
static_assert(kM == kN, "Q^T and K^T share a row stride");

struct SimtSmem {
  float qt[kD * kTS];           // Q^T: qt[d * kTS + m]
  float kt[kD * kTS];           // K^T: kt[d * kTS + n]; after the scores, P: kt[m * kTS + n]
  float v[kN * kVS];            // V: v[n * kVS + d]
  long long key_row[kN];        // tile key n: slab row (>= 0), -2 - current row, or -1 (none)
  int seg_start[kMaxSegments];
  int seg_cum[kMaxSegments + 1];  // keys before segment i
  int nseg;
};

// Four consecutive elements as fp32 (one 16- or 8-byte load when kVec).
template <typename T, bool kVec>
__device__ __forceinline__ float4 load4(const T* p) {
  if constexpr (kVec && sizeof(T) == 4) {
    return __ldg(reinterpret_cast<const float4*>(p));
  } else if constexpr (kVec && sizeof(T) == 2) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
    return make_float4(Elem<T>::to_float(e[0]), Elem<T>::to_float(e[1]), Elem<T>::to_float(e[2]),
                       Elem<T>::to_float(e[3]));
  } else {
    return make_float4(Elem<T>::to_float(p[0]), Elem<T>::to_float(p[1]), Elem<T>::to_float(p[2]),
                       Elem<T>::to_float(p[3]));
  }
}

// rows x 128 tile -> transposed shared tile t[d * kTS + r]. A warp covers 16 rows x 2 column
// quads: 32-byte global segments per row, and stores to 32 distinct banks.
template <typename T, bool kVec, typename RowPtr>
__device__ __forceinline__ void load_transposed(float* t, RowPtr row_ptr) {
  for (int u = threadIdx.x; u < kN * (kD / 4); u += kThreads) {
    const int r = (u % 16) + 16 * (u / 512);
    const int d4 = (u / 16) % 32;
    const T* src = row_ptr(r);
    const float4 x = src ? load4<T, kVec>(src + d4 * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    float* dst = t + (d4 * 4) * kTS + r;
    dst[0] = x.x;
    dst[kTS] = x.y;
    dst[2 * kTS] = x.z;
    dst[3 * kTS] = x.w;
  }
}

template <typename TQ, typename TK, typename TV, bool kVec>
__global__ void __launch_bounds__(kThreads, 2) attn_simt_kernel(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SimtSmem& sm = *reinterpret_cast<SimtSmem*>(smem_raw);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int ty = tid / 16;  // rows 4ty..4ty+3
  const int tx = tid % 16;  // keys 4tx..4tx+3 (scores), columns 4tx.., 64+4tx.. (output)
  const int64_t Lq = a.q_len;
  const int64_t bh = int64_t(b) * a.heads + h;
  const int64_t m0 = int64_t(blockIdx.x) * kM;

  // head h's segment list, clipped to the slab, empty entries removed, with running key counts
  if (tid == 0) {
    const int cnt = max(0, min(a.seg_counts[h], int(a.max_segments)));
    int n = 0, cum = 0;
    bool clipped = false;
    for (int i = 0; i < cnt; ++i) {
      int s = a.seg_starts[int64_t(h) * a.max_segments + i];
      int e = a.seg_ends[int64_t(h) * a.max_segments + i];
      if (s >= e) continue;
      if (s < 0 || e > a.capacity) clipped = true;
      s = max(s, 0);
      e = int(min64(e, a.capacity));
      if (s >= e) continue;
      sm.seg_start[n] = s;
      sm.seg_cum[n] = cum;
      cum += e - s;
      ++n;
    }
    sm.seg_cum[n] = cum;
    sm.nseg = n;
    if (clipped && blockIdx.x == 0 && b == 0) raise_status(a.status, HEATKV_DEVICE_BAD_SEGMENT);
  }
  const TQ* qp = static_cast<const TQ*>(a.q) + (bh * Lq + m0) * kD;
  load_transposed<TQ, kVec>(sm.qt, [&](int r) -> const TQ* {
    return (m0 + r < Lq) ? qp + int64_t(r) * kD : nullptr;
  });
  __syncthreads();

  const TK* slab_k = static_cast<const TK*>(a.slab_k);
  const TV* slab_v = static_cast<const TV*>(a.slab_v);
  const TK* cur_k = static_cast<const TK*>(a.cur_k);
  const TV* cur_v = static_cast<const TV*>(a.cur_v);
  const int nseg = sm.nseg;
  const int64_t n_slab = sm.seg_cum[nseg];
  // with current_in_segments the current keys already end the head's segments
  const int64_t total = n_slab + ((a.current_in_segments && nseg > 0) ? 0 : Lq);
  const float scale = a.scale;

  float o[4][8];
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
  }

  for (int64_t t0 = 0; t0 < total; t0 += kN) {
    if (tid < kN) {
      const int64_t t = t0 + tid;
      long long r = -1;
      if (t < n_slab) {
        int lo = 0, hi = nseg - 1;  // last segment with seg_cum <= t
        while (lo < hi) {
          const int mid = (lo + hi + 1) / 2;
          if (sm.seg_cum[mid] <= t) lo = mid; else hi = mid - 1;
        }
        r = int64_t(b) * a.capacity + sm.seg_start[lo] + (t - sm.seg_cum[lo]);
      } else if (t < total) {
        r = -2 - (bh * Lq + (t - n_slab));
      }
      sm.key_row[tid] = r;
    }
    __syncthreads();
    load_transposed<TK, kVec>(sm.kt, [&](int n) -> const TK* {
      const long long r = sm.key_row[n];
      return r >= 0 ? slab_k + r * kD : (r <= -2 ? cur_k + (-2 - r) * kD : nullptr);
    });
    for (int u = tid; u < kN * (kD / 4); u += kThreads) {
      const int n = u / 32, d4 = u % 32;
      const long long r = sm.key_row[n];
      const TV* src = r >= 0 ? slab_v + r * kD : (r <= -2 ? cur_v + (-2 - r) * kD : nullptr);
      *reinterpret_cast<float4*>(&sm.v[n * kVS + d4 * 4]) =
          src ? load4<TV, kVec>(src + d4 * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();

    // S = Q K^T for rows 4ty..+3, keys 4tx..+3
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < kD; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(&sm.qt[d * kTS + ty * 4]);
      const float4 kb = *reinterpret_cast<const float4*>(&sm.kt[d * kTS + tx * 4]);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
      const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
    // online softmax per row over the tile's valid keys
    const int nvalid = static_cast<int>(min64(kN, total - t0));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (tx * 4 + j < nvalid) ? s[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run[i], mx);
      const float alpha = expf(m_run[i] - m_new);  // 0 on the first tile (m_run = -inf)
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = expf(s[i][j] - m_new);
        ps += s[i][j];
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l_run[i] = l_run[i] * alpha + ps;
      m_run[i] = m_new;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] *= alpha;
    }
    __syncthreads();  // every thread is done with K^T: P goes over it
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4*>(&sm.kt[(ty * 4 + i) * kTS + tx * 4]) =
          make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
    __syncthreads();

    // O += P V for rows 4ty..+3, columns 4tx..+3 and 64+4tx..+3
#pragma unroll 2
    for (int n = 0; n < kN; n += 4) {
      float4 pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        pr[i] = *reinterpret_cast<const float4*>(&sm.kt[(ty * 4 + i) * kTS + n]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 va = *reinterpret_cast<const float4*>(&sm.v[(n + k) * kVS + tx * 4]);
        const float4 vb = *reinterpret_cast<const float4*>(&sm.v[(n + k) * kVS + 64 + tx * 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float pv = k == 0 ? pr[i].x : k == 1 ? pr[i].y : k == 2 ? pr[i].z : pr[i].w;
          o[i][0] = fmaf(pv, va.x, o[i][0]);
          o[i][1] = fmaf(pv, va.y, o[i][1]);
          o[i][2] = fmaf(pv, va.z, o[i][2]);
          o[i][3] = fmaf(pv, va.w, o[i][3]);
          o[i][4] = fmaf(pv, vb.x, o[i][4]);
          o[i][5] = fmaf(pv, vb.y, o[i][5]);
          o[i][6] = fmaf(pv, vb.z, o[i][6]);
          o[i][7] = fmaf(pv, vb.w, o[i][7]);
        }
      }
    }
    __syncthreads();  // the next tile's rows, K^T and V overwrite this tile's
  }

  // out[b, m, h*D + c] = O / l
  TQ* op = static_cast<TQ*>(a.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= Lq) continue;
    const float inv = 1.f / l_run[i];
    TQ* row = op + ((int64_t(b) * Lq + m) * a.heads + h) * kD;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      row[tx * 4 + j] = Elem<TQ>::from_float(o[i][j] * inv);
      row[64 + tx * 4 + j] = Elem<TQ>::from_float(o[i][4 + j] * inv);
    }
  }
}

template <typename TQ, typename TK, typename TV>
static cudaError_t launch_simt_t(const AttnArgs& a, cudaStream_t st) {
  // 4-element vector loads when every base pointer allows them (rows are 128 elements)
  auto aligned = [](const void* p, size_t esize) {
    return (reinterpret_cast<uintptr_t>(p) % (4 * esize)) == 0;
  };
  const bool vec = aligned(a.q, sizeof(TQ)) && aligned(a.cur_k, sizeof(TK)) &&
                   aligned(a.cur_v, sizeof(TV)) && aligned(a.slab_k, sizeof(TK)) &&
                   aligned(a.slab_v, sizeof(TV));
  auto kern = vec ? attn_simt_kernel<TQ, TK, TV, true> : attn_simt_kernel<TQ, TK, TV, false>;
  const int smem = static_cast<int>(sizeof(SimtSmem));
  // opt in to >48 KiB dynamic shared memory once per device and variant (never inside a graph
  // capture)
  static std::atomic<uint64_t> configured[2] = {{0}, {0}};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured[vec].load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[vec].fetch_or(bit);
  }
  dim3 grid(static_cast<unsigned>((a.q_len + kM - 1) / kM), static_cast<unsigned>(a.heads),
            static_cast<unsigned>(a.batch));
  kern<<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

template <typename TQ, typename TK>
static cudaError_t dispatch_v(int v_dtype, const AttnArgs& a, cudaStream_t st) {
  switch (v_dtype) {
    case HEATKV_DTYPE_F32: return launch_simt_t<TQ, TK, float>(a, st);
    case HEATKV_DTYPE_F16: return launch_simt_t<TQ, TK, __half>(a, st);
    default: return launch_simt_t<TQ, TK, __nv_bfloat16>(a, st);
  }
}
template <typename TQ>
static cudaError_t dispatch_k(int k_dtype, int v_dtype, const AttnArgs& a, cudaStream_t st) {
  switch (k_dtype) {
    case HEATKV_DTYPE_F32: return dispatch_v<TQ, float>(v_dtype, a, st);
    case HEATKV_DTYPE_F16: return dispatch_v<TQ, __half>(v_dtype, a, st);
    default: return dispatch_v<TQ, __nv_bfloat16>(v_dtype, a, st);
  }
}

}  // namespace

cudaError_t launch_attention_simt(const AttnArgs& a, int q_dtype, int k_dtype, int v_dtype,
                                  cudaStream_t st) {
  switch (q_dtype) {
    case HEATKV_DTYPE_F32: return dispatch_k<float>(k_dtype, v_dtype, a, st);
    case HEATKV_DTYPE_F16: return dispatch_k<__half>(k_dtype, v_dtype, a, st);
    default: return dispatch_k<__nv_bfloat16>(k_dtype, v_dtype, a, st);
  }
}

}  // namespace heatkv
