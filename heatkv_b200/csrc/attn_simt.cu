// Exact segmented attention on CUDA cores: fp32 products, fp32 accumulation, expf softmax.
//
// Semantics of _fused_real_pruning_segmented_attention_kernel (real_pruning_fused_attention.py:76-267)
// with its fp32 dot modes (QK_DOT_MODE "fp32"/"ieee", VALUE_DOT_MODE "fp32"): for batch row b and
// head h the keys are the head's slab segments [start, end) in segment order, then the current
// scale's K/V; online softmax over 32-key tiles; output [B, Lq, H*D] in q's dtype. This kernel
// serves every dtype combination (inputs are widened to fp32 on load) and is the path of the fp32
// configuration, whose tolerance (1e-5) rules out tensor-core TF32/bf16 products.
//
// Block = 256 threads computes 64 query rows of one (b, h). Per 32-key tile: S = Q K^T with each
// thread owning 4 rows x 2 keys (K staged transposed in shared memory), row statistics reduced over
// the 16 threads of a half-warp, then O += P V with each thread owning 4 rows x 8 columns.
#include <atomic>

#include "attn.h"
#include "common.cuh"

namespace heatkv {

constexpr int kSimtM = 64;
constexpr int kSimtN = 32;
constexpr int kSimtD = 128;
constexpr int kSimtThreads = 256;
constexpr int kSimtMaxSeg = kMaxSegments;
constexpr int kQStride = kSimtD + 4;   // padded row stride of Q (floats)
constexpr int kKtStride = kSimtN + 1;  // padded row stride of K^T (floats)
constexpr int kVStride = kSimtD + 4;
constexpr int kPStride = kSimtN + 1;

struct SimtSmem {
  float q[kSimtM * kQStride];
  float kt[kSimtD * kKtStride];
  float v[kSimtN * kVStride];
  float p[kSimtM * kPStride];
  int seg_start[kSimtMaxSeg];
  int seg_end[kSimtMaxSeg];
  int nseg;
};


template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i) {
  return Elem<T>::to_float(p[i]);
}
template <>
__device__ __forceinline__ float ldf<float>(const float* p, int64_t i) {
  return p[i];
}

// Load `rows` (<= kSimtN) key/value rows starting at element offset `row_base * D`; K is stored
// transposed (kt[d][n]), V row-major. Rows past `rows` are zero.
template <typename TK, typename TV>
__device__ void load_kv_tile(SimtSmem& sm, const TK* kbase, const TV* vbase, int rows) {
  for (int idx = threadIdx.x; idx < kSimtN * kSimtD; idx += kSimtThreads) {
    const int n = idx / kSimtD;
    const int d = idx % kSimtD;
    float kv = 0.f, vv = 0.f;
    if (n < rows) {
      kv = ldf(kbase, int64_t(n) * kSimtD + d);
      vv = ldf(vbase, int64_t(n) * kSimtD + d);
    }
    sm.kt[d * kKtStride + n] = kv;
    sm.v[n * kVStride + d] = vv;
  }
}

template <typename TQ, typename TK, typename TV>
__global__ void __launch_bounds__(kSimtThreads) attn_simt_kernel(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SimtSmem& sm = *reinterpret_cast<SimtSmem*>(smem_raw);
  const int mblk = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int ty = tid / 16;  // 16 row groups of 4 rows
  const int tx = tid % 16;  // 16 key pairs (S) / 16 column groups of 8 (O)
  const int64_t Lq = a.q_len;
  const int64_t bh = int64_t(b) * a.heads + h;
  const int64_t m0 = int64_t(mblk) * kSimtM;

  // head h's segment list, clipped to the slab, empty entries removed
  if (tid == 0) {
    int cnt = a.seg_counts[h];
    cnt = max(0, min(cnt, int(a.max_segments)));
    int n = 0;
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
      sm.seg_end[n] = e;
      ++n;
    }
    sm.nseg = n;
    if (clipped && mblk == 0 && b == 0) raise_status(a.status, HEATKV_DEVICE_BAD_SEGMENT);
  }
  // Q rows (zero past Lq)
  const TQ* qp = static_cast<const TQ*>(a.q) + (bh * Lq + m0) * kSimtD;
  for (int idx = tid; idx < kSimtM * kSimtD; idx += kSimtThreads) {
    const int r = idx / kSimtD, d = idx % kSimtD;
    sm.q[r * kQStride + d] = (m0 + r < Lq) ? ldf(qp, int64_t(r) * kSimtD + d) : 0.f;
  }
  __syncthreads();

  float o[4][8];
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
  }
  const float scale = a.scale;
  const int nseg = sm.nseg;
  const TK* slab_k = static_cast<const TK*>(a.slab_k);
  const TV* slab_v = static_cast<const TV*>(a.slab_v);
  const TK* cur_k = static_cast<const TK*>(a.cur_k) + bh * Lq * kSimtD;
  const TV* cur_v = static_cast<const TV*>(a.cur_v) + bh * Lq * kSimtD;

  // tiles: every segment in order, then the current scale
  int seg = 0;
  int64_t pos = nseg > 0 ? sm.seg_start[0] : 0;
  bool in_current = (nseg == 0);
  if (in_current) pos = 0;
  while (true) {
    int rows;
    const TK* kb;
    const TV* vb;
    if (!in_current) {
      rows = int(min64(kSimtN, sm.seg_end[seg] - pos));
      kb = slab_k + (int64_t(b) * a.capacity + pos) * kSimtD;
      vb = slab_v + (int64_t(b) * a.capacity + pos) * kSimtD;
    } else {
      if (pos >= Lq) break;
      rows = int(min64(kSimtN, Lq - pos));
      kb = cur_k + pos * kSimtD;
      vb = cur_v + pos * kSimtD;
    }
    load_kv_tile(sm, kb, vb, rows);
    __syncthreads();

    // S = Q K^T for rows ty*4..+3, keys tx*2..+1
    float s[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.f;
#pragma unroll 8
    for (int d = 0; d < kSimtD; ++d) {
      const float k0 = sm.kt[d * kKtStride + tx * 2];
      const float k1 = sm.kt[d * kKtStride + tx * 2 + 1];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qv = sm.q[(ty * 4 + i) * kQStride + d];
        s[i][0] = fmaf(qv, k0, s[i][0]);
        s[i][1] = fmaf(qv, k1, s[i][1]);
      }
    }
    // online softmax per row over the tile's valid keys
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v0 = (tx * 2 < rows) ? s[i][0] * scale : -INFINITY;
      float v1 = (tx * 2 + 1 < rows) ? s[i][1] * scale : -INFINITY;
      float mx = fmaxf(v0, v1);
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run[i], mx);
      const float alpha = expf(m_run[i] - m_new);  // 0 on the first tile (m_run = -inf)
      const float p0 = expf(v0 - m_new);
      const float p1 = expf(v1 - m_new);
      float ps = p0 + p1;
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l_run[i] = l_run[i] * alpha + ps;
      m_run[i] = m_new;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] *= alpha;
      sm.p[(ty * 4 + i) * kPStride + tx * 2] = p0;
      sm.p[(ty * 4 + i) * kPStride + tx * 2 + 1] = p1;
    }
    __syncthreads();
    // O += P V for rows ty*4..+3, columns tx*8..+7
#pragma unroll 4
    for (int n = 0; n < kSimtN; ++n) {
      const float4 va = *reinterpret_cast<const float4*>(&sm.v[n * kVStride + tx * 8]);
      const float4 vb4 = *reinterpret_cast<const float4*>(&sm.v[n * kVStride + tx * 8 + 4]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pv = sm.p[(ty * 4 + i) * kPStride + n];
        o[i][0] = fmaf(pv, va.x, o[i][0]);
        o[i][1] = fmaf(pv, va.y, o[i][1]);
        o[i][2] = fmaf(pv, va.z, o[i][2]);
        o[i][3] = fmaf(pv, va.w, o[i][3]);
        o[i][4] = fmaf(pv, vb4.x, o[i][4]);
        o[i][5] = fmaf(pv, vb4.y, o[i][5]);
        o[i][6] = fmaf(pv, vb4.z, o[i][6]);
        o[i][7] = fmaf(pv, vb4.w, o[i][7]);
      }
    }
    __syncthreads();

    // advance the tile cursor
    pos += rows;
    if (!in_current) {
      if (pos >= sm.seg_end[seg]) {
        ++seg;
        if (seg < nseg) {
          pos = sm.seg_start[seg];
        } else {
          in_current = true;
          pos = 0;
        }
      }
    }
  }

  // out[b, m, h*D + c] = O / l
  TQ* op = static_cast<TQ*>(a.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= Lq) continue;
    const float inv = 1.f / l_run[i];
    TQ* row = op + ((int64_t(b) * Lq + m) * a.heads + h) * kSimtD + tx * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) row[j] = Elem<TQ>::from_float(o[i][j] * inv);
  }
}

template <typename TQ, typename TK, typename TV>
static cudaError_t launch_simt_t(const AttnArgs& a, cudaStream_t st) {
  auto kern = attn_simt_kernel<TQ, TK, TV>;
  const int smem = static_cast<int>(sizeof(SimtSmem));
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
  dim3 grid(static_cast<unsigned>((a.q_len + kSimtM - 1) / kSimtM), static_cast<unsigned>(a.heads),
            static_cast<unsigned>(a.batch));
  kern<<<grid, kSimtThreads, smem, st>>>(a);
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

cudaError_t launch_attention_simt(const AttnArgs& a, int q_dtype, int k_dtype, int v_dtype,
                                  cudaStream_t st) {
  switch (q_dtype) {
    case HEATKV_DTYPE_F32: return dispatch_k<float>(k_dtype, v_dtype, a, st);
    case HEATKV_DTYPE_F16: return dispatch_k<__half>(k_dtype, v_dtype, a, st);
    default: return dispatch_k<__nv_bfloat16>(k_dtype, v_dtype, a, st);
  }
}

}  // namespace heatkv
