// S-CAS accumulation: per-(head, source scale) attention mass of one scale's queries, without
// materialising the probabilities.
//
// tools/compute_scas.py:114-128 (ScasAccumulator.update) takes, for batch row 0, the probabilities
// probs = softmax(q k^T * scale) of the current scale's queries over every key so far (the cached
// scales, then the current one; fp32 scores, :217-218) and adds, for each source scale s in
// [sink_scales, min(scale_ind, num_scales - 1)),
//   mass[h][s] = mean over the queries of sum over the keys of scale s of probs
// to accum[layer][h][s] (float64). Here each query row keeps an online softmax - running max,
// row sum - and one partial sum per source scale, rescaled with the row sum whenever the max
// rises, so mass = partial / row sum at the end; fp32 products and accumulation as the reference's
// fp32 matmul and softmax.
//
// Block = 256 threads, 64 query rows of one head, keys in tiles of 64 (Q and the K tile staged
// transposed in shared memory, each thread 4 rows x 4 keys as in attn_simt.cu). The 16 threads of
// a row reduce each source scale's share of a tile with warp shuffles; the row's partial sums live
// in shared memory. At the end every row's masses are summed over the block and added to
// mass_out[h * mass_stride + s] (float64 atomics), already divided by the number of queries.
#include <atomic>

#include "attn.h"
#include "common.cuh"

namespace heatkv {

namespace {

constexpr int kM = 64;
constexpr int kN = 64;
constexpr int kD = 128;
constexpr int kThreads = 256;
constexpr int kTS = kM + 4;
constexpr int kMaxSrc = 32;  // source scales

struct ScasSmem {
  float qt[kD * kTS];
  float kt[kD * kTS];
  float part[kM][kMaxSrc];   // per row: sum over keys of source s of exp(score - running max)
  int bounds[kMaxSrc + 1];   // source s = keys [bounds[s], bounds[s + 1])
};

template <typename T>
__device__ __forceinline__ float4 ld4(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return __ldg(reinterpret_cast<const float4*>(p));
  } else {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
    return make_float4(Elem<T>::to_float(e[0]), Elem<T>::to_float(e[1]), Elem<T>::to_float(e[2]),
                       Elem<T>::to_float(e[3]));
  }
}

// rows x 128 -> transposed tile t[d * kTS + r] (16 rows x 2 column quads per warp)
template <typename T>
__device__ __forceinline__ void stage_t(float* t, const T* base, int64_t rows_valid) {
  for (int u = threadIdx.x; u < 64 * (kD / 4); u += kThreads) {
    const int r = (u % 16) + 16 * (u / 512);
    const int d4 = (u / 16) % 32;
    const float4 x = r < rows_valid ? ld4(base + int64_t(r) * kD + d4 * 4)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    float* dst = t + (d4 * 4) * kTS + r;
    dst[0] = x.x;
    dst[kTS] = x.y;
    dst[2 * kTS] = x.z;
    dst[3 * kTS] = x.w;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    scas_mass_kernel(const T* __restrict__ q, const T* __restrict__ k, int64_t heads,
                     int64_t q_len, int64_t k_len, float scale, const int32_t* __restrict__ bounds,
                     int n_src, double* __restrict__ mass_out, int64_t mass_stride) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ScasSmem& sm = *reinterpret_cast<ScasSmem*>(smem_raw);
  pdl_wait();
  const int h = blockIdx.y;
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int64_t m0 = int64_t(blockIdx.x) * kM;
  for (int i = tid; i <= n_src; i += kThreads) sm.bounds[i] = bounds[i];
  for (int i = tid; i < kM * kMaxSrc; i += kThreads) sm.part[i / kMaxSrc][i % kMaxSrc] = 0.f;
  stage_t(sm.qt, q + (int64_t(h) * q_len + m0) * kD, q_len - m0);
  __syncthreads();
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
  }
  const T* kh = k + int64_t(h) * k_len * kD;
  for (int64_t t0 = 0; t0 < k_len; t0 += kN) {
    stage_t(sm.kt, kh + t0 * kD, k_len - t0);
    __syncthreads();
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
    const int nvalid = static_cast<int>(min64(kN, k_len - t0));
    // source scales that intersect this tile
    int s_first = 0;
    while (s_first < n_src && sm.bounds[s_first + 1] <= t0) ++s_first;
    int s_last = s_first;
    while (s_last + 1 < n_src && sm.bounds[s_last + 1] < t0 + nvalid) ++s_last;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (tx * 4 + j < nvalid) ? s[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run[i], mx);
      const float alpha = expf(m_run[i] - m_new);  // 0 on the first tile
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
      // the row's partial sums: rescale, then add this tile's share of every source it meets
      if (alpha != 1.f && tx == 0) {
        for (int src = 0; src < n_src; ++src) sm.part[r][src] *= alpha;
      }
      for (int src = s_first; src <= s_last && src < n_src; ++src) {
        const int lo = sm.bounds[src], hi = sm.bounds[src + 1];
        float share = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t key = t0 + tx * 4 + j;
          share += (key >= lo && key < hi) ? s[i][j] : 0.f;
        }
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) share += __shfl_xor_sync(0xffffffffu, share, off);
        if (tx == 0) sm.part[r][src] += share;
      }
    }
    __syncthreads();  // the next tile overwrites K^T
  }
  // mass of every row = partial / row sum; sum the block's rows per source, then one atomic each
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty * 4 + i;
    const bool live = m0 + r < q_len;
    if (tx == 0) {
      const float inv = live ? 1.f / l_run[i] : 0.f;
      for (int src = 0; src < n_src; ++src) sm.part[r][src] *= inv;
    }
  }
  __syncthreads();
  for (int src = tid; src < n_src; src += kThreads) {
    double acc = 0.0;
    for (int r = 0; r < kM; ++r) acc += sm.part[r][src];
    atomicAdd(mass_out + int64_t(h) * mass_stride + src, acc / double(q_len));
  }
}

}  // namespace

cudaError_t launch_scas_mass(const void* q, const void* k, int dtype, int64_t heads, int64_t q_len,
                             int64_t k_len, float scale, const int32_t* bounds, int n_src,
                             double* mass_out, int64_t mass_stride, cudaStream_t st) {
  const int smem = static_cast<int>(sizeof(ScasSmem));
  dim3 grid(static_cast<unsigned>((q_len + kM - 1) / kM), static_cast<unsigned>(heads));
  auto go = [&](auto kern, auto qp, auto kp) -> cudaError_t {
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
    e = launch_pdl(kern, grid, dim3(kThreads), static_cast<size_t>(smem), st, qp, kp, heads,
                   q_len, k_len, scale, bounds, n_src, mass_out, mass_stride);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  };
  switch (dtype) {
    case HEATKV_DTYPE_F32:
      return go(scas_mass_kernel<float>, static_cast<const float*>(q), static_cast<const float*>(k));
    case HEATKV_DTYPE_F16:
      return go(scas_mass_kernel<__half>, static_cast<const __half*>(q), static_cast<const __half*>(k));
    default:
      return go(scas_mass_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(q),
                static_cast<const __nv_bfloat16*>(k));
  }
}

}  // namespace heatkv
