// q/k/v preparation between the QKV projection and the segmented attention, in one pass.
//
// The patched attention forward (enable_real_pruning_fast.py:2040-2072) turns the projection
// output qkv [B, L, 3, H, D] into contiguous q, k, v [B, H, L, D] with a chain of PyTorch ops:
// unbind + permute + contiguous; with cos-attention q = normalize(q) * scale_mul[h] and
// k = normalize(k) (F.normalize: x / max(||x||_2, eps); under autocast the norm and the quotient are
// fp32); then the 2-D rotary embedding of infinity/models/basic.py:97-117, computed with autocast
// off in fp32: for each pair (x0, x1) = (x[2i], x[2i+1]) and the scale's rope row (c, s),
//   out[2i] = c*x0 - s*x1,   out[2i+1] = s*x0 + c*x1
// (each product and the sum rounded separately, as the elementwise ops round them). v is copied
// as is. This kernel reads qkv once and writes q, k, v once.
//
// One warp per (token, head): lane t holds elements 4t..4t+3 (two rotary pairs) of q, k and v;
// the squared norm is reduced over the warp. Rows are 128 elements (the only head dim of the
// path). HBM-bound: per (token, head) it reads 3 x 128 input elements (+ the rope row, shared by
// the heads of a token and served by L1/L2) and writes q, k in their dtype and v in the input's.
//
// Slab append (optional): the append after the attention (enable_real_pruning_fast.py:2218-2225 ->
// :969-1024) copies the scale's K/V rows of every retained head into that head's slab segment,
// slab[b, offset[h] + l, :] = k[b, h, l, :] (and v). For the heads whose segment shares no slot
// with the segments the attention of this scale reads, the caller passes offset[h] >= 0 and this
// kernel writes those rows here, from the registers that hold the final k and v; the slab ends up
// with the same bytes as after the reference's copy. offset[h] = -1 leaves head h to that copy.
// A segment that would leave the slab (offset + seq_len > slab_rows) is skipped and raises
// HEATKV_DEVICE_PACK_OUT_OF_RANGE.
#include "attn.h"
#include "common.cuh"

namespace heatkv {

namespace {

constexpr int kD = 128;
constexpr int kWarpsPerBlock = 8;

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);  // four 16-bit elements
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = Elem<T>::to_float(e[i]);
}

template <typename T>
__device__ __forceinline__ void store4(T* p, const float (&x)[4]) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  } else {
    T e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = Elem<T>::from_float(x[i]);
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(e);
  }
}

// x / max(||x||, eps) with the row's squared norm reduced over the warp
__device__ __forceinline__ void normalize(float (&x)[4], float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float n = fmaxf(sqrtf(ss), eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = __fdiv_rn(x[i], n);
}

__device__ __forceinline__ void rope(float (&x)[4], const float2 c, const float2 s) {
  const float a0 = x[0], a1 = x[1], b0 = x[2], b1 = x[3];
  x[0] = __fsub_rn(__fmul_rn(c.x, a0), __fmul_rn(s.x, a1));
  x[1] = __fadd_rn(__fmul_rn(s.x, a0), __fmul_rn(c.x, a1));
  x[2] = __fsub_rn(__fmul_rn(c.y, b0), __fmul_rn(s.y, b1));
  x[3] = __fadd_rn(__fmul_rn(s.y, b0), __fmul_rn(c.y, b1));
}

template <typename TIn, typename TQK, bool kCos, bool kRope>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    qkv_prepare_kernel(const TIn* __restrict__ qkv, TQK* __restrict__ q, TQK* __restrict__ k,
                       TIn* __restrict__ v, int64_t batch, int64_t seq_len, int64_t heads,
                       const float* __restrict__ scale_mul, float eps,
                       const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                       int64_t rope_row_stride, TQK* __restrict__ slab_k, TIn* __restrict__ slab_v,
                       int64_t slab_rows, const int64_t* __restrict__ slab_offset,
                       unsigned int* status) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x % 32;
  const int64_t units = batch * seq_len * heads;  // (b, l, h) in qkv order
  for (int64_t u = int64_t(blockIdx.x) * kWarpsPerBlock + threadIdx.x / 32; u < units;
       u += int64_t(gridDim.x) * kWarpsPerBlock) {
    const int64_t h = u % heads;
    const int64_t bl = u / heads;
    const int64_t l = bl % seq_len;
    const int64_t b = bl / seq_len;
    const TIn* src = qkv + bl * 3 * heads * kD + h * kD + 4 * lane;
    float xq[4], xk[4], xv[4];
    load4(src, xq);
    load4(src + heads * kD, xk);
    load4(src + 2 * heads * kD, xv);
    if constexpr (kCos) {
      normalize(xq, eps);
      normalize(xk, eps);
      const float sm = __ldg(scale_mul + h);
#pragma unroll
      for (int i = 0; i < 4; ++i) xq[i] = __fmul_rn(xq[i], sm);
    }
    if constexpr (kRope) {
      // pairs 2t and 2t+1 of the scale's rope row l
      const float2 c = __ldg(reinterpret_cast<const float2*>(rope_cos + l * rope_row_stride) + lane);
      const float2 s = __ldg(reinterpret_cast<const float2*>(rope_sin + l * rope_row_stride) + lane);
      rope(xq, c, s);
      rope(xk, c, s);
    }
    const int64_t dst = ((b * heads + h) * seq_len + l) * kD + 4 * lane;
    store4(q + dst, xq);
    store4(k + dst, xk);
    store4(v + dst, xv);
    if (slab_offset != nullptr) {
      const int64_t off = __ldg(slab_offset + h);
      if (off >= 0) {
        if (off > slab_rows - seq_len) {
          if (lane == 0 && l == 0 && status) atomicOr(status, HEATKV_DEVICE_PACK_OUT_OF_RANGE);
        } else {
          const int64_t row = (b * slab_rows + off + l) * kD + 4 * lane;
          store4(slab_k + row, xk);
          store4(slab_v + row, xv);
        }
      }
    }
  }
}

template <typename TIn, typename TQK>
cudaError_t launch_t(const void* qkv, void* q, void* k, void* v, int64_t batch, int64_t seq_len,
                     int64_t heads, const float* scale_mul, float eps, const float* rope_cos,
                     const float* rope_sin, int64_t rope_row_stride, void* slab_k, void* slab_v,
                     int64_t slab_rows, const int64_t* slab_offset, int sms, unsigned int* status,
                     cudaStream_t st) {
  const int64_t units = batch * seq_len * heads;
  const int64_t want = (units + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int grid = static_cast<int>(std::min<int64_t>(want, int64_t(sms) * 8));
  const TIn* in = static_cast<const TIn*>(qkv);
  TQK* qo = static_cast<TQK*>(q);
  TQK* ko = static_cast<TQK*>(k);
  TIn* vo = static_cast<TIn*>(v);
  TQK* sk = static_cast<TQK*>(slab_k);
  TIn* sv = static_cast<TIn*>(slab_v);
  const bool cos = scale_mul != nullptr, rp = rope_cos != nullptr;
  auto go = [&](auto kern) {
    return launch_pdl(kern, dim3(grid), dim3(kWarpsPerBlock * 32), 0, st, in, qo, ko, vo, batch,
                      seq_len, heads, scale_mul, eps, rope_cos, rope_sin, rope_row_stride, sk, sv,
                      slab_rows, slab_offset, status);
  };
  cudaError_t e;
  if (cos && rp) e = go(qkv_prepare_kernel<TIn, TQK, true, true>);
  else if (cos) e = go(qkv_prepare_kernel<TIn, TQK, true, false>);
  else if (rp) e = go(qkv_prepare_kernel<TIn, TQK, false, true>);
  else e = go(qkv_prepare_kernel<TIn, TQK, false, false>);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qkv_prepare(const void* qkv, void* q, void* k, void* v, int in_dtype,
                               int qk_dtype, int64_t batch, int64_t seq_len, int64_t heads,
                               const float* scale_mul, float eps, const float* rope_cos,
                               const float* rope_sin, int64_t rope_row_stride, void* slab_k,
                               void* slab_v, int64_t slab_rows, const int64_t* slab_offset,
                               int sms, unsigned int* status, cudaStream_t st) {
  const bool bf16 = in_dtype == HEATKV_DTYPE_BF16;
#define HEATKV_QKV_PREP(TI, TQ)                                                               \
  launch_t<TI, TQ>(qkv, q, k, v, batch, seq_len, heads, scale_mul, eps, rope_cos, rope_sin,   \
                   rope_row_stride, slab_k, slab_v, slab_rows, slab_offset, sms, status, st)
  cudaError_t e;
  switch (qk_dtype) {
    case HEATKV_DTYPE_F32:
      e = bf16 ? HEATKV_QKV_PREP(__nv_bfloat16, float) : HEATKV_QKV_PREP(__half, float);
      break;
    case HEATKV_DTYPE_BF16:
      e = bf16 ? HEATKV_QKV_PREP(__nv_bfloat16, __nv_bfloat16)
               : HEATKV_QKV_PREP(__half, __nv_bfloat16);
      break;
    default:
      e = bf16 ? HEATKV_QKV_PREP(__nv_bfloat16, __half) : HEATKV_QKV_PREP(__half, __half);
      break;
  }
#undef HEATKV_QKV_PREP
  return e;
}

}  // namespace heatkv
