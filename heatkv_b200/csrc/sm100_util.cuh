// Device and host helpers shared by the tcgen05 kernels (attn_sm100_cs.cu, attn_sm100_cs64.cu,
// qkv_proj.cu): the key-tile cursor over a head's slab segments, TMEM row loads, row maxima,
// packed fp32x2 arithmetic, bounded drain waits, and tensor-map encoding.
#pragma once

#include "common.cuh"

#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

namespace heatkv {
namespace sm100 {

constexpr int kKeyTile = 128;  // keys per K/V tile of both kernels
constexpr int kHeadDim = 128;  // the only head dim of the path
constexpr int kNumSms = 148;

// Walks the key tiles of one head: each segment in kTile-row steps, then the current scale. The
// end of the segment being walked is held in a register: shared-memory loads wait behind the
// tensor core's operand reads, so the table is read only when the walk enters a segment.
template <int kTile>
struct TileCursorT {
  const int* st;
  const int* en;
  int nseg, seg, pos, end;
  bool current;
  // position on tile j0 of head h
  template <class SmemT>
  __device__ void begin(const SmemT& sm, int h, int stride, int j0) {
    st = sm.seg_start + h * stride;
    en = sm.seg_end + h * stride;
    nseg = sm.head_nseg[h];
    seg = 0;
    current = false;
    while (seg < nseg) {
      const int t = (en[seg] - st[seg] + kTile - 1) / kTile;
      if (j0 < t) break;
      j0 -= t;
      ++seg;
    }
    if (seg < nseg) {
      pos = st[seg] + j0 * kTile;
      end = en[seg];
    } else {
      current = true;
      pos = j0 * kTile;
      end = 0;
    }
  }
  __device__ int valid(int q_len) const {
    return current ? min(kTile, q_len - pos) : min(kTile, end - pos);
  }
  __device__ void next() {
    pos += kTile;
    if (!current && pos >= end) {
      ++seg;
      if (seg < nseg) {
        pos = st[seg];
        end = en[seg];
      } else {
        current = true;
        pos = 0;
      }
    }
  }
};
using TileCursor = TileCursorT<kKeyTile>;

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

__device__ __forceinline__ void tmem_ld16_sync(uint32_t taddr, float (&x)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(r[i]);
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


__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&x)[N]) {
  if constexpr (N == 64) {
    tmem_ld_row64(taddr, x);
  } else {
    static_assert(N == 32, "32 or 64 columns per warpgroup");
    tmem_ld32_sync(taddr, x);
  }
}

// Row max of N (a multiple of 16) scores: 8 independent chains of 3-input max.
template <int N>
__device__ __forceinline__ float row_max(const float (&x)[N]) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = fmaxf(x[k], x[k + 8]);
#pragma unroll
  for (int i = 2; i < N / 8; i += 2) {
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = max3f(a[k], x[k + 8 * i], x[k + 8 * i + 8]);
  }
  return max3f(max3f(a[0], a[1], a[2]), max3f(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}


// packed pairs of fp32 (sm_100 f32x2 arithmetic)
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// A drain wait for the error path: bounded, ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, unsigned int* status) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles / 4) {
      raise_status(status, HEATKV_DEVICE_WAIT_TIMEOUT);
      return;
    }
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

// rows x 128 16-bit matrix, box 64 columns x box_rows rows with 128-byte swizzle
static bool encode_rows(CUtensorMap* map, const void* base, int64_t rows, bool bf16,
                        int box_rows = kKeyTile) {
  auto enc = get_encode();
  if (!enc) return false;
  if (rows <= 0) rows = 1;  // an empty tensor is never read; keep the map well-formed
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHeadDim * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int sm_count() {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kNumSms;
  int v = cached[dev & 63].load();
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = kNumSms;
    cached[dev & 63].store(v);
  }
  return v;
}

}  // namespace sm100
}  // namespace heatkv
