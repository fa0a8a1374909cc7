// Cross-GPU barrier for the sharded hot path's peer-to-peer exchange.
//
// After a rank's attention kernel has stored its output rows into every rank's output tensor over
// NVLink, this one-warp kernel publishes the rank's next epoch into every rank's flag array
// (release, system scope) and then waits until every rank's epoch has arrived in its own array
// (acquire, system scope): once it returns, all peers' rows of this step are visible here. The
// epoch is a device-side counter, so a CUDA graph replaying the step advances it on every replay.
// The wait is bounded: when a peer does not arrive within ~2 s the kernel raises
// HEATKV_DEVICE_WAIT_TIMEOUT and returns, and the host sees the flag.
#include "attn.h"
#include "common.cuh"

namespace heatkv {

namespace {

constexpr long long kBarrierBudgetCycles = 4000000000LL;  // ~2 s at B200 clocks

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(uint32_t* const* flag_ptrs,
                                                          uint32_t* counter, int world, int rank,
                                                          unsigned int* status) {
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    epoch = *counter + 1u;
    *counter = epoch;
  }
  __syncthreads();
  const uint32_t e = epoch;
  const int i = threadIdx.x;
  if (i < world) {
    __threadfence_system();
    st_release_sys(flag_ptrs[i] + rank, e);  // "rank has reached epoch e", in rank i's array
  }
  if (i < world) {
    const uint32_t* mine = flag_ptrs[rank] + i;
    const long long t0 = clock64();
    while (static_cast<int32_t>(ld_acquire_sys(mine) - e) < 0) {
      if (clock64() - t0 > kBarrierBudgetCycles) {
        raise_status(status, HEATKV_DEVICE_WAIT_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
}

}  // namespace

cudaError_t launch_peer_barrier(uint32_t* const* flag_ptrs, uint32_t* counter, int world,
                                int rank, unsigned int* status, cudaStream_t stream) {
  peer_barrier_kernel<<<1, 32, 0, stream>>>(flag_ptrs, counter, world, rank, status);
  return cudaGetLastError();
}

}  // namespace heatkv
