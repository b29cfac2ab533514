// Device side of the exchange waits folded into consuming kernels (EpSync in kernels.h).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace aipu {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..n-1 wait (bounded) for flag q to reach *seq + 1, then the CTA synchronises. Returns false
// (status set) when a wait gave up; the caller then skips its reads of the exchanged data.
__device__ __forceinline__ bool ep_sync_wait(const EpSync& w) {
  __shared__ int ep_ok;
  if (threadIdx.x == 0) ep_ok = 1;
  __syncthreads();
  if (threadIdx.x < w.n) {
    const uint32_t target = *w.seq + 1u;
    const uint32_t* f = w.flags + threadIdx.x;
    const long long t0 = clock64();
    long long limit = 0;
    while (static_cast<int32_t>(ld_acquire_sys(f) - target) < 0) {
      const long long el = clock64() - t0;
      if (el > kWaitGrace && limit == 0) limit = wait_limit(w.status);
      if (el > kWaitGrace && el > limit) {
        atomicOr(w.status, ST_TIMEOUT_FULL);
        ep_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ep_ok != 0;
}

// End of the layer call: the last CTA of the kernel to arrive advances *seq (after every CTA has read it).
__device__ __forceinline__ void ep_sync_bump(const EpSync& w) {
  if (!w.bump_arrive) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(w.bump_arrive, 1u) == gridDim.x - 1) {
      *w.bump_arrive = 0u;
      *w.seq += 1u;
    }
  }
}

}  // namespace aipu
