// Expert-parallel exchange over NVLink peer memory (one process per GPU, CUDA IPC mappings).
//
// Every rank owns one symmetric buffer (same layout on every rank) that its peers map:
//   flags   [2][G] uint32   dispatch / return arrival flags, written by peers (sequence numbers)
//   in_sel  [G][M][T]       selections of every rank's tokens (M = this call's tokens per rank, the
//   in_x    [G][M][H]       bf16 tokens of every rank          same on every rank, <= capacity)
//   out     [G][M][T][H]    bf16 per-slot expert outputs for this rank's tokens, one piece per rank
// A layer call bumps a device-side sequence number; writers store data with plain peer stores,
// make them visible system-wide, then release the flag (st.release.sys); readers acquire the flags
// with a bounded spin (no wait can run forever: on expiry the status word is set and the kernel
// returns). No TMA and no multicast touches peer memory; only plain loads and stores.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace aipu {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// seq += 1 (one thread); every later kernel of the layer reads it
__global__ void ep_bump_kernel(uint32_t* seq) { *seq += 1u; }

// CTA q: copy this rank's M tokens and selections into peer q's inbox slot `rank`, then release
// peer q's dispatch flag[rank] = seq.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpParams p, const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ sel, int M) {
  const int q = blockIdx.x;
  const uint32_t seq = *p.seq;
  uint8_t* peer = p.peers[q];
  uint16_t* dx = reinterpret_cast<uint16_t*>(peer + p.off_in_x) + static_cast<int64_t>(p.rank) * M * p.H;
  int32_t* ds = reinterpret_cast<int32_t*>(peer + p.off_in_sel) + static_cast<int64_t>(p.rank) * M * p.T;
  const int64_t nv = static_cast<int64_t>(M) * p.H / 8;
  for (int64_t i = threadIdx.x; i < nv; i += blockDim.x)
    reinterpret_cast<uint4*>(dx)[i] = __ldg(reinterpret_cast<const uint4*>(x) + i);
  for (int i = threadIdx.x; i < M * p.T; i += blockDim.x) ds[i] = sel[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) st_release_sys(reinterpret_cast<uint32_t*>(peer + p.off_flags) + p.rank, seq);
}

// Wait until flags[which][0..G) of this rank's buffer reach seq (bounded).
__global__ void ep_wait_kernel(const EpParams p, int which) {
  const int q = threadIdx.x;
  if (q >= p.G) return;
  const uint32_t seq = *p.seq;
  const uint32_t* f = reinterpret_cast<const uint32_t*>(p.peers[p.rank] + p.off_flags) + which * p.G + q;
  const long long limit = wait_limit(p.status);
  const long long t0 = clock64();
  while (static_cast<int32_t>(ld_acquire_sys(f) - seq) < 0) {
    if (clock64() - t0 > limit) {
      atomicOr(p.status, ST_TIMEOUT_FULL);
      return;
    }
  }
}

// Return: for gathered token t (owner q = t / M, local row m = t % M), every slot s
// whose expert is local (index >= 0 into the union rows `rows` [U][Gtok][H]) is stored into peer q's
// out[rank][m][s]. Then each CTA makes its stores visible; ep_release_kernel sets the flags.
__global__ void __launch_bounds__(256) ep_return_kernel(const EpParams p, const int32_t* __restrict__ slot_map,
                                                        const uint16_t* __restrict__ rows, int M, int Gtok) {
  const int64_t hv = p.H / 8;
  const int64_t total = static_cast<int64_t>(Gtok) * p.T * hv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t ts = i / hv, v = i - ts * hv;
    const int t = static_cast<int>(ts / p.T), s = static_cast<int>(ts - static_cast<int64_t>(t) * p.T);
    const int q = t / M, m = t - q * M;
    const int ix = slot_map[ts];
    if (ix < 0) continue;
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(rows + (static_cast<int64_t>(ix) * Gtok + t) * p.H) + v);
    uint16_t* dst = reinterpret_cast<uint16_t*>(p.peers[q] + p.off_out) +
                    ((static_cast<int64_t>(p.rank) * M + m) * p.T + s) * p.H;
    reinterpret_cast<uint4*>(dst)[v] = val;
  }
  __threadfence_system();
}

__global__ void ep_release_kernel(const EpParams p, int which) {
  const int q = threadIdx.x;
  if (q >= p.G) return;
  __threadfence_system();
  st_release_sys(reinterpret_cast<uint32_t*>(p.peers[q] + p.off_flags) + which * p.G + p.rank, *p.seq);
}

int ep_bump_launch(const EpParams& p, cudaStream_t s) {
  ep_bump_kernel<<<1, 1, 0, s>>>(p.seq);
  return set_cuda_error(cudaGetLastError(), "ep_bump_kernel");
}
int ep_dispatch_launch(const EpParams& p, const uint16_t* x, const int32_t* sel, int M, cudaStream_t s) {
  if (p.H % 8) return set_error(EINVAL_, "ep: H % 8 != 0");
  ep_dispatch_kernel<<<p.G, 256, 0, s>>>(p, x, sel, M);
  return set_cuda_error(cudaGetLastError(), "ep_dispatch_kernel");
}
int ep_wait_launch(const EpParams& p, int which, cudaStream_t s) {
  ep_wait_kernel<<<1, 32, 0, s>>>(p, which);
  return set_cuda_error(cudaGetLastError(), "ep_wait_kernel");
}
int ep_return_launch(const EpParams& p, const int32_t* slot_map, const uint16_t* rows, int M, int Gtok,
                     cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(Gtok) * p.T * (p.H / 8);
  const int blocks = static_cast<int>(std::min<int64_t>(std::max<int64_t>((total + 255) / 256, 1), 1024));
  ep_return_kernel<<<blocks, 256, 0, s>>>(p, slot_map, rows, M, Gtok);
  int rc = set_cuda_error(cudaGetLastError(), "ep_return_kernel");
  if (rc) return rc;
  ep_release_kernel<<<1, 32, 0, s>>>(p, 1);
  return set_cuda_error(cudaGetLastError(), "ep_release_kernel");
}

}  // namespace aipu
