// Expert-parallel exchange over NVLink peer memory (one process per GPU, CUDA IPC mappings).
//
// Every rank owns one symmetric buffer (same layout on every rank) that its peers map:
//   flags   [2][G] uint32   dispatch / return arrival flags, written by peers (sequence numbers)
//   in_sel  [G][M][T]       selections of every rank's tokens (M = this call's tokens per rank, the
//   in_x    [G][M][H]       bf16 tokens of every rank          same on every rank, <= capacity)
//   out     [G][M][T][H]    bf16 per-slot expert outputs for this rank's tokens, one piece per rank
// A layer call runs with the sequence number *seq + 1 (the device counter holds the last completed
// call; the combine kernel advances it at the end); writers store data with plain peer stores, make
// them visible system-wide, then release the flag (st.release.sys); the consuming kernels (union,
// combine) acquire the flags with a bounded spin before reading (no wait can run forever: on expiry
// the status word is set and the kernel skips the exchanged data). No TMA and no multicast touches peer memory; only plain loads and stores.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "ep_sync.cuh"
#include "kernels.h"
#include "launch.h"

namespace aipu {

// CTA q: copy this rank's M tokens and selections into peer q's inbox slot `rank`, then release
// peer q's dispatch flag[rank] = seq.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpParams p, const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ sel, int M) {
  const int q = blockIdx.x;
  const uint32_t seq = *p.seq + 1u;
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

// Return: for gathered token t (owner q = t / M, local row m = t % M), every slot s
// whose expert is local (index >= 0 into the union rows `rows` [U][Gtok][H]) is stored into peer q's
// out[rank][m][s]. Each CTA makes its stores visible system-wide; the last CTA to arrive releases the
// return flags of every peer.
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
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(p.seq + 1, 1u) == gridDim.x - 1) {
    p.seq[1] = 0u;
    __threadfence_system();
    const uint32_t seq = *p.seq + 1u;
    for (int q = 0; q < p.G; ++q)
      st_release_sys(reinterpret_cast<uint32_t*>(p.peers[q] + p.off_flags) + p.G + p.rank, seq);
  }
}

EpSync ep_sync(const EpParams& p, int which, bool bump) {
  EpSync w;
  w.flags = reinterpret_cast<const uint32_t*>(p.peers[p.rank] + p.off_flags) + which * p.G;
  w.n = p.G;
  w.seq = p.seq;
  w.status = p.status;
  w.bump_arrive = bump ? p.seq + 2 : nullptr;
  return w;
}
int ep_dispatch_launch(const EpParams& p, const uint16_t* x, const int32_t* sel, int M, cudaStream_t s) {
  if (p.H % 8) return set_error(EINVAL_, "ep: H % 8 != 0");
  ep_dispatch_kernel<<<p.G, 256, 0, s>>>(p, x, sel, M);
  return set_cuda_error(cudaGetLastError(), "ep_dispatch_kernel");
}
int ep_return_launch(const EpParams& p, const int32_t* slot_map, const uint16_t* rows, int M, int Gtok,
                     cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(Gtok) * p.T * (p.H / 8);
  const int blocks = static_cast<int>(std::min<int64_t>(std::max<int64_t>((total + 255) / 256, 1), 1024));
  ep_return_kernel<<<blocks, 256, 0, s>>>(p, slot_map, rows, M, Gtok);
  return set_cuda_error(cudaGetLastError(), "ep_return_kernel");
}

}  // namespace aipu
