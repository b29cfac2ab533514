// Decode-time dequant GEMV / small-M GEMM for B200 (sm_100a).
//
//   y[m, n] = bf16( sum_k x[m, k] * w[n, k] ),   w stored as GGUF rows (Q4_K / Q6_K / Q8_0 / F16)
//
// Contract followed: tools/q4k_ref.py:67-92 (exact ggml dequant, fp32 MAC, bf16 RNE out). The MAC
// order differs from the reference's sequential K order (this kernel is within 1 bf16 ulp; the
// strict kernel in kernels.cu is the bit-exact one).
//
// Design (HBM-bound: ~0.56 B/weight for Q4_K, so the budget is ~3 thread-ops per weight):
//   * Persistent grid, one CTA per SM, NW (8..16) fully decoupled warps. There is no producer warp
//     and no CTA-wide barrier in the main loop: every warp is its own "worker".
//   * Work unit = 16 weight rows x 256 weights (one super-block column). The units of all tiles are
//     laid end to end and split evenly over all workers of the grid ("stream-K" at warp level); a
//     tile cut between workers is finished by the last worker to arrive, which sums the partials in
//     worker order (deterministic).
//   * Each warp streams its own chunks (16 rows x up to UPC units) into a private S-slot ring with
//     1-D bulk copies (cp.async.bulk, the untiled TMA path; no multicast): lanes 0..15 each copy one
//     row, completion on a per-slot mbarrier. Weights do not depend on the previous kernel, so with
//     programmatic dependent launch the first slots fill before griddepcontrol.wait.
//   * Consumers turn packed codes into exact fp16 operands with LOP3/PRMT magic-number tricks and
//     use mma.sync m16n8k16 (fp16 in, fp32 accumulate) as an exact-product dot engine: weight rows
//     are the 16 MMA rows, activation columns (tokens, or hi/lo halves of fp32 tokens) the 8 MMA
//     columns.
//   * Activations are staged once per CTA (per group the CTA touches, when groups have their own
//     activations) as fp16 with a per-token power-of-two prescale (exact for bf16 input; fp32
//     input is split into hi + lo fp16 columns).
//   * Q4_K: A = sc*q (exact in fp16, <= 945), so one fp32 accumulator per super-block, then
//     acc += d*P - dmin*Cm, where Cm = sum_j m_j * sum_{k in j} x_k comes from one more MMA with
//     A = m (6-bit mins) and B = per-sub-block activation sums (hi/lo fp16).
#pragma once
#include <cuda.h>

#include "act.cuh"
#include "common.cuh"

namespace aipu {

constexpr int GEMV_MAXW = 16;   // warps per CTA (each an independent worker)
constexpr int GEMV_MAXS = 4;    // ring slots per warp
constexpr int GEMV_MAXXG = 4;   // activation groups staged per CTA

enum Epi : int { EPI_STORE = 0, EPI_SWIGLU = 1 };

struct GemvParams {
  const uint8_t* w0;         // rows of the matrix (or the gate rows for EPI_SWIGLU)
  const uint8_t* w1;         // up rows (EPI_SWIGLU)
  int64_t row_bytes;         // bytes per row
  int64_t expert_stride;     // bytes between consecutive experts of w0/w1
  const int* group_ids;      // device: expert id of each group, or nullptr (group g = expert g)
  const int* n_groups_dev;   // device: number of groups, or nullptr (use n_groups)
  int n_groups;              // number of groups (upper bound when n_groups_dev is set)
  int N;                     // rows per matrix
  int K;                     // reduction length (multiple of 256)
  const void* x;             // activations [M, K] (fp32 or bf16), group g at x + g*x_group_stride
  int64_t x_group_stride;    // elements
  int M;                     // tokens (<= 8 bf16, <= 4 fp32)
  uint16_t* y;               // bf16 out [M, N] per group (EPI_SWIGLU: h [M, N])
  int64_t y_group_stride;    // elements
  float* partials;           // stream-K workspace [grid][2][32][4]
  int* counters;             // stream-K arrival counters, one per tile, zero between launches
  int* status;               // device status word
  int upc;                   // units (256-weight columns) per ring slot
  int pitch;                 // shared-memory row pitch of a slot
  int nslots;                // ring slots per warp
  int xpitch;                // shared-memory bytes per activation column
  int xg;                    // activation groups staged per CTA (1 when x is shared by all groups)
  int n_experts;             // extent of the expert dimension of w0/w1 (tensor maps)
  int use_tmap;              // 1: each slot is filled by one tiled TMA request (two for EPI_SWIGLU)
  int ids_ready;             // 1: group_ids / n_groups_dev were complete before the launch preceding this
                             // one began, so they are read (and weights prefetched) before
                             // griddepcontrol.wait
  int tm_esz;                // tensor-map element size (bytes)
  int tm_box;                // tensor-map box width (elements)
  int cta_mode;              // 1: whole tiles per CTA, tiles cut between its warps summed in shared memory
  alignas(64) CUtensorMap tmap0;  // [expert][row][row bytes / esz] over w0
  alignas(64) CUtensorMap tmap1;  // same over w1 (EPI_SWIGLU)
};

__host__ __device__ inline int gemv_slot_pitch(int wt, int upc) {
  // room for the unit bytes plus a possible 16-byte-alignment head, rounded so that rows start
  // 32 or 96 bytes mod 128 (rows g = 0..3 of a half-warp then hit distinct banks)
  int p = (upc * unit_bytes(wt) + ((wt == WT_Q6K) ? 15 : 0) + 15) & ~15;
  while (p % 128 != 32 && p % 128 != 96) p += 16;
  return p;
}

// ---------------------------------------------------------------------------------- x staging
// Q4_K/Q6_K/Q8_0 operands are built as pairs (k0,k2) and (k1,k3) of every aligned group of four
// weights, so the activation columns are stored with the same order (0,2,1,3) in each group.
__device__ __forceinline__ int xswz(int k, bool swz) { return swz ? ((k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1)) : k; }

}  // namespace aipu
