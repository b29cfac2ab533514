// bf16 GEMV under the reference's bf16 dot-product contract (tools/glm_model_q4k_ref.py:474-486,
// matmul_bf16_dot; the LM head at :826): for token row x and weight row w (both bf16),
//   p_l = sequential fp32 sum over k = l, l + 7, l + 14, ... of fl(x_k * w_k)   (l = 0..6)
//   out = bf16( (fl(p0 + p1) + fl(p2 + p3)) + (fl(p4 + p5) + fl(p6 + 0)) )
// (bf16 x bf16 products are exact in fp32; every add rounds separately).
//
// HBM-bound: every weight byte is read once. One thread per weight row keeps the row's 7 partial
// sums (per token) in registers, so the 7 dependent add chains interleave; the row is read in
// 56-weight pieces (7 x 16-byte loads, 56 = lcm(7, 8) keeps every weight's chain index a
// compile-time constant). The activations are staged once per CTA in shared memory as fp32 (all
// lanes of a warp read the same element: broadcast).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace aipu {

template <int MT>
__device__ __forceinline__ void dot7_word(float (&ps)[MT][7], const float* xs, int K, int kbase, uint32_t wd,
                                          int lane_lo, int lane_hi) {
  const float wlo = __uint_as_float(wd << 16), whi = __uint_as_float(wd & 0xFFFF0000u);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    ps[m][lane_lo] = __fadd_rn(ps[m][lane_lo], __fmul_rn(xs[m * K + kbase], wlo));
    ps[m][lane_hi] = __fadd_rn(ps[m][lane_hi], __fmul_rn(xs[m * K + kbase + 1], whi));
  }
}

struct Dot7Params {
  const uint16_t* w;  // [V, K] bf16 rows
  int64_t V;
  int K;
  const uint16_t* x;  // [M, K] bf16
  int M;
  uint16_t* y;        // [M, V] bf16
};

template <int MT>
__global__ void __launch_bounds__(256) bf16_dot7_kernel(const __grid_constant__ Dot7Params p) {
  const uint16_t* __restrict__ w = p.w;
  const uint16_t* __restrict__ x = p.x;
  uint16_t* __restrict__ y = p.y;
  const int64_t V = p.V;
  const int K = p.K, M = p.M;
  extern __shared__ float xs[];  // [MT][K] fp32
  pdl_wait();
  for (int i = threadIdx.x; i < MT * K; i += blockDim.x) {
    const int m = i / K;
    xs[i] = (m < M) ? bf16_bits_to_f32(x[static_cast<int64_t>(m) * K + (i - m * K)]) : 0.f;
  }
  __syncthreads();
  const int K56 = K / 56 * 56;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < V;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4* row = reinterpret_cast<const uint4*>(w + v * K);
    float ps[MT][7];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int l = 0; l < 7; ++l) ps[m][l] = 0.f;
    for (int k0 = 0; k0 < K56; k0 += 56) {
      uint4 q[7];
#pragma unroll
      for (int j = 0; j < 7; ++j) q[j] = __ldg(row + (k0 >> 3) + j);
#pragma unroll
      for (int j = 0; j < 7; ++j) {
        const uint32_t wd[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const int kk = 8 * j + 2 * h;  // k0 is a multiple of 7: chain index = kk % 7
          dot7_word<MT>(ps, xs, K, k0 + kk, wd[h], kk % 7, (kk + 1) % 7);
        }
      }
    }
    // tail: K % 8 == 0, at most 6 more 8-weight pieces; piece t starts at K56 + 8 t, whose chain
    // index is t (8 = 1 mod 7)
#pragma unroll
    for (int t = 0; t < 6; ++t) {
      const int k0 = K56 + 8 * t;
      if (k0 < K) {
        const uint4 qt = __ldg(row + (k0 >> 3));
        const uint32_t wd[4] = {qt.x, qt.y, qt.z, qt.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) dot7_word<MT>(ps, xs, K, k0 + 2 * h, wd[h], (t + 2 * h) % 7, (t + 2 * h + 1) % 7);
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M) {
        const float a01 = __fadd_rn(ps[m][0], ps[m][1]), a23 = __fadd_rn(ps[m][2], ps[m][3]);
        const float a45 = __fadd_rn(ps[m][4], ps[m][5]), a6 = __fadd_rn(ps[m][6], 0.f);
        y[static_cast<int64_t>(m) * V + v] = bf16_rne_bits(__fadd_rn(__fadd_rn(a01, a23), __fadd_rn(a45, a6)));
      }
    }
  }
  pdl_launch_dependents();
}

template <int MT>
static int bf16_dot7_launch_mt(const uint16_t* w, int64_t V, int K, const uint16_t* x, int M, uint16_t* y,
                               int num_sms, cudaStream_t s, bool pdl) {
  const int smem = MT * K * 4;
  static bool attr[64] = {false};
  {
    const int arc = set_smem_attr_once(reinterpret_cast<const void*>(bf16_dot7_kernel<MT>), 227 * 1024, attr, "cudaFuncSetAttribute(bf16_dot7)");
    if (arc) return arc;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bf16_dot7_kernel<MT>, 256, smem);
  if (e != cudaSuccess) return set_cuda_error(e, "occupancy(bf16_dot7)");
  const int64_t need = (V + 255) / 256;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, static_cast<int64_t>(std::max(1, per_sm)) * num_sms)));
  Dot7Params p = {w, V, K, x, M, y};
  return launch_kernel(reinterpret_cast<const void*>(bf16_dot7_kernel<MT>), dim3(grid), dim3(256), smem, s, pdl, &p);
}

int bf16_dot7_launch(const uint16_t* w, int64_t V, int64_t K, const uint16_t* x, int64_t M, uint16_t* y, int num_sms,
                     cudaStream_t s, bool pdl) {
  if (V <= 0 || K <= 0 || M <= 0 || K % 8 || K > 14336 || (reinterpret_cast<uintptr_t>(w) & 15u))
    return set_error(EINVAL_, "bf16 dot GEMV: need K % 8 == 0, K <= 14336, 16-byte aligned weights");
  for (int64_t m0 = 0; m0 < M; m0 += 4) {
    const int mb = static_cast<int>(std::min<int64_t>(4, M - m0));
    const uint16_t* xm = x + m0 * K;
    uint16_t* ym = y + m0 * V;
    int rc;
    if (mb == 1)
      rc = bf16_dot7_launch_mt<1>(w, V, static_cast<int>(K), xm, 1, ym, num_sms, s, pdl);
    else if (mb == 2)
      rc = bf16_dot7_launch_mt<2>(w, V, static_cast<int>(K), xm, 2, ym, num_sms, s, pdl);
    else
      rc = bf16_dot7_launch_mt<4>(w, V, static_cast<int>(K), xm, mb, ym, num_sms, s, pdl);
    if (rc) return rc;
  }
  return OK;
}

}  // namespace aipu
