// Bit-exact device restatement of the reference's activation numerics:
//   fp32_rsqrt  -- Quake seed 0x5F3759DF + exactly 2 Newton steps (tools/glm_model_q4k_ref.py:96-116,
//                  RTL src/glm_fp.vh:324-348)
//   sigmoid/silu -- glm_act: sanitize, clamp +-16, k = round-half-up(z*log2e) clamped to +-64,
//                  r = z - k*ln2, degree-5 Horner exp, exponent add, 1/(1+e) as rsqrt^2
//                  (tools/glm_model_q4k_ref.py:214-299, RTL src/glm_act.v:19-72)
// Every fp32 op is a separate round-to-nearest op (__fmul_rn/__fadd_rn), matching the numpy
// golden op for op; none of CUDA's math library functions is used.
#pragma once
#include "common.cuh"

namespace aipu {

__device__ __forceinline__ float quake_rsqrt(float x) {
  uint32_t u = __float_as_uint(x);
  uint32_t e = (u >> 23) & 0xFFu, man = u & 0x7FFFFFu, sign = u >> 31;
  if ((e == 0xFFu && man != 0u) || sign == 1u || e == 0u) return __uint_as_float(0x7FC00000u);
  if (e == 0xFFu && man == 0u) return 0.0f;
  float xhalf = __fmul_rn(0.5f, x);
  float y = __uint_as_float(0x5F3759DFu - (u >> 1));
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float yy = __fmul_rn(y, y);
    float xyy = __fmul_rn(xhalf, yy);
    float t = __fadd_rn(1.5f, -xyy);
    y = __fmul_rn(y, t);
  }
  return y;
}

__device__ __forceinline__ float act_sanitize(float x) {
  uint32_t u = __float_as_uint(x);
  if (((u >> 23) & 0xFFu) == 0xFFu) return __uint_as_float((u & 0x80000000u) | 0x41800000u);
  return x;
}
__device__ __forceinline__ float act_clamp(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) >= 0x41800000u) return __uint_as_float((u & 0x80000000u) | 0x41800000u);
  return x;
}
__device__ __forceinline__ int act_round_to_int(float f) {
  uint32_t u = __float_as_uint(f);
  uint32_t s = u >> 31, e = (u >> 23) & 0xFFu, m = 0x800000u | (u & 0x7FFFFFu);
  int r;
  if (e < 127u) {
    r = (e == 126u) ? 1 : 0;
  } else {
    int rsh = 23 - static_cast<int>(e - 127u);
    rsh = rsh < 1 ? 1 : rsh;
    r = static_cast<int>((m >> rsh) & 0xFFu) + static_cast<int>((m >> (rsh - 1)) & 1u);
  }
  return s ? -r : r;
}
__device__ __forceinline__ float act_scale_pow2(float v, int k) {
  uint32_t u = __float_as_uint(v);
  int e_new = static_cast<int>((u >> 23) & 0xFFu) + k;
  uint32_t sgn = u & 0x80000000u;
  if (e_new >= 255) return __uint_as_float(sgn | (0xFEu << 23) | (u & 0x7FFFFFu));
  if (e_new <= 0) return __uint_as_float(sgn);
  return __uint_as_float(sgn | (static_cast<uint32_t>(e_new) << 23) | (u & 0x7FFFFFu));
}

// glm_act sigmoid core (fp32, unrounded)
__device__ __forceinline__ float glm_sigmoid_f32(float xbf) {
  float xcl = act_clamp(act_sanitize(xbf));
  float z = __uint_as_float(__float_as_uint(xcl) ^ 0x80000000u);
  float kf = __fmul_rn(z, __uint_as_float(0x3FB8AA3Bu));
  int k = act_round_to_int(kf);
  k = k < -64 ? -64 : (k > 64 ? 64 : k);
  float kfl = static_cast<float>(k);  // exact, |k| <= 64
  float r = __fadd_rn(z, -__fmul_rn(kfl, __uint_as_float(0x3F317218u)));
  float p = __fadd_rn(__uint_as_float(0x3D2AAAABu), __fmul_rn(r, __uint_as_float(0x3C088889u)));
  p = __fadd_rn(__uint_as_float(0x3E2AAAABu), __fmul_rn(r, p));
  p = __fadd_rn(__uint_as_float(0x3F000000u), __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  float ex = act_scale_pow2(p, k);
  float d = __fadd_rn(1.0f, ex);
  float t = quake_rsqrt(d);
  return __fmul_rn(t, t);
}
// bf16(sigmoid(x)) as a bf16-valued float
__device__ __forceinline__ float glm_sigmoid_bf(float xbf) { return bf16_round_f(glm_sigmoid_f32(xbf)); }
// bf16(sigmoid(x) * sanitize(x))
__device__ __forceinline__ float glm_silu_bf(float xbf) {
  float s = glm_sigmoid_f32(xbf);
  return bf16_round_f(__fmul_rn(s, act_sanitize(xbf)));
}

// order-preserving uint32 key of an fp32 (tools/glm_model_q4k_ref.py:684-688)
__device__ __forceinline__ uint32_t f32_order_key(float x) {
  uint32_t u = __float_as_uint(x);
  return (u >> 31) == 0u ? (u ^ 0x80000000u) : ~u;
}

}  // namespace aipu
