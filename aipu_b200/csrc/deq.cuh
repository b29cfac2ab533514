// Exact per-weight dequantisation of one GGUF row (bit-exact to the reference golden).
//
// Q4_K: tools/q4k_ref.py:27-61   w = fsub(fmul(fmul(d, sc), q), fmul(dmin, m))
// Q6_K: tools/q4k_ref.py:105-124 w = fmul(fmul(d, f32(int8 sc[p/16])), f32(q - 32))
// Q8_0: tools/q4k_ref.py:126-129 w = fmul(d, f32(int8 q))
// F16 : exact widen;  F32: as stored.
// Used by the dequant kernel and by the strict (sequential, bit-exact) GEMM / router kernels.
#pragma once
#include "common.cuh"

namespace aipu {

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
}

// 6-bit (scale, min) of sub-block j of a Q4_K super-block (get_scale_min_k4, q4k_ref.py:27-37)
__device__ __forceinline__ void q4k_scale_min(const uint8_t* q, int j, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = q[j] & 63u;
    m = q[j + 4] & 63u;
  } else {
    sc = (q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// weight k of a row stored in type wt (row points at the row's first byte)
__device__ __forceinline__ float deq_one(int wt, const uint8_t* row, int64_t k) {
  switch (wt) {
    case WT_Q4K: {
      const uint8_t* b = row + (k >> 8) * 144;
      int kk = static_cast<int>(k & 255);
      int sub = kk >> 5, grp = kk >> 6, l = kk & 31;
      float d = f16_bits_to_f32(ld_u16(b));
      float dmin = f16_bits_to_f32(ld_u16(b + 2));
      uint32_t sc, m;
      q4k_scale_min(b + 4, sub, sc, m);
      uint32_t byte = b[16 + 32 * grp + l];
      uint32_t q = (sub & 1) ? (byte >> 4) : (byte & 0xFu);
      float d1 = __fmul_rn(d, static_cast<float>(sc));
      float m1 = __fmul_rn(dmin, static_cast<float>(m));
      return __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
    }
    case WT_Q6K: {
      const uint8_t* b = row + (k >> 8) * 210;
      int p = static_cast<int>(k & 255);
      int hf = p >> 7, r = p & 127, j = r >> 5, l = r & 31;
      const uint8_t* ql = b + 64 * hf;
      const uint8_t* qh = b + 128 + 32 * hf;
      uint32_t lowq = (j & 1) ? ql[32 + l] : ql[l];
      uint32_t nib = (j >= 2) ? (lowq >> 4) : (lowq & 0xFu);
      uint32_t hi2 = (qh[l] >> (2 * j)) & 3u;
      int q = static_cast<int>(nib | (hi2 << 4)) - 32;
      int sc = static_cast<int>(static_cast<int8_t>(b[192 + (p >> 4)]));
      float d = f16_bits_to_f32(ld_u16(b + 208));
      return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q));
    }
    case WT_Q80: {
      const uint8_t* b = row + (k >> 5) * 34;
      float d = f16_bits_to_f32(ld_u16(b));
      int q = static_cast<int>(static_cast<int8_t>(b[2 + (k & 31)]));
      return __fmul_rn(d, static_cast<float>(q));
    }
    case WT_F16:
      return f16_bits_to_f32(ld_u16(row + 2 * k));
    default: {
      uint32_t u = static_cast<uint32_t>(row[4 * k]) | (static_cast<uint32_t>(row[4 * k + 1]) << 8) |
                   (static_cast<uint32_t>(row[4 * k + 2]) << 16) | (static_cast<uint32_t>(row[4 * k + 3]) << 24);
      return __uint_as_float(u);
    }
  }
}

__host__ __device__ inline int64_t row_bytes_of(int wt, int64_t K) {
  switch (wt) {
    case WT_Q4K: return (K / 256) * 144;
    case WT_Q6K: return (K / 256) * 210;
    case WT_Q80: return (K / 32) * 34;
    case WT_F16: return K * 2;
    default: return K * 4;
  }
}

}  // namespace aipu
