// Bit-exact dequant GEMV on sequential fp32 chains (the reference's GEMM contract, tools/q4k_ref.py:86-92:
// acc = fl(acc + fl(x_k * w_k)) for k = 0..K-1 in order, then bf16 RNE), fast enough to be the MoE
// decode path.
//
// Why it can be fast: for Q4_K, w = fl(fl(d*sc)*q - fl(dmin*m)) (tools/q4k_ref.py:39-61) where d*sc and
// dmin*m are exact in fp32 (11-bit fp16 times 6-bit integer) and d*sc*q is exact too (21 bits), so
// w = fma(d*sc, q, -dmin*m) with one rounding -- the same value. For Q6_K, w = fl(d*sc)*q is exact
// (18 + 6 bits). A code q at bit position p of a packed word becomes the float 2^23 + q * 2^p with one
// LOP3 (mask the code, OR the exponent of 2^23), one FADD removes 2^23, and the 2^p is folded into the
// (exact, power-of-two scaled) sub-block scale. Every fp32 operation is an IEEE round-to-nearest op in
// the reference's order; the packed f32x2 forms of sm_100 (one instruction, two independent lanes)
// carry two rows per thread, so a weight pair costs about 2 integer ops + 4 packed fp32 ops + x.
//
// Structure: persistent CTAs of NT consumer threads (two rows each: rows a, b of a 2 NT-row tile, or the
// gate and up rows n of a SwiGLU tile) and one producer warp. Per stage (one 256-weight super-block
// column of the tile) the producer issues one tiled TMA per operand (no multicast) and converts the
// stage's activations of the item's tokens to fp32 pairs (x, x) in shared memory; the consumers run
// their chains through the stage in k order. Items = (group, row tile, pass of <= MT tokens).
#include <algorithm>
#include <cstdio>

#include "act.cuh"
#include "common.cuh"
#include "deq.cuh"
#include "kernels.h"
#include "launch.h"

namespace aipu {

constexpr int CH_MAXS = 6;       // ring stages
constexpr uint32_t MAG = 0x4B000000u;   // 2^23
constexpr float MAGF = 8388608.0f;

template <int WT>
struct ChainGeom {
  static constexpr int BOX = (WT == WT_Q4K) ? 18 : 30;  // 8-byte elements per row per stage
  static constexpr int PITCH = BOX * 8;                  // 144 / 240 bytes: 16 x odd, conflict-free LDS.128
};

// Packed fp32 pair arithmetic (sm_100 f32x2) with explicit .rn rounding. Every product and sum must
// round separately, as the reference's numpy float32 ops do, but a packed multiply whose result feeds a
// packed add is contracted into one packed fma by the assembler even with .rn on both and -fmad=false
// (measured on B200: most long chains then end one fp32 ulp off). The product x * w is therefore
// formed as fma(x, w, z) with z = -0.0 read from the kernel parameters: x * w + (-0) is exactly
// fl(x * w) (signed zeros included), and an fma with an addend unknown at compile time is not merged
// into the following add.
__device__ __forceinline__ unsigned long long pk(float2 a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
__device__ __forceinline__ float2 upk(unsigned long long r) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
  return a;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
  return upk(d);
}
__device__ __forceinline__ float2 f2(uint32_t a, uint32_t b) { return make_float2(__uint_as_float(a), __uint_as_float(b)); }
__device__ __forceinline__ float2 f2s(float a) { return make_float2(a, a); }

__device__ __forceinline__ uint4 ch_lds4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t ch_lds1(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 ch_ldsf4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lop_mag(uint32_t w, uint32_t mask) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "r"(mask), "r"(MAG));
  return d;
}
// byte `b` of `tab` as the float 2^23 + byte (PRMT with 0x4B000000 as the upper source)
__device__ __forceinline__ uint32_t byte_mag(uint32_t tab, int b) { return prmt(tab, MAG, 0x7440u | b); }

// one chain step for a weight pair (rows a, b) given as magic floats: q = Q - C (exact),
// w = fma(s, q, nm) (one rounding: the reference's fl(fl(s*q) - m) when s*q is exact) or s * q,
// then per token acc = fl(acc + fl(x * w)).
template <int CNT>
__device__ __forceinline__ void chain_tok(float2 (&acc)[8], const float2 w, const float2 (&xv)[8], const float2 nz) {
#pragma unroll
  for (int t = 0; t < CNT; ++t) acc[t] = add2(acc[t], fma2(xv[t], w, nz));
}

// x pairs (x_k, x_k) of the CNT tokens for k and k + 1 (stage x block: [MT][256] float2)
template <int CNT>
__device__ __forceinline__ void load_x2(uint32_t xs, int k, float2 (&x0)[8], float2 (&x1)[8]) {
#pragma unroll
  for (int t = 0; t < CNT; ++t) {
    const float4 v = ch_ldsf4(xs + t * 2048 + 8 * k);
    x0[t] = make_float2(v.x, v.y);
    x1[t] = make_float2(v.z, v.w);
  }
}

// ------------------------------------------------------------------ Q4_K super-block (256 k)
template <int CNT>
__device__ __forceinline__ void q4k_sb(uint32_t ra, uint32_t rb, uint32_t xs, float2 (&acc)[8], const float2 nz) {
  const uint4 ha = ch_lds4(ra), hb = ch_lds4(rb);
  const float2 d = make_float2(f16_bits_to_f32(ha.x), f16_bits_to_f32(hb.x));
  const float2 dm = make_float2(f16_bits_to_f32(ha.x >> 16), f16_bits_to_f32(hb.x >> 16));
  // the 6-bit scale/min tables of get_scale_min_k4 (tools/q4k_ref.py:27-37), byte j = entry j
  const uint32_t sa03 = ha.y & 0x3F3F3F3Fu, ma03 = ha.z & 0x3F3F3F3Fu;
  const uint32_t sa47 = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
  const uint32_t ma47 = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
  const uint32_t sb03 = hb.y & 0x3F3F3F3Fu, mb03 = hb.z & 0x3F3F3F3Fu;
  const uint32_t sb47 = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
  const uint32_t mb47 = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
  const float2 nmag = f2s(-MAGF);
  // two 64-weight groups per iteration (measured: one per iteration leaves latency exposed, all four
  // overflow the instruction cache)
#pragma unroll 2
  for (int g = 0; g < 4; ++g) {
    // sub-blocks 2g (low nibbles) and 2g + 1 (high nibbles): d1 = d*sc, m1 = dmin*m, both exact
    const bool hi4 = g >= 2;
    const uint32_t tsa = hi4 ? sa47 : sa03, tsb = hi4 ? sb47 : sb03;
    const uint32_t tma = hi4 ? ma47 : ma03, tmb = hi4 ? mb47 : mb03;
    const int bl = (2 * g) & 3, bh = (2 * g + 1) & 3;
    const float2 scl = add2(f2(byte_mag(tsa, bl), byte_mag(tsb, bl)), nmag);
    const float2 mnl = add2(f2(byte_mag(tma, bl), byte_mag(tmb, bl)), nmag);
    const float2 sch = add2(f2(byte_mag(tsa, bh), byte_mag(tsb, bh)), nmag);
    const float2 mnh = add2(f2(byte_mag(tma, bh), byte_mag(tmb, bh)), nmag);
    const float2 d1l = mul2(d, scl), d1h = mul2(d, sch);
    const float2 nm1l = mul2(dm, make_float2(-mnl.x, -mnl.y));
    const float2 nm1h = mul2(dm, make_float2(-mnh.x, -mnh.y));
    // power-of-two scaled copies for the bit position of each code (exact)
    const float2 l0 = d1l, l8 = mul2(d1l, f2s(0x1p-8f)), l16 = mul2(d1l, f2s(0x1p-16f));
    const float2 h4 = mul2(d1h, f2s(0x1p-4f)), h12 = mul2(d1h, f2s(0x1p-12f));
    const uint4 a0 = ch_lds4(ra + 16 + 32 * g), a1 = ch_lds4(ra + 32 + 32 * g);
    const uint4 b0 = ch_lds4(rb + 16 + 32 * g), b1 = ch_lds4(rb + 32 + 32 * g);
    const uint32_t A[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t B[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    // low nibbles: weights 64g + 4w + b, b = 0..3 (byte b of word w)
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int k = 64 * g + 4 * w;
      const uint32_t As = A[w] >> 16, Bs = B[w] >> 16;
      float2 x0[8], x1[8], x2[8], x3[8];
      load_x2<CNT>(xs, k, x0, x1);
      load_x2<CNT>(xs, k + 2, x2, x3);
      float2 q, wv;
      q = add2(f2(lop_mag(A[w], 0xFu), lop_mag(B[w], 0xFu)), nmag);
      wv = fma2(l0, q, nm1l);
      chain_tok<CNT>(acc, wv, x0, nz);
      q = add2(f2(lop_mag(A[w], 0xF00u), lop_mag(B[w], 0xF00u)), nmag);
      wv = fma2(l8, q, nm1l);
      chain_tok<CNT>(acc, wv, x1, nz);
      q = add2(f2(lop_mag(A[w], 0xF0000u), lop_mag(B[w], 0xF0000u)), nmag);
      wv = fma2(l16, q, nm1l);
      chain_tok<CNT>(acc, wv, x2, nz);
      q = add2(f2(lop_mag(As, 0xF00u), lop_mag(Bs, 0xF00u)), nmag);
      wv = fma2(l8, q, nm1l);
      chain_tok<CNT>(acc, wv, x3, nz);
    }
    // high nibbles: weights 64g + 32 + 4w + b
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int k = 64 * g + 32 + 4 * w;
      const uint32_t As = A[w] >> 16, Bs = B[w] >> 16;
      float2 x0[8], x1[8], x2[8], x3[8];
      load_x2<CNT>(xs, k, x0, x1);
      load_x2<CNT>(xs, k + 2, x2, x3);
      float2 q, wv;
      q = add2(f2(lop_mag(A[w], 0xF0u), lop_mag(B[w], 0xF0u)), nmag);
      wv = fma2(h4, q, nm1h);
      chain_tok<CNT>(acc, wv, x0, nz);
      q = add2(f2(lop_mag(A[w], 0xF000u), lop_mag(B[w], 0xF000u)), nmag);
      wv = fma2(h12, q, nm1h);
      chain_tok<CNT>(acc, wv, x1, nz);
      q = add2(f2(lop_mag(As, 0xF0u), lop_mag(Bs, 0xF0u)), nmag);
      wv = fma2(h4, q, nm1h);
      chain_tok<CNT>(acc, wv, x2, nz);
      q = add2(f2(lop_mag(As, 0xF000u), lop_mag(Bs, 0xF000u)), nmag);
      wv = fma2(h12, q, nm1h);
      chain_tok<CNT>(acc, wv, x3, nz);
    }
  }
}

// ------------------------------------------------------------------ Q6_K super-block (256 k)
// Layout [ql 128][qh 64][int8 sc 16][fp16 d] (tools/q4k_ref.py:105-124): for half h and l = 0..31,
// weight 128h + 32c + l has code c = 0: ql[64h+l] low | qh[32h+l] bits 0-1 << 4, c = 1: ql[64h+32+l] low |
// bits 2-3, c = 2: ql[64h+l] high | bits 4-5, c = 3: ql[64h+32+l] high | bits 6-7; scale sc[8h + 2c + l/16];
// w = fl(d * sc) * (code - 32), exact.
__device__ __forceinline__ uint32_t sext_byte(uint32_t w, int b) {
  const uint32_t s = 8u | static_cast<uint32_t>(b);
  return prmt(w, 0u, static_cast<uint32_t>(b) | (s << 4) | (s << 8) | (s << 12));
}
// Words i = 0..n-1 starting `head` bytes (even, < 16) into a window of 16-byte chunks loaded with
// conflict-free LDS.128 from a 16-byte-aligned row address (rows 240 bytes apart: an odd number of
// 16-byte units, so the 8 lanes of each LDS.128 phase hit distinct banks).
template <int NW, int NCH>
__device__ __forceinline__ void q6k_words(uint32_t row16, int head, uint32_t (&out)[NW]) {
  uint32_t win[4 * NCH];
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const uint4 v = ch_lds4(row16 + 16 * j);
    win[4 * j] = v.x;
    win[4 * j + 1] = v.y;
    win[4 * j + 2] = v.z;
    win[4 * j + 3] = v.w;
  }
  // realign by head bytes: word offset head >> 2 (warp-uniform, 4 cases), then half-word shift
  const uint32_t sel = (head & 2) ? 0x5432u : 0x3210u;
  switch (head >> 2) {
#define AIPU_Q6W(O)                                                                               \
  case O:                                                                                         \
    _Pragma("unroll") for (int i = 0; i < NW; ++i) out[i] = __byte_perm(win[i + O], win[i + O + 1], sel); \
    break;
    AIPU_Q6W(0)
    AIPU_Q6W(1)
    AIPU_Q6W(2)
    default:
      _Pragma("unroll") for (int i = 0; i < NW; ++i) out[i] = __byte_perm(win[i + 3], win[i + 4], sel);
      break;
#undef AIPU_Q6W
  }
}

template <int CNT>
__device__ __forceinline__ void q6k_sb(uint32_t ra16, uint32_t rb16, int head, uint32_t xs, float2 (&acc)[8],
                                       const float2 nz) {
  // scales and d: bytes 192..209 of the super-block
  uint32_t ta[5], tb[5];
  q6k_words<5, 3>(ra16 + 192, head, ta);
  q6k_words<5, 3>(rb16 + 192, head, tb);
  const float2 d = make_float2(f16_bits_to_f32(ta[4]), f16_bits_to_f32(tb[4]));
  const float2 c0 = f2s(-(MAGF + 32.f)), c1 = f2s(-(MAGF + 8192.f)), c2 = f2s(-(MAGF + 2097152.f));
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    // ql[64h .. 64h + 64) and qh[32h .. 32h + 32) of both rows, realigned into registers
    uint32_t A[16], Q[8], B2[16], Q2[8];
    q6k_words<16, 5>(ra16 + 64 * h, head, A);
    q6k_words<8, 3>(ra16 + 128 + 32 * h, head, Q);
    q6k_words<16, 5>(rb16 + 64 * h, head, B2);
    q6k_words<8, 3>(rb16 + 128 + 32 * h, head, Q2);
    const uint32_t sa_lo = h ? ta[2] : ta[0], sa_hi = h ? ta[3] : ta[1];
    const uint32_t sb_lo = h ? tb[2] : tb[0], sb_hi = h ? tb[3] : tb[1];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      // sub-block scales sc[8h + 2c + l/16], l/16 = 0 (words 0..3) and 1 (words 4..7): exact d * sc
      float2 dsc[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 2 * c + hh;
        const int ia = static_cast<int>(sext_byte(i < 4 ? sa_lo : sa_hi, i & 3));
        const int ib = static_cast<int>(sext_byte(i < 4 ? sb_lo : sb_hi, i & 3));
        // int8 -> float via 1.5 * 2^23 + v (exact for |v| < 2^22)
        const float2 sv = add2(f2(0x4B400000u + static_cast<uint32_t>(ia), 0x4B400000u + static_cast<uint32_t>(ib)),
                               f2s(-12582912.0f));
        dsc[hh] = mul2(d, sv);
      }
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const int k = 128 * h + 32 * c + 4 * w;  // h is a loop variable: k is an offset into xs
        const uint32_t qla = A[8 * (c & 1) + w], qlb = B2[8 * (c & 1) + w];
        const uint32_t qha = Q[w], qhb = Q2[w];
        uint32_t ca, cb;
        if (c == 0) {
          ca = (qla & 0x0F0F0F0Fu) | ((qha << 4) & 0x30303030u);
          cb = (qlb & 0x0F0F0F0Fu) | ((qhb << 4) & 0x30303030u);
        } else if (c == 1) {
          ca = (qla & 0x0F0F0F0Fu) | ((qha << 2) & 0x30303030u);
          cb = (qlb & 0x0F0F0F0Fu) | ((qhb << 2) & 0x30303030u);
        } else if (c == 2) {
          ca = ((qla >> 4) & 0x0F0F0F0Fu) | (qha & 0x30303030u);
          cb = ((qlb >> 4) & 0x0F0F0F0Fu) | (qhb & 0x30303030u);
        } else {
          ca = ((qla >> 4) & 0x0F0F0F0Fu) | ((qha >> 2) & 0x30303030u);
          cb = ((qlb >> 4) & 0x0F0F0F0Fu) | ((qhb >> 2) & 0x30303030u);
        }
        const uint32_t cas = ca >> 16, cbs = cb >> 16;
        const float2 s0 = dsc[w >> 2];
        const float2 s8 = mul2(s0, f2s(0x1p-8f)), s16 = mul2(s0, f2s(0x1p-16f));
        float2 x0[8], x1[8], x2[8], x3[8];
        load_x2<CNT>(xs, k, x0, x1);
        load_x2<CNT>(xs, k + 2, x2, x3);
        float2 q, wv;
        q = add2(f2(lop_mag(ca, 0x3Fu), lop_mag(cb, 0x3Fu)), c0);
        wv = mul2(s0, q);
        chain_tok<CNT>(acc, wv, x0, nz);
        q = add2(f2(lop_mag(ca, 0x3F00u), lop_mag(cb, 0x3F00u)), c1);
        wv = mul2(s8, q);
        chain_tok<CNT>(acc, wv, x1, nz);
        q = add2(f2(lop_mag(ca, 0x3F0000u), lop_mag(cb, 0x3F0000u)), c2);
        wv = mul2(s16, q);
        chain_tok<CNT>(acc, wv, x2, nz);
        q = add2(f2(lop_mag(cas, 0x3F00u), lop_mag(cbs, 0x3F00u)), c1);
        wv = mul2(s8, q);
        chain_tok<CNT>(acc, wv, x3, nz);
      }
    }
  }
}

// ------------------------------------------------------------------ items
struct ChainItem {
  int g, tile, pass, cnt;
  int tok[8];
};

// Token set of group g: bit m set when some slot of token m maps to g (all M tokens without a slot map).
__device__ __forceinline__ uint32_t group_token_mask(const ChainParams& p, int g, int lane) {
  if (!p.slot_map) return 0u;
  uint32_t m = 0u;
  for (int i = lane; i < p.M * p.topk; i += 32)
    if (p.slot_map[i] == g) m |= 1u << (i / p.topk);
  return __reduce_or_sync(0xffffffffu, m);
}

__device__ __forceinline__ int chain_passes(const ChainParams& p) {
  if (p.tiles) return 1;
  return ((p.slot_map ? min(p.M, 32) : p.M) + p.mt - 1) / p.mt;
}

// Item idx = (group, row tile, pass): pass p takes tokens [p mt, (p + 1) mt) of the group's token
// list (the set bits of its mask in ascending order, or tokens 0..M-1 without a slot map). In tile
// mode the group is a perm tile (one expert, <= 8 tokens). Every warp enumerates the same sequence;
// items without tokens are skipped by all of them. xrow/yrow: activation and output row of token j.
__device__ __forceinline__ void item_at(const ChainParams& p, int idx, int lane, ChainItem& ci, int (&xrow)[8],
                                        int (&yrow)[8], int& expert) {
  const int passes = chain_passes(p);
  const int per_g = p.tiles_per_group * passes;
  ci.g = idx / per_g;
  const int r = idx - ci.g * per_g;
  ci.tile = r / passes;
  ci.pass = r - ci.tile * passes;
  if (p.tiles) {
    const int4 t = p.tiles[ci.g];
    expert = t.x;
    ci.cnt = min(t.z, 8);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int pos = t.y + min(c, max(ci.cnt - 1, 0));
      yrow[c] = pos;
      xrow[c] = p.x_by_pos ? pos : max(p.perm_tok[pos], 0);
    }
    return;
  }
  expert = p.group_ids ? p.group_ids[ci.g] : ci.g;
  if (p.slot_map) {
    uint32_t m = group_token_mask(p, ci.g, lane);
    for (int i = 0; i < ci.pass * p.mt && m; ++i) m &= m - 1;
    int c = 0;
    while (m && c < p.mt) {
      ci.tok[c++] = __ffs(m) - 1;
      m &= m - 1;
    }
    ci.cnt = c;
  } else {
    const int m0 = ci.pass * p.mt;
    ci.cnt = min(p.mt, p.M - m0);
#pragma unroll
    for (int c = 0; c < 8; ++c) ci.tok[c] = m0 + c;
  }
  const int64_t ys = p.y_group_stride / max(p.N, 1);  // output rows per group
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int t = ci.tok[min(c, max(ci.cnt - 1, 0))];
    xrow[c] = static_cast<int>(static_cast<int64_t>(ci.g) * (p.x_group_stride / p.K) + t);
    yrow[c] = static_cast<int>(static_cast<int64_t>(ci.g) * ys + t);
  }
}

template <int WT, int EPI, int MT, int CH_NT>
__global__ void __launch_bounds__(CH_NT + 32) aipu_chain_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int PITCH = ChainGeom<WT>::PITCH;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + CH_MAXS;
  uint8_t* ring = smem + 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.nstages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);            // producer lane 0's expect_tx arrival + 32 x-writer lanes
      mbar_init(&empty[s], CH_NT / 32);   // one arrival per consumer warp
    }
    fence_mbar_init();
  }
  __syncthreads();
  // the token lists and activations come from the preceding kernels (programmatic dependent launch
  // only for grids of at most one CTA per SM, see chain_launch)
  pdl_wait();
  const int ngroups = p.tiles ? min(*p.n_tiles_dev, p.max_tiles)
                              : (p.n_groups_dev ? min(*p.n_groups_dev, p.n_groups) : p.n_groups);
  const int n_items = ngroups * p.tiles_per_group * chain_passes(p);
  const int nsb = p.K >> 8;
  const int rows_tile = (EPI == CHAIN_SWIGLU) ? CH_NT : 2 * CH_NT;

  if (warp == CH_NT / 32) {
    // ---------------------------------------------------------------- producer warp
    int it = 0;
    bool ok = true;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
      ChainItem ci;
      int xrow[8], yrow[8], e;
      item_at(p, idx, lane, ci, xrow, yrow, e);
      if (ci.cnt == 0) continue;
      const int row0 = ci.tile * rows_tile;
      const int esz = p.x_f32 ? 4 : 2;
      const uint8_t* xg = static_cast<const uint8_t*>(p.x);
      for (int sb = 0; sb < nsb; ++sb, ++it) {
        const int s = it % S;
        if (it >= S && !mbar_wait_bounded(&empty[s], ((it / S) - 1) & 1, p.status, ST_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        uint8_t* st = ring + s * p.stage_bytes;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(p.w_bytes));
          const int xc = (WT == WT_Q4K) ? 18 * sb : ((210 * sb) & ~15) / 8;
          if (EPI == CHAIN_SWIGLU) {
            tma_load_3d(st, &p.tmap0, xc, row0, e, &full[s]);
            tma_load_3d(st + CH_NT * PITCH, &p.tmap1, xc, row0, e, &full[s]);
          } else {
            tma_load_3d(st, &p.tmap0, xc, row0, e, &full[s]);
          }
        }
        // activations of the item's tokens for k in [256 sb, 256 sb + 256) as (x, x) fp32 pairs
        float2* xs = reinterpret_cast<float2*>(st + p.w_bytes);
        for (int t = 0; t < ci.cnt; ++t) {
          const uint8_t* xr = xg + (static_cast<int64_t>(xrow[t]) * p.K + 256 * sb) * esz;
          float4* dst = reinterpret_cast<float4*>(xs + t * 256 + 8 * lane);
          if (p.x_f32) {
            const float4 v0 = __ldg(reinterpret_cast<const float4*>(xr) + 2 * lane);
            const float4 v1 = __ldg(reinterpret_cast<const float4*>(xr) + 2 * lane + 1);
            dst[0] = make_float4(v0.x, v0.x, v0.y, v0.y);
            dst[1] = make_float4(v0.z, v0.z, v0.w, v0.w);
            dst[2] = make_float4(v1.x, v1.x, v1.y, v1.y);
            dst[3] = make_float4(v1.z, v1.z, v1.w, v1.w);
          } else {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr) + lane);
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float lo = __uint_as_float(w4[i] << 16), hi = __uint_as_float(w4[i] & 0xFFFF0000u);
              dst[i] = make_float4(lo, lo, hi, hi);
            }
          }
        }
        mbar_arrive(&full[s]);
      }
    }
    if (!ok) {
      // a consumer stopped: wait (bounded) for the copies already issued before leaving
      for (int j = max(0, it - S); j < it; ++j)
        mbar_wait_bounded(&full[j % S], (j / S) & 1, p.status, ST_TIMEOUT_FULL, 200000000LL);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int tid = threadIdx.x;
  const float2 nz = make_float2(p.neg_zero, p.neg_zero);
  int it = 0;
  bool ok = true;
  for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
    ChainItem ci;
    int xrow[8], yrow[8], e;
    item_at(p, idx, lane, ci, xrow, yrow, e);
    if (ci.cnt == 0) continue;
    float2 acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = make_float2(0.f, 0.f);
    for (int sb = 0; sb < nsb; ++sb, ++it) {
      const int s = it % S;
      if (!mbar_wait_bounded(&full[s], (it / S) & 1, p.status, ST_TIMEOUT_FULL)) {
        ok = false;
        break;
      }
      const uint8_t* st = ring + s * p.stage_bytes;
      const uint32_t xs = smem_u32(st + p.w_bytes);
      if (WT == WT_Q4K) {
        const uint32_t ra = smem_u32(st + tid * PITCH);
        const uint32_t rb = ra + CH_NT * PITCH;
        switch (ci.cnt) {
          case 1: q4k_sb<1>(ra, rb, xs, acc, nz); break;
          case 2: if (MT >= 2) q4k_sb<(MT >= 2 ? 2 : 1)>(ra, rb, xs, acc, nz); break;
          case 3: if (MT >= 4) q4k_sb<(MT >= 4 ? 3 : 1)>(ra, rb, xs, acc, nz); break;
          case 4: if (MT >= 4) q4k_sb<(MT >= 4 ? 4 : 1)>(ra, rb, xs, acc, nz); break;
          case 5: if (MT >= 8) q4k_sb<(MT >= 8 ? 5 : 1)>(ra, rb, xs, acc, nz); break;
          case 6: if (MT >= 8) q4k_sb<(MT >= 8 ? 6 : 1)>(ra, rb, xs, acc, nz); break;
          case 7: if (MT >= 8) q4k_sb<(MT >= 8 ? 7 : 1)>(ra, rb, xs, acc, nz); break;
          default: if (MT >= 8) q4k_sb<(MT >= 8 ? 8 : 1)>(ra, rb, xs, acc, nz); break;
        }
      } else {
        const int head = (210 * sb) & 15;
        const uint32_t ra = smem_u32(st + tid * PITCH);
        const uint32_t rb = ra + CH_NT * PITCH;
#define AIPU_Q6(C) q6k_sb<C>(ra, rb, head, xs, acc, nz);
        switch (ci.cnt) {
          case 1: AIPU_Q6(1) break;
          case 2: if (MT >= 2) { AIPU_Q6((MT >= 2 ? 2 : 1)) } break;
          case 3: if (MT >= 4) { AIPU_Q6((MT >= 4 ? 3 : 1)) } break;
          case 4: if (MT >= 4) { AIPU_Q6((MT >= 4 ? 4 : 1)) } break;
          case 5: if (MT >= 8) { AIPU_Q6((MT >= 8 ? 5 : 1)) } break;
          case 6: if (MT >= 8) { AIPU_Q6((MT >= 8 ? 6 : 1)) } break;
          case 7: if (MT >= 8) { AIPU_Q6((MT >= 8 ? 7 : 1)) } break;
          default: if (MT >= 8) { AIPU_Q6((MT >= 8 ? 8 : 1)) } break;
        }
#undef AIPU_Q6
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!ok) break;
    // ---------------------------------------------------------------- epilogue
    if (EPI == CHAIN_SWIGLU) {
      const int n = ci.tile * CH_NT + tid;
      if (n < p.N) {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (t < ci.cnt) {
            // h = bf16( fl(silu(bf16 g) * bf16 u) ) (tools/glm_model_q4k_ref.py:702-708)
            const float gb = bf16_round_f(acc[t].x), ub = bf16_round_f(acc[t].y);
            p.y[static_cast<int64_t>(yrow[t]) * p.N + n] = bf16_rne_bits(__fmul_rn(glm_silu_bf(gb), ub));
          }
        }
      }
    } else {
      const int na = ci.tile * 2 * CH_NT + tid, nb = na + CH_NT;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t < ci.cnt) {
          const int64_t o = static_cast<int64_t>(yrow[t]) * p.N;
          if (na < p.N) {
            if (p.y) p.y[o + na] = bf16_rne_bits(acc[t].x);
            if (p.y_f32) p.y_f32[o + na] = acc[t].x;
          }
          if (nb < p.N) {
            if (p.y) p.y[o + nb] = bf16_rne_bits(acc[t].y);
            if (p.y_f32) p.y_f32[o + nb] = acc[t].y;
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------ host
bool chain_supported(int wt, int64_t K, int64_t row_bytes) {
  return (wt == WT_Q4K || wt == WT_Q6K) && K > 0 && K % 256 == 0 && row_bytes % 16 == 0;
}

template <int WT, int EPI, int MT, int NT>
static int chain_launch_t(ChainParams& p, int grid, int smem, cudaStream_t s, bool pdl) {
  auto kern = aipu_chain_kernel<WT, EPI, MT, NT>;
  static bool attr[64] = {false};
  // the attribute is the largest dynamic shared memory any launch of this kernel uses (launches size it
  // differently: one or several CTAs per SM)
  const int rc = set_smem_attr_once(reinterpret_cast<const void*>(kern), 232448 - 1024, attr, "cudaFuncSetAttribute(chain)");
  if (rc) return rc;
  return launch_kernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NT + 32), smem, s, pdl, &p);
}

int chain_launch(int wt, int epi, ChainParams p, int num_sms, cudaStream_t s, bool pdl) {
  p.neg_zero = -0.0f;
  if (!chain_supported(wt, p.K, p.row_bytes)) return CHAIN_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(p.w0) % 16 || (p.w1 && reinterpret_cast<uintptr_t>(p.w1) % 16) ||
      reinterpret_cast<uintptr_t>(p.x) % 16)
    return CHAIN_UNSUPPORTED;
  if (p.N <= 0 || p.M <= 0 || (!p.tiles && p.n_groups <= 0) || (p.tiles && p.max_tiles <= 0)) return OK;
  if (p.x_group_stride % p.K || p.y_group_stride % std::max(p.N, 1))
    return set_error(EINVAL_, "chain: group strides must be whole rows");
  if (p.slot_map && (p.M > 32 || p.topk <= 0)) return CHAIN_UNSUPPORTED;
  const int ne = p.n_experts > 0 ? p.n_experts : p.n_groups;
  if (ne > 1 && p.expert_stride % 16) return CHAIN_UNSUPPORTED;
  const int pitch = (wt == WT_Q4K) ? ChainGeom<WT_Q4K>::PITCH : ChainGeom<WT_Q6K>::PITCH;
  const int box = pitch / 8;
  const int mneed = p.tiles ? 8 : std::min(p.M, 8);
  const int mt = mneed <= 1 ? 1 : mneed <= 2 ? 2 : mneed <= 4 ? 4 : 8;
  p.mt = mt;
  const int64_t passes = p.tiles ? 1 : ((p.slot_map ? std::min(p.M, 32) : p.M) + mt - 1) / mt;
  const int64_t ngr = p.tiles ? p.max_tiles : p.n_groups;
  // 128 consumer threads (one CTA per SM), or 64 with several CTAs per SM when 128-thread tiles would
  // leave SMs idle or need a second round (the Q6_K down projection of a decode layer)
  auto items_of = [&](int nt) {
    const int rt = (epi == CHAIN_SWIGLU) ? nt : 2 * nt;
    return ngr * ((p.N + rt - 1) / rt) * passes;
  };
  const int NT = (epi == CHAIN_STORE && items_of(128) > num_sms / 2) ? 64 : 128;
  const int rows_tile = (epi == CHAIN_SWIGLU) ? NT : 2 * NT;
  const int box_rows = rows_tile;
  p.tiles_per_group = (p.N + rows_tile - 1) / rows_tile;
  p.w_bytes = 2 * NT * pitch;
  p.stage_bytes = p.w_bytes + mt * 256 * 8;
  const int limit = 232448 - 1024;
  // Several CTAs per SM when there are more items than SMs (more warps per scheduler hide the chains'
  // latencies): NT = 64 tiles three per SM, NT = 128 tiles two per SM, two or more stages each.
  const int ctas_per_sm = (NT == 64) ? 3 : (items_of(NT) > num_sms ? 2 : 1);
  const int per_cta = std::max(2 * p.stage_bytes + 128, (limit - ctas_per_sm * 1024) / ctas_per_sm);
  p.nstages = std::min(CH_MAXS, (std::min(per_cta, limit) - 128) / p.stage_bytes);
  if (p.nstages < 2) {
    p.nstages = std::min(CH_MAXS, (limit - 128) / p.stage_bytes);
    if (p.nstages < 2) return set_error(EINVAL_, "chain: stage too large for shared memory");
  }
  const int smem = 128 + p.nstages * p.stage_bytes;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.row_bytes / 8), static_cast<cuuint64_t>(p.N),
                              static_cast<cuuint64_t>(ne)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.row_bytes),
                                 static_cast<cuuint64_t>(ne > 1 ? p.expert_stride : p.row_bytes * p.N)};
  const cuuint32_t boxd[3] = {static_cast<cuuint32_t>(box), static_cast<cuuint32_t>(box_rows), 1};
  int rc = encode_tiled(&p.tmap0, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, p.w0, dims, strides, boxd);
  if (!rc && epi == CHAIN_SWIGLU) rc = encode_tiled(&p.tmap1, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, p.w1, dims, strides, boxd);
  if (rc) return rc;
  const int64_t items = items_of(NT);
  if (items > (1ll << 30)) return set_error(EINVAL_, "chain: too many items");
  const int64_t slots = static_cast<int64_t>(num_sms) * std::max(1, limit / smem);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(slots, items)));
  // Programmatic dependent launch only for a grid of at most one CTA per SM: its CTAs wait on SMs the
  // preceding kernel leaves free. A larger grid would park waiting CTAs on SMs the preceding kernel
  // still needs for its own later CTAs (measured: slower at four tokens).
  const bool pdl_one = pdl && grid <= num_sms;
#define AIPU_CHAIN_CASE(W, E, M_, N_)                                                      \
  if (wt == W && epi == E && mt == M_ && NT == N_) return chain_launch_t<W, E, M_, N_>(p, grid, smem, s, pdl_one);
#define AIPU_CHAIN_MT(W, E, N_) \
  AIPU_CHAIN_CASE(W, E, 1, N_) AIPU_CHAIN_CASE(W, E, 2, N_) AIPU_CHAIN_CASE(W, E, 4, N_) AIPU_CHAIN_CASE(W, E, 8, N_)
  AIPU_CHAIN_MT(WT_Q4K, CHAIN_STORE, 128)
  AIPU_CHAIN_MT(WT_Q4K, CHAIN_STORE, 64)
  AIPU_CHAIN_MT(WT_Q4K, CHAIN_SWIGLU, 128)
  AIPU_CHAIN_MT(WT_Q6K, CHAIN_STORE, 128)
  AIPU_CHAIN_MT(WT_Q6K, CHAIN_STORE, 64)
#undef AIPU_CHAIN_MT
#undef AIPU_CHAIN_CASE
  return CHAIN_UNSUPPORTED;
}

}  // namespace aipu
