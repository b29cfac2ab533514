// Decode dequant GEMV kernel bodies and host launchers (design notes in gemv.cuh).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "deq.cuh"
#include "gemv.cuh"
#include "launch.h"

namespace aipu {

// ------------------------------------------------------------------ shared-memory layout
// [mbarriers: NW x S][misc: prescale shifts per (group slot, column)][activations: XG x ncols fp16
// columns][Q4_K sub-block sums: per (column, super-block) 64 bytes = fp16 hi[8], lo[8], lo2[8], pad]
// [per-warp rings: NW x S slots x 16 rows x pitch]
struct GemvLayout {
  int off_misc, off_xs, off_sxs, off_ring, off_part, total;
};

// part_nw: warps whose tile pieces are summed in shared memory (cta mode), 1 KB each
__host__ __device__ inline GemvLayout gemv_layout(int wt, int ncols, int K, int xg, int nw, int nslots, int pitch,
                                                  int xpitch, int part_nw) {
  GemvLayout L;
  L.off_misc = GEMV_MAXW * GEMV_MAXS * 8;
  L.off_xs = L.off_misc + 256;
  L.off_sxs = L.off_xs + xg * ncols * xpitch;
  // Q4_K: f16-engine sub-block sums (>= the integer engine's K / 32 floats); Q6_K: the integer engine's
  // K / 16 floats
  const int sx = (wt == WT_Q4K) ? xg * ncols * (K / 256) * 64 : (wt == WT_Q6K ? xg * (K / 4) : 0);
  L.off_ring = (L.off_sxs + sx + 127) & ~127;
  L.off_part = L.off_ring + nw * nslots * 16 * pitch;
  L.total = L.off_part + part_nw * 2 * 32 * 16;
  return L;
}

// ------------------------------------------------------------------ shared-memory loads
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
  if ((reinterpret_cast<uintptr_t>(p) & 3u) == 0u) return *reinterpret_cast<const uint32_t*>(p);
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[1]) << 16);
}

constexpr uint32_t H2_1024 = 0x64006400u;   // (1024, 1024)
constexpr uint32_t H2_1056 = 0x64206420u;   // (1056, 1056)
constexpr uint32_t H2_1152 = 0x64806480u;   // (1152, 1152)

__device__ __forceinline__ uint32_t byte_pair_sel(int idx) {
  return 0x4040u | static_cast<uint32_t>(idx) | (static_cast<uint32_t>(idx) << 8);
}

// ------------------------------------------------------------------ per-type unit compute
// A unit = 16 weight rows (g and g+8 of this thread) x 256 weights at super-block column `sb`.
// xcol: this thread's activation column (fp16) in shared memory; colok: the column is a live
// token column (others feed zeros).

// Q4_K operand build: for a 32-bit word of packed nibbles, (w & 0x000F000F) holds two codes q in
// separate 16-bit lanes; one integer multiply-add by the 6-bit scale sc and the magic 0x6400 gives,
// in each lane, the fp16 bit pattern of 1024 + sc*q (sc*q <= 945 < 1024, so no carry between lanes
// and the value is exact: the sum lands in the 10-bit mantissa field of 1024.0). High nibbles are
// shifted down first and built the same way. The constant offset (1024 per weight) is removed with
// one extra MMA that sums the activations of the super-block.
__device__ __forceinline__ uint32_t imad_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4_K unit (16 rows x one super-block). Each code becomes an fp16 MMA operand 1024 + f q in the
// upper mantissa bits, so the 1024 offset costs little precision: low nibbles by a mask and an integer
// multiply-add (f = 64), high nibbles by one LOP3 on the nibble in place at bits 4-7 (f = 16); PRMT
// moves bytes 1 and 3 down for the other half of the k positions. No scale multiply per code: every
// MMA covers one 32-weight sub-block of every row, so D_j = sum_k x_k (1024 + f_j q_k) and
//   sum_k x_k sc_j q_k = (sc_j / f_j) (D_j - 1024 S_j),
// accumulated in fp32 with the row's 6-bit scale. The offsets 1024 sum_j (sc_j / f_j) S_j come from
// MMAs of A = sc_j / f_j against the sub-block sums S_j held as three fp16 parts (33 bits), the min
// term Cm = sum_j m_j S_j from one more MMA (two parts). acc += d * P - dmin * Cm.
__device__ __forceinline__ float half_lo_f(uint32_t h2) { return __half2float(__ushort_as_half(h2 & 0xFFFFu)); }
__device__ __forceinline__ float half_hi_f(uint32_t h2) { return __half2float(__ushort_as_half(h2 >> 16)); }

// Shared-memory operands addressed by 32-bit shared-window addresses (no 64-bit generic address
// arithmetic per load). The loads are volatile so they stay behind the slot's mbarrier wait.
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_v1(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

// rg, rg8: shared addresses of the unit's bytes in rows g and g + 8; xcol: of the lane's activation
// column; sxcol: of the column's sub-block sums (64 bytes per super-block)
__device__ __forceinline__ void unit_q4k(uint32_t rg, uint32_t rg8, uint32_t xcol, uint32_t sxcol, int sb, int t,
                                         float (&acc)[4]) {
  const uint4 hg = lds_v4(rg);
  const uint4 h8 = lds_v4(rg8);
  // 8 six-bit scales / mins per row, as packed bytes (get_scale_min_k4 for j = 0..7 at once)
  const uint32_t sc03g = hg.y & 0x3F3F3F3Fu, m03g = hg.z & 0x3F3F3F3Fu;
  const uint32_t sc47g = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
  const uint32_t m47g = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
  const uint32_t sc038 = h8.y & 0x3F3F3F3Fu, m038 = h8.z & 0x3F3F3F3Fu;
  const uint32_t sc478 = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
  const uint32_t m478 = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
  // fp16 (sc_2p / 64, sc_2p+1 / 16) pairs of both rows for the 4 groups p: 1024 + sc via PRMT, - 1024,
  // * (1/64, 1/16)
  const uint32_t h2_1_16 = 0x2C002400u;  // (1/64, 1/16)
  uint32_t sg[4], s8[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t sel = (p & 1) ? 0x4342u : 0x4140u;
    sg[p] = hmul2_u32(hsub2_u32(prmt((p < 2) ? sc03g : sc47g, 0x64u, sel), H2_1024), h2_1_16);
    s8[p] = hmul2_u32(hsub2_u32(prmt((p < 2) ? sc038 : sc478, 0x64u, sel), H2_1024), h2_1_16);
  }

  float P[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t xb = xcol + 2 * (sb * 256 + 8 * t);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint2 qg = lds_v2(rg + 16 + 32 * p + 8 * t);
    const uint2 q8 = lds_v2(rg8 + 16 + 32 * p + 8 * t);
    const uint4 xl = lds_v4(xb + 2 * (64 * p));
    const uint4 xh = lds_v4(xb + 2 * (64 * p + 32));
    float Dlo[4] = {0.f, 0.f, 0.f, 0.f}, Dhi[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t w = j ? qg.y : qg.x, v = j ? q8.y : q8.x;
      const uint32_t ws = prmt(w, 0u, 0x4341u), vs = prmt(v, 0u, 0x4341u);  // bytes 1, 3 -> low bytes
      uint32_t a[4];
      a[0] = imad_u32(w & 0x000F000Fu, 64u, H2_1024);
      a[1] = imad_u32(v & 0x000F000Fu, 64u, H2_1024);
      a[2] = imad_u32(ws & 0x000F000Fu, 64u, H2_1024);
      a[3] = imad_u32(vs & 0x000F000Fu, 64u, H2_1024);
      mma_f16_16816(Dlo, a, j ? xl.z : xl.x, j ? xl.w : xl.y);
      a[0] = lop3_and_or(w, 0x00F000F0u, H2_1024);
      a[1] = lop3_and_or(v, 0x00F000F0u, H2_1024);
      a[2] = lop3_and_or(ws, 0x00F000F0u, H2_1024);
      a[3] = lop3_and_or(vs, 0x00F000F0u, H2_1024);
      mma_f16_16816(Dhi, a, j ? xh.z : xh.x, j ? xh.w : xh.y);
    }
    const float slg = half_lo_f(sg[p]), shg = half_hi_f(sg[p]);
    const float sl8 = half_lo_f(s8[p]), sh8 = half_hi_f(s8[p]);
    P[0] = fmaf(shg, Dhi[0], fmaf(slg, Dlo[0], P[0]));
    P[1] = fmaf(shg, Dhi[1], fmaf(slg, Dlo[1], P[1]));
    P[2] = fmaf(sh8, Dhi[2], fmaf(sl8, Dlo[2], P[2]));
    P[3] = fmaf(sh8, Dhi[3], fmaf(sl8, Dlo[3], P[3]));
  }
  // offsets Cs = sum_j (sc_j / f_j) S_j and the min term Cm = sum_j m_j S_j (k positions of this
  // lane: sub-blocks 2t', 2t'+1 of the hi sums (b0) and of the lo sums (b1), t' = t & 3)
  float Cm[4] = {0.f, 0.f, 0.f, 0.f}, Cs[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const uint32_t sel = (t & 1) ? 0x4342u : 0x4140u;
    const uint32_t mg = hsub2_u32(prmt((t < 2) ? m03g : m47g, 0x64u, sel), H2_1024);
    const uint32_t m8 = hsub2_u32(prmt((t < 2) ? m038 : m478, 0x64u, sel), H2_1024);
    const uint32_t sx = sxcol + 4 * (sb * 16 + t);
    const uint32_t b0 = lds_v1(sx), b1 = lds_v1(sx + 16), b2 = lds_v1(sx + 32);
    const uint32_t am[4] = {mg, m8, mg, m8};
    mma_f16_16816(Cm, am, b0, b1);
    const uint32_t sgt = (t & 2) ? ((t & 1) ? sg[3] : sg[2]) : ((t & 1) ? sg[1] : sg[0]);
    const uint32_t s8t = (t & 2) ? ((t & 1) ? s8[3] : s8[2]) : ((t & 1) ? s8[1] : s8[0]);
    const uint32_t as[4] = {sgt, s8t, sgt, s8t};
    mma_f16_16816(Cs, as, b0, b1);
    mma_f16_16816(Cs, as, b2, 0u);  // third parts of the sums (k positions 8.. of A multiply zero)
  }
  const float dg = f16_bits_to_f32(hg.x), dmg = f16_bits_to_f32(hg.x >> 16);
  const float d8 = f16_bits_to_f32(h8.x), dm8 = f16_bits_to_f32(h8.x >> 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float Pi = fmaf(-1024.f, Cs[i], P[i]);  // sum_k x_k * sc * q
    const float d = (i < 2) ? dg : d8, dm = (i < 2) ? dmg : dm8;
    acc[i] = fmaf(-dm, Cm[i], fmaf(d, Pi, acc[i]));
  }
}

__device__ __forceinline__ void unit_q6k(const uint8_t* rg, const uint8_t* rg8, const uint8_t* xcol, bool colok,
                                         int sb, int t, float (&acc)[4]) {
  const float dg = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg + 208));
  const float d8 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg8 + 208));
  const int8_t* scg = reinterpret_cast<const int8_t*>(rg + 192);
  const int8_t* sc8 = reinterpret_cast<const int8_t*>(rg8 + 192);
  const uint8_t* xb = xcol + 2 * (sb * 256 + 4 * t);
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
    for (int lh = 0; lh < 2; ++lh) {
      const int off = 16 * lh + 4 * t;
      const uint32_t qa = lds_u32_any(rg + 64 * hf + off), qb = lds_u32_any(rg + 64 * hf + 32 + off);
      const uint32_t qh = lds_u32_any(rg + 128 + 32 * hf + off);
      const uint32_t ra = lds_u32_any(rg8 + 64 * hf + off), rb = lds_u32_any(rg8 + 64 * hf + 32 + off);
      const uint32_t rh = lds_u32_any(rg8 + 128 + 32 * hf + off);
      uint32_t cg[4], c8[4];
      cg[0] = (qa & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
      cg[1] = (qb & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
      cg[2] = ((qa >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
      cg[3] = ((qb >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
      c8[0] = (ra & 0x0F0F0F0Fu) | ((rh << 4) & 0x30303030u);
      c8[1] = (rb & 0x0F0F0F0Fu) | ((rh << 2) & 0x30303030u);
      c8[2] = ((ra >> 4) & 0x0F0F0F0Fu) | (rh & 0x30303030u);
      c8[3] = ((rb >> 4) & 0x0F0F0F0Fu) | ((rh >> 2) & 0x30303030u);
#pragma unroll
      for (int qi = 0; qi < 4; ++qi) {
        const int grp = 8 * hf + 2 * qi + lh;
        uint32_t a[4];
        a[0] = hsub2_u32(lop3_and_or(cg[qi], 0x003F003Fu, H2_1024), H2_1056);
        a[1] = hsub2_u32(lop3_and_or(c8[qi], 0x003F003Fu, H2_1024), H2_1056);
        a[2] = hsub2_u32(lop3_and_or(cg[qi] >> 8, 0x003F003Fu, H2_1024), H2_1056);
        a[3] = hsub2_u32(lop3_and_or(c8[qi] >> 8, 0x003F003Fu, H2_1024), H2_1056);
        uint2 xv = make_uint2(0, 0);
        if (colok) xv = *reinterpret_cast<const uint2*>(xb + 2 * (128 * hf + 32 * qi + 16 * lh));
        float P[4] = {0.f, 0.f, 0.f, 0.f};
        mma_f16_16816(P, a, xv.x, xv.y);
        const float sg = __fmul_rn(dg, static_cast<float>(scg[grp]));
        const float s8 = __fmul_rn(d8, static_cast<float>(sc8[grp]));
        acc[0] = fmaf(sg, P[0], acc[0]);
        acc[1] = fmaf(sg, P[1], acc[1]);
        acc[2] = fmaf(s8, P[2], acc[2]);
        acc[3] = fmaf(s8, P[3], acc[3]);
      }
    }
  }
}

// 4 bytes at a shared address known to be 4-byte aligned (A4) or 2 mod 4 (two aligned words and a
// byte permute).
template <bool A4>
__device__ __forceinline__ uint32_t lds4(uint32_t a) {
  if (A4) return lds_v1(a);
  return __byte_perm(lds_v1(a - 2), lds_v1(a + 2), 0x5432);
}
__device__ __forceinline__ int lds_s8(uint32_t a) {
  int v;
  asm volatile("ld.shared.s8 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

// Q6_K unit for up to 4 live columns (MP = 1, 2 or 4 columns padded to a power of two): the MMA's
// 8 output columns hold 8 / MP scale groups x MP columns, so the 16-weight groups of a super-block
// accumulate in 2 MP sets of fp32 accumulators and are scaled once per unit (one multiply-add per
// accumulator instead of one per group). Lane (g, t) feeds B column g: column g % MP, group slot
// g / MP (zeros for the MMAs of other slots). acc holds per-lane partial sums over groups until
// q6k_fold combines the lanes at the end of a tile. rg, rg8, xcolm: shared addresses.
template <int MP, bool A4>
__device__ __forceinline__ void unit_q6k_mp(uint32_t rg, uint32_t rg8, uint32_t xcolm, bool mok, int gslot, int sb,
                                            int t, float (&acc)[4]) {
  constexpr int NGM = 8 / MP;    // groups per accumulator set
  constexpr int NSET = 16 / NGM;
  float D[NSET][4];
#pragma unroll
  for (int i = 0; i < NSET; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = 0.f;
  const uint32_t xb = xcolm + 2 * (sb * 256 + 4 * t);
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
    for (int lh = 0; lh < 2; ++lh) {
      const int off = 16 * lh + 4 * t;
      const uint32_t qa = lds4<A4>(rg + 64 * hf + off), qb = lds4<A4>(rg + 64 * hf + 32 + off);
      const uint32_t qh = lds4<A4>(rg + 128 + 32 * hf + off);
      const uint32_t ra = lds4<A4>(rg8 + 64 * hf + off), rb = lds4<A4>(rg8 + 64 * hf + 32 + off);
      const uint32_t rh = lds4<A4>(rg8 + 128 + 32 * hf + off);
      uint32_t cg[4], c8[4];
      cg[0] = (qa & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
      cg[1] = (qb & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
      cg[2] = ((qa >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
      cg[3] = ((qb >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
      c8[0] = (ra & 0x0F0F0F0Fu) | ((rh << 4) & 0x30303030u);
      c8[1] = (rb & 0x0F0F0F0Fu) | ((rh << 2) & 0x30303030u);
      c8[2] = ((ra >> 4) & 0x0F0F0F0Fu) | (rh & 0x30303030u);
      c8[3] = ((rb >> 4) & 0x0F0F0F0Fu) | ((rh >> 2) & 0x30303030u);
#pragma unroll
      for (int qi = 0; qi < 4; ++qi) {
        const int grp = 8 * hf + 2 * qi + lh;
        uint32_t a[4];
        a[0] = hsub2_u32(lop3_and_or(cg[qi], 0x003F003Fu, H2_1024), H2_1056);
        a[1] = hsub2_u32(lop3_and_or(c8[qi], 0x003F003Fu, H2_1024), H2_1056);
        a[2] = hsub2_u32(lop3_and_or(cg[qi] >> 8, 0x003F003Fu, H2_1024), H2_1056);
        a[3] = hsub2_u32(lop3_and_or(c8[qi] >> 8, 0x003F003Fu, H2_1024), H2_1056);
        uint2 xv = make_uint2(0, 0);
        if (mok && gslot == grp % NGM) xv = lds_v2(xb + 2 * (128 * hf + 32 * qi + 16 * lh));
        mma_f16_16816(D[grp / NGM], a, xv.x, xv.y);
      }
    }
  }
  const float dg = f16_bits_to_f32(lds_u16(rg + 208));
  const float d8 = f16_bits_to_f32(lds_u16(rg8 + 208));
#pragma unroll
  for (int st = 0; st < NSET; ++st) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int gc = st * NGM + (2 * t + h) / MP;  // the group of this lane's output column 2t + h
      acc[h] = fmaf(__fmul_rn(dg, static_cast<float>(lds_s8(rg + 192 + gc))), D[st][h], acc[h]);
      acc[2 + h] = fmaf(__fmul_rn(d8, static_cast<float>(lds_s8(rg8 + 192 + gc))), D[st][2 + h], acc[2 + h]);
    }
  }
}

// End of a tile for unit_q6k_mp: sum each column's partials over the lanes holding its group slots
// and leave column c in the standard layout (lane t = c / 2, element h = c % 2).
template <int MP>
__device__ __forceinline__ void q6k_fold(float (&acc)[4]) {
  if (MP == 1) {
    float v0 = __fadd_rn(acc[0], acc[1]), v2 = __fadd_rn(acc[2], acc[3]);
    v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, 1));
    v2 = __fadd_rn(v2, __shfl_xor_sync(0xffffffffu, v2, 1));
    v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, 2));
    v2 = __fadd_rn(v2, __shfl_xor_sync(0xffffffffu, v2, 2));
    acc[0] = v0;
    acc[2] = v2;
    acc[1] = acc[3] = 0.f;
  } else if (MP == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 1));
      acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 2));
    }
  } else if (MP == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 2));
  }
}

__device__ __forceinline__ void unit_q80(const uint8_t* rg, const uint8_t* rg8, const uint8_t* xcol, bool colok,
                                         int sb, int t, float (&acc)[4]) {
  const uint8_t* xb = xcol + 2 * (sb * 256 + 4 * t);
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint8_t* bg = rg + 34 * b;
    const uint8_t* b8 = rg8 + 34 * b;
    const float dg = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bg));
    const float d8 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(b8));
    float P[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2) {
      const uint32_t u = lds_u32_any(bg + 2 + 16 * j2 + 4 * t) ^ 0x80808080u;
      const uint32_t v = lds_u32_any(b8 + 2 + 16 * j2 + 4 * t) ^ 0x80808080u;
      uint32_t a[4];
      a[0] = hsub2_u32(prmt(u, 0x64u, 0x4240u), H2_1152);
      a[1] = hsub2_u32(prmt(v, 0x64u, 0x4240u), H2_1152);
      a[2] = hsub2_u32(prmt(u, 0x64u, 0x4341u), H2_1152);
      a[3] = hsub2_u32(prmt(v, 0x64u, 0x4341u), H2_1152);
      uint2 xv = make_uint2(0, 0);
      if (colok) xv = *reinterpret_cast<const uint2*>(xb + 2 * (32 * b + 16 * j2));
      mma_f16_16816(P, a, xv.x, xv.y);
    }
    acc[0] = fmaf(dg, P[0], acc[0]);
    acc[1] = fmaf(dg, P[1], acc[1]);
    acc[2] = fmaf(d8, P[2], acc[2]);
    acc[3] = fmaf(d8, P[3], acc[3]);
  }
}

__device__ __forceinline__ void unit_f16(const uint8_t* rg, const uint8_t* rg8, const uint8_t* xcol, bool colok,
                                         int sb, int t, float (&acc)[4]) {
  const uint8_t* xb = xcol + 2 * (sb * 256 + 4 * t);
  float P4[4][4] = {};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint2 wg = *reinterpret_cast<const uint2*>(rg + 2 * (16 * i + 4 * t));
    const uint2 w8 = *reinterpret_cast<const uint2*>(rg8 + 2 * (16 * i + 4 * t));
    uint32_t a[4] = {wg.x, w8.x, wg.y, w8.y};
    uint2 xv = make_uint2(0, 0);
    if (colok) xv = *reinterpret_cast<const uint2*>(xb + 2 * (16 * i));
    mma_f16_16816(P4[i & 3], a, xv.x, xv.y);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    acc[j] = __fadd_rn(acc[j], __fadd_rn(__fadd_rn(P4[0][j], P4[1][j]), __fadd_rn(P4[2][j], P4[3][j])));
}

// ------------------------------------------------------------------ integer dot engine (Q4_K, one token)
// The activation row is rounded once to integers X = rn(x * 2^-s) with max |X| in [2^21, 2^22] (a
// power-of-two prescale s per row), and X is written as three balanced base-256 digits (int8,
// X = d0 + 2^8 d1 + 2^16 d2). Q4_K codes need no conversion: masking the packed bytes gives u8
// operands q (low nibbles) and 16 q (high nibbles), and one m16n8k32 u8 x s8 MMA covers 16 rows x one
// 32-weight sub-block with exact int32 sums (the integer MMA runs natively; an fp8 MMA issued through
// mma.sync costs a dozen operand conversions on this GPU). The MMA's 8 columns are (sub-block parity,
// digit): the activation columns hold the digits only at the k of their parity, so the low-nibble
// sub-block 2g and the high-nibble sub-block 2g + 1 of a 64-weight group share one accumulator set.
// Each lane scales its sets by the 6-bit integer sub-block scales with integer multiply-adds (|sum| <
// 2^28: exact), converts once per row and super-block and applies d; the min term dmin * sum_j m_j S_j
// uses the sub-block sums S_j of X. The only roundings are X itself (2^-22 of the row's largest
// value) and the fp32 steps per super-block.
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Stage one token row (group grp) as 8 masked int8 digit columns + fp32 sub-block sums of X (all
// threads). Column c = 4 * parity + digit (digit < 3; columns 3 and 7 stay zero) holds, at every k
// whose sub-block j has j % 2 == parity, digit `digit` of X; zero elsewhere (the columns are zero on
// entry). misc[0..1] = prescale shift s (value = sum * 2^s). Leaves with a __syncthreads.
// Q4_K: 32-weight sub-blocks, sums sxs[j]; Q6_K: 16-weight sub-blocks, sums per super-block in
// parity-major order (sxs[16 sb + 8 (j % 2) + (j % 16) / 2] for sub-block j).
template <int WT, int XT>
__device__ void gemv_stage_x_i8(const GemvParams& p, uint8_t* smem, const GemvLayout& L, int grp, int xs_slot,
                                float* red) {
  const int tid = threadIdx.x, NT = blockDim.x, NW = NT >> 5;
  const int K = p.K;
  int* misc = reinterpret_cast<int*>(smem + L.off_misc) + xs_slot * 8;
  uint8_t* xs = smem + L.off_xs + xs_slot * 8 * p.xpitch;
  float* sxs = reinterpret_cast<float*>(smem + L.off_sxs) + xs_slot * (WT == WT_Q6K ? K / 16 : K / 32);
  const uint8_t* xr = static_cast<const uint8_t*>(p.x) +
                      static_cast<int64_t>(grp) * p.x_group_stride * (XT == XT_F32 ? 4 : 2);
  const int nvec = K / 8;  // 8 activations per vector
  auto load8 = [&](int v, float (&f)[8]) {
    if (XT == XT_F32) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(xr) + 2 * v);
      const float4 b = __ldg(reinterpret_cast<const float4*>(xr) + 2 * v + 1);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr) + v);
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w4[i] << 16);
        f[2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
      }
    }
  };
  // up to kRegVec vectors per thread are loaded once, all at the same time, and kept in registers for
  // the second pass (one L2 round trip instead of one per loop iteration and pass)
  constexpr int kRegVec = 4;
  const bool in_regs = nvec <= kRegVec * NT;
  float fr[kRegVec][8];
  float mx = 0.f;
  if (in_regs) {
#pragma unroll
    for (int r = 0; r < kRegVec; ++r) {
      const int v = tid + r * NT;
      if (v < nvec) {
        load8(v, fr[r]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) fr[r][i] = 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < kRegVec; ++r)
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(fr[r][i]));
  } else {
    for (int v = tid; v < nvec; v += NT) {
      float f[8];
      load8(v, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(f[i]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  float m = 0.f;
  for (int w = 0; w < NW; ++w) m = fmaxf(m, red[w]);
  // max * 2^-s in [2^21, 2^22): |X| <= 2^22 after rounding, so d2 stays within [-65, 65] and every
  // integer sum below stays exact
  const int e = static_cast<int>((__float_as_uint(m) >> 23) & 0xFFu);
  int sh = (m == 0.f) ? 0 : (e - 127 - 21);
  sh = sh < -100 ? -100 : (sh > 100 ? 100 : sh);
  if (tid == 0) {
    misc[0] = sh;
    misc[1] = sh;
  }
  const float sc = exp2i(-sh);
  auto stage8 = [&](int v, const float (&f)[8]) {
    int sum = 0;
    // balanced base-256 digits of X at once: the bytes of X + 0x808080 (in [0, 2^24) for |X| <= 2^22)
    // are d_i + 128, so XOR with 0x808080 leaves d0, d1, d2 as int8 in bytes 0..2
    uint32_t e[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // round to the nearest integer (ties to even): |x * 2^-s| < 2^22, so adding 1.5 * 2^23 leaves
      // the integer in the low mantissa bits
      const int X = static_cast<int>(__float_as_uint(__fadd_rn(__fmul_rn(f[i], sc), 12582912.f)) - 0x4B400000u);
      sum += X;
      e[i] = (static_cast<uint32_t>(X) + 0x808080u) ^ 0x808080u;
    }
    // digit planes: byte c of elements 0..3 and 4..7
    uint32_t dig[3][2];
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t lo = prmt(e[4 * h], e[4 * h + 1], static_cast<uint32_t>(c | ((4 + c) << 4)));
        const uint32_t hi = prmt(e[4 * h + 2], e[4 * h + 3], static_cast<uint32_t>(c | ((4 + c) << 4)));
        dig[c][h] = prmt(lo, hi, 0x5410u);
      }
    // the threads of a sub-block (4 for 32 weights, 2 for 16) add their integer sums (exact)
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    const int k0 = 8 * v;
    int par;
    if (WT == WT_Q6K) {
      const int j = k0 >> 4;
      par = j & 1;
      if ((v & 1) == 0) sxs[16 * (j >> 4) + 8 * par + ((j & 15) >> 1)] = static_cast<float>(sum);
    } else {
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      const int j = k0 >> 5;
      par = j & 1;
      if ((v & 3) == 0) sxs[j] = static_cast<float>(sum);
    }
    // the live digits only (column 4 * parity + digit); the kernel cleared all columns beforehand
    uint8_t* xc = xs + 4 * par * p.xpitch + k0;
#pragma unroll
    for (int c = 0; c < 3; ++c) *reinterpret_cast<uint2*>(xc + c * p.xpitch) = make_uint2(dig[c][0], dig[c][1]);
  };
  // (nvec and the warps' first vectors are multiples of 32, so every lane of a warp runs the same
  // iterations: the sub-block sums shuffle across 4 lanes)
  if (in_regs) {
#pragma unroll
    for (int r = 0; r < kRegVec; ++r)
      if (tid + r * NT < nvec) stage8(tid + r * NT, fr[r]);
  } else {
    for (int v = tid; v < nvec; v += NT) {
      float f[8];
      load8(v, f);
      stage8(v, f);
    }
  }
  __syncthreads();
}

// Q4_K unit (16 rows g, g + 8 x one super-block) on the integer engine, one token. acc[0] / acc[2]:
// this lane's partial sums of rows g / g + 8 (its digit columns, and the min terms of sub-blocks 2t,
// 2t + 1); q4k_i8_fold sums the 4 lanes. xb: the lane's activation column at this super-block (+ 8t);
// sxb: the super-block's sub-block sums; w0 / w1: the digit weights of the lane's two columns (1/16
// folded in for the high-nibble columns); ssel0/1: PRMT selectors of the lane's scale bytes, msel0/1:
// of its min bytes.
__device__ __forceinline__ void unit_q4k_i8(uint32_t rg, uint32_t rg8, uint32_t xb, uint32_t sxb, int t, float w0,
                                            float w1, uint32_t ssel0, uint32_t ssel1, uint32_t msel0, uint32_t msel1,
                                            float (&acc)[4]) {
  const uint4 hg = lds_v4(rg), h8 = lds_v4(rg8);
  int D[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint2 wg = lds_v2(rg + 16 + 32 * g + 8 * t), w8 = lds_v2(rg8 + 16 + 32 * g + 8 * t);
    const uint2 xl = lds_v2(xb + 64 * g), xh = lds_v2(xb + 64 * g + 32);
    const uint32_t alo[4] = {wg.x & 0x0F0F0F0Fu, w8.x & 0x0F0F0F0Fu, wg.y & 0x0F0F0F0Fu, w8.y & 0x0F0F0F0Fu};
    mma_u8s8_16832(D[g], alo, xl.x, xl.y);
    const uint32_t ahi[4] = {wg.x & 0xF0F0F0F0u, w8.x & 0xF0F0F0F0u, wg.y & 0xF0F0F0F0u, w8.y & 0xF0F0F0F0u};
    mma_u8s8_16832(D[g], ahi, xh.x, xh.y);
  }
  // 6-bit scale / min tables of both rows (get_scale_min_k4 for j = 0..7 at once)
  const uint32_t sc03g = hg.y & 0x3F3F3F3Fu, m03g = hg.z & 0x3F3F3F3Fu;
  const uint32_t sc47g = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
  const uint32_t m47g = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
  const uint32_t sc038 = h8.y & 0x3F3F3F3Fu, m038 = h8.z & 0x3F3F3F3Fu;
  const uint32_t sc478 = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
  const uint32_t m478 = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
  // set g covers sub-block 2g + parity: g = 0, 1 from the 0-3 tables, g = 2, 3 from the 4-7 tables
  int c0g = 0, c1g = 0, c08 = 0, c18 = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t sl = (g & 1) ? ssel1 : ssel0;
    const int sg = static_cast<int>(prmt(g < 2 ? sc03g : sc47g, 0u, sl));
    const int s8 = static_cast<int>(prmt(g < 2 ? sc038 : sc478, 0u, sl));
    c0g += sg * D[g][0];
    c1g += sg * D[g][1];
    c08 += s8 * D[g][2];
    c18 += s8 * D[g][3];
  }
  const float vg = fmaf(__int2float_rn(c1g), w1, __fmul_rn(__int2float_rn(c0g), w0));
  const float v8 = fmaf(__int2float_rn(c18), w1, __fmul_rn(__int2float_rn(c08), w0));
  acc[0] = fmaf(f16_bits_to_f32(hg.x & 0xFFFFu), vg, acc[0]);
  acc[2] = fmaf(f16_bits_to_f32(h8.x & 0xFFFFu), v8, acc[2]);
  // min term: this lane takes sub-blocks 2t and 2t + 1 (table m03 for t < 2, m47 otherwise)
  float2 S;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(S.x), "=f"(S.y) : "r"(sxb + 8 * t));
  constexpr uint32_t MAG = 0x4B000000u;
  auto ent = [&](uint32_t tab, uint32_t sl) { return __fsub_rn(__uint_as_float(prmt(tab, MAG, sl)), 8388608.f); };
  const uint32_t tmg = (t < 2) ? m03g : m47g, tm8 = (t < 2) ? m038 : m478;
  const float cmg = fmaf(ent(tmg, msel0), S.x, __fmul_rn(ent(tmg, msel1), S.y));
  const float cm8 = fmaf(ent(tm8, msel0), S.x, __fmul_rn(ent(tm8, msel1), S.y));
  acc[0] = fmaf(-f16_bits_to_f32(hg.x >> 16), cmg, acc[0]);
  acc[2] = fmaf(-f16_bits_to_f32(h8.x >> 16), cm8, acc[2]);
}

// End of a tile for unit_q4k_i8: rows g and g + 8 summed over the 4 lanes, left in the standard
// layout (column 0 of every lane; the other column slots zero).
__device__ __forceinline__ void q4k_i8_fold(float (&acc)[4]) {
  float v0 = acc[0], v2 = acc[2];
  v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, 1));
  v2 = __fadd_rn(v2, __shfl_xor_sync(0xffffffffu, v2, 1));
  v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, 2));
  v2 = __fadd_rn(v2, __shfl_xor_sync(0xffffffffu, v2, 2));
  acc[0] = v0;
  acc[2] = v2;
  acc[1] = acc[3] = 0.f;
}

// Q6_K unit (16 rows g, g + 8 x one super-block) on the integer engine, one token. Block layout
// [ql 128][qh 64][int8 sc 16][fp16 d] (tools/q4k_ref.py:99-124): weight w = 128 n + 32 c + l has the
// 6-bit code (ql[64 n + 32 (c & 1) + l] >> 4 (c >> 1)) & 15 | ((qh[32 n + l] >> 2 c) & 3) << 4 and the
// value d * sc[w / 16] * (code - 32). One u8 x s8 MMA per (n, c) covers 32 weights = two 16-weight
// sub-blocks, told apart by the parity columns (activation k order = weight order). The codes are
// assembled four at a time (mask the nibble plane, mask the 2-bit plane shifted into bits 4-5, OR);
// the -32 offset is applied once per sub-block on the sums S_j of the staged activations. AL: the
// unit's start offset mod 8 (the same for every row of a tiled slot, so the choice is warp-uniform).
// 8 bytes at a shared address whose offset mod 8 is AL (0, 4, or 2 for 2 / 6 mod 8)
template <int AL>
__device__ __forceinline__ uint2 q6_ld8(uint32_t a) {
  if (AL == 0) return lds_v2(a);
  if (AL == 4) return make_uint2(lds_v1(a), lds_v1(a + 4));
  const uint32_t w0 = lds_v1(a - 2), w1 = lds_v1(a + 2), w2 = lds_v1(a + 6);
  return make_uint2(__byte_perm(w0, w1, 0x5432), __byte_perm(w1, w2, 0x5432));
}

template <int AL>
__device__ __forceinline__ void unit_q6k_i8(uint32_t rg, uint32_t rg8, uint32_t xb, uint32_t sxb, int t, float w0,
                                            float w1, float (&acc)[4]) {
  const int par = t >> 1;
  int D[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = 0;
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    // MMA k rows 4t..4t+3 (a0, a1) <-> weights l = 8t..8t+3, rows 16+4t.. (a2, a3) <-> l = 8t+4..8t+7 of
    // the 32-weight group (the activation columns are read with the same permutation): one 8-byte
    // load per row and plane
    uint32_t la[2][2], lb[2][2], qh[2][2];  // [row g / g + 8][half: l = 8t.. / 8t+4..]
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const uint32_t b = (rr ? rg8 : rg) + 8 * t;
      const uint2 va = q6_ld8<AL>(b + 64 * n), vb = q6_ld8<AL>(b + 64 * n + 32), vh = q6_ld8<AL>(b + 128 + 32 * n);
      la[rr][0] = va.x; la[rr][1] = va.y;
      lb[rr][0] = vb.x; lb[rr][1] = vb.y;
      qh[rr][0] = vh.x; qh[rr][1] = vh.y;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t a[4];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t lw = (c & 1) ? lb[rr][hh] : la[rr][hh];
          const uint32_t nib = (c >> 1) ? ((lw >> 4) & 0x0F0F0F0Fu) : (lw & 0x0F0F0F0Fu);
          const uint32_t hw = qh[rr][hh];
          const uint32_t hb = (c == 0) ? (hw << 4) : (c == 1) ? (hw << 2) : (c == 2) ? hw : (hw >> 2);
          a[2 * hh + rr] = nib | (hb & 0x30303030u);
        }
      const uint2 xv = lds_v2(xb + 128 * n + 32 * c + 8 * t);
      mma_u8s8_16832(D[4 * n + c], a, xv.x, xv.y);
    }
  }
  // sub-block j = 8 n + 2 c + parity: this lane's sets use the scales of its column parity
  int scg[8], sc8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    scg[i] = lds_s8(rg + 192 + 2 * i + par);
    sc8[i] = lds_s8(rg8 + 192 + 2 * i + par);
  }
  int c0g = 0, c1g = 0, c08 = 0, c18 = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c0g += scg[i] * D[i][0];
    c1g += scg[i] * D[i][1];
    c08 += sc8[i] * D[i][2];
    c18 += sc8[i] * D[i][3];
  }
  // the -32 offset: this lane takes the sub-blocks 2 m + parity, m = 4 (t & 1) .. + 3 (sets n = t & 1)
  const uint4 S = lds_v4(sxb + 4 * (8 * par + 4 * (t & 1)));
  const float Sv[4] = {__uint_as_float(S.x), __uint_as_float(S.y), __uint_as_float(S.z), __uint_as_float(S.w)};
  float og = 0.f, o8 = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int sg = (t & 1) ? scg[4 + c] : scg[c], s8 = (t & 1) ? sc8[4 + c] : sc8[c];
    og = fmaf(static_cast<float>(sg), Sv[c], og);
    o8 = fmaf(static_cast<float>(s8), Sv[c], o8);
  }
  const float vg = fmaf(__int2float_rn(c1g), w1, __fmul_rn(__int2float_rn(c0g), w0));
  const float v8 = fmaf(__int2float_rn(c18), w1, __fmul_rn(__int2float_rn(c08), w0));
  const float dg = f16_bits_to_f32(lds_u16(rg + 208)), d8 = f16_bits_to_f32(lds_u16(rg8 + 208));
  acc[0] = fmaf(dg, fmaf(-32.f, og, vg), acc[0]);
  acc[2] = fmaf(d8, fmaf(-32.f, o8, v8), acc[2]);
}

// ------------------------------------------------------------------ kernel
template <int WT, int XT, int EPI>
struct GemvGeom {
  static constexpr int RPT = (EPI == EPI_SWIGLU) ? 8 : 16;  // matrix rows per tile
  static constexpr int UB = unit_bytes(WT);
};

template <int WT, int XT, int EPI>
__device__ __forceinline__ const uint8_t* gemv_row_ptr(const GemvParams& p, int grp, int lt, int r) {
  constexpr int RPT = GemvGeom<WT, XT, EPI>::RPT;
  const int e = p.group_ids ? p.group_ids[grp] : grp;
  int n = lt * RPT + (EPI == EPI_SWIGLU ? (r & 7) : r);
  n = n < p.N ? n : p.N - 1;
  const uint8_t* base = (EPI == EPI_SWIGLU && r >= 8) ? p.w1 : p.w0;
  return base + static_cast<int64_t>(e) * p.expert_stride + static_cast<int64_t>(n) * p.row_bytes;
}

__device__ __forceinline__ int cta_of_unit(int64_t u, int64_t U, int G) {
  return static_cast<int>(((u + 1) * G - 1) / U);
}

template <int WT, int XT, int EPI>
__device__ void gemv_epilogue(const GemvParams& p, const int* misc, int grp, int lt, const float (&v)[4], int lane) {
  const int g = lane >> 2, t = lane & 3;
  uint16_t* y = p.y + static_cast<int64_t>(grp) * p.y_group_stride;
  if (EPI == EPI_STORE) {
    const int n0 = lt * 16 + g, n1 = n0 + 8;
    if (XT == XT_BF16) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = 2 * t + h;
        if (c < p.M) {
          const float s = exp2i(misc[c]);
          if (n0 < p.N) y[static_cast<int64_t>(c) * p.N + n0] = bf16_rne_bits(__fmul_rn(v[h], s));
          if (n1 < p.N) y[static_cast<int64_t>(c) * p.N + n1] = bf16_rne_bits(__fmul_rn(v[2 + h], s));
        }
      }
    } else {
      if (t < p.M) {
        const float s = exp2i(misc[2 * t]);
        if (n0 < p.N) y[static_cast<int64_t>(t) * p.N + n0] = bf16_rne_bits(__fmul_rn(__fadd_rn(v[0], v[1]), s));
        if (n1 < p.N) y[static_cast<int64_t>(t) * p.N + n1] = bf16_rne_bits(__fmul_rn(__fadd_rn(v[2], v[3]), s));
      }
    }
  } else {  // EPI_SWIGLU: rows g = gate row n, g+8 = up row n; h = bf16(silu(bf16 g) * bf16 u)
    const int n = lt * 8 + g;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = 2 * t + h;
      if (c < p.M && n < p.N) {
        const float s = exp2i(misc[c]);
        const float gb = bf16_round_f(__fmul_rn(v[h], s));
        const float ub = bf16_round_f(__fmul_rn(v[2 + h], s));
        y[static_cast<int64_t>(c) * p.N + n] = bf16_rne_bits(__fmul_rn(glm_silu_bf(gb), ub));
      }
    }
  }
}

// fp32 or bf16 16-byte vector -> fp16 values scaled by `sc` (hi, and lo for fp32 input), written to
// the activation columns in the per-type k order; returns the sum(s) of the written fp16 values.
template <int XT, bool SWZ>
__device__ __forceinline__ void stage_vec(const uint4 q, float sc, uint8_t* colhi, uint8_t* collo, int v,
                                          float& sum_hi, float& sum_lo) {
  if (XT == XT_F32) {
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
    uint32_t hb[4], lb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float f = __fmul_rn(__uint_as_float(w4[i]), sc);
      const __half hi = __float2half_rn(f);
      const float hf = __half2float(hi);
      const __half lo = __float2half_rn(__fsub_rn(f, hf));
      hb[i] = __half_as_ushort(hi);
      lb[i] = __half_as_ushort(lo);
      sum_hi = __fadd_rn(sum_hi, hf);
      sum_lo = __fadd_rn(sum_lo, __half2float(lo));
    }
    const int a1 = SWZ ? 2 : 1, a2 = SWZ ? 1 : 2;
    *reinterpret_cast<uint2*>(colhi + 8 * v) = make_uint2(hb[0] | (hb[a1] << 16), hb[a2] | (hb[3] << 16));
    *reinterpret_cast<uint2*>(collo + 8 * v) = make_uint2(lb[0] | (lb[a1] << 16), lb[a2] | (lb[3] << 16));
  } else {
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half a = __float2half_rn(__fmul_rn(__uint_as_float(w4[i] << 16), sc));
      const __half b = __float2half_rn(__fmul_rn(__uint_as_float(w4[i] & 0xFFFF0000u), sc));
      h[2 * i] = __half_as_ushort(a);
      h[2 * i + 1] = __half_as_ushort(b);
      sum_hi = __fadd_rn(sum_hi, __fadd_rn(__half2float(a), __half2float(b)));
    }
    uint4 o;
    if (SWZ) {
      o = make_uint4(h[0] | (h[2] << 16), h[1] | (h[3] << 16), h[4] | (h[6] << 16), h[5] | (h[7] << 16));
    } else {
      o = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
    }
    *reinterpret_cast<uint4*>(colhi + 16 * v) = o;
  }
}

__device__ __forceinline__ float vec_absmax(const uint4 q, bool f32, float mx) {
  const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (f32) {
      mx = fmaxf(mx, fabsf(__uint_as_float(w4[i])));
    } else {
      mx = fmaxf(mx, fabsf(__uint_as_float(w4[i] << 16)));
      mx = fmaxf(mx, fabsf(__uint_as_float(w4[i] & 0xFFFF0000u)));
    }
  }
  return mx;
}

__device__ __forceinline__ int prescale_shift(float mx) {
  // max * 2^-s in [2^9, 2^10): sub-block sums of 32 values stay below 2^15 (fp16-safe)
  const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu);
  int s = (mx == 0.f) ? 0 : (e - 127 - 9);
  return s < -100 ? -100 : (s > 100 ? 100 : s);
}

// Stage the activations of group `grp` into shared memory as fp16 columns (see gemv.cuh). Tokens
// are handled two at a time: 16-byte vectors are loaded once into registers (up to 4 per thread per
// token), reduced for the per-token power-of-two prescale, converted and stored; for Q4_K the
// 32-weight sub-block sums are reduced across the 4 (bf16) or 8 (fp32) lanes holding a sub-block.
// Stage the activations of group `grp` into group slot `xs_slot` as fp16 columns (all threads of
// the CTA). Tokens two at a time: 16-byte vectors are loaded once into registers (up to 4 per
// thread per token), reduced for the per-token power-of-two prescale, converted and stored; for
// Q4_K the 32-weight sub-block sums are reduced across the 4 (bf16) or 8 (fp32) lanes holding a
// sub-block. Leaves with a __syncthreads.
template <int WT, int XT, int EPI>
__device__ void gemv_stage_x(const GemvParams& p, uint8_t* smem, const GemvLayout& L, int grp, int xs_slot,
                             int ncols, float* red) {
  const int tid = threadIdx.x;
  const int NT = blockDim.x, NW = NT >> 5;
  constexpr int VEC = (XT == XT_F32) ? 4 : 8;
  constexpr int VPT = 4;
  constexpr bool SWZ = (WT != WT_F16);
  constexpr int LPS = 32 / VEC;  // lanes holding one 32-weight sub-block
  int* misc = reinterpret_cast<int*>(smem + L.off_misc) + xs_slot * 8;
  uint8_t* xs = smem + L.off_xs + xs_slot * ncols * p.xpitch;
  const int K = p.K, M = p.M, nv = K / VEC, nsb = K / 256;
  uint8_t* sxs = smem + L.off_sxs + xs_slot * ncols * nsb * 64;
  const uint4* xv = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.x) +
                                                   static_cast<int64_t>(grp) * p.x_group_stride * (XT == XT_F32 ? 4 : 2));
  const bool one_pass = nv <= VPT * NT;
  for (int m0 = 0; m0 < M; m0 += 2) {
    const int mt = min(2, M - m0);
    uint4 q[2][VPT];
    float mx[2] = {0.f, 0.f};
#pragma unroll
    for (int t2 = 0; t2 < 2; ++t2) {
      if (t2 < mt) {
        const uint4* row = xv + static_cast<int64_t>(m0 + t2) * nv;
        if (one_pass) {
#pragma unroll
          for (int j = 0; j < VPT; ++j) {
            const int v = tid + j * NT;
            q[t2][j] = (v < nv) ? __ldg(row + v) : make_uint4(0, 0, 0, 0);
            mx[t2] = vec_absmax(q[t2][j], XT == XT_F32, mx[t2]);
          }
        } else {
          for (int v = tid; v < nv; v += NT) mx[t2] = vec_absmax(__ldg(row + v), XT == XT_F32, mx[t2]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx[t2] = fmaxf(mx[t2], __shfl_xor_sync(0xffffffffu, mx[t2], o));
        if ((tid & 31) == 0) red[(tid >> 5) * 2 + t2] = mx[t2];
      }
    }
    __syncthreads();
    int sh[2];
#pragma unroll
    for (int t2 = 0; t2 < 2; ++t2) {
      float m = 0.f;
      for (int w = 0; w < NW; ++w) m = fmaxf(m, red[w * 2 + t2]);
      sh[t2] = prescale_shift(m);
    }
    if (tid == 0) {
      for (int t2 = 0; t2 < mt; ++t2) {
        if (XT == XT_F32) {
          misc[2 * (m0 + t2)] = sh[t2];
          misc[2 * (m0 + t2) + 1] = sh[t2];
        } else {
          misc[m0 + t2] = sh[t2];
        }
      }
    }
#pragma unroll
    for (int t2 = 0; t2 < 2; ++t2) {
      if (t2 >= mt) continue;
      const int m = m0 + t2;
      const float sc = exp2i(-sh[t2]);
      const int chi = (XT == XT_F32) ? 2 * m : m;
      uint8_t* colhi = xs + chi * p.xpitch;
      uint8_t* collo = (XT == XT_F32) ? xs + (chi + 1) * p.xpitch : colhi;
      const uint4* row = xv + static_cast<int64_t>(m) * nv;
      const int nrounds = one_pass ? 1 : (nv + VPT * NT - 1) / (VPT * NT);
      for (int rd = 0; rd < nrounds; ++rd) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int v = tid + (rd * VPT + j) * NT;
          if (!one_pass && v < nv) q[t2][j] = __ldg(row + v);
          float shi = 0.f, slo = 0.f;
          if (v < nv) stage_vec<XT, SWZ>(q[t2][j], sc, colhi, collo, v, shi, slo);
          if (WT == WT_Q4K) {
#pragma unroll
            for (int o = 1; o < LPS; o <<= 1) {
              shi = __fadd_rn(shi, __shfl_xor_sync(0xffffffffu, shi, o));
              if (XT == XT_F32) slo = __fadd_rn(slo, __shfl_xor_sync(0xffffffffu, slo, o));
            }
            if (v < nv && (v % LPS) == 0) {
              const int sub = v / LPS;
              // the fp32 sum as three fp16 parts (33 significant bits)
              const __half hh = __float2half_rn(shi);
              const float r1 = __fsub_rn(shi, __half2float(hh));
              const __half hl = __float2half_rn(r1);
              const __half hl2 = __float2half_rn(__fsub_rn(r1, __half2float(hl)));
              __half* dst = reinterpret_cast<__half*>(sxs + (chi * nsb + sub / 8) * 64);
              dst[sub & 7] = hh;
              dst[8 + (sub & 7)] = hl;
              dst[16 + (sub & 7)] = hl2;
              if (XT == XT_F32) {
                const __half lh = __float2half_rn(slo);
                const float q1 = __fsub_rn(slo, __half2float(lh));
                const __half ll = __float2half_rn(q1);
                const __half ll2 = __float2half_rn(__fsub_rn(q1, __half2float(ll)));
                __half* d2 = reinterpret_cast<__half*>(sxs + ((chi + 1) * nsb + sub / 8) * 64);
                d2[sub & 7] = lh;
                d2[8 + (sub & 7)] = ll;
                d2[16 + (sub & 7)] = ll2;
              }
            }
          }
        }
      }
    }
    __syncthreads();
  }
}

// floor(a * b / c) for a * b < 2^53 and c < 2^20, in double precision (exact: a quotient within
// 1/c below an integer is not rounded up to it), instead of an emulated 64-bit integer division
__device__ __forceinline__ int muldiv_floor(int64_t a, int64_t b, int64_t c) {
  return static_cast<int>(floor(__ddiv_rn(static_cast<double>(a * b), static_cast<double>(c))));
}

__device__ __forceinline__ int worker_of_unit(int64_t u, int64_t U, int W) {
  return static_cast<int>(((u + 1) * W - 1) / U);
}

// A warp walks its unit range with an incremental cursor (no divisions in the loop); a chunk is up
// to `upc` consecutive units of one tile inside the range.
struct Cursor {
  int u, tile, sb, grp, lt;
};
struct Chunk {
  int tile, sb, n, grp, lt;
};
__device__ __forceinline__ Cursor cursor_at(int u, int nsb, int tpg) {
  Cursor c;
  c.u = u;
  c.tile = u / nsb;
  c.sb = u - c.tile * nsb;
  c.grp = c.tile / tpg;
  c.lt = c.tile - c.grp * tpg;
  return c;
}
__device__ __forceinline__ Chunk chunk_at(const Cursor& c, int b, int nsb, int upc) {
  Chunk ch;
  ch.tile = c.tile;
  ch.sb = c.sb;
  ch.grp = c.grp;
  ch.lt = c.lt;
  ch.n = min(min(upc, nsb - c.sb), b - c.u);
  return ch;
}
__device__ __forceinline__ void advance(Cursor& c, int n, int nsb, int tpg) {
  c.u += n;
  c.sb += n;
  if (c.sb == nsb) {
    c.sb = 0;
    ++c.tile;
    if (++c.lt == tpg) {
      c.lt = 0;
      ++c.grp;
    }
  }
}

template <int WT, int XT, int EPI>
__device__ __forceinline__ void issue_chunk(const GemvParams& p, const Chunk& ch, int tpg, uint8_t* slot,
                                            uint64_t* bar, int lane) {
  constexpr int UB = GemvGeom<WT, XT, EPI>::UB;
  constexpr int RPT = GemvGeom<WT, XT, EPI>::RPT;
  if (p.use_tmap) {
    // one tiled request covers all 16 rows (two 8-row requests for gate/up), aligned down to 16 B
    if (lane == 0) {
      const int grp = ch.grp, lt = ch.lt;
      const int e = p.group_ids ? p.group_ids[grp] : grp;
      const int x = ((ch.sb * UB) & ~15) / p.tm_esz;
      mbar_arrive_expect_tx(bar, static_cast<uint32_t>(16 * p.tm_box * p.tm_esz));
      tma_load_3d(slot, &p.tmap0, x, lt * RPT, e, bar);
      if (EPI == EPI_SWIGLU) tma_load_3d(slot + 8 * p.pitch, &p.tmap1, x, lt * RPT, e, bar);
    }
    __syncwarp();
    return;
  }
  uint32_t bytes = 0;
  const uint8_t* lo = nullptr;
  if (lane < 16) {
    const int grp = ch.grp, lt = ch.lt;
    const uint8_t* src = gemv_row_ptr<WT, XT, EPI>(p, grp, lt, lane) + static_cast<int64_t>(ch.sb) * UB;
    lo = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~static_cast<uintptr_t>(15));
    bytes = (static_cast<uint32_t>(src - lo) + ch.n * UB + 15u) & ~15u;
  }
  uint32_t total = bytes;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  total = __shfl_sync(0xffffffffu, total, 0);
  if (lane == 0) mbar_arrive_expect_tx(bar, total);
  __syncwarp();
  if (lane < 16) bulk_g2s(slot + lane * p.pitch, lo, bytes, bar);
}

template <int WT, int XT, int EPI, int ENG>
__global__ void __launch_bounds__(GEMV_MAXW * 32, 1) aipu_kq_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RPT = GemvGeom<WT, XT, EPI>::RPT;
  constexpr int UB = GemvGeom<WT, XT, EPI>::UB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NW = blockDim.x >> 5, S = p.nslots;
  // ENG = 1: the integer engine (Q4_K, one token) stages 8 masked int8 digit columns
  const int ncols = ENG ? 8 : ((XT == XT_F32) ? 2 * p.M : p.M);
  const GemvLayout L = gemv_layout(WT, ncols, p.K, p.xg, NW, S, p.pitch, p.xpitch, p.cta_mode ? NW : 0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * GEMV_MAXS;
  uint8_t* ring = smem + L.off_ring + warp * S * 16 * p.pitch;
  __shared__ float red[2 * GEMV_MAXW];

  if (lane < S) mbar_init(&bars[lane], 1);
  fence_mbar_init();
  __syncwarp();
  // the next kernel may be scheduled now; it reads our outputs only after its griddepcontrol.wait
  pdl_launch_dependents();

  const bool dyn = (p.group_ids != nullptr) || (p.n_groups_dev != nullptr);
  const int nsb = p.K >> 8;
  const int tpg = (p.N + RPT - 1) / RPT;
  const int G = gridDim.x, W = G * NW, wid = blockIdx.x * NW + warp;
  const int stride_slot = 16 * p.pitch;

  // weights are static: without a data-dependent group list, prefetch before waiting on the
  // previous kernel
  int U = 0, a = 0, b = 0;  // unit counts fit in 32 bits (checked on the host)
  Cursor ci;                // issue cursor
  int issued = 0, consumed = 0, islot = 0;  // islot = issued % S, kept without a division
  int ua = 0, ub = 0;  // cta mode: this CTA's units (whole tiles)
  auto setup_range = [&](int ngroups) {
    U = ngroups * tpg * nsb;
    if (p.cta_mode) {
      const int T = ngroups * tpg;
      ua = muldiv_floor(T, blockIdx.x, G) * nsb;
      ub = muldiv_floor(T, blockIdx.x + 1, G) * nsb;
      a = ua + (ub - ua) * warp / NW;
      b = ua + (ub - ua) * (warp + 1) / NW;
    } else {
      a = muldiv_floor(U, wid, W);
      b = muldiv_floor(U, wid + 1, W);
    }
    ci = cursor_at(a, nsb, tpg);
  };
  auto prefetch = [&]() {
    while (ci.u < b && issued - consumed < S) {
      const Chunk ch = chunk_at(ci, b, nsb, p.upc);
      issue_chunk<WT, XT, EPI>(p, ch, tpg, ring + islot * stride_slot, &bars[islot], lane);
      advance(ci, ch.n, nsb, tpg);
      ++issued;
      if (++islot == S) islot = 0;
    }
  };
  // (a dynamic group list is read before the wait only when the host marks it as already complete)
  const bool early = !dyn || p.ids_ready;
  if (early) {
    setup_range(p.n_groups_dev ? min(*p.n_groups_dev, p.n_groups) : p.n_groups);
    prefetch();
  }
  if (ENG) {
    // the digit columns are zero outside their sub-blocks: clear them all before the wait (the
    // staging after it writes only the live digits; its first __syncthreads orders the two)
    uint4* z = reinterpret_cast<uint4*>(smem + L.off_xs);
    const int nz = p.xg * 8 * p.xpitch / 16;
    for (int i = threadIdx.x; i < nz; i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  if (!early) {
    setup_range(p.n_groups_dev ? min(*p.n_groups_dev, p.n_groups) : p.n_groups);
    prefetch();
  }
  // stage the activations of every group this CTA touches (one group when x is shared)
  const int c0 = p.cta_mode ? ua : muldiv_floor(U, blockIdx.x * NW, W);
  const int c1 = p.cta_mode ? ub : muldiv_floor(U, (blockIdx.x + 1) * NW, W);
  const int gfirst = (c1 > c0) ? (c0 / nsb) / tpg : 0;
  const int glast = (c1 > c0) ? ((c1 - 1) / nsb) / tpg : 0;
  if (ENG) {
    if (p.x_group_stride == 0) {
      gemv_stage_x_i8<WT, XT>(p, smem, L, 0, 0, red);
    } else {
      for (int g = gfirst; g <= glast && g - gfirst < p.xg; ++g) gemv_stage_x_i8<WT, XT>(p, smem, L, g, g - gfirst, red);
    }
  } else if (p.x_group_stride == 0) {
    gemv_stage_x<WT, XT, EPI>(p, smem, L, 0, 0, ncols, red);
  } else {
    for (int g = gfirst; g <= glast && g - gfirst < p.xg; ++g) gemv_stage_x<WT, XT, EPI>(p, smem, L, g, g - gfirst, ncols, red);
  }

  // integer engine: the digit weights of this lane's two MMA columns (t = 0: digits 0, 1; t = 1: digit
  // 2 and a zero column; t = 2, 3 the same for the high-nibble columns, whose codes carry a factor 16),
  // and the PRMT selectors of its scale bytes (sub-block 2g + t / 2 of the 0-3 / 4-7 tables: byte
  // t / 2 for g even, 2 + t / 2 for g odd) and min bytes (sub-blocks 2t, 2t + 1)
  const int tl = lane & 3;
  // (Q6_K codes are assembled whole: no factor 16 in either parity)
  const bool x16 = (WT == WT_Q4K) && (tl & 2);
  const float w0 = (tl & 1) ? (x16 ? 4096.f : 65536.f) : (x16 ? 0.0625f : 1.f);
  const float w1 = (tl & 1) ? 0.f : (x16 ? 16.f : 256.f);
  const uint32_t ssel0 = 0x4440u | static_cast<uint32_t>(tl >> 1);
  const uint32_t ssel1 = 0x4440u | static_cast<uint32_t>(2 + (tl >> 1));
  const uint32_t msel0 = 0x7440u | static_cast<uint32_t>((2 * tl) & 3);
  const uint32_t msel1 = 0x7440u | static_cast<uint32_t>((2 * tl + 1) & 3);

  // ------------------------------------------------------------------ per-warp main loop
  const int g = lane >> 2, t = lane & 3;
  const bool colok = g < ncols;
  const int gx = colok ? g : 0;  // lanes of dead columns read column 0 (their results are never stored)
  // Q6_K with at most 4 columns: B column g = (group slot g / mp, column g % mp). Only with the tiled
  // copies, where every row of a slot starts at the same offset, so the unit's alignment variant is
  // the same for the whole warp (its MMAs must not diverge).
  const int mp = (WT == WT_Q6K && p.use_tmap) ? (ncols == 1 ? 1 : ncols == 2 ? 2 : ncols <= 4 ? 4 : 8) : 8;
  const int gslot = g / mp;
  const bool mok = (g % mp) < ncols;
  const int gxm = mok ? g % mp : 0;
  const int* misc0 = reinterpret_cast<const int*>(smem + L.off_misc);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  bool ok = true;
  int fin_tile = -1, fin_grp = 0, fin_lt = 0, fin_xsl = 0;  // cta mode: the tile this warp finishes
  Cursor cc = cursor_at(a, nsb, tpg);  // consume cursor
  int slot = 0, phase = 0;
  while (cc.u < b) {
    const Chunk ch = chunk_at(cc, b, nsb, p.upc);
    ok = mbar_wait_bounded(&bars[slot], phase, p.status, ST_TIMEOUT_FULL);
    if (!ok) break;
    const int grp = ch.grp, lt = ch.lt;
    const int xsl = (p.x_group_stride == 0) ? 0 : grp - gfirst;
    const uint8_t* st = ring + slot * stride_slot;
    uint32_t hg, h8;
    if (p.use_tmap) {
      hg = h8 = static_cast<uint32_t>(ch.sb * UB) & 15u;  // rows are 16-byte multiples: same head for all
    } else {
      hg = reinterpret_cast<uintptr_t>(gemv_row_ptr<WT, XT, EPI>(p, grp, lt, g) + static_cast<int64_t>(ch.sb) * UB) & 15u;
      h8 = reinterpret_cast<uintptr_t>(gemv_row_ptr<WT, XT, EPI>(p, grp, lt, g + 8) + static_cast<int64_t>(ch.sb) * UB) &
           15u;
    }
    const uint8_t* rg = st + g * p.pitch + hg;
    const uint8_t* r8 = st + (g + 8) * p.pitch + h8;
    const uint8_t* xcol = smem + L.off_xs + (xsl * ncols + gx) * p.xpitch;
    const uint8_t* xcolm = smem + L.off_xs + (xsl * ncols + gxm) * p.xpitch;
    // a chunk is one or two units (upc <= 2): straight-line calls, no loop over a runtime count
    auto do_unit = [&](const int i) {
      const int sb = ch.sb + i;
      if (ENG && WT == WT_Q4K) {
        const uint32_t xc8 = smem_u32(smem + L.off_xs + (xsl * 8 + g) * p.xpitch) + 256 * sb + 8 * t;
        const uint32_t sxb = smem_u32(smem + L.off_sxs) + 4 * (xsl * (p.K / 32) + 8 * sb);
        unit_q4k_i8(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, xc8, sxb, t, w0, w1, ssel0, ssel1, msel0, msel1, acc);
      } else if (ENG && WT == WT_Q6K) {
        const uint32_t xc8 = smem_u32(smem + L.off_xs + (xsl * 8 + g) * p.xpitch) + 256 * sb;
        const uint32_t sxb = smem_u32(smem + L.off_sxs) + 4 * (xsl * (p.K / 16) + 16 * sb);
        const int al = __shfl_sync(0xffffffffu, static_cast<int>((reinterpret_cast<uintptr_t>(rg) + i * UB) & 7u), 0);
        if (al == 0) unit_q6k_i8<0>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, xc8, sxb, t, w0, w1, acc);
        else if (al == 4) unit_q6k_i8<4>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, xc8, sxb, t, w0, w1, acc);
        else unit_q6k_i8<2>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, xc8, sxb, t, w0, w1, acc);
      } else if (WT == WT_Q4K) {
        const uint32_t sxcol = smem_u32(smem + L.off_sxs + (xsl * ncols + gx) * nsb * 64);
        unit_q4k(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcol), sxcol, sb, t, acc);
      } else if (WT == WT_Q6K) {
        // warp-uniform (lane 0's row; all rows share the offset when mp < 8)
        const bool a4 = __shfl_sync(0xffffffffu, ((reinterpret_cast<uintptr_t>(rg) + i * UB) & 3u) == 0u, 0);
        if (mp == 1) {
          if (a4) unit_q6k_mp<1, true>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcolm), mok, gslot, sb, t, acc);
          else unit_q6k_mp<1, false>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcolm), mok, gslot, sb, t, acc);
        } else if (mp == 2) {
          if (a4) unit_q6k_mp<2, true>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcolm), mok, gslot, sb, t, acc);
          else unit_q6k_mp<2, false>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcolm), mok, gslot, sb, t, acc);
        } else if (mp == 4) {
          if (a4) unit_q6k_mp<4, true>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcolm), mok, gslot, sb, t, acc);
          else unit_q6k_mp<4, false>(smem_u32(rg) + i * UB, smem_u32(r8) + i * UB, smem_u32(xcolm), mok, gslot, sb, t, acc);
        } else {
          unit_q6k(rg + i * UB, r8 + i * UB, xcol, colok, sb, t, acc);
        }
      } else if (WT == WT_Q80) {
        unit_q80(rg + i * UB, r8 + i * UB, xcol, colok, sb, t, acc);
      } else {
        unit_f16(rg + i * UB, r8 + i * UB, xcol, colok, sb, t, acc);
      }
    };
    do_unit(0);
    if (ch.n > 1) do_unit(1);
    __syncwarp();
    ++consumed;
    if (++slot == S) {
      slot = 0;
      phase ^= 1;
    }
    advance(cc, ch.n, nsb, tpg);
    prefetch();  // refill the slot just freed
    if (ch.sb + ch.n == nsb || cc.u == b) {
      // ---------------- this worker's piece of `tile` is done
      if (ENG) q4k_i8_fold(acc);
      if (WT == WT_Q6K) {
        if (mp == 1) q6k_fold<1>(acc);
        else if (mp == 2) q6k_fold<2>(acc);
        else if (mp == 4) q6k_fold<4>(acc);
      }
      const int seg0 = max(a, ch.tile * nsb);
      const bool whole = (seg0 == ch.tile * nsb) && (cc.u == (ch.tile + 1) * nsb);
      const int* misc = misc0 + xsl * 8;
      if (whole) {
        gemv_epilogue<WT, XT, EPI>(p, misc, grp, lt, acc, lane);
      } else if (p.cta_mode) {
        // piece of a tile cut between warps of this CTA: slot 0 = this warp's first tile, 1 = its last;
        // the warp holding the tile's last unit sums the pieces after the loop
        const int slot2 = (seg0 == a) ? 0 : 1;
        *reinterpret_cast<float4*>(smem + L.off_part + ((warp * 2 + slot2) * 32 + lane) * 16) =
            make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (cc.u == (ch.tile + 1) * nsb) {
          fin_tile = ch.tile;
          fin_grp = grp;
          fin_lt = lt;
          fin_xsl = xsl;
        }
      } else {
        // this worker holds units [seg0, cc.u) of the tile: slot 0 = its first tile, 1 = its last
        const int slot2 = (seg0 == a) ? 0 : 1;
        *reinterpret_cast<float4*>(p.partials + ((static_cast<int64_t>(wid) * 2 + slot2) * 32 + lane) * 4) =
            make_float4(acc[0], acc[1], acc[2], acc[3]);
        __threadfence();
        __syncwarp();
        // arrivals count units: the piece that completes the tile's nsb units finishes it
        int old = 0;
        if (lane == 0) old = atomicAdd(&p.counters[ch.tile], cc.u - seg0);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old + (cc.u - seg0) == nsb) {
          __threadfence();
          // walk the workers whose ranges meet the tile, in worker order (range starts by
          // floor(U w / W), stepped incrementally from the first one)
          const int64_t t0u = static_cast<int64_t>(ch.tile) * nsb, t1u = t0u + nsb;
          int w2 = worker_of_unit(t0u, U, W);
          int64_t s = static_cast<int64_t>(U) * w2 / W;
          int64_t frac = (static_cast<int64_t>(U) * w2) % W;
          const int64_t qs = U / W, rs = U % W;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          while (s < t1u && w2 < W) {
            int64_t e = s + qs;
            frac += rs;
            if (frac >= W) {
              frac -= W;
              ++e;
            }
            if (e > s) {  // non-empty range [s, e) of worker w2
              const int s2 = (s < t0u) ? 1 : 0;  // the tile is w2's first tile unless w2 began earlier
              const float4 r = __ldcg(reinterpret_cast<const float4*>(
                  p.partials + ((static_cast<int64_t>(w2) * 2 + s2) * 32 + lane) * 4));
              v[0] = __fadd_rn(v[0], r.x);
              v[1] = __fadd_rn(v[1], r.y);
              v[2] = __fadd_rn(v[2], r.z);
              v[3] = __fadd_rn(v[3], r.w);
            }
            s = e;
            ++w2;
          }
          gemv_epilogue<WT, XT, EPI>(p, misc, grp, lt, v, lane);
          if (lane == 0) p.counters[ch.tile] = 0;
        }
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
  }
  if (!ok) {
    // a bounded wait gave up: never leave with this warp's copies in flight
    for (int j = consumed; j < issued; ++j)
      mbar_wait_bounded(&bars[j % S], (j / S) & 1, p.status, ST_TIMEOUT_FULL, 200000000LL);
  }
  if (p.cta_mode) {
    __syncthreads();
    if (fin_tile >= 0) {
      // the pieces of the tile in warp order (a warp's slot: 0 when the tile is its first tile)
      const int t0u = fin_tile * nsb, t1u = t0u + nsb;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w2 = 0; w2 < NW; ++w2) {
        const int a2 = ua + (ub - ua) * w2 / NW, b2 = ua + (ub - ua) * (w2 + 1) / NW;
        if (a2 < b2 && a2 < t1u && b2 > t0u) {
          const float4 r = *reinterpret_cast<const float4*>(smem + L.off_part +
                                                            ((w2 * 2 + (a2 >= t0u ? 0 : 1)) * 32 + lane) * 16);
          v[0] = __fadd_rn(v[0], r.x);
          v[1] = __fadd_rn(v[1], r.y);
          v[2] = __fadd_rn(v[2], r.z);
          v[3] = __fadd_rn(v[3], r.w);
        }
      }
      gemv_epilogue<WT, XT, EPI>(p, misc0 + fin_xsl * 8, fin_grp, fin_lt, v, lane);
    }
  }
}

// ------------------------------------------------------------------ host launch
template <int WT, int XT, int EPI, int ENG = 0>
static int launch_one(GemvParams p, int grid, int nw, int smem, cudaStream_t stream, bool pdl) {
  auto kern = aipu_kq_gemv_kernel<WT, XT, EPI, ENG>;
  static bool attr_set[64] = {false};
  const int arc = set_smem_attr_once(reinterpret_cast<const void*>(kern), 232448 - 1024, attr_set, "cudaFuncSetAttribute(gemv)");
  if (arc) return arc;
  return launch_kernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(nw * 32), smem, stream, pdl, &p);
}

// units per slot: rows of at least ~288 bytes per bulk copy keep the copy engine efficient
// (at most 2: the kernel processes a chunk as one or two straight-line units)
static int gemv_upc(int wt) { return wt == WT_Q4K ? 2 : wt == WT_Q6K ? 2 : wt == WT_Q80 ? 2 : 1; }

int gemv_launch(int wt, int xt, int epi, GemvParams p, int num_sms, cudaStream_t stream, bool pdl, int min_smem) {
  if (p.K % 256 != 0 || p.K <= 0 || p.N <= 0 || p.M <= 0 || ((xt == XT_F32) ? 2 * p.M : p.M) > 8)
    return set_error(-1, "gemv: bad shape");
  // the integer dot engine for Q4_K and Q6_K rows and one token (the decode GEMV); the f16 engine
  // otherwise
  // (Q6_K: only with tiled copies, where every row of a slot starts at the same offset)
  const bool tiled_rows = (p.row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(p.w0) % 16 == 0) &&
                          (!p.w1 || reinterpret_cast<uintptr_t>(p.w1) % 16 == 0) &&
                          ((p.n_experts > 0 ? p.n_experts : p.n_groups) <= 1 || p.expert_stride % 16 == 0);
  const bool engi = (wt == WT_Q4K || (wt == WT_Q6K && tiled_rows)) && p.M == 1 && (epi == EPI_STORE || xt == XT_BF16);
  const int ncols = engi ? 8 : ((xt == XT_F32) ? 2 * p.M : p.M);
  if (epi == EPI_SWIGLU && xt != XT_BF16) return set_error(-1, "gemv: swiglu needs bf16 activations");
  if ((reinterpret_cast<uintptr_t>(p.x) & 15u) != 0) return set_error(-1, "gemv: activations must be 16-byte aligned");
  const int rpt = (epi == EPI_SWIGLU) ? 8 : 16;
  const int64_t upg = static_cast<int64_t>((p.N + rpt - 1) / rpt) * (p.K / 256);
  const int64_t U = static_cast<int64_t>(p.n_groups) * upg;
  if (U > (1ll << 30)) return set_error(-1, "gemv: problem too large for one launch (units exceed 2^30)");
  // at least one unit per worker of a full CTA, so small problems do not spread into empty workers
  int grid = static_cast<int>(std::min<int64_t>(num_sms, (U + GEMV_MAXW - 1) / GEMV_MAXW));
  if (grid < 1) grid = 1;
  p.upc = gemv_upc(wt);
  p.pitch = gemv_slot_pitch(wt, p.upc);
  // tiled TMA path when rows (and experts) start on 16-byte boundaries
  const int ne_map = p.n_experts > 0 ? p.n_experts : p.n_groups;
  const bool aligned = (p.row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(p.w0) % 16 == 0) &&
                       (!p.w1 || reinterpret_cast<uintptr_t>(p.w1) % 16 == 0) &&
                       (ne_map <= 1 || p.expert_stride % 16 == 0);
  p.use_tmap = aligned ? 1 : 0;
  if (p.use_tmap) {
    p.tm_esz = (wt == WT_Q6K) ? 2 : 8;
    p.tm_box = (wt == WT_Q4K) ? 18 * p.upc : (wt == WT_Q6K) ? 240 : 68;
    p.pitch = p.tm_box * p.tm_esz;
    const int ne = ne_map;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.row_bytes / p.tm_esz), static_cast<cuuint64_t>(p.N),
                                static_cast<cuuint64_t>(ne)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.row_bytes),
                                   static_cast<cuuint64_t>(ne > 1 ? p.expert_stride : p.row_bytes * p.N)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(p.tm_box), static_cast<cuuint32_t>(rpt), 1};
    const CUtensorMapDataType dt = (wt == WT_Q6K) ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT64;
    int rc = encode_tiled(&p.tmap0, dt, 3, p.w0, dims, strides, box);
    if (!rc && epi == EPI_SWIGLU) rc = encode_tiled(&p.tmap1, dt, 3, p.w1, dims, strides, box);
    if (rc) return rc;
  }
  // f16 engine: K fp16 values per column; integer engine: K bytes per column, +32 so that the 8 columns
  // read by a half-warp start 8 banks apart
  p.xpitch = engi ? p.K + 32 : ((p.K * 2 + 127) & ~127) + 64;
  // at least ~4 units per worker: fewer pieces per tile when a launch has few units
  const int64_t want_w = std::max<int64_t>(4, std::min<int64_t>(16, U / (4 * static_cast<int64_t>(grid))));
  // A launch with few units per CTA (a single decode GEMV) is latency-bound: its weights are on the
  // way before it may start, and what remains is the activation staging, each warp's short run of
  // units and the sums of tiles cut between warps. It runs in cta mode: whole tiles per CTA, pieces
  // summed in shared memory (no global partials, fences or arrival counters), down to one ring slot
  // per warp.
  const bool small = want_w < 16;
  const int64_t T = static_cast<int64_t>(p.n_groups) * ((p.N + rpt - 1) / rpt);
  p.cta_mode = small ? 1 : 0;
  // (up to two CTAs per SM: a tile each where there are more tiles than SMs, so no CTA holds two)
  if (small) grid = static_cast<int>(std::min<int64_t>(2 * static_cast<int64_t>(num_sms), T));
  // 8 warps and at most half an SM's shared memory, so that the next launch's CTAs become resident
  // beside this one and prefetch their weights while it finishes (measured: 3.98 / 6.18 us per launch
  // of 16 / 4096 rows x 4096 against 4.82 / 6.44 us with 16 warps that fill the SM)
  const int small_w = 8;
  if (p.x_group_stride == 0) {
    p.xg = 1;
  } else {
    const int64_t per_cta = small ? ((T + grid - 1) / grid) * (p.K / 256) : (U + grid - 1) / grid;
    p.xg = static_cast<int>(std::min<int64_t>(p.n_groups, (per_cta + upg - 1) / upg + 1));
    if (p.xg > GEMV_MAXXG) return set_error(-1, "gemv: too many activation groups per CTA");
  }
  const int full_limit = 232448 - 1024 - 2 * GEMV_MAXW * 4;  // dynamic smem limit minus static
  int limit = full_limit;
  int nw = 0, ns = 0;
  // small launches try half an SM first (unless the caller asks for a minimum), then the whole SM
  for (int pass = (small && min_smem == 0) ? 0 : 1; pass < 2 && !nw; ++pass) {
    limit = pass == 0 ? 232448 / 2 - 1024 - 2 * GEMV_MAXW * 4 : full_limit;
    for (int cand_w : {16, 12, 8, 4}) {
      if (!small && cand_w > want_w && cand_w > 4) continue;
      if (small && cand_w > small_w) continue;
      for (int cand_s = GEMV_MAXS; cand_s >= (small ? 1 : 2); --cand_s) {
        if (gemv_layout(wt, ncols, p.K, p.xg, cand_w, cand_s, p.pitch, p.xpitch, p.cta_mode ? cand_w : 0).total <=
            limit) {
          nw = cand_w;
          ns = cand_s;
          break;
        }
      }
      if (nw) break;
    }
  }
  if (!nw) return set_error(-1, "gemv: activation block too large for shared memory");
  p.nslots = ns;
  const int smem = std::min(limit, std::max(min_smem, gemv_layout(wt, ncols, p.K, p.xg, nw, ns, p.pitch, p.xpitch, p.cta_mode ? nw : 0).total));
  if (engi && wt == WT_Q4K) {
    if (xt == XT_F32) return launch_one<WT_Q4K, XT_F32, EPI_STORE, 1>(p, grid, nw, smem, stream, pdl);
    if (xt == XT_BF16 && epi == EPI_STORE) return launch_one<WT_Q4K, XT_BF16, EPI_STORE, 1>(p, grid, nw, smem, stream, pdl);
    if (xt == XT_BF16 && epi == EPI_SWIGLU) return launch_one<WT_Q4K, XT_BF16, EPI_SWIGLU, 1>(p, grid, nw, smem, stream, pdl);
  }
  if (engi && wt == WT_Q6K) {
    if (xt == XT_F32) return launch_one<WT_Q6K, XT_F32, EPI_STORE, 1>(p, grid, nw, smem, stream, pdl);
    if (xt == XT_BF16 && epi == EPI_STORE) return launch_one<WT_Q6K, XT_BF16, EPI_STORE, 1>(p, grid, nw, smem, stream, pdl);
    if (xt == XT_BF16 && epi == EPI_SWIGLU) return launch_one<WT_Q6K, XT_BF16, EPI_SWIGLU, 1>(p, grid, nw, smem, stream, pdl);
  }
#define AIPU_GEMV_CASE(W, X, E)                                              \
  if (wt == W && xt == X && epi == E) return launch_one<W, X, E>(p, grid, nw, smem, stream, pdl);
  AIPU_GEMV_CASE(WT_Q4K, XT_BF16, EPI_STORE)
  AIPU_GEMV_CASE(WT_Q4K, XT_F32, EPI_STORE)
  AIPU_GEMV_CASE(WT_Q6K, XT_BF16, EPI_STORE)
  AIPU_GEMV_CASE(WT_Q6K, XT_F32, EPI_STORE)
  AIPU_GEMV_CASE(WT_Q80, XT_BF16, EPI_STORE)
  AIPU_GEMV_CASE(WT_Q80, XT_F32, EPI_STORE)
  AIPU_GEMV_CASE(WT_F16, XT_BF16, EPI_STORE)
  AIPU_GEMV_CASE(WT_F16, XT_F32, EPI_STORE)
  AIPU_GEMV_CASE(WT_Q4K, XT_BF16, EPI_SWIGLU)
  AIPU_GEMV_CASE(WT_Q6K, XT_BF16, EPI_SWIGLU)
#undef AIPU_GEMV_CASE
  return set_error(-1, "gemv: unsupported weight/activation type combination");
}

// ------------------------------------------------------------------ allocation-free variant
// Scratch for aipu_q4k_gemm_noalloc, owned by the library for the lifetime of the process on every
// device that loads it: stream-K partials for up to kNoAllocSms CTAs of GEMV_MAXW workers, one
// arrival counter per 16-row tile for up to kNoAllocTiles tiles (N <= 65536 rows), then one status
// word (set when a bounded wait in the kernel gave up).
constexpr int kNoAllocSms = 160;
constexpr int kNoAllocTiles = 4096;
constexpr size_t kNoAllocPartialBytes = sizeof(float) * kNoAllocSms * GEMV_MAXW * 2 * 128;  // 2.5 MiB
constexpr size_t kNoAllocCounterBytes = sizeof(int) * kNoAllocTiles;                        // 16 KiB
constexpr size_t kNoAllocBytes = kNoAllocPartialBytes + kNoAllocCounterBytes + 256;        // + status word
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of the scratch array and SM count, looked up once per device with that device
// current (in host code the array's name is only a host-side stand-in, never a device address).
// The lookup is guarded by a mutex, so first calls from several threads do not race.
struct NoAllocDev {
  unsigned char* ptr = nullptr;
  int sms = 0;
};
static int noalloc_device(NoAllocDev& out) {
  static std::mutex mu;
  static NoAllocDev table[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "gemm_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(EINVAL_, "gemm_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!table[dev].ptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error(e, "gemm_noalloc: cudaGetSymbolAddress");
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_cuda_error(e, "gemm_noalloc: cudaDeviceGetAttribute");
    table[dev].sms = n < kNoAllocSms ? n : kNoAllocSms;
    table[dev].ptr = static_cast<unsigned char*>(ptr);
  }
  out = table[dev];
  return OK;
}

}  // namespace aipu

extern "C" int aipu_q4k_gemm_noalloc(int wtype, const void* w, int64_t N, int64_t K, const void* x, int x_dtype,
                                     int64_t M, void* y, void* stream) {
  using namespace aipu;
  if (!w || !x || !y || N <= 0 || M <= 0 || K <= 0 || K % 256 || K > INT32_MAX ||
      (wtype != WT_Q4K && wtype != WT_Q6K && wtype != WT_Q80 && wtype != WT_F16) ||
      (x_dtype != XT_F32 && x_dtype != XT_BF16))
    return set_error(EINVAL_, "gemm_noalloc: bad arguments");
  if ((N + 15) / 16 > kNoAllocTiles)
    return set_error(EINVAL_, "gemm_noalloc: N exceeds the static scratch limit of 65536 rows");
  if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0) return set_error(EINVAL_, "gemm_noalloc: weights must be 16-byte aligned");
  NoAllocDev nd;
  int rc = noalloc_device(nd);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partials = reinterpret_cast<float*>(nd.ptr);
  int* counters = reinterpret_cast<int*>(nd.ptr + kNoAllocPartialBytes);
  int* status = reinterpret_cast<int*>(nd.ptr + kNoAllocPartialBytes + kNoAllocCounterBytes);
  const int mb = (x_dtype == XT_F32) ? 4 : 8;
  const int esz = (x_dtype == XT_F32) ? 4 : 2;
  for (int64_t m0 = 0; m0 < M; m0 += mb) {
    // the counters must start at zero; an earlier call that gave up a bounded wait may have left
    // some set, so clear them before every launch (no allocation involved)
    cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int) * ((N + 15) / 16), s);
    if (e != cudaSuccess) return set_cuda_error(e, "gemm_noalloc: cudaMemsetAsync");
    GemvParams p = {};
    p.w0 = static_cast<const uint8_t*>(w);
    p.row_bytes = row_bytes_of(wtype, K);
    p.n_groups = 1;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.x = static_cast<const uint8_t*>(x) + m0 * K * esz;
    p.M = static_cast<int>(M - m0 < mb ? M - m0 : mb);
    p.y = static_cast<uint16_t*>(y) + m0 * N;
    p.partials = partials;
    p.counters = counters;
    p.status = status;
    rc = gemv_launch(wtype, x_dtype, EPI_STORE, p, nd.sms, s, false, 0);
    if (rc) return rc;
  }
  return OK;
}

extern "C" int aipu_q4k_gemm_noalloc_status(int* status) {
  using namespace aipu;
  if (!status) return set_error(EINVAL_, "gemm_noalloc_status: null pointer");
  NoAllocDev nd;
  int rc = noalloc_device(nd);
  if (rc) return rc;
  int* dst = reinterpret_cast<int*>(nd.ptr + kNoAllocPartialBytes + kNoAllocCounterBytes);
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, dst, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_cuda_error(e, "gemm_noalloc_status: read");
  const int zero = 0;
  e = cudaMemcpy(dst, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return set_cuda_error(e, "gemm_noalloc_status: clear");
  *status = v;
  return OK;
}

namespace aipu {

// stream-K workspace: one partial tile (32 lanes x 4 floats) per (worker, first/last tile)
int gemv_partials_floats(int num_sms) { return num_sms * GEMV_MAXW * 2 * 128; }

}  // namespace aipu
