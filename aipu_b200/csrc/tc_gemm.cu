// Prefill-sized dequant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   y[tok, n] = bf16( sum_k x[tok, k] * w[n, k] ),  w = GGUF Q4_K or Q6_K rows, many tokens
//
// Contract followed: tools/q4k_ref.py:67-92 (exact ggml dequant, fp32 accumulation, bf16 RNE); the
// accumulation order differs from the reference's sequential K order (same 1-ulp bar as the fast
// decode GEMV).
//
// Exactness on the tensor core: the MMA operands must be exact fp16 values.
//   * tokens: fp16 with a per-token power-of-two prescale (exact for bf16 input), produced once by
//     prescale_rows_kernel together with the 32-weight sub-block sums of every token;
//   * Q4_K: A = 1024 + sc*q built with one packed integer multiply-add per two weights (exact,
//     sc*q <= 945); per super-block the accumulator holds sum_k x (1024 + sc q); the epilogue applies
//     d*(C - 1024*S) - dmin*Cm, where S is the token's super-block sum and Cm = sum_j m_j S_j comes
//     from one more small MMA (A = 6-bit mins, B = the token's sub-block sums as fp16 hi + lo);
//   * Q6_K: sc*q spans 13 bits, so A = 8*sc*a + sc*b with q = 8a + b (a in -4..3, b in 0..7): two
//     exact operands, two MMAs into the same accumulator, epilogue d*C.
// One super-block (256 k) is one TMEM accumulator; two accumulator buffers alternate so the MMA of
// the next super-block overlaps the epilogue of the previous one.
//
// CTA = 128 output rows x a tile of NT tokens (NT = 64 or 128) of one group (expert):
//   warps 0-3  producers: build A (128 rows x 128 k per stage) and B (NT tokens x 128 k) in shared
//              memory in the UMMA K-major, no-swizzle core-matrix layout (8 rows x 16 bytes);
//   warps 4-7  epilogue: TMEM lane = output row, register accumulators over the super-blocks;
//   warp 8     TMEM allocation and the single MMA-issuing thread.
// No TMA multicast, no clusters.
#include <algorithm>
#include <cstdio>

#include "act.cuh"
#include "deq.cuh"
#include "kernels.h"
#include "launch.h"
#include "tc.cuh"

namespace aipu {

// ------------------------------------------------------------------ activation prescale
// rows [R, K] bf16 -> fp16 [R, K] scaled by 2^-shift[r] (max |x| * 2^-s in [2^9, 2^10)), stored with
// the (0,2,1,3) order inside every aligned group of four k (the order the weight operands use);
// sx[r, sb, 0..15] = fp16 hi (0..7) / lo (8..15) parts of the 8 sub-block sums of super-block sb;
// sxsb[r, sb] = fp32 sum over the super-block. One CTA per row.
__global__ void __launch_bounds__(256) prescale_rows_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                            const int* __restrict__ rows, int n_rows_dev_max,
                                                            const int* __restrict__ n_rows_dev,
                                                            __half* __restrict__ xh, int* __restrict__ shift,
                                                            __half* __restrict__ sx, float* __restrict__ sxsb) {
  pdl_wait();
  const int r = blockIdx.x;
  const int nrows = n_rows_dev ? min(*n_rows_dev, n_rows_dev_max) : R;
  if (r >= nrows) return;
  const int src = rows ? rows[r] : r;
  const int tid = threadIdx.x;
  const int nv = K / 8, nsb = K / 256;
  const uint4* xv = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(src) * K);
  __shared__ float red[8];
  float mx = 0.f;
  for (int v = tid; v < nv; v += 256) {
    const uint4 q = __ldg(xv + v);
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mx = fmaxf(mx, fabsf(__uint_as_float(w4[i] << 16)));
      mx = fmaxf(mx, fabsf(__uint_as_float(w4[i] & 0xFFFF0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = 0.f;
  for (int w = 0; w < 8; ++w) mx = fmaxf(mx, red[w]);
  const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu);
  int s = (mx == 0.f) ? 0 : (e - 127 - 9);
  s = s < -100 ? -100 : (s > 100 ? 100 : s);
  if (tid == 0) shift[r] = s;
  const float sc = exp2i(-s);
  uint4* out = reinterpret_cast<uint4*>(xh + static_cast<int64_t>(r) * K);
  // nv is a multiple of 32 (K % 256 == 0): every warp-iteration covers whole sub-blocks (4 vectors)
  for (int v0 = 0; v0 < nv; v0 += 256) {
    const int v = v0 + tid;
    float sum = 0.f;
    if (v < nv) {
      const uint4 q = __ldg(xv + v);
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
      uint32_t h[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half a = __float2half_rn(__fmul_rn(__uint_as_float(w4[i] << 16), sc));
        const __half b = __float2half_rn(__fmul_rn(__uint_as_float(w4[i] & 0xFFFF0000u), sc));
        h[2 * i] = __half_as_ushort(a);
        h[2 * i + 1] = __half_as_ushort(b);
        sum = __fadd_rn(sum, __fadd_rn(__half2float(a), __half2float(b)));
      }
      out[v] = make_uint4(h[0] | (h[2] << 16), h[1] | (h[3] << 16), h[4] | (h[6] << 16), h[5] | (h[7] << 16));
    }
    // sub-block sum over the 4 lanes holding it
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
    if (v < nv && (v & 3) == 0 && sx) {
      const int sub = v >> 2, sb = sub >> 3, j = sub & 7;
      const __half hh = __float2half_rn(sum);
      const __half hl = __float2half_rn(__fsub_rn(sum, __half2float(hh)));
      __half* d = sx + (static_cast<int64_t>(r) * nsb + sb) * 16;
      d[j] = hh;
      d[8 + j] = hl;
    }
    // super-block sum over the 32 lanes holding it (8 sub-blocks)
    float ssb = sum;
    ssb = __fadd_rn(ssb, __shfl_xor_sync(0xffffffffu, ssb, 4));
    ssb = __fadd_rn(ssb, __shfl_xor_sync(0xffffffffu, ssb, 8));
    ssb = __fadd_rn(ssb, __shfl_xor_sync(0xffffffffu, ssb, 16));
    if (v < nv && (v & 31) == 0 && sxsb) sxsb[static_cast<int64_t>(r) * nsb + (v >> 5)] = ssb;
  }
  pdl_launch_dependents();
}

// ------------------------------------------------------------------ GEMM kernel
constexpr int TC_THREADS = 288;
constexpr int TC_KS = 128;  // k per stage (half a super-block)

struct TcLayout {
  int a_bytes, a2_bytes, b_bytes, amin_bytes, bmin_bytes, stage_bytes, nst, off_stage, total;
};
__host__ __device__ inline TcLayout tc_layout(int wt, int NT, int nst) {
  TcLayout L;
  L.a_bytes = 128 * TC_KS * 2;
  L.a2_bytes = (wt == WT_Q6K) ? L.a_bytes : 0;
  L.b_bytes = NT * TC_KS * 2;
  L.amin_bytes = (wt == WT_Q4K) ? 128 * 16 * 2 : 0;
  L.bmin_bytes = (wt == WT_Q4K) ? NT * 16 * 2 : 0;
  L.stage_bytes = L.a_bytes + L.a2_bytes + L.b_bytes + L.amin_bytes + L.bmin_bytes;
  L.nst = nst;
  L.off_stage = 1024;
  L.total = L.off_stage + nst * L.stage_bytes;
  return L;
}

// byte offset of (row r, 16-byte chunk c) in a K-major no-swizzle operand whose 8-row groups are
// `sbo` bytes apart (chunks of one 8-row group are 128 bytes apart)
__device__ __forceinline__ int core_off(int r, int c, int sbo) { return (r >> 3) * sbo + c * 128 + (r & 7) * 16; }

template <int WT, int NT, bool SWIGLU>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NST = (WT == WT_Q6K) ? 2 : 3;
  const TcLayout L = tc_layout(WT, NT, NST);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 4;
  uint64_t* accful = empty + 4;
  uint64_t* accempty = accful + 2;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(accempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- which (group, token tile) this CTA computes
  pdl_wait();
  int grp = 0, t0 = 0, tn = 0;
  if (!p.tiles) {
    t0 = blockIdx.y * NT;
    tn = min(NT, p.M - t0);
    if (tn <= 0) return;
  } else {
    const int ntiles = p.tile_count ? *p.tile_count : 1;
    if (static_cast<int>(blockIdx.y) >= ntiles) return;
    const int4 tl = p.tiles[blockIdx.y];  // (group, first position, tokens, -)
    grp = tl.x;
    t0 = tl.y;
    tn = tl.z;
  }
  const int e = p.group_ids ? p.group_ids[grp] : grp;
  const int rt = blockIdx.x;
  const int nsb = p.K / 256;
  const int nstage = 2 * nsb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accful[b], 1);
      mbar_init(&accempty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 8) tmem_alloc(tmem_base_s, 4 * NT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  // TMEM columns: C[0] at 0, C[1] at NT, Cm[0] at 2NT, Cm[1] at 3NT

  if (warp < 4) {
    // ================================================================= producers
    const int r = threadIdx.x;  // A row
    int nrow;
    const uint8_t* wsrc;
    if (SWIGLU) {
      nrow = rt * 64 + (r & 63);
      wsrc = (r < 64) ? p.w0 : p.w1;
    } else {
      nrow = rt * 128 + r;
      wsrc = p.w0;
    }
    nrow = nrow < p.N ? nrow : p.N - 1;
    const uint8_t* wrow = wsrc + static_cast<int64_t>(e) * p.expert_stride + static_cast<int64_t>(nrow) * p.row_bytes;
    for (int s = 0; s < nstage; ++s) {
      const int slot = s % NST;
      if (s >= NST) mbar_wait_bounded(&empty[slot], ((s / NST) - 1) & 1, p.status, ST_TIMEOUT_EMPTY);
      uint8_t* st = smem + L.off_stage + slot * L.stage_bytes;
      uint8_t* A = st;
      uint8_t* A2 = st + L.a_bytes;
      uint8_t* B = A2 + L.a2_bytes;
      uint8_t* Amin = B + L.b_bytes;
      uint8_t* Bmin = Amin + L.amin_bytes;
      const int sb = s >> 1, h = s & 1;
      if (WT == WT_Q4K) {
        const uint8_t* blk = wrow + static_cast<int64_t>(sb) * 144;
        const uint4 hd = __ldg(reinterpret_cast<const uint4*>(blk));
        const uint32_t sc03 = hd.y & 0x3F3F3F3Fu, m03 = hd.z & 0x3F3F3F3Fu;
        const uint32_t sc47 = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
        const uint32_t m47 = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        const uint32_t scw = h ? sc47 : sc03;  // sub-blocks 4h .. 4h+3
        uint4 qv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qv[i] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 64 * h + 16 * i));
        const uint32_t* qw = reinterpret_cast<const uint32_t*>(qv);  // 64 bytes = groups 2h, 2h+1
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int pl = c >> 3, kk = (c * 8) & 63;  // group within the half, k within the group
          const bool hi = kk >= 32;
          const int off = pl * 32 + (hi ? kk - 32 : kk);  // byte offset inside the 64 loaded bytes
          const int jl = 2 * pl + (hi ? 1 : 0);           // sub-block within the half
          const uint32_t sc = (scw >> (8 * jl)) & 0xFFu;
          const uint32_t w0 = qw[off >> 2], w1 = qw[(off >> 2) + 1];
          uint4 o;
          if (!hi) {
            o.x = (w0 & 0x000F000Fu) * sc + 0x64006400u;
            o.y = ((w0 >> 8) & 0x000F000Fu) * sc + 0x64006400u;
            o.z = (w1 & 0x000F000Fu) * sc + 0x64006400u;
            o.w = ((w1 >> 8) & 0x000F000Fu) * sc + 0x64006400u;
          } else {
            o.x = ((w0 >> 4) & 0x000F000Fu) * sc + 0x64006400u;
            o.y = ((w0 >> 12) & 0x000F000Fu) * sc + 0x64006400u;
            o.z = ((w1 >> 4) & 0x000F000Fu) * sc + 0x64006400u;
            o.w = ((w1 >> 12) & 0x000F000Fu) * sc + 0x64006400u;
          }
          *reinterpret_cast<uint4*>(A + core_off(r, c, 2048)) = o;
        }
        if (h == 1) {
          // min-term operand: row r = the 8 six-bit mins, twice (for the hi and lo sums)
          uint32_t mh[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t mw = (i < 2) ? m03 : m47;
            const int b0 = 2 * (i & 1);
            const uint32_t lo16 = __half_as_ushort(__uint2half_rn((mw >> (8 * b0)) & 0xFFu));
            const uint32_t hi16 = __half_as_ushort(__uint2half_rn((mw >> (8 * (b0 + 1))) & 0xFFu));
            mh[i] = lo16 | (hi16 << 16);
          }
          const uint4 mv = make_uint4(mh[0], mh[1], mh[2], mh[3]);
          *reinterpret_cast<uint4*>(Amin + core_off(r, 0, 256)) = mv;
          *reinterpret_cast<uint4*>(Amin + core_off(r, 1, 256)) = mv;
        }
      } else {  // Q6_K: q = 8a + b, A = 8 sc a, A2 = sc b (both exact in fp16)
        const uint8_t* blk = wrow + static_cast<int64_t>(sb) * 210;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int kk = 8 * c;                 // k inside this half (0..127)
          const int qi = kk >> 5, l0 = kk & 31;  // which of q1..q4, position l
          const uint8_t* ql = blk + 64 * h + ((qi & 1) ? 32 : 0) + l0;
          const uint8_t* qh = blk + 128 + 32 * h + l0;
          const int8_t scv = static_cast<int8_t>(blk[192 + 8 * h + 2 * qi + (l0 >> 4)]);
          const __half2 sc2 = __half2half2(__int2half_rn(scv));
          const __half2 sc8 = __half2half2(__int2half_rn(8 * scv));
          uint32_t code[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t nib = (qi >= 2) ? (ql[i] >> 4) : (ql[i] & 0xFu);
            code[i] = nib | (((qh[i] >> (2 * qi)) & 3u) << 4);
          }
          // weights of the chunk in the (0,2,1,3) order: pairs (0,2),(1,3),(4,6),(5,7)
          const int ord[8] = {0, 2, 1, 3, 4, 6, 5, 7};
          uint32_t oa[4], ob[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t c0 = code[ord[2 * i]], c1 = code[ord[2 * i + 1]];
            // a = (code >> 3) - 4 in -4..3, b = code & 7
            const uint32_t av = ((c0 >> 3) | ((c1 >> 3) << 16)) | 0x64006400u;  // 1024 + (a + 4)
            const uint32_t bv = ((c0 & 7u) | ((c1 & 7u) << 16)) | 0x64006400u;  // 1024 + b
            __half2 ah = __hsub2(*reinterpret_cast<const __half2*>(&av), __floats2half2_rn(1028.f, 1028.f));
            __half2 bh = __hsub2(*reinterpret_cast<const __half2*>(&bv), __floats2half2_rn(1024.f, 1024.f));
            ah = __hmul2(ah, sc8);
            bh = __hmul2(bh, sc2);
            oa[i] = *reinterpret_cast<uint32_t*>(&ah);
            ob[i] = *reinterpret_cast<uint32_t*>(&bh);
          }
          *reinterpret_cast<uint4*>(A + core_off(r, c, 2048)) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
          *reinterpret_cast<uint4*>(A2 + core_off(r, c, 2048)) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
        }
      }
      // ---- B: NT tokens x 128 k (16 chunks each), zeros past the tile's tokens
      const int kbase = sb * 256 + h * TC_KS;
      for (int idx = threadIdx.x; idx < NT * 16; idx += 128) {
        const int n = idx >> 4, c = idx & 15;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n < tn) {
          const int pos = t0 + n;
          const int xr = p.x_rows ? p.x_rows[pos] : pos;
          v = __ldg(reinterpret_cast<const uint4*>(p.xh + static_cast<int64_t>(xr) * p.K + kbase + 8 * c));
        }
        *reinterpret_cast<uint4*>(B + core_off(n, c, 2048)) = v;
      }
      if (WT == WT_Q4K && h == 1) {
        for (int idx = threadIdx.x; idx < NT * 2; idx += 128) {
          const int n = idx >> 1, c = idx & 1;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (n < tn) {
            const int pos = t0 + n;
            const int xr = p.x_rows ? p.x_rows[pos] : pos;
            v = __ldg(reinterpret_cast<const uint4*>(p.sx + (static_cast<int64_t>(xr) * nsb + sb) * 16 + 8 * c));
          }
          *reinterpret_cast<uint4*>(Bmin + core_off(n, c, 256)) = v;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[slot]);
    }
  } else if (warp == 8) {
    // ================================================================= MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(128, NT);
      for (int s = 0; s < nstage; ++s) {
        const int slot = s % NST, sb = s >> 1, h = s & 1, buf = sb & 1;
        mbar_wait_bounded(&full[slot], (s / NST) & 1, p.status, ST_TIMEOUT_FULL);
        if (h == 0 && sb >= 2) mbar_wait_bounded(&accempty[buf], ((sb >> 1) - 1) & 1, p.status, ST_TIMEOUT_EMPTY);
        tc_fence_after();
        const uint32_t st = smem_u32(smem + L.off_stage + slot * L.stage_bytes);
        const uint32_t A = st, A2 = st + L.a_bytes, B = A2 + L.a2_bytes, Amin = B + L.b_bytes,
                       Bmin = Amin + L.amin_bytes;
        const uint32_t dC = tmem + buf * NT;
#pragma unroll 1
        for (int ks = 0; ks < TC_KS / 16; ++ks) {
          const uint64_t bd = umma_desc(B + ks * 256, 128, 2048);
          umma_f16(dC, umma_desc(A + ks * 256, 128, 2048), bd, idesc, (h == 0 && ks == 0) ? 0u : 1u);
          if (WT == WT_Q6K) umma_f16(dC, umma_desc(A2 + ks * 256, 128, 2048), bd, idesc, 1u);
        }
        if (WT == WT_Q4K && h == 1)
          umma_f16(tmem + 2 * NT + buf * NT, umma_desc(Amin, 128, 256), umma_desc(Bmin, 128, 256), idesc, 0u);
        umma_commit(&empty[slot]);
        if (h == 1) umma_commit(&accful[buf]);
      }
    }
    __syncwarp();
  } else {
    // ================================================================= epilogue
    const int q = warp - 4;
    const int r = q * 32 + lane;  // TMEM lane = A row
    int nrow;
    const uint8_t* wsrc;
    if (SWIGLU) {
      nrow = rt * 64 + (r & 63);
      wsrc = (r < 64) ? p.w0 : p.w1;
    } else {
      nrow = rt * 128 + r;
      wsrc = p.w0;
    }
    const int nrc = nrow < p.N ? nrow : p.N - 1;
    const uint8_t* wrow = wsrc + static_cast<int64_t>(e) * p.expert_stride + static_cast<int64_t>(nrc) * p.row_bytes;
    float acc[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n] = 0.f;
    for (int sb = 0; sb < nsb; ++sb) {
      const int buf = sb & 1;
      mbar_wait_bounded(&accful[buf], (sb >> 1) & 1, p.status, ST_TIMEOUT_FULL);
      tc_fence_after();
      float d, dmin = 0.f;
      if (WT == WT_Q4K) {
        const uint32_t hd = __ldg(reinterpret_cast<const uint32_t*>(wrow + static_cast<int64_t>(sb) * 144));
        d = f16_bits_to_f32(hd);
        dmin = f16_bits_to_f32(hd >> 16);
      } else {
        d = f16_bits_to_f32(ld_u16(wrow + static_cast<int64_t>(sb) * 210 + 208));
      }
      const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
      for (int n0 = 0; n0 < NT; n0 += 16) {
        float c[16];
        tmem_ld16(tl + buf * NT + n0, c);
        if (WT == WT_Q4K) {
          float cm[16];
          tmem_ld16(tl + 2 * NT + buf * NT + n0, cm);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = n0 + i;
            float S = 0.f;
            if (n < tn) {
              const int pos = t0 + n;
              const int xr = p.x_rows ? p.x_rows[pos] : pos;
              S = __ldg(p.sxsb + static_cast<int64_t>(xr) * nsb + sb);
            }
            acc[n] = fmaf(-dmin, cm[i], fmaf(d, fmaf(-1024.f, S, c[i]), acc[n]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[n0 + i] = fmaf(d, c[i], acc[n0 + i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[buf]);
    }
    // ---- output
    if (SWIGLU) {
      // up rows (TMEM lanes 64..127) hand their accumulators to the gate rows through shared memory
      float* ex = reinterpret_cast<float*>(smem + L.off_stage);
      named_bar_sync(2, 128);  // all MMAs are complete: every accumulator was read above
      if (r >= 64) {
#pragma unroll
        for (int n = 0; n < NT; ++n) ex[n * 64 + (r - 64)] = acc[n];
      }
      named_bar_sync(2, 128);
      if (r < 64 && nrow < p.N) {
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (n >= tn) continue;
          const int pos = t0 + n;
          const int xr = p.x_rows ? p.x_rows[pos] : pos;
          const float s = exp2i(p.xshift[xr]);
          const float gb = bf16_round_f(__fmul_rn(acc[n], s));
          const float ub = bf16_round_f(__fmul_rn(ex[n * 64 + r], s));
          p.y[static_cast<int64_t>(pos) * p.N + nrow] = bf16_rne_bits(__fmul_rn(glm_silu_bf(gb), ub));
        }
      }
    } else if (nrow < p.N) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if (n >= tn) continue;
        const int pos = t0 + n;
        const int xr = p.x_rows ? p.x_rows[pos] : pos;
        p.y[static_cast<int64_t>(pos) * p.N + nrow] = bf16_rne_bits(__fmul_rn(acc[n], exp2i(p.xshift[xr])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 4 * NT);
    tmem_relinquish();
  }
}

// ------------------------------------------------------------------ host
template <int WT, int NT, bool SW>
static int tc_launch_one(const TcParams& p, dim3 grid, cudaStream_t s, bool pdl) {
  constexpr int NST = (WT == WT_Q6K) ? 2 : 3;
  const int smem = tc_layout(WT, NT, NST).total;
  auto kern = tc_gemm_kernel<WT, NT, SW>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(tc_gemm)");
    attr = true;
  }
  TcParams q = p;
  return launch_kernel(reinterpret_cast<const void*>(kern), grid, dim3(TC_THREADS), smem, s, pdl, &q);
}

int tc_gemm_launch(const TcParams& p, int nt, int max_tiles, cudaStream_t s, bool pdl) {
  if (p.K % 256 || p.K <= 0 || p.N <= 0 || (p.wt != WT_Q4K && p.wt != WT_Q6K) || (p.swiglu && p.wt != WT_Q4K))
    return set_error(EINVAL_, "tc_gemm: needs Q4_K or Q6_K weights, K % 256 == 0 (SwiGLU: Q4_K)");
  const int rows_per_cta = p.swiglu ? 64 : 128;
  dim3 grid((p.N + rows_per_cta - 1) / rows_per_cta, max_tiles);
  if (p.wt == WT_Q4K) {
    if (p.swiglu) return nt == 64 ? tc_launch_one<WT_Q4K, 64, true>(p, grid, s, pdl)
                                  : tc_launch_one<WT_Q4K, 128, true>(p, grid, s, pdl);
    return nt == 64 ? tc_launch_one<WT_Q4K, 64, false>(p, grid, s, pdl) : tc_launch_one<WT_Q4K, 128, false>(p, grid, s, pdl);
  }
  return nt == 64 ? tc_launch_one<WT_Q6K, 64, false>(p, grid, s, pdl) : tc_launch_one<WT_Q6K, 128, false>(p, grid, s, pdl);
}

int prescale_launch(const uint16_t* x, int R, int K, const int* rows, const int* n_rows_dev, __half* xh, int* shift,
                    __half* sx, float* sxsb, cudaStream_t s, bool pdl) {
  if (K % 256 || R <= 0) return set_error(EINVAL_, "prescale: K % 256 != 0");
  struct Args {
    const uint16_t* x;
    int R, K;
    const int* rows;
    int n_max;
    const int* n_dev;
    __half* xh;
    int* shift;
    __half* sx;
    float* sxsb;
  };
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(R);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return set_cuda_error(cudaLaunchKernelEx(&cfg, prescale_rows_kernel, x, R, K, rows, R, n_rows_dev, xh, shift, sx, sxsb),
                        "prescale_rows_kernel");
}

}  // namespace aipu
