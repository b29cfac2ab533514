// Prefill-sized dequant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   y[pos, n] = bf16( sum_k x[pos, k] * w[e, n, k] ),  w = GGUF Q4_K or Q6_K rows, many tokens
//
// Contract followed: tools/q4k_ref.py:67-92 (exact ggml dequant, fp32 accumulation, bf16 RNE); the
// accumulation order differs from the reference's sequential K order (same 1-ulp bar as the fast
// decode GEMV).
//
// Exactness on the tensor core: the MMA operands are fp16 values.
//   * tokens: fp16 with a per-token power-of-two prescale (exact for bf16 input), written once by
//     prescale_tiled_kernel in the swizzled UMMA operand layout, with the 32-weight sub-block sums
//     of every token (fp16 hi + lo) appended to each super-block;
//   * Q4_K: A = sc*q (exact, <= 945): one packed integer multiply-add per two weights gives the fp16
//     bits of 1024 + sc*q, one HSUB2 removes the 1024. Per super-block the accumulator C gets
//     sum_k x sc q and a second accumulator Cm = sum_j m_j S_j (A = 6-bit mins, B = the sub-block
//     sums). Epilogue: acc += d*C - dmin*Cm;
//   * Q6_K: A = fp16(sc * (q - 32)), exact except odd magnitudes in (2048, 4096], which round to the
//     nearest even value (relative change <= 2^-12 of that weight); epilogue acc += d*C.
//
// Persistent kernel, one CTA per SM, items = (token tile, 128-row tile) taken round-robin:
//   warp 17      raw-weight loader: one tiled TMA (or per-row bulk copies) per 64 rows x super-block
//   warp 18      activation loader: per 64-k stage, one 1 KB bulk copy per 8-token group (+ sums)
//   warps 0-7    dequant: raw super-block bytes (smem) -> A operand in TMEM (tcgen05.st; warp w
//                writes rows 32 (w % 4).. and k half w / 4 of each 64-k stage), per-row scales
//   warp 16      TMEM allocation and the single MMA-issuing thread (A from TMEM, B from smem)
//   warps 8-15   epilogue: TMEM lane = output row, 64 token columns each; register accumulators
//                over the super-blocks, output (or the SwiGLU of a gate/up row pair) per item.
// TMEM: two accumulators C (128 columns each) alternate between super-blocks so the MMAs of one
// super-block overlap the epilogue of the previous one; Cm (Q4_K, 128 columns); a ring of A stages.
// No TMA multicast, no clusters. Every wait is bounded; on expiry the CTA sets the status word, every
// role leaves its loop, the copies and MMAs in flight are drained (bounded) and TMEM is freed.
#include <algorithm>
#include <cstdio>

#include "act.cuh"
#include "deq.cuh"
#include "kernels.h"
#include "launch.h"
#include "tc.cuh"

namespace aipu {

// Tiled activation layout, per (8-token group, super-block) XT_SB = 4352 bytes: four 1024-byte
// 128-byte-swizzled K-major atoms (64 k each: token row t at 128 t, 16-byte chunk c at (c ^ t) * 16),
// then 256 bytes of sub-block sums in the no-swizzle core-matrix layout (fp16 hi parts of the 8
// sub-block sums at 16 t, lo parts at 128 + 16 t).
constexpr int XT_SB = 4352;

// ------------------------------------------------------------------ SiLU table
// bf16(silu(x)) for every bf16 x (the reference's step sequence, glm_silu_bf), written once per
// device at context creation: the SwiGLU epilogue of the prefill GEMM looks its gate values up
// (one load instead of the ~60-instruction sequence per output), with identical bits.
__device__ uint16_t g_silu_tab[65536];

__global__ void silu_table_kernel() {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536u) g_silu_tab[i] = static_cast<uint16_t>(__float_as_uint(glm_silu_bf(__uint_as_float(i << 16))) >> 16);
}

int silu_table_init(cudaStream_t s) {
  silu_table_kernel<<<256, 256, 0, s>>>();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "silu_table_kernel");
  return set_cuda_error(cudaStreamSynchronize(s), "silu_table_kernel");
}

__device__ __forceinline__ float silu_lookup(float xbf) {
  return __uint_as_float(static_cast<uint32_t>(__ldg(&g_silu_tab[__float_as_uint(xbf) >> 16])) << 16);
}

// ------------------------------------------------------------------ activation prescale (tiled)
// Row p of the output (p < n_pos) takes source row src = rows ? rows[p] : p (rows_mask: src = p when
// rows[p] >= 0); src < 0 or src >= R gives a zero row. fp16 values x * 2^-shift[p] (max |x| * 2^-s
// in [2^9, 2^10)), written in the (0,2,1,3) order inside every aligned group of four k, as UMMA
// the tiled layout above (XT_SB). One CTA per row.
__global__ void __launch_bounds__(256) prescale_tiled_kernel(const uint16_t* __restrict__ x, int R, int K,
                                                             const int* __restrict__ rows, int rows_mask,
                                                             int n_pos_host, const int* __restrict__ n_pos_dev,
                                                             uint8_t* __restrict__ xt, int* __restrict__ shift) {
  pdl_wait();
  const int p = blockIdx.x;
  const int n_pos = n_pos_dev ? *n_pos_dev : n_pos_host;
  if (p >= n_pos) {
    pdl_launch_dependents();
    return;
  }
  int src = p;
  if (rows) {
    const int v = rows[p];
    src = rows_mask ? (v >= 0 ? p : -1) : v;
  }
  if (src >= R) src = -1;
  const int tid = threadIdx.x;
  const int nv = K / 8, nsb = K / 256;
  const int t = p & 7;
  uint8_t* grp = xt + static_cast<int64_t>(p >> 3) * nsb * XT_SB;
  if (src < 0) {
    for (int v = tid; v < nsb * 34; v += 256) {
      const int sb = v / 34, c = v - sb * 34;
      const int off = c < 32 ? (c >> 3) * 1024 + t * 128 + (((c & 7) ^ t) << 4) : 4096 + (c - 32) * 128 + t * 16;
      *reinterpret_cast<uint4*>(grp + static_cast<int64_t>(sb) * XT_SB + off) = make_uint4(0, 0, 0, 0);
    }
    if (tid == 0) shift[p] = 0;
    pdl_launch_dependents();
    return;
  }
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
  if (tid == 0) shift[p] = s;
  const float sc = exp2i(-s);
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
      const int sb = v >> 5, c = v & 31;
      *reinterpret_cast<uint4*>(grp + static_cast<int64_t>(sb) * XT_SB + (c >> 3) * 1024 + t * 128 +
                                (((c & 7) ^ t) << 4)) =
          make_uint4(h[0] | (h[2] << 16), h[1] | (h[3] << 16), h[4] | (h[6] << 16), h[5] | (h[7] << 16));
    }
    // sub-block sum over the 4 lanes holding it
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
    if (v < nv && (v & 3) == 0) {
      const int sb = v >> 5, j = (v >> 2) & 7;
      const __half hh = __float2half_rn(sum);
      const __half hl = __float2half_rn(__fsub_rn(sum, __half2float(hh)));
      __half* d = reinterpret_cast<__half*>(grp + static_cast<int64_t>(sb) * XT_SB + 4096 + t * 16);
      d[j] = hh;
      d[64 + j] = hl;  // the lo parts start 128 bytes (64 halfs) later
    }
  }
  pdl_launch_dependents();
}

// ------------------------------------------------------------------ GEMM kernel
constexpr int TC_THREADS = 608;  // 19 warps
constexpr int W_EPI = 8, W_MMA = 16, W_RAW = 17, W_BLD = 18;

template <int WT, int NT>
struct TcCfg {
  // smem pitch of one row's super-block window: 144 (Q4_K) / 240 (Q6_K: a 16-byte aligned window of
  // 224 bytes holds the 210-byte block; 15 chunks keep 16-byte loads of 8 consecutive rows on
  // distinct banks)
  static constexpr int RAW = (WT == WT_Q4K) ? 144 : 240;
  static constexpr int RAW_SLOT = 128 * RAW;
  static constexpr int NRAW = (WT == WT_Q4K) ? 4 : 3;
  // one stage = 128 k (half a super-block). B slot: 8-token group g at 2048 g (two swizzled 64-k
  // atoms), then (Q4_K) the sub-block sums of the group at B_X + 256 g
  static constexpr int B_X = (NT / 8) * 2048;
  static constexpr int B_SLOT = B_X + ((WT == WT_Q4K) ? (NT / 8) * 256 : 0);
  static constexpr int NB = (NT == 64) ? 4 : ((WT == WT_Q4K) ? 3 : 4);
  static constexpr int NDS = 8;                             // scale ring (super-blocks)
  static constexpr int NMIN = 2;                            // min-operand ring (super-blocks)
  static constexpr int OFF_B = 1024;
  static constexpr int OFF_RAW = OFF_B + NB * B_SLOT;
  static constexpr int OFF_AOFF = OFF_RAW + NRAW * RAW_SLOT;
  static constexpr int OFF_AMIN = OFF_AOFF;
  static constexpr int OFF_DS = OFF_AMIN + ((WT == WT_Q4K) ? NMIN * 4096 : 0);
  static constexpr int TOTAL = OFF_DS + NDS * 128 * 8;
  // TMEM (512 columns): accumulators C[b] at NT b (b = 0, 1); Q4_K min accumulators Cm: NT = 64:
  // Cm[b] at 128 + 64 b (double-buffered), NT = 128: one Cm at 256; then the ring of A stages
  // (64 columns each) up to column 512.
  static constexpr bool CM2 = (NT == 64);
  static constexpr uint32_t COL_CM = 2 * NT;
  static constexpr uint32_t COL_A = (WT == WT_Q4K && !CM2) ? 384 : 256;
  static constexpr int NA = static_cast<int>((512 - COL_A) / 64);
  // NT = 64: A and B rings hold two super-blocks, so the MMAs of a super-block commit once
  // (acc_full), which also releases both of its stages; NT = 128: one commit per stage
  static constexpr bool SBREL = (NA == 4 && NB == 4);
  static_assert(NA == 2 || NA == 4, "A ring of 2 or 4 stages");
};
static_assert(TcCfg<WT_Q4K, 128>::TOTAL <= 232448 && TcCfg<WT_Q4K, 64>::TOTAL <= 232448, "Q4_K tc smem");
static_assert(TcCfg<WT_Q6K, 128>::TOTAL <= 232448 && TcCfg<WT_Q6K, 64>::TOTAL <= 232448, "Q6_K tc smem");

// byte offset of (row r, 16-byte chunk c) in a K-major no-swizzle operand whose 8-row groups are
// `sbo` bytes apart (chunks of one 8-row group are 128 bytes apart)
__device__ __forceinline__ int core_off(int r, int c, int sbo) { return (r >> 3) * sbo + c * 128 + (r & 7) * 16; }

struct TcBars {
  uint64_t raw_full[4], raw_empty[4];
  uint64_t stage_full[4];  // stage k: 8 dequant-warp arrivals + the activation bytes
  // stage release: the MMAs of the first half of super-block s complete on stage_done[s & 1], those
  // of the second half (and so the whole accumulator of s) on acc_full[s & 1]
  uint64_t stage_done[2], acc_full[2], acc_empty[2], cm_empty, ds_full[8], ds_empty[8], drain;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(TcBars) <= 1024, "barrier block");

// bounded wait that also gives up as soon as another role of the CTA gave up
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, TcBars* sb, int* status, int bit) {
  if (mbar_try_wait(bar, parity)) return true;
  long long limit = 0;  // the context's limit, read once the wait outlasts the grace period
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(&sb->abort)) return false;
    const long long el = clock64() - t0;
    if (el > kWaitGrace && limit == 0) limit = wait_limit(status);
    if (el > kWaitGrace && el > limit) {
      *reinterpret_cast<volatile int*>(&sb->abort) = 1;
      if (status) atomicOr(status, bit);
      return false;
    }
  }
  return true;
}
// short bounded drain wait at exit (copies or MMAs in flight after an abort)
__device__ __forceinline__ void tc_drain_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > 200000000LL) return;
}

// Optional role timing (compile with -DTC_TRACE): cycles each role spends waiting, summed over CTAs.
#ifdef TC_TRACE
__device__ unsigned long long g_tc_trace[64];
#define TW(acc, expr)               \
  ([&]() {                          \
    const long long t_ = clock64(); \
    const bool r_ = (expr);         \
    acc += clock64() - t_;          \
    return r_;                      \
  }())
#define TFLUSH(base, arr, n)                                                                                     \
  do {                                                                                                            \
    if (lane == 0)                                                                                                \
      for (int k_ = 0; k_ < (n); ++k_) atomicAdd(&g_tc_trace[(base) + k_ + (SWIGLU ? 32 : 0)], static_cast<unsigned long long>(arr[k_])); \
  } while (0)
#define TT(acc, stmt)         \
  do {                        \
    const long long t_ = clock64(); \
    stmt;                     \
    acc += clock64() - t_;    \
  } while (0)
#else
#define TT(acc, stmt) \
  do {                \
    stmt;             \
  } while (0)
#define TW(acc, expr) (expr)
#define TFLUSH(base, arr, n) \
  do {                       \
  } while (0)
#endif

struct TcItem {
  int e, t0, tn, rt;
};
template <int NT>
__device__ __forceinline__ TcItem tc_item(const TcParams& p, int i, int n_rt) {
  TcItem it;
  const int tile = i / n_rt;
  it.rt = i - tile * n_rt;
  if (p.tiles) {
    const int4 tl = p.tiles[tile];
    it.e = tl.x;
    it.t0 = tl.y;
    it.tn = tl.z;
  } else {
    it.e = 0;
    it.t0 = tile * NT;
    it.tn = min(NT, p.M - it.t0);
  }
  return it;
}

__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
// NW consecutive 32-bit words starting o bytes (o even, 0..14) after a 16-byte aligned shared
// address p16, read as 16-byte vectors; the word shift by o / 4 is two select levels (o is uniform
// per super-block, so no branches), the 2-byte remainder a funnel shift.
template <int NW>
__device__ __forceinline__ void lds_words_at(const uint8_t* p16, int o, uint32_t (&out)[NW]) {
  constexpr int NV = (4 * NW + 14) / 16 + 1;
  uint32_t w[4 * NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint4 t = reinterpret_cast<const uint4*>(p16)[i];
    w[4 * i] = t.x;
    w[4 * i + 1] = t.y;
    w[4 * i + 2] = t.z;
    w[4 * i + 3] = t.w;
  }
  const bool s2 = (o & 8) != 0, s1 = (o & 4) != 0;
  const uint32_t sh = static_cast<uint32_t>(o & 3) * 8;
  uint32_t a[NW + 2], b[NW + 1];
#pragma unroll
  for (int i = 0; i < NW + 2; ++i) a[i] = s2 ? w[i + 2] : w[i];
#pragma unroll
  for (int i = 0; i < NW + 1; ++i) b[i] = s1 ? a[i + 1] : a[i];
#pragma unroll
  for (int j = 0; j < NW; ++j) out[j] = __funnelshift_r(b[j], b[j + 1], sh);
}

// Release of stage k (= 2 * super-block s + half h) of a ring: the MMAs that read it are complete.
template <bool SBREL>
__device__ __forceinline__ bool tc_wait_stage_done(TcBars* bars, uint32_t k, int* status) {
  const uint32_t s = k >> 1;
  uint64_t* bar = (SBREL || (k & 1)) ? &bars->acc_full[s & 1] : &bars->stage_done[s & 1];
  return tc_wait(bar, (s >> 1) & 1, bars, status, ST_TIMEOUT_EMPTY);
}

template <int WT, int NT, bool SWIGLU>
__global__ void __launch_bounds__(TC_THREADS, 1) aipu_tc_gemm_kernel(const __grid_constant__ TcParams p) {
  using C = TcCfg<WT, NT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  TcBars* bars = reinterpret_cast<TcBars*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = p.K / 256;
  const int rows_per_item = SWIGLU ? 64 : 128;
  const int n_rt = (p.N + rows_per_item - 1) / rows_per_item;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; ++s) {
      mbar_init(&bars->raw_full[s], 1);
      mbar_init(&bars->raw_empty[s], 8);
      mbar_init(&bars->stage_full[s], 9);
    }
    for (int s = 0; s < 8; ++s) {
      mbar_init(&bars->ds_full[s], 8);
      mbar_init(&bars->ds_empty[s], 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->stage_done[b], 1);
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 8);
    }
    mbar_init(&bars->cm_empty, 8);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == W_MMA) tmem_alloc(&bars->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  pdl_wait();
  const int n_tiles = p.tiles ? (p.tile_count ? *p.tile_count : 0) : (p.M + NT - 1) / NT;
  const int n_items = n_tiles * n_rt;

  if (warp == W_RAW) {
    // ============================================================ raw-weight loader
    long long tw[4] = {0, 0, 0, 0};
    const long long t_role = clock64();
    uint32_t kr = 0;
    bool ok = true;
    for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
      const TcItem it = tc_item<NT>(p, i, n_rt);
      const bool shared = (it.e == p.shared_id);
      const int ez = shared ? 0 : it.e;
      const int row0 = it.rt * rows_per_item;
      for (int sb = 0; sb < nsb; ++sb, ++kr) {
        const int slot = kr % C::NRAW;
        if (kr >= static_cast<uint32_t>(C::NRAW) && lane == 0)
          ok = TW(tw[0], tc_wait(&bars->raw_empty[slot], ((kr / C::NRAW) + 1) & 1, bars, p.status, ST_TIMEOUT_EMPTY));
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        uint8_t* dst = smem + C::OFF_RAW + slot * C::RAW_SLOT;
        if (p.use_tmap) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&bars->raw_full[slot], C::RAW_SLOT);
            const int x = (WT == WT_Q4K) ? sb * 18 : ((sb * 210) >> 4) * 8;  // 16-byte aligned start
            const CUtensorMap* m0 = shared ? &p.smap[0] : &p.wmap[0];
            const CUtensorMap* m1 = SWIGLU ? (shared ? &p.smap[1] : &p.wmap[1]) : m0;
            tma_load_3d(dst, m0, x, row0, ez, &bars->raw_full[slot]);
            tma_load_3d(dst + 64 * C::RAW, m1, x, SWIGLU ? row0 : row0 + 64, ez, &bars->raw_full[slot]);
          }
        } else {
          // per-row 16-byte aligned windows (rows whose start is not 16-byte aligned: Q6_K)
          const uint8_t* b0 = shared ? p.ws[0] : p.w[0] + static_cast<int64_t>(ez) * p.expert_stride;
          const uint8_t* b1 = SWIGLU ? (shared ? p.ws[1] : p.w[1] + static_cast<int64_t>(ez) * p.expert_stride) : b0;
          const int valid_half = max(0, min(64, p.N - row0));
          const int nvalid = SWIGLU ? 2 * valid_half : max(0, min(128, p.N - row0));
          if (lane == 0) mbar_arrive_expect_tx(&bars->raw_full[slot], nvalid * ((WT == WT_Q4K) ? 144 : 224));
          __syncwarp();
          for (int r = lane; r < 128; r += 32) {
            const int nrow = SWIGLU ? row0 + (r & 63) : row0 + r;
            if (nrow >= p.N) continue;
            const uint8_t* src = ((SWIGLU && r >= 64) ? b1 : b0) + static_cast<int64_t>(nrow) * p.row_bytes +
                                 static_cast<int64_t>(sb) * ((WT == WT_Q4K) ? 144 : 210);
            src = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~static_cast<uintptr_t>(15));
            bulk_g2s(dst + r * C::RAW, src, (WT == WT_Q4K) ? 144 : 224, &bars->raw_full[slot]);
          }
        }
      }
    }
    // drain copies still in flight (only after an abort; a normal exit has consumed them all)
    if (lane == 0)
      for (uint32_t j = kr > static_cast<uint32_t>(C::NRAW) ? kr - C::NRAW : 0; j < kr; ++j)
        tc_drain_wait(&bars->raw_full[j % C::NRAW], (j / C::NRAW) & 1);
    tw[3] = clock64() - t_role;
    TFLUSH(0, tw, 4);
  } else if (warp == W_BLD) {
    // ============================================================ activation loader
    long long tw[4] = {0, 0, 0, 0};
    const long long t_role = clock64();
    uint32_t kb = 0;
    bool ok = true;
    const int64_t gstride = static_cast<int64_t>(nsb) * XT_SB;
    for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
      const TcItem it = tc_item<NT>(p, i, n_rt);
      const int ngroups = ((it.tn + 15) & ~15) >> 3;
      const uint8_t* xg = p.xt + static_cast<int64_t>(it.t0 >> 3) * gstride;
      for (int sb = 0; ok && sb < nsb; ++sb) {
        for (int h = 0; h < 2; ++h, ++kb) {
          const int slot = kb % C::NB;
          if (kb >= static_cast<uint32_t>(C::NB) && lane == 0)
            ok = TW(tw[0], tc_wait_stage_done<C::SBREL>(bars, kb - C::NB, p.status));
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          const bool sums = (WT == WT_Q4K && h == 1);
          uint64_t* full = &bars->stage_full[kb & 3];
          if (lane == 0) mbar_arrive_expect_tx(full, ngroups * (sums ? 2304 : 2048));
          __syncwarp();
          uint8_t* dst = smem + C::OFF_B + slot * C::B_SLOT;
          if (lane < ngroups) {
            const uint8_t* src = xg + lane * gstride + static_cast<int64_t>(sb) * XT_SB;
            bulk_g2s(dst + lane * 2048, src + h * 2048, 2048, full);
            if (sums) bulk_g2s(dst + C::B_X + lane * 256, src + 4096, 256, full);
          }
        }
      }
    }
    if (lane == 0)
      for (uint32_t j = kb > static_cast<uint32_t>(C::NB) ? kb - C::NB : 0; j < kb; ++j)
        tc_drain_wait(&bars->stage_full[j & 3], (j >> 2) & 1);
    tw[3] = clock64() - t_role;
    TFLUSH(4, tw, 4);
  } else if (warp < W_EPI) {
    // ============================================================ dequant -> TMEM A operand
    // warp w: TMEM lanes (rows) 32 (w % 4) .. +31, k half hk = w / 4 of every 128-k stage
    const int q = warp & 3, hk = warp >> 2;
    const int r = q * 32 + lane;
    // raw row; SwiGLU: lanes 0-15 of warp q are gate rows 16q.., lanes 16-31 the up rows of the same
    // outputs (a gate/up pair is 16 lanes apart in one warp)
    const int rr = SWIGLU ? ((lane & 16) ? 64 + 16 * q + (lane & 15) : 16 * q + (lane & 15)) : r;
    const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float2* dsc = reinterpret_cast<float2*>(smem + C::OFF_DS);
    long long tw[6] = {0, 0, 0, 0, 0, 0};
    const long long t_role = clock64();
    uint32_t kr = 0, kd = 0;
    bool ok = true;
    for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
      const TcItem it = tc_item<NT>(p, i, n_rt);
      const bool shared = (it.e == p.shared_id);
      const int ez = shared ? 0 : it.e;
      int nrow = SWIGLU ? it.rt * 64 + (rr & 63) : it.rt * 128 + rr;
      nrow = min(nrow, p.N - 1);
      const uint8_t* wbase = (SWIGLU && rr >= 64) ? (shared ? p.ws[1] : p.w[1]) : (shared ? p.ws[0] : p.w[0]);
      const uintptr_t growaddr = reinterpret_cast<uintptr_t>(wbase) +
                                 static_cast<uintptr_t>(shared ? 0 : static_cast<int64_t>(ez) * p.expert_stride) +
                                 static_cast<uintptr_t>(static_cast<int64_t>(nrow) * p.row_bytes);
      for (int sb = 0; ok && sb < nsb; ++sb, ++kr) {
        const int rslot = kr % C::NRAW;
        ok = __all_sync(0xffffffffu,
                        TW(tw[0], tc_wait(&bars->raw_full[rslot], (kr / C::NRAW) & 1, bars, p.status, ST_TIMEOUT_FULL)));
        if (!ok) break;
        const uint8_t* raw = smem + C::OFF_RAW + rslot * C::RAW_SLOT + rr * C::RAW;
        float d, dmin = 0.f;
        uint32_t scw[2] = {0, 0}, m03 = 0, m47 = 0;
        int o = 0;
        if (WT == WT_Q4K) {
          const uint4 hd = *reinterpret_cast<const uint4*>(raw);
          d = f16_bits_to_f32(hd.x & 0xFFFFu);
          dmin = f16_bits_to_f32(hd.x >> 16);
          scw[0] = hd.y & 0x3F3F3F3Fu;
          m03 = hd.z & 0x3F3F3F3Fu;
          scw[1] = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
          m47 = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        } else {
          o = static_cast<int>((growaddr + static_cast<uintptr_t>(sb) * 210u) & 15u);
          d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(raw + o + 208));
        }
        // per-(row, super-block) scales for the epilogue
        {
          const int ds = kd % C::NDS;
          if (kd >= static_cast<uint32_t>(C::NDS))
            ok = __all_sync(0xffffffffu, TW(tw[1], tc_wait(&bars->ds_empty[ds], ((kd / C::NDS) + 1) & 1, bars,
                                                           p.status, ST_TIMEOUT_EMPTY)));
          if (!ok) break;
          if (hk == 0) dsc[ds * 128 + r] = make_float2(d, dmin);
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->ds_full[ds]);
          ++kd;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t ka = 2 * kr + h;
          const int aslot = ka % C::NA;
          if (ka >= static_cast<uint32_t>(C::NA))
            ok = __all_sync(0xffffffffu, TW(tw[2], tc_wait_stage_done<C::SBREL>(bars, ka - C::NA, p.status)));
          if (!ok) break;
          tc_fence_after();
          uint32_t v[32];
#ifdef TC_TRACE
          const long long t_c = clock64();
#endif
          if (WT == WT_Q4K) {
            // 64 k of this warp = qs group g = 2h + hk (32 bytes): low nibbles sub-block 2g, high 2g+1
            const int g = 2 * h + hk;
            const uint4 q0 = *reinterpret_cast<const uint4*>(raw + 16 + 32 * g);
            const uint4 q1 = *reinterpret_cast<const uint4*>(raw + 32 + 32 * g);
            const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            const uint32_t scp = scw[g >> 1] >> (16 * (g & 1));
            const uint32_t sclo = scp & 0xFFu, schi = (scp >> 8) & 0xFFu;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              // 1024 + sc q by one integer multiply-add per two codes, then - 1024 (exact: sc q <= 945)
              const uint32_t w0 = qw[2 * c], w1 = qw[2 * c + 1], o1024 = 0x64006400u;
              v[4 * c + 0] = hsub2_u32((w0 & 0x000F000Fu) * sclo + o1024, o1024);
              v[4 * c + 1] = hsub2_u32(((w0 >> 8) & 0x000F000Fu) * sclo + o1024, o1024);
              v[4 * c + 2] = hsub2_u32((w1 & 0x000F000Fu) * sclo + o1024, o1024);
              v[4 * c + 3] = hsub2_u32(((w1 >> 8) & 0x000F000Fu) * sclo + o1024, o1024);
              v[16 + 4 * c + 0] = hsub2_u32(((w0 >> 4) & 0x000F000Fu) * schi + o1024, o1024);
              v[16 + 4 * c + 1] = hsub2_u32(((w0 >> 12) & 0x000F000Fu) * schi + o1024, o1024);
              v[16 + 4 * c + 2] = hsub2_u32(((w1 >> 4) & 0x000F000Fu) * schi + o1024, o1024);
              v[16 + 4 * c + 3] = hsub2_u32(((w1 >> 12) & 0x000F000Fu) * schi + o1024, o1024);
            }
            if (h == 1 && hk == 0) {
              // min-term operand: the 8 six-bit mins, twice (against the hi and the lo sums)
              uint32_t mh[4];
#pragma unroll
              for (int i2 = 0; i2 < 4; ++i2) {
                const uint32_t mw = (i2 < 2) ? m03 : m47;
                const int b0 = 2 * (i2 & 1);
                const uint32_t lo16 = __half_as_ushort(__uint2half_rn((mw >> (8 * b0)) & 0xFFu));
                const uint32_t hi16 = __half_as_ushort(__uint2half_rn((mw >> (8 * (b0 + 1))) & 0xFFu));
                mh[i2] = lo16 | (hi16 << 16);
              }
              const uint4 mv = make_uint4(mh[0], mh[1], mh[2], mh[3]);
              uint8_t* amin = smem + C::OFF_AMIN + (kr % C::NMIN) * 4096;
              *reinterpret_cast<uint4*>(amin + core_off(r, 0, 256)) = mv;
              *reinterpret_cast<uint4*>(amin + core_off(r, 1, 256)) = mv;
              fence_async_smem();
            }
          } else {
            // Q6_K half h of the super-block; this warp: runs 2hk, 2hk+1 (32 weights each, ql nibble hk).
            // A = fp16(sc * (q - 32)): exact except odd magnitudes in (2048, 4096], rounded to even.
            uint32_t Lw[16], Qw[8], Sw[2];
            lds_words_at<16>(raw + 64 * h, o, Lw);
            lds_words_at<8>(raw + 128 + 32 * h, o, Qw);
            lds_words_at<2>(raw + 192 + ((o + 8 * h) & 16), (o + 8 * h) & 15, Sw);  // the 8 scales of half h
#pragma unroll
            for (int rl = 0; rl < 2; ++rl) {
              const int run = 2 * hk + rl;
              uint32_t scv2[2];
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                // scale byte 2 run + j = 4 hk + (2 rl + j) of the 8
                const uint32_t sw = hk ? Sw[1] : Sw[0];
                const int s8 = static_cast<int8_t>((sw >> (8 * (2 * rl + j))) & 0xFFu);
                const __half2 s2 = __half2half2(__int2half_rn(s8));
                scv2[j] = *reinterpret_cast<const uint32_t*>(&s2);
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) {  // word j: weights l = 4j .. 4j+3 of the run
                const uint32_t n4 = (Lw[8 * rl + j] >> (4 * hk)) & 0x0F0F0F0Fu;
                const uint32_t hb = (Qw[j] >> (2 * run)) & 0x03030303u;
                const uint32_t code = hb * 16u + n4;  // 6-bit codes, one per byte
                // fp16 bits 0x6400 | code (= 1024 + code) for codes 0, 2 and 1, 3 of the word
                const uint32_t c02 = prmt(code, 0x64u, 0x4240u);
                const uint32_t c13 = prmt(code, 0x64u, 0x4341u);
                const uint32_t sc2 = scv2[j >> 2];
                v[16 * rl + 2 * j] = hmul2_u32(hsub2_u32(c02, 0x64206420u), sc2);
                v[16 * rl + 2 * j + 1] = hmul2_u32(hsub2_u32(c13, 0x64206420u), sc2);
              }
            }
          }
#ifdef TC_TRACE
          tw[4] += clock64() - t_c;
#endif
          uint32_t v0[16], v1[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v0[j] = v[j];
            v1[j] = v[16 + j];
          }
          const uint32_t ta = trow + C::COL_A + aslot * 64 + hk * 32;
          TT(tw[5], {
            tmem_st16(ta, v0);
            tmem_st16(ta + 16, v1);
          });
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->stage_full[ka & 3]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->raw_empty[rslot]);
      }
    }
    tw[3] = clock64() - t_role;
    if (warp == 0) TFLUSH(8, tw, 4);
    if (warp == 0) TFLUSH(24, (tw + 4), 2);
  } else if (warp == W_MMA) {
    // ============================================================ MMA issuer
    uint32_t ksb = 0;
    bool ok = true, issued = false;
    long long tw[6] = {0, 0, 0, 0, 0, 0};
    const long long t_role = clock64();
    if (lane == 0) {
      for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
        const TcItem it = tc_item<NT>(p, i, n_rt);
        const uint32_t idesc = umma_idesc_f16(128, (it.tn + 15) & ~15);
        for (int sb = 0; ok && sb < nsb; ++sb, ++ksb) {
          const int buf = ksb & 1;
          if (ksb >= 2)
            ok = TW(tw[0], tc_wait(&bars->acc_empty[buf], ((ksb >> 1) + 1) & 1, bars, p.status, ST_TIMEOUT_EMPTY));
          if (!ok) break;
          const uint32_t dC = tmem + buf * NT;
          const uint32_t dCm = tmem + C::COL_CM + (C::CM2 ? buf * 64 : 0);
          for (int h = 0; h < 2; ++h) {
            const uint32_t k = 2 * ksb + h;
            const int aslot = k % C::NA, bslot = k % C::NB;
            ok = TW(tw[1], tc_wait(&bars->stage_full[k & 3], (k >> 2) & 1, bars, p.status, ST_TIMEOUT_FULL));
            if (WT == WT_Q4K && !C::CM2 && h == 1 && ksb >= 1 && ok)
              ok = TW(tw[0], tc_wait(&bars->cm_empty, (ksb - 1) & 1, bars, p.status, ST_TIMEOUT_EMPTY));
            if (!ok) break;
            tc_fence_after();
            const uint32_t At = tmem + C::COL_A + aslot * 64;
            const uint32_t B = smem_u32(smem + C::OFF_B + bslot * C::B_SLOT);
            TT(tw[4], {
#pragma unroll
              for (int ks = 0; ks < 8; ++ks)
                umma_f16_ts(dC, At + 8 * ks, umma_desc_sw128(B + (ks >> 2) * 1024 + 32 * (ks & 3), 2048), idesc,
                            (h | ks) ? 1u : 0u);
            });
            if (WT == WT_Q4K && h == 1)
              umma_f16(dCm, umma_desc(smem_u32(smem + C::OFF_AMIN + (ksb % C::NMIN) * 4096), 128, 256),
                       umma_desc(B + C::B_X, 128, 256), idesc, 0u);
            issued = true;
            if (h) TT(tw[5], umma_commit(&bars->acc_full[buf]));
            else if (!C::SBREL) TT(tw[5], umma_commit(&bars->stage_done[buf]));
          }
        }
      }
      if (issued) {
        umma_commit(&bars->drain);
        tc_drain_wait(&bars->drain, 0);
      }
      tw[3] = clock64() - t_role;
      TFLUSH(12, tw, 4);
      TFLUSH(20, (tw + 4), 2);
    }
    __syncwarp();
  } else {
    // ============================================================ epilogue (warps 8..15)
    const int ew = warp - W_EPI;
    const int q = ew & 3, half = ew >> 2;
    const int r = q * 32 + lane;  // TMEM lane = A row
    const float2* dsc = reinterpret_cast<const float2*>(smem + C::OFF_DS);
    uint32_t ksb = 0, kd = 0;
    bool ok = true;
    long long tw[4] = {0, 0, 0, 0};
    const long long t_role = clock64();
    for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
      const TcItem it = tc_item<NT>(p, i, n_rt);
      const int nm = (it.tn + 15) & ~15;
      constexpr int HC = NT / 2;  // columns of this warp
      // prescale of this warp's columns: lane l holds column half * HC + l (HC <= 64: two per lane)
      int shl0 = 0, shl1 = 0;
      {
        const int c0 = half * HC + lane, c1 = c0 + 32;
        if (lane < HC && c0 < it.tn) shl0 = p.xshift[it.t0 + c0];
        if (HC > 32 && lane + 32 < HC && c1 < it.tn) shl1 = p.xshift[it.t0 + c1];
      }
      float acc[HC];
#pragma unroll
      for (int n = 0; n < HC; ++n) acc[n] = 0.f;
      for (int sb = 0; sb < nsb; ++sb, ++ksb, ++kd) {
        const int buf = ksb & 1, ds = kd % C::NDS;
        ok = __all_sync(0xffffffffu,
                        TW(tw[0], tc_wait(&bars->acc_full[buf], (ksb >> 1) & 1, bars, p.status, ST_TIMEOUT_FULL) &&
                                      tc_wait(&bars->ds_full[ds], (kd / C::NDS) & 1, bars, p.status, ST_TIMEOUT_FULL)));
        if (!ok) break;
        tc_fence_after();
        const float2 dd = dsc[ds * 128 + r];
        const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const uint32_t tc0 = tl + buf * NT + half * HC;
        const uint32_t tcm = tl + C::COL_CM + (C::CM2 ? buf * 64 : 0) + half * HC;
#pragma unroll
        for (int j = 0; j < HC / 16; ++j) {
          if (half * HC + 16 * j >= nm) continue;  // warp-uniform
          uint32_t c[16], cm[16];
          tmem_ld16_nw(tc0 + 16 * j, c);
          if (WT == WT_Q4K) tmem_ld16_nw(tcm + 16 * j, cm);
          tmem_wait_ld();
#pragma unroll
          for (int i2 = 0; i2 < 16; ++i2) {
            float a = fmaf(dd.x, __uint_as_float(c[i2]), acc[16 * j + i2]);
            if (WT == WT_Q4K) a = fmaf(-dd.y, __uint_as_float(cm[i2]), a);
            acc[16 * j + i2] = a;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars->acc_empty[buf]);
          mbar_arrive(&bars->ds_empty[ds]);
          if (WT == WT_Q4K && !C::CM2) mbar_arrive(&bars->cm_empty);
        }
      }
      if (!ok) break;
      const long long t_out = clock64();
      // ---- output of the item
      if (SWIGLU) {
        // lanes l and l + 16 hold the gate and up accumulators of one output row; per column pair
        // (2m, 2m + 1) the gate lane finishes column 2m and the up lane column 2m + 1
        const int nrow = it.rt * 64 + 16 * q + (lane & 15);
        const bool upl = lane >= 16;
#pragma unroll
        for (int m = 0; m < HC / 2; ++m) {
          if (half * HC + 2 * m >= it.tn) break;  // warp-uniform
          const float send = upl ? acc[2 * m] : acc[2 * m + 1];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
          const float g = upl ? recv : acc[2 * m];
          const float u = upl ? acc[2 * m + 1] : recv;
          const int n = 2 * m + (upl ? 1 : 0);
          const int shn = __shfl_sync(0xffffffffu, (2 * m < 32) ? shl0 : shl1, n & 31);
          const int col = half * HC + n;
          if (col < it.tn && nrow < p.N) {
            const float s = exp2i(shn);
            const float gb = bf16_round_f(__fmul_rn(g, s));
            const float ub = bf16_round_f(__fmul_rn(u, s));
            p.y[static_cast<int64_t>(it.t0 + col) * p.N + nrow] = bf16_rne_bits(__fmul_rn(silu_lookup(gb), ub));
          }
        }
      } else {
        const int nrow = it.rt * 128 + r;
#pragma unroll
        for (int n = 0; n < HC; ++n) {
          const int col = half * HC + n;
          if (col >= it.tn) break;  // warp-uniform
          const int shn = __shfl_sync(0xffffffffu, n < 32 ? shl0 : shl1, n & 31);
          const int pos = it.t0 + col;
          if (nrow < p.N) p.y[static_cast<int64_t>(pos) * p.N + nrow] = bf16_rne_bits(__fmul_rn(acc[n], exp2i(shn)));
        }
      }
      tw[1] += clock64() - t_out;
    }
    tw[3] = clock64() - t_role;
    if (warp == W_EPI) TFLUSH(16, tw, 4);
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
    tmem_relinquish();
  }
}

// ------------------------------------------------------------------ host
template <int WT, int NT, bool SW>
static int tc_launch_one(const TcParams& p, int grid, cudaStream_t s, bool pdl) {
  constexpr int smem = TcCfg<WT, NT>::TOTAL;
  auto kern = aipu_tc_gemm_kernel<WT, NT, SW>;
  static bool attr[64] = {false};
  {
    const int arc = set_smem_attr_once(reinterpret_cast<const void*>(kern), smem, attr, "cudaFuncSetAttribute(tc_gemm)");
    if (arc) return arc;
  }
  TcParams q = p;
  return launch_kernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(TC_THREADS), smem, s, pdl, &q);
}

static int tc_encode(CUtensorMap* map, int wt, const uint8_t* base, int64_t row_bytes, int N, int ne,
                     int64_t expert_stride) {
  const int esz = (wt == WT_Q4K) ? 8 : 2;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_bytes / esz), static_cast<cuuint64_t>(N),
                              static_cast<cuuint64_t>(ne)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes),
                                 static_cast<cuuint64_t>(ne > 1 ? expert_stride : row_bytes * N)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(wt == WT_Q4K ? 18 : 120), 64, 1};
  return encode_tiled(map, wt == WT_Q4K ? CU_TENSOR_MAP_DATA_TYPE_UINT64 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, base,
                      dims, strides, box);
}

int tc_gemm_launch(TcParams& p, int nt, int n_experts, int max_tiles, int num_sms, cudaStream_t s, bool pdl) {
  if (nt != 64 && nt != 128) return set_error(EINVAL_, "tc_gemm: tile width must be 64 or 128");
  if (p.K % 256 || p.K <= 0 || p.N <= 0 || (p.wt != WT_Q4K && p.wt != WT_Q6K) || (p.swiglu && p.wt != WT_Q4K) ||
      !p.w[0] || (p.swiglu && !p.w[1]) || !p.xt || !p.xshift || !p.y)
    return set_error(EINVAL_, "tc_gemm: needs Q4_K or Q6_K weights, K % 256 == 0 (SwiGLU: Q4_K)");
  if (max_tiles <= 0) return OK;
  const bool has_shared = p.shared_id >= 0;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  bool aligned = p.row_bytes % 16 == 0 && (n_experts <= 1 || p.expert_stride % 16 == 0) && al16(p.w[0]) &&
                 (!p.swiglu || al16(p.w[1]));
  if (has_shared) aligned = aligned && al16(p.ws[0]) && (!p.swiglu || al16(p.ws[1]));
  p.use_tmap = aligned ? 1 : 0;
  if (aligned) {
    int rc = tc_encode(&p.wmap[0], p.wt, p.w[0], p.row_bytes, p.N, n_experts, p.expert_stride);
    if (!rc && p.swiglu) rc = tc_encode(&p.wmap[1], p.wt, p.w[1], p.row_bytes, p.N, n_experts, p.expert_stride);
    if (!rc && has_shared) rc = tc_encode(&p.smap[0], p.wt, p.ws[0], p.row_bytes, p.N, 1, 0);
    if (!rc && has_shared && p.swiglu) rc = tc_encode(&p.smap[1], p.wt, p.ws[1], p.row_bytes, p.N, 1, 0);
    if (rc) return rc;
  } else if (p.wt == WT_Q4K) {
    return set_error(EINVAL_, "tc_gemm: Q4_K weights must be 16-byte aligned");
  }
  const int rows_per_item = p.swiglu ? 64 : 128;
  const int64_t items = static_cast<int64_t>(max_tiles) * ((p.N + rows_per_item - 1) / rows_per_item);
  const int grid = static_cast<int>(std::min<int64_t>(num_sms, items));
  if (nt == 64) {
    if (p.wt == WT_Q4K)
      return p.swiglu ? tc_launch_one<WT_Q4K, 64, true>(p, grid, s, pdl) : tc_launch_one<WT_Q4K, 64, false>(p, grid, s, pdl);
    return tc_launch_one<WT_Q6K, 64, false>(p, grid, s, pdl);
  }
  if (p.wt == WT_Q4K)
    return p.swiglu ? tc_launch_one<WT_Q4K, 128, true>(p, grid, s, pdl) : tc_launch_one<WT_Q4K, 128, false>(p, grid, s, pdl);
  return tc_launch_one<WT_Q6K, 128, false>(p, grid, s, pdl);
}

size_t xt_bytes(int64_t R, int64_t K) {
  const int64_t groups = (R + 7) / 8 + 2;  // +2 groups: the MMA may read one 8-token group past a tile
  return static_cast<size_t>(groups) * (K / 256) * XT_SB;
}

int prescale_tiled_launch(const uint16_t* x, int R, int K, const int* rows, int rows_mask, int n_pos_max,
                          const int* n_pos_dev, uint8_t* xt, int* shift, cudaStream_t s, bool pdl) {
  if (K % 256 || R <= 0 || n_pos_max <= 0) return set_error(EINVAL_, "prescale: K % 256 != 0");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_pos_max);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return set_cuda_error(
      cudaLaunchKernelEx(&cfg, prescale_tiled_kernel, x, R, K, rows, rows_mask, n_pos_max, n_pos_dev, xt, shift),
      "prescale_tiled_kernel");
}

}  // namespace aipu

#ifdef TC_TRACE
// role timing readout of a -DTC_TRACE build (cycles summed over CTAs; see g_tc_trace)
extern "C" int aipu_debug_tc_trace(unsigned long long* out, int reset) {
  if (cudaMemcpyFromSymbol(out, aipu::g_tc_trace, sizeof(aipu::g_tc_trace)) != cudaSuccess) return -1;
  if (reset) {
    static const unsigned long long z[64] = {};
    cudaMemcpyToSymbol(aipu::g_tc_trace, z, sizeof(z));
  }
  return 0;
}
#endif
