// Exact (bit-for-bit) kernels: dequant, strict sequential GEMM, strict router with sigmoid
// top-K, and the MoE weighted combine. Each follows the reference golden op for op.
#include <algorithm>
#include <cstdio>


#include "act.cuh"
#include "deq.cuh"
#include "kernels.h"
#include "ep_sync.cuh"
#include "launch.h"

namespace aipu {

// ------------------------------------------------------------------ dequant
// out[r, k] = exact dequant of weight k of row r (fp32, or bf16 RNE of that fp32)
__global__ void dequant_kernel(int wt, const uint8_t* __restrict__ w, int64_t nrows, int64_t K, int64_t row_bytes,
                               void* __restrict__ out, int out_bf16) {
  const int64_t total = nrows * K;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / K, k = i - r * K;
    const float v = deq_one(wt, w + r * row_bytes, k);
    if (out_bf16)
      reinterpret_cast<uint16_t*>(out)[i] = bf16_rne_bits(v);
    else
      reinterpret_cast<float*>(out)[i] = v;
  }
}

int dequant_launch(int wt, const void* w, int64_t nrows, int64_t K, void* out, int out_bf16, cudaStream_t s) {
  const int64_t total = nrows * K;
  if (total <= 0) return OK;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  dequant_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(wt, static_cast<const uint8_t*>(w), nrows, K,
                                                          row_bytes_of(wt, K), out, out_bf16);
  return set_cuda_error(cudaGetLastError(), "dequant_kernel");
}

// ------------------------------------------------------------------ failure-detection self-test
// One bounded wait on an mbarrier that nothing arrives at: it gives up at the context's wait limit,
// sets ST_TIMEOUT_FULL in the status word and the kernel returns (the context stays usable).
__global__ void wait_selftest_kernel(int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  mbar_wait_bounded(&bar, 0, status, ST_TIMEOUT_FULL);
}

int wait_selftest_launch(int* status, cudaStream_t s) {
  wait_selftest_kernel<<<1, 32, 0, s>>>(status);
  return set_cuda_error(cudaGetLastError(), "wait_selftest_kernel");
}

// ------------------------------------------------------------------ strict GEMM
// y[m, n] = bf16( sequential fp32 sum_k fmul(x[m,k], w[n,k]) ), the reference's exact contract
// (tools/q4k_ref.py:86-92). 32 rows per block, one thread per (row, token); weights of a 256-wide
// K chunk are dequantised exactly into shared memory, then every thread runs its own chain.
constexpr int STRICT_ROWS = 32;
__global__ void strict_gemm_kernel(const StrictParams p) {
  __shared__ float ws[STRICT_ROWS][257];
  const int g = blockIdx.z;
  if (p.n_groups_dev && g >= *p.n_groups_dev) return;
  const int e = p.group_ids ? p.group_ids[g] : g;
  const uint8_t* w = p.w + static_cast<int64_t>(e) * p.w_group_stride;
  const int64_t row_bytes = row_bytes_of(p.wt, p.K);
  const int r = threadIdx.x & 31;
  const int mloc = threadIdx.x >> 5;
  const int m = blockIdx.y * 8 + mloc;
  const int n = blockIdx.x * STRICT_ROWS + r;
  const int nthr = blockDim.x;
  const int esz = (p.xt == XT_F32) ? 4 : 2;
  const uint8_t* x = static_cast<const uint8_t*>(p.x) + static_cast<int64_t>(g) * p.x_group_stride * esz;
  float acc = 0.f;
  for (int k0 = 0; k0 < p.K; k0 += 256) {
    const int kl = min(256, p.K - k0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < STRICT_ROWS * kl; idx += nthr) {
      const int rr = idx / kl, kk = idx - rr * kl;
      const int nn = blockIdx.x * STRICT_ROWS + rr;
      ws[rr][kk] = (nn < p.N) ? deq_one(p.wt, w + static_cast<int64_t>(nn) * row_bytes, k0 + kk) : 0.f;
    }
    __syncthreads();
    if (m < p.M) {
      const int64_t xo = static_cast<int64_t>(m) * p.K + k0;
      for (int kk = 0; kk < kl; ++kk) {
        const float xv = (p.xt == XT_F32) ? __ldg(reinterpret_cast<const float*>(x) + xo + kk)
                                          : bf16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(x) + xo + kk));
        acc = __fadd_rn(acc, __fmul_rn(xv, ws[r][kk]));
      }
    }
  }
  if (m < p.M && n < p.N) {
    const int64_t o = static_cast<int64_t>(g) * p.y_group_stride + static_cast<int64_t>(m) * p.N + n;
    if (p.y) p.y[o] = bf16_rne_bits(acc);
    if (p.y_f32) p.y_f32[o] = acc;
  }
}

int strict_gemm_grouped_launch(const StrictParams& p, int n_groups, cudaStream_t s) {
  if (p.N <= 0 || p.M <= 0 || p.K <= 0 || n_groups <= 0) return OK;
  const int mb = p.M < 8 ? p.M : 8;
  dim3 grid((p.N + STRICT_ROWS - 1) / STRICT_ROWS, (p.M + 7) / 8, n_groups);
  if (grid.y > 65535 || grid.z > 65535) return set_error(EINVAL_, "strict gemm: too many tokens or groups");
  StrictParams q = p;
  return launch_kernel(reinterpret_cast<const void*>(strict_gemm_kernel), grid, dim3(32 * mb), 0, s, false, &q);
}

int strict_gemm_launch(int wt, const void* w, int N, int K, const void* x, int xt, int M, uint16_t* y, float* y_f32,
                       cudaStream_t s) {
  StrictParams p = {};
  p.wt = wt;
  p.w = static_cast<const uint8_t*>(w);
  p.N = N;
  p.K = K;
  p.M = M;
  p.x = x;
  p.xt = xt;
  p.y = y;
  p.y_f32 = y_f32;
  return strict_gemm_grouped_launch(p, 1, s);
}

// h = bf16( fp32(silu_bf(g)) * fp32(u) ): the SwiGLU product of tools/glm_model_q4k_ref.py:706
__global__ void swiglu_elem_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u, int64_t n,
                                   uint16_t* __restrict__ h) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    h[i] = bf16_rne_bits(__fmul_rn(glm_silu_bf(bf16_bits_to_f32(g[i])), bf16_bits_to_f32(u[i])));
}

int swiglu_elem_launch(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* h, cudaStream_t s) {
  if (n <= 0) return OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 8192) blocks = 8192;
  swiglu_elem_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(g, u, n, h);
  return set_cuda_error(cudaGetLastError(), "swiglu_elem_kernel");
}

// ------------------------------------------------------------------ strict router
// Stage 1 (one warp per 32 experts per token): logit = bf16(sequential fp32 chain) exactly as
// moe_router's matmul_q4k (tools/glm_model_q4k_ref.py:667-668), gate = bf16 glm sigmoid.
// Stage 2 (the last warp to finish a token): top-K by (order key of gate [+ bias], lower index
// wins ties), balanced add tree, Quake rsqrt^2 renormalisation x SCALE (glm_model_q4k_ref.py:669-681).
// Stage 3 (the last token to finish): the sorted union of selected experts over all tokens and
// each (token, slot)'s index into it, for the grouped expert GEMVs and the combine.
// One warp per token. Lane l holds experts [l*per, (l+1)*per) (per = ceil(E/32)) as (order key of
// the score, 0x7FFFFFFF - e) and its own best; each of the T rounds takes the warp maximum with two
// redux.sync (key, then the lowest index among equal keys), the winner's lane replaces its best.
// The T winning gates stay in registers; the balanced tree is the zero-padded 16-leaf tree, which
// equals the reference's 2^ceil(log2 T)-leaf tree (the padding contributes exact +0 additions).
template <int MAXPL>  // experts per lane: 8 (E <= 256) or 32 (E <= 1024)
__device__ void router_topk_token_pl(const RouterParams& p, int m, const float* bias_pre, int* sel_s) {
  const int lane = threadIdx.x & 31;
  const int E = p.E, T = p.topk;
  const int per = (E + 31) / 32;
  const int eb = lane * per;
  uint32_t kh[MAXPL];
  uint16_t gb[MAXPL];
  const uint16_t* g = p.gate + static_cast<int64_t>(m) * E;
#pragma unroll
  for (int j = 0; j < MAXPL; ++j) {
    kh[j] = 0u;
    gb[j] = 0;
    const int e = eb + j;
    if (j < per && e < E) {
      gb[j] = __ldcg(g + e);
      const float gate = bf16_bits_to_f32(gb[j]);
      const float score = p.bias ? __fadd_rn(gate, bias_pre ? bias_pre[j] : __ldg(p.bias + e)) : gate;
      kh[j] = f32_order_key(score);
    }
  }
  // the lane's best: highest key, lowest index among equal keys (strict > keeps the first)
  uint32_t bk;
  int bj;
  bk = 0u;
  bj = -1;
#pragma unroll
  for (int j = 0; j < MAXPL; ++j)
    if (j < per && eb + j < E && (bj < 0 || kh[j] > bk)) {
      bk = kh[j];
      bj = j;
    }
  float win[16];
  int my_sel = 0;       // lane s keeps the s-th selection
  float my_win = 0.f;
  uint32_t taken = 0u;  // this lane's selected entries (bit j)
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    win[s] = 0.f;
    if (s < T) {
      const bool has = bj >= 0;
      const uint32_t top = __reduce_max_sync(0xffffffffu, has ? bk : 0u);
      const uint32_t lo = (has && bk == top) ? static_cast<uint32_t>(0x7FFFFFFF - (eb + bj)) : 0u;
      const uint32_t best_lo = __reduce_max_sync(0xffffffffu, lo);
      const int e = 0x7FFFFFFF - static_cast<int>(best_lo);
      const int wl = e / per;
      uint16_t gsel = 0;
#pragma unroll
      for (int j = 0; j < MAXPL; ++j)
        if (j == bj) gsel = gb[j];
      win[s] = bf16_bits_to_f32(__shfl_sync(0xffffffffu, gsel, wl));
      if (lane == s) {
        my_sel = e;
        my_win = win[s];
      }
      if (lane == wl) {
        taken |= 1u << bj;
        bj = -1;
        bk = 0u;
#pragma unroll
        for (int j = 0; j < MAXPL; ++j)
          if (j < per && eb + j < E && !((taken >> j) & 1u) && (bj < 0 || kh[j] > bk)) {
            bk = kh[j];
            bj = j;
          }
      }
    }
  }
  // balanced fp32 add tree (glm_model_q4k_ref.py:691-699), 16 leaves, +0 padded
  float node[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) node[i] = win[i];
#pragma unroll
  for (int n = 16; n > 1; n >>= 1)
#pragma unroll
    for (int i = 0; i < n / 2; ++i) node[i] = __fadd_rn(node[2 * i], node[2 * i + 1]);
  const float rr = quake_rsqrt(node[0]);
  const float rs = __fmul_rn(__fmul_rn(rr, rr), p.scale);
  if (lane < T) {
    p.sel[m * T + lane] = my_sel;
    p.sel_w[m * T + lane] = bf16_rne_bits(__fmul_rn(my_win, rs));
    sel_s[lane] = my_sel;
  }
}

// wide routers out of line, so their 32 keys per lane do not raise the kernel's register count
__device__ __noinline__ void router_topk_token_wide(const RouterParams& p, int m, int* sel_s) {
  router_topk_token_pl<32>(p, m, nullptr, sel_s);
}

// the score bias of this lane's experts (E <= 256: lane l holds [l*per, (l+1)*per)), loaded before
// the cross-CTA hand-off so the top-k does not wait on it
__device__ __forceinline__ void router_bias_pre(const RouterParams& p, float (&b)[8]) {
  const int lane = threadIdx.x & 31, per = (p.E + 31) / 32;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane * per + j;
    b[j] = (p.bias && j < per && e < p.E) ? __ldg(p.bias + e) : 0.f;
  }
}

__device__ void router_topk_token(const RouterParams& p, int m, const float (&bias_pre)[8], int* sel_s) {
  if (p.E <= 256)
    router_topk_token_pl<8>(p, m, bias_pre, sel_s);
  else
    router_topk_token_wide(p, m, sel_s);
}

// sel_s: the selections in shared memory (one token block), or null (read p.sel from L2)
__device__ void router_union(const RouterParams& p, const int* sel_s) {
  // one warp: mark selected experts, emit them in ascending expert order
  const int lane = threadIdx.x & 31;
  const int T = p.topk, M = p.M;
  __shared__ uint32_t mask[32];
  mask[lane] = 0u;
  __syncwarp();
  for (int i = lane; i < M * T; i += 32) {
    const int e = sel_s ? sel_s[i] : __ldcg(p.sel + i);
    atomicOr(&mask[e >> 5], 1u << (e & 31));
  }
  __syncwarp();
  // prefix counts over the 32 mask words
  const uint32_t mw = mask[lane];
  int cnt = __popc(mw), pre = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, pre, o);
    if (lane >= o) pre += v;
  }
  const int base = pre - cnt;
  int idx = base;
  for (int b = 0; b < 32; ++b)
    if (mw & (1u << b)) p.union_ids[idx++] = lane * 32 + b;
  if (lane == 31) *p.n_union = pre;
  __syncwarp();
  for (int i = lane; i < M * T; i += 32) {
    const int e = sel_s ? sel_s[i] : __ldcg(p.sel + i);
    const int wd = e >> 5, bit = e & 31;
    // rank of e = (count of set bits in words < wd) + popcount(mask[wd] & ((1<<bit)-1))
    int rank = 0;
    for (int w2 = 0; w2 < wd; ++w2) rank += __popc(mask[w2]);
    rank += __popc(mask[wd] & ((1u << bit) - 1u));
    p.slot_map[i] = rank;
  }
}

// One CTA = EG experts x a block of up to 8 tokens; one chain warp per token (lane = expert), each
// lane running the sequential fp32 chain of its (token, expert) logit. For the dense fp32 router
// ([K, E]) a producer warp streams 128-row x EG-expert boxes of W by tiled TMA (and the matching
// activation slices by bulk copies) into a shared-memory ring, so the chains never wait on DRAM
// latency. GGUF-row routers dequantise each weight exactly in the chain.
constexpr int RT_CHUNK = 128;   // k rows per stage
// Packed f32x2 chain step (router_many_kernel: two experts per lane): fl(acc + fl(x * w)) per lane of
// the pair with one product and one add instruction for both. The product is fma(x, w, -0) with -0
// read from the parameters (exactly fl(x * w), signed zeros included), so the assembler cannot
// contract it with the following add.
__device__ __forceinline__ unsigned long long rt_pk(float2 a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
__device__ __forceinline__ float2 rt_upk(unsigned long long r) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
  return a;
}
__device__ __forceinline__ float2 rt_step2(float2 acc, float2 x, float2 w, float2 nz) {
  unsigned long long pr, d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(pr) : "l"(rt_pk(x)), "l"(rt_pk(w)), "l"(rt_pk(nz)));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(rt_pk(acc)), "l"(pr));
  return rt_upk(d);
}
// experts per CTA: 8 for few tokens (lanes 0..7 run the chains, four times the CTAs stream the
// router), 32 for many tokens (every lane runs a chain)
constexpr int RT_MB = 8;        // tokens per CTA
constexpr int RT_XBYTES = RT_MB * RT_CHUNK * 2;
// EG = 8 (decode) splits each token over warps: product warps write the chunk's 1024 fp32 products
// into a per-token shared ring, the chain warp runs only the dependent adds (one warp doing both is
// issue-bound at ~10 cycles per k; the add chain alone runs near the add latency)
template <int EG>
struct RtCfg {
  static constexpr bool SPLIT = (EG == 8);
  static constexpr int NST = SPLIT ? 8 : 6;  // input ring depth
  static constexpr int WBYTES = RT_CHUNK * EG * 4;
  static constexpr int NWARP = SPLIT ? 2 * RT_MB + 1 : RT_MB + 1;
  static constexpr int PSTR = 132;            // floats per expert row of a product slot (padded)
  static constexpr int PSLOT = EG * PSTR * 4;  // bytes of one product slot
  static constexpr int NPS = 4;               // product slots per token at 8 tokens (fewer tokens: more)
  static constexpr int OFF_RING = 1024;
  static constexpr int OFF_PROD = OFF_RING + NST * (WBYTES + RT_XBYTES);
  static constexpr int SMEM = OFF_PROD + (SPLIT ? RT_MB * NPS * PSLOT : 0);
};

// Debug builds only (-DRT_GT): globaltimer marks of one router call, read back by
// aipu_debug_rt_gt (not part of the product library).
#ifdef RT_GT
// globaltimer marks of one call: ~min start, max chain end, top-k end, union end
__device__ unsigned long long g_rt_gt[4];
__device__ __forceinline__ unsigned long long rt_gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
extern "C" int aipu_debug_rt_gt(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, g_rt_gt, sizeof(g_rt_gt));
  static const unsigned long long z[4] = {};
  cudaMemcpyToSymbol(g_rt_gt, z, sizeof(z));
  return 0;
}
#endif
template <int RT_EG>
__global__ void __launch_bounds__(32 * RtCfg<RT_EG>::NWARP) router_strict_kernel(const __grid_constant__ RouterParams p) {
  using RC = RtCfg<RT_EG>;
  constexpr int RT_NST = RC::NST;
  constexpr int RT_WBYTES = RC::WBYTES;
#ifdef RT_GT
  if (threadIdx.x == 0) atomicMax(&g_rt_gt[0], ~rt_gtime());
#endif
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + RT_NST;
  uint8_t* ring = smem + RC::OFF_RING;  // barriers first; TMA destinations 128-byte aligned
  __shared__ int last_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * RT_EG, e = e0 + lane;
  const bool live = (lane < RT_EG) && (e < p.E);
  const int m0 = blockIdx.y * RT_MB;
  const int mb = min(RT_MB, p.M - m0);
  // SPLIT: product slots per token (the RT_MB * NPS slots shared by the block's tokens, at most 16
  // each; chunk c of token t in slot t * nps + c % nps), and per token the chunks whose products are
  // written (pready[t]) and the chunks the chain has consumed (pdone[t])
  const int nps = min(16, (RT_MB * RC::NPS) / mb);
  uint32_t* pready = reinterpret_cast<uint32_t*>(empty + RT_NST);
  uint32_t* pdone = pready + RT_MB;
  const int K = p.K, E = p.E;
  const bool dense = (p.wt == WT_F32);
  const int nchunk = (K + RT_CHUNK - 1) / RT_CHUNK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < RT_NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], mb);
    }
    for (int s = 0; s < 2 * RT_MB; ++s) pready[s] = 0u;  // pready and pdone
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == RT_MB) {
    // producer: W[k0:k0+128, e0:e0+EG] boxes and x[m0+m, k0:k0+128] slices. The first RT_NST W boxes
    // are requested before griddepcontrol.wait (the router weights are not written by the kernel
    // this launch may overlap), the activations after it.
    if (!dense) {
      pdl_wait();
      return;
    }
    const int npre = min(RT_NST, nchunk);
    auto issue_w = [&](int c) {
      const int slot = c % RT_NST;
      const int k0 = c * RT_CHUNK, kl = min(RT_CHUNK, K - k0);
      const uint32_t xrow = static_cast<uint32_t>((kl * 2 + 15) & ~15);
      uint8_t* st = ring + slot * (RT_WBYTES + RT_XBYTES);
      // one tiled TMA request for the whole 128-row x EG-expert box (out-of-range parts read 0)
      mbar_arrive_expect_tx(&full[slot], RT_WBYTES + xrow * mb);
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
              "r"(smem_u32(st)),
          "l"(reinterpret_cast<uint64_t>(&p.wmap)), "r"(e0), "r"(k0), "r"(smem_u32(&full[slot]))
          : "memory");
    };
    auto issue_x = [&](int c) {
      const int slot = c % RT_NST;
      const int k0 = c * RT_CHUNK, kl = min(RT_CHUNK, K - k0);
      const uint32_t xrow = static_cast<uint32_t>((kl * 2 + 15) & ~15);
      uint8_t* st = ring + slot * (RT_WBYTES + RT_XBYTES);
      if (lane < mb)
        bulk_g2s(st + RT_WBYTES + lane * RT_CHUNK * 2, p.x + static_cast<int64_t>(m0 + lane) * K + k0, xrow,
                 &full[slot]);
    };
    if (lane == 0)
      for (int c = 0; c < npre; ++c) issue_w(c);
    __syncwarp();
    pdl_wait();
    for (int c = 0; c < npre; ++c) issue_x(c);
    for (int c = npre; c < nchunk; ++c) {
      const int slot = c % RT_NST;
      bool ok = true;
      if (lane == 0) ok = mbar_wait_bounded(&empty[slot], ((c / RT_NST) - 1) & 1, p.status, ST_TIMEOUT_EMPTY);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
      if (lane == 0) issue_w(c);
      __syncwarp();
      issue_x(c);
    }
    return;
  }
  pdl_wait();
  if (RC::SPLIT && warp > RT_MB) {
    // product warp of token m0 + pw: the products of each chunk into the token's product slots
    const int pw = warp - RT_MB - 1;
    if (pw >= mb || !dense) return;
    uint32_t done_seen = 0u;
    for (int c = 0; c < nchunk; ++c) {
      const int slot = c % RT_NST, ps = pw * nps + c % nps;
      const int kl = min(RT_CHUNK, K - c * RT_CHUNK);
      bool ok = mbar_wait_bounded(&full[slot], (c / RT_NST) & 1, p.status, ST_TIMEOUT_FULL);
      if (!__all_sync(0xffffffffu, ok)) return;
      // the slot's previous chunk (c - nps) must be consumed; re-read the chain's counter only when
      // the last value seen does not cover it
      if (c - nps + 1 > static_cast<int>(done_seen)) {
        const uint32_t want = static_cast<uint32_t>(c - nps + 1);
        done_seen = warp_wait_counter(&pdone[pw], want, p.status, ST_TIMEOUT_EMPTY);
        if (static_cast<int32_t>(done_seen - want) < 0) return;
      }
      const uint8_t* st = ring + slot * (RT_WBYTES + RT_XBYTES);
      const float4* ws = reinterpret_cast<const float4*>(st);
      const uint16_t* xs = reinterpret_cast<const uint16_t*>(st + RT_WBYTES + pw * RT_CHUNK * 2);
      float* pb = reinterpret_cast<float*>(smem + RC::OFF_PROD + ps * RC::PSLOT);
      // lane = k within each 32-row group: the row's 8 weights (two float4) times x[k], stored
      // expert-major (bank (4 e + k) mod 32: conflict-free). All operands are loaded before the first
      // store (the stores could alias the loads as far as the compiler knows).
      constexpr int NJ = RT_CHUNK / 32;
      float4 w0[NJ], w1[NJ];
      float xv[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int k = lane + 32 * j;
        w0[j] = ws[2 * k];
        w1[j] = ws[2 * k + 1];
        xv[j] = (k < kl) ? bf16_bits_to_f32(xs[k]) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int k = lane + 32 * j;
        pb[0 * RC::PSTR + k] = __fmul_rn(xv[j], w0[j].x);
        pb[1 * RC::PSTR + k] = __fmul_rn(xv[j], w0[j].y);
        pb[2 * RC::PSTR + k] = __fmul_rn(xv[j], w0[j].z);
        pb[3 * RC::PSTR + k] = __fmul_rn(xv[j], w0[j].w);
        pb[4 * RC::PSTR + k] = __fmul_rn(xv[j], w1[j].x);
        pb[5 * RC::PSTR + k] = __fmul_rn(xv[j], w1[j].y);
        pb[6 * RC::PSTR + k] = __fmul_rn(xv[j], w1[j].z);
        pb[7 * RC::PSTR + k] = __fmul_rn(xv[j], w1[j].w);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[slot]);
        st_release_cta_shared(&pready[pw], static_cast<uint32_t>(c + 1));
      }
    }
    return;
  }
  // consumer warp `warp` = token m0 + warp
  const int m = m0 + warp;
  if (warp < mb) {
    float acc = 0.f;
    if (RC::SPLIT && dense) {
      // the chain over the products, in k order; 32 of them loaded ahead of the adds
      bool ok = true;
      uint32_t ready_seen = 0u;
      // the token's product slots, stepped without a division on the chain's path
      const uint8_t* pbase = smem + RC::OFF_PROD + warp * nps * RC::PSLOT + (lane & (RT_EG - 1)) * RC::PSTR * 4;
      const uint8_t* pend = pbase + nps * RC::PSLOT;
      const uint8_t* pcur = pbase;
      static_assert(RT_CHUNK == 128, "four batches of 32 products per chunk");
      float4 a0[8], a1[8];
      bool pre = false;  // a0 already holds the first 32 products of chunk c
      auto add8 = [&](const float4 (&v)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc = __fadd_rn(acc, v[i].x);
          acc = __fadd_rn(acc, v[i].y);
          acc = __fadd_rn(acc, v[i].z);
          acc = __fadd_rn(acc, v[i].w);
        }
      };
      for (int c = 0; c < nchunk && ok; ++c) {
        // the counter is re-read only when the chunks seen ready so far are used up (a hand-off costs
        // a few hundred cycles on the critical chain; one read often covers several chunks)
        if (c >= static_cast<int>(ready_seen)) {
          const uint32_t want = static_cast<uint32_t>(c + 1);
          ready_seen = warp_wait_counter(&pready[warp], want, p.status, ST_TIMEOUT_FULL);
          ok = static_cast<int32_t>(ready_seen - want) >= 0;
        }
        if (!ok) break;
        const float4* pr = reinterpret_cast<const float4*>(pcur);
        pcur += RC::PSLOT;
        if (pcur == pend) pcur = pbase;
        // batches of 32 products, the next batch loaded while the current one is added
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (!pre) a0[i] = pr[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) a1[i] = pr[8 + i];
        add8(a0);
#pragma unroll
        for (int i = 0; i < 8; ++i) a0[i] = pr[16 + i];
        add8(a1);
#pragma unroll
        for (int i = 0; i < 8; ++i) a1[i] = pr[24 + i];
        add8(a0);
        // the next chunk's first batch, when its products are already known to be written
        pre = (c + 1 < nchunk) && (c + 1 < static_cast<int>(ready_seen));
        if (pre) {
          const float4* pn = reinterpret_cast<const float4*>(pcur);
#pragma unroll
          for (int i = 0; i < 8; ++i) a0[i] = pn[i];
        }
        add8(a1);
        // (a short last chunk has zero products past its end; adding them leaves the sum unchanged)
        __syncwarp();
        if (lane == 0) st_release_cta_shared(&pdone[warp], static_cast<uint32_t>(c + 1));
      }
    } else if (dense) {
      bool ok = true;
      for (int c = 0; c < nchunk; ++c) {
        const int slot = c % RT_NST;
        const int kl = min(RT_CHUNK, K - c * RT_CHUNK);
        if (ok) ok = mbar_wait_bounded(&full[slot], (c / RT_NST) & 1, p.status, ST_TIMEOUT_FULL);
        if (ok) {
          const uint8_t* st = ring + slot * (RT_WBYTES + RT_XBYTES);
          const float* ws = reinterpret_cast<const float*>(st);
          const uint16_t* xs = reinterpret_cast<const uint16_t*>(st + RT_WBYTES + warp * RT_CHUNK * 2);
          if (kl == RT_CHUNK) {
            // batches of 32 k, the operands of the next batch loaded while the dependent adds of
            // this batch run in k order (the chain runs near the add latency)
            const int pe = lane & (RT_EG - 1);
            float wv[32];
            uint4 xv[4];
#pragma unroll
            for (int i = 0; i < 32; ++i) wv[i] = ws[i * RT_EG + pe];
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = reinterpret_cast<const uint4*>(xs)[i];
#pragma unroll
            for (int k0b = 0; k0b < RT_CHUNK; k0b += 32) {
              float pr[32];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  pr[8 * i + 2 * h] = __fmul_rn(__uint_as_float(xw[h] << 16), wv[8 * i + 2 * h]);
                  pr[8 * i + 2 * h + 1] = __fmul_rn(__uint_as_float(xw[h] & 0xFFFF0000u), wv[8 * i + 2 * h + 1]);
                }
              }
              if (k0b + 32 < RT_CHUNK) {
#pragma unroll
                for (int i = 0; i < 32; ++i) wv[i] = ws[(k0b + 32 + i) * RT_EG + pe];
#pragma unroll
                for (int i = 0; i < 4; ++i) xv[i] = reinterpret_cast<const uint4*>(xs + k0b + 32)[i];
              }
#pragma unroll
              for (int i = 0; i < 32; ++i) acc = __fadd_rn(acc, pr[i]);
            }
          } else {
            for (int k = 0; k < kl; ++k)
              acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(xs[k]), ws[k * RT_EG + (lane & (RT_EG - 1))]));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    } else if (live) {
      const uint8_t* row = p.w + static_cast<int64_t>(e) * row_bytes_of(p.wt, K);
      const int64_t xo = static_cast<int64_t>(m) * K;
      for (int k = 0; k < K; ++k)
        acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(__ldg(p.x + xo + k)), deq_one(p.wt, row, k)));
    }
    if (live) {
      const float logit = bf16_round_f(acc);
      p.gate[static_cast<int64_t>(m) * E + e] = bf16_rne_bits(glm_sigmoid_bf(logit));
      if (p.logits) p.logits[static_cast<int64_t>(m) * E + e] = bf16_rne_bits(logit);
    }
  }
#ifdef RT_GT
  if (threadIdx.x == 0) atomicMax(&g_rt_gt[1], rt_gtime());
#endif
  // the last CTA of this token block selects top-K for its tokens; the last block builds the union
  __shared__ int sel_s[RT_MB * 16];
  float bias_pre[8];
  router_bias_pre(p, bias_pre);
  named_bar_sync(1, 32 * RT_MB);
  if (threadIdx.x == 0)
    last_flag = (atom_add_acq_rel_gpu(&p.counters[blockIdx.y], 1) == static_cast<int>(gridDim.x) - 1);
  named_bar_sync(1, 32 * RT_MB);
  if (!last_flag) return;
  if (warp < mb) router_topk_token(p, m, bias_pre, sel_s + warp * p.topk);
#ifdef RT_GT
  if (threadIdx.x == 0) atomicMax(&g_rt_gt[2], rt_gtime());
#endif
  named_bar_sync(1, 32 * RT_MB);
  if (gridDim.y > 1) {
    if (threadIdx.x == 0) {
      p.counters[blockIdx.y] = 0;
      last_flag = (atom_add_acq_rel_gpu(&p.counters[gridDim.y], 1) == static_cast<int>(gridDim.y) - 1);
    }
    named_bar_sync(1, 32 * RT_MB);
    if (!last_flag) return;
  }
  if (warp == 0) {
    if (lane == 0) p.counters[gridDim.y > 1 ? gridDim.y : blockIdx.y] = 0;
    if (p.union_ids) router_union(p, gridDim.y > 1 ? nullptr : sel_s);
#ifdef RT_GT
    if (lane == 0) atomicMax(&g_rt_gt[3], rt_gtime());
#endif
  }
}

// ------------------------------------------------------------------ router, many tokens (dense fp32)
// One CTA = 64 experts x 56 tokens. A producer warp streams 128 k x 64 expert boxes of W (tiled TMA)
// and the tokens' matching activation slices (bulk copies) into a 3-stage ring; each of the 7
// compute warps runs the chains of 8 tokens, every lane two experts as packed f32x2 chains
// (fl(acc + fl(x w)) per lane of the pair, k in order). A weight pair loaded once serves 8 tokens from
// registers, so the loop costs about 1.2 instructions per (token, expert-pair, k) step.
// (7 warps x 8 tokens: 2048 tokens x 256 experts make 37 x 4 = 148 CTAs, one per SM)
constexpr int RM_WARPS = 7, RM_TOK = 8 * RM_WARPS, RM_EG = 64, RM_NST = 3;
constexpr int RM_WB = RT_CHUNK * RM_EG * 4;   // 32 KB of W per stage
constexpr int RM_XB = RM_TOK * RT_CHUNK * 2;  // 16 KB of activations per stage
constexpr int RM_OFF_RING = 1024;
constexpr int RM_SMEM = RM_OFF_RING + RM_NST * (RM_WB + RM_XB);

template <int TPW>
__global__ void __launch_bounds__(32 * (RM_WARPS + 1), 1) router_many_kernel(const __grid_constant__ RouterParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + RM_NST;
  uint8_t* ring = smem + RM_OFF_RING;
  __shared__ int last_flag;
  __shared__ int sel_s[RM_TOK * 16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * RM_EG, e = e0 + 2 * lane;
  constexpr int tpw = TPW;
  const int tok_cta = RM_WARPS * tpw;
  const int m0 = blockIdx.y * tok_cta;
  const int mb = min(tok_cta, p.M - m0);
  const int K = p.K, E = p.E;
  const int nchunk = (K + RT_CHUNK - 1) / RT_CHUNK;
  if (threadIdx.x == 0) {
    for (int st = 0; st < RM_NST; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], RM_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == RM_WARPS) {
    // producer: the first stages' W boxes before griddepcontrol.wait (static weights), activations after
    auto issue_w = [&](int c) {
      const int st = c % RM_NST;
      const int k0 = c * RT_CHUNK, kl = min(RT_CHUNK, K - k0);
      const uint32_t xrow = static_cast<uint32_t>((kl * 2 + 15) & ~15);
      uint8_t* dst = ring + st * (RM_WB + RM_XB);
      mbar_arrive_expect_tx(&full[st], RM_WB + xrow * mb);
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
              "r"(smem_u32(dst)),
          "l"(reinterpret_cast<uint64_t>(&p.wmap)), "r"(e0), "r"(k0), "r"(smem_u32(&full[st]))
          : "memory");
    };
    auto issue_x = [&](int c) {
      const int st = c % RM_NST;
      const int k0 = c * RT_CHUNK, kl = min(RT_CHUNK, K - k0);
      const uint32_t xrow = static_cast<uint32_t>((kl * 2 + 15) & ~15);
      uint8_t* dst = ring + st * (RM_WB + RM_XB) + RM_WB;
      for (int t = lane; t < mb; t += 32)
        bulk_g2s(dst + t * RT_CHUNK * 2, p.x + static_cast<int64_t>(m0 + t) * K + k0, xrow, &full[st]);
    };
    const int npre = min(RM_NST, nchunk);
    if (lane == 0)
      for (int c = 0; c < npre; ++c) issue_w(c);
    __syncwarp();
    pdl_wait();
    for (int c = 0; c < npre; ++c) issue_x(c);
    for (int c = npre; c < nchunk; ++c) {
      const int st = c % RM_NST;
      bool ok = true;
      if (lane == 0) ok = mbar_wait_bounded(&empty[st], ((c / RM_NST) - 1) & 1, p.status, ST_TIMEOUT_EMPTY);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
      if (lane == 0) issue_w(c);
      __syncwarp();
      issue_x(c);
    }
    return;
  }
  pdl_wait();
  // compute warp: tokens t0 .. t0 + tpw - 1 of the block (rows past mb compute on the ring's stale
  // bytes and are never stored)
  const int t0 = warp * tpw;
  const float2 nz = make_float2(p.neg_zero, p.neg_zero);
  float2 acc[TPW];
#pragma unroll
  for (int j = 0; j < TPW; ++j) acc[j] = make_float2(0.f, 0.f);
  bool ok = true;
  for (int c = 0; c < nchunk && ok; ++c) {
    const int st = c % RM_NST;
    const int kl = min(RT_CHUNK, K - c * RT_CHUNK);
    ok = mbar_wait_bounded(&full[st], (c / RM_NST) & 1, p.status, ST_TIMEOUT_FULL);
    if (!ok) break;
    const uint8_t* base = ring + st * (RM_WB + RM_XB);
    const float2* ws = reinterpret_cast<const float2*>(base) + lane;
    const uint8_t* xs = base + RM_WB + t0 * RT_CHUNK * 2;
    // k in groups of 4, then the rest of a short last chunk one by one (k < kl only)
    const int kq = kl & ~3;
    for (int k = 0; k < kq; k += 4) {
      const float2 w0 = ws[(k + 0) * 32], w1 = ws[(k + 1) * 32], w2 = ws[(k + 2) * 32], w3 = ws[(k + 3) * 32];
#pragma unroll
      for (int j = 0; j < TPW; ++j) {
        const uint2 xv = *reinterpret_cast<const uint2*>(xs + j * RT_CHUNK * 2 + 2 * k);
        const float x0 = __uint_as_float(xv.x << 16), x1 = __uint_as_float(xv.x & 0xFFFF0000u);
        const float x2 = __uint_as_float(xv.y << 16), x3 = __uint_as_float(xv.y & 0xFFFF0000u);
        acc[j] = rt_step2(acc[j], make_float2(x0, x0), w0, nz);
        acc[j] = rt_step2(acc[j], make_float2(x1, x1), w1, nz);
        acc[j] = rt_step2(acc[j], make_float2(x2, x2), w2, nz);
        acc[j] = rt_step2(acc[j], make_float2(x3, x3), w3, nz);
      }
    }
    for (int k = kq; k < kl; ++k) {
      const float2 wk = ws[k * 32];
#pragma unroll
      for (int j = 0; j < TPW; ++j) {
        const float xk = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(xs + j * RT_CHUNK * 2 + 2 * k));
        acc[j] = rt_step2(acc[j], make_float2(xk, xk), wk, nz);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (ok) {
#pragma unroll
    for (int j = 0; j < TPW; ++j) {
      const int t = t0 + j;
      if (t < mb) {
        const int64_t m = m0 + t;
        const float l0 = bf16_round_f(acc[j].x), l1 = bf16_round_f(acc[j].y);
        if (e < E) {
          p.gate[m * E + e] = bf16_rne_bits(glm_sigmoid_bf(l0));
          if (p.logits) p.logits[m * E + e] = bf16_rne_bits(l0);
        }
        if (e + 1 < E) {
          p.gate[m * E + e + 1] = bf16_rne_bits(glm_sigmoid_bf(l1));
          if (p.logits) p.logits[m * E + e + 1] = bf16_rne_bits(l1);
        }
      }
    }
  }
  // the last CTA of this token block selects top-K for its tokens; the last block builds the union
  float bias_pre[8];
  router_bias_pre(p, bias_pre);
  named_bar_sync(1, 32 * RM_WARPS);
  if (threadIdx.x == 0)
    last_flag = (atom_add_acq_rel_gpu(&p.counters[blockIdx.y], 1) == static_cast<int>(gridDim.x) - 1);
  named_bar_sync(1, 32 * RM_WARPS);
  if (!last_flag) return;
  for (int j = 0; j < tpw; ++j)
    if (t0 + j < mb) router_topk_token(p, m0 + t0 + j, bias_pre, sel_s + (t0 + j) * p.topk);
  named_bar_sync(1, 32 * RM_WARPS);
  if (gridDim.y > 1) {
    if (threadIdx.x == 0) {
      p.counters[blockIdx.y] = 0;
      last_flag = (atom_add_acq_rel_gpu(&p.counters[gridDim.y], 1) == static_cast<int>(gridDim.y) - 1);
    }
    named_bar_sync(1, 32 * RM_WARPS);
    if (!last_flag) return;
  }
  if (warp == 0) {
    if (lane == 0) p.counters[gridDim.y > 1 ? gridDim.y : blockIdx.y] = 0;
    if (p.union_ids) router_union(p, gridDim.y > 1 ? nullptr : sel_s);
  }
}

// tokens per compute warp: the fewest CTAs that still give every SM one (8 at 2048 tokens x 256 experts)
static int router_many_tpw(const RouterParams& p) {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms[dev] = 148;
  const int64_t eg = (p.E + RM_EG - 1) / RM_EG;
  const int64_t want = (static_cast<int64_t>(p.M) * eg + static_cast<int64_t>(RM_WARPS) * sms[dev] - 1) /
                       (static_cast<int64_t>(RM_WARPS) * sms[dev]);
  const int64_t w = std::max<int64_t>(1, std::min<int64_t>(8, want));
  return w <= 1 ? 1 : w <= 2 ? 2 : w <= 4 ? 4 : 8;  // the kernel's instantiations
}

template <int TPW>
static int router_launch_many_t(RouterParams q, cudaStream_t s, bool pdl) {
  static bool attr[64] = {false};
  const int arc = set_smem_attr_once(reinterpret_cast<const void*>(router_many_kernel<TPW>), RM_SMEM, attr,
                                     "cudaFuncSetAttribute(router_many)");
  if (arc) return arc;
  return launch_kernel(reinterpret_cast<const void*>(router_many_kernel<TPW>),
                       dim3((q.E + RM_EG - 1) / RM_EG, (q.M + RM_WARPS * TPW - 1) / (RM_WARPS * TPW)),
                       dim3(32 * (RM_WARPS + 1)), RM_SMEM, s, pdl, &q);
}

static int router_launch_many(const RouterParams& p, cudaStream_t s, bool pdl) {
  RouterParams q = p;
  q.neg_zero = -0.0f;
  q.tpw = router_many_tpw(p);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.E), static_cast<cuuint64_t>(p.K)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.E) * 4};
  const cuuint32_t box[2] = {RM_EG, RT_CHUNK};
  const int rc = encode_tiled(&q.wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.w, dims, strides, box);
  if (rc) return rc;
  switch (q.tpw) {
    case 1: return router_launch_many_t<1>(q, s, pdl);
    case 2: return router_launch_many_t<2>(q, s, pdl);
    case 4: return router_launch_many_t<4>(q, s, pdl);
    default: return router_launch_many_t<8>(q, s, pdl);
  }
}

template <int EG>
static int router_launch_eg(const RouterParams& p, cudaStream_t s, bool pdl) {
  using RC = RtCfg<EG>;
  static_assert(2 * RC::NST * 8 + 2 * RT_MB * 4 <= RC::OFF_RING, "router barriers fit before the ring");
  static_assert(RC::SMEM <= 227 * 1024, "router shared memory");
  const int smem = RC::SMEM;
  static bool attr[64] = {false};
  {
    const int arc = set_smem_attr_once(reinterpret_cast<const void*>(router_strict_kernel<EG>), smem, attr, "cudaFuncSetAttribute(router)");
    if (arc) return arc;
  }
  RouterParams q = p;
  q.neg_zero = -0.0f;
  if (p.wt == WT_F32) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.E), static_cast<cuuint64_t>(p.K)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.E) * 4};
    const cuuint32_t box[2] = {EG, RT_CHUNK};
    const int rc = encode_tiled(&q.wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.w, dims, strides, box);
    if (rc) return rc;
  }
  return launch_kernel(reinterpret_cast<const void*>(router_strict_kernel<EG>),
                       dim3((p.E + EG - 1) / EG, (p.M + RT_MB - 1) / RT_MB), dim3(32 * RC::NWARP), smem, s, pdl, &q);
}

int router_launch(const RouterParams& p, cudaStream_t s, bool pdl) {
  if (p.E <= 0 || p.E > 1024 || p.topk <= 0 || p.topk > 16 || p.topk > p.E || p.M <= 0)
    return set_error(EINVAL_, "router: need 1 <= topk <= min(16, E), E <= 1024");
  if (p.wt == WT_F32 && (p.E % 4 != 0 || (reinterpret_cast<uintptr_t>(p.w) & 15u) ||
                         (reinterpret_cast<uintptr_t>(p.x) & 15u) || (p.K % 8)))
    return set_error(EINVAL_, "router: fp32 router needs E % 4 == 0, K % 8 == 0 and 16-byte aligned w, x");
  // few token blocks: spread the router over more SMs; many: every lane of a CTA runs a packed chain
  // over two experts (dense fp32 router) or one (GGUF-row router)
  if (p.M <= 4 * RT_MB) return router_launch_eg<8>(p, s, pdl);
  return (p.wt == WT_F32) ? router_launch_many(p, s, pdl) : router_launch_eg<32>(p, s, pdl);
}

int router_grid_ctas(const RouterParams& p) {
  if (p.M > 4 * RT_MB && p.wt == WT_F32) {
    const int tok = RM_WARPS * router_many_tpw(p);
    return ((p.E + RM_EG - 1) / RM_EG) * ((p.M + tok - 1) / tok);
  }
  const int eg = (p.M <= 4 * RT_MB) ? 8 : 32;
  return ((p.E + eg - 1) / eg) * ((p.M + RT_MB - 1) / RT_MB);
}

int router_smem_bytes(const RouterParams& p) {
  if (p.M <= 4 * RT_MB) return RtCfg<8>::SMEM;
  return (p.wt == WT_F32) ? RM_SMEM : RtCfg<32>::SMEM;
}

// ------------------------------------------------------------------ combine
// out[m, d] = bf16( (sum over slots in slot order of fmul(w_slot, y_slot[d])) + y_shared[d] )
// (tools/glm_model_q4k_ref.py:799-809)
__global__ void combine_kernel(const CombineParams p) {
  pdl_wait();
  // 8 consecutive outputs per thread (H % 8 == 0): 16-byte loads of every expert row
  const int hv = p.H >> 3;
  const int64_t total = static_cast<int64_t>(p.M) * hv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / hv);
    const int d8 = static_cast<int>(i - static_cast<int64_t>(m) * hv);
    float facc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) facc[j] = 0.f;
    for (int s = 0; s < p.topk; ++s) {
      const int u = p.slot_map[m * p.topk + s];
      const float wv = bf16_bits_to_f32(p.sel_w[m * p.topk + s]);
      const int64_t row = p.rows_are_positions ? static_cast<int64_t>(u) : static_cast<int64_t>(u) * p.M + m;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.y_union + row * p.H) + d8);
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        facc[2 * j] = __fadd_rn(facc[2 * j], __fmul_rn(wv, bf16_bits_to_f32(w4[j] & 0xFFFFu)));
        facc[2 * j + 1] = __fadd_rn(facc[2 * j + 1], __fmul_rn(wv, bf16_bits_to_f32(w4[j] >> 16)));
      }
    }
    const uint16_t* sh = nullptr;
    if (p.shared_rows) sh = p.y_union + static_cast<int64_t>(p.shared_rows[m]) * p.H;
    else if (p.y_shared) sh = p.y_shared + static_cast<int64_t>(m) * p.H;
    if (sh) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(sh) + d8);
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        facc[2 * j] = __fadd_rn(facc[2 * j], bf16_bits_to_f32(w4[j] & 0xFFFFu));
        facc[2 * j + 1] = __fadd_rn(facc[2 * j + 1], bf16_bits_to_f32(w4[j] >> 16));
      }
    }
    uint4 o;
    o.x = bf16_rne_bits(facc[0]) | (static_cast<uint32_t>(bf16_rne_bits(facc[1])) << 16);
    o.y = bf16_rne_bits(facc[2]) | (static_cast<uint32_t>(bf16_rne_bits(facc[3])) << 16);
    o.z = bf16_rne_bits(facc[4]) | (static_cast<uint32_t>(bf16_rne_bits(facc[5])) << 16);
    o.w = bf16_rne_bits(facc[6]) | (static_cast<uint32_t>(bf16_rne_bits(facc[7])) << 16);
    reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(m) * p.H)[d8] = o;
  }
  pdl_launch_dependents();
}

int combine_launch(const CombineParams& p, cudaStream_t s, bool pdl) {
  if (p.H % 8) return set_error(EINVAL_, "combine: H % 8 != 0");
  const int64_t total = static_cast<int64_t>(p.M) * (p.H / 8);
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  CombineParams q = p;
  return launch_kernel(reinterpret_cast<const void*>(combine_kernel), dim3(blocks), dim3(256), 0, s, pdl, &q);
}

// ------------------------------------------------------------------ prefill permutation
// One CTA per segment (local expert e < E; segment E = shared expert over a token range). Every CTA
// counts the local selections of all experts (shared-memory histogram), takes its segment's start as
// the padded prefix of the counts, then walks the tokens in order, 256 at a time, and places each
// token that selected its expert with a block-wide prefix of flags, so the order inside a segment is
// ascending and the result deterministic. A position is never shared: a token selects an expert at
// most once. CTA 0 also writes the tile list (segments in order, nt tokens per tile) and the
// position count; slots whose expert is not local get position -1.
__global__ void __launch_bounds__(256) perm_kernel(const PermParams p) {
  pdl_wait();
  __shared__ int cnt[1025];
  __shared__ int wsum[8];
  __shared__ int s_off;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = blockIdx.x;
  const int nseg = p.E + (p.with_shared ? 1 : 0);
  for (int e = tid; e < nseg; e += 256) cnt[e] = (e == p.E) ? p.shared_n : 0;
  __syncthreads();
  for (int i = tid; i < p.T * p.topk; i += 256) {
    const int le = p.sel[i] - p.expert_lo;
    if (le >= 0 && le < p.E) atomicAdd(&cnt[le], 1);
  }
  __syncthreads();
  // start of this segment: sum over earlier segments of the count rounded up to 8
  int part = 0;
  for (int e = tid; e < seg; e += 256) part += (cnt[e] + 7) & ~7;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) wsum[warp] = part;
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int w = 0; w < 8; ++w) acc += wsum[w];
    s_off = acc;
  }
  __syncthreads();
  const int off = s_off;
  if (seg == 0 && tid == 0) {
    int acc = 0, nt = 0;
    for (int e = 0; e < nseg; ++e) {
      for (int t0 = 0; t0 < cnt[e]; t0 += p.nt) p.tiles[nt++] = make_int4(e, acc + t0, min(p.nt, cnt[e] - t0), 0);
      acc += (cnt[e] + 7) & ~7;
    }
    *p.n_tiles = nt;
    *p.n_pos = acc;
  }
  const bool shared_seg = (seg == p.E);
  const int t_lo = shared_seg ? p.shared_t0 : 0, t_hi = shared_seg ? p.shared_t0 + p.shared_n : p.T;
  int base = off;
  for (int t0 = t_lo; t0 < t_hi; t0 += 256) {
    const int t = t0 + tid;
    int slot = -1;
    if (t < t_hi) {
      if (shared_seg) {
        slot = p.topk;
      } else {
        for (int s = 0; s < p.topk; ++s)
          if (p.sel[t * p.topk + s] - p.expert_lo == seg) slot = s;
      }
    }
    const unsigned m = __ballot_sync(0xffffffffu, slot >= 0);
    __syncthreads();  // wsum reuse
    if (lane == 0) wsum[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 8; ++w) {
      before += (w < warp) ? wsum[w] : 0;
      total += wsum[w];
    }
    if (slot >= 0) {
      const int pos = base + before + __popc(m & ((1u << lane) - 1u));
      p.perm_tok[pos] = t;
      if (slot == p.topk) p.shared_pos[t - p.shared_t0] = pos;
      else p.pos_of[t * p.topk + slot] = pos;
    }
    base += total;
  }
  for (int pos = base + tid; pos < off + (((base - off) + 7) & ~7); pos += 256) p.perm_tok[pos] = -1;
  // slots of non-local experts (each written by exactly one CTA: the one of segment 0)
  if (seg == 0)
    for (int i = tid; i < p.T * p.topk; i += 256) {
      const int le = p.sel[i] - p.expert_lo;
      if (le < 0 || le >= p.E) p.pos_of[i] = -1;
    }
  pdl_launch_dependents();
}

int perm_launch(const PermParams& p, cudaStream_t s) {
  if (p.E > 1024 || p.E <= 0 || p.nt <= 0) return set_error(EINVAL_, "perm: E must be 1..1024");
  PermParams q = p;
  return launch_kernel(reinterpret_cast<const void*>(perm_kernel), dim3(p.E + (p.with_shared ? 1 : 0)), dim3(256), 0,
                       s, true, &q);
}

// ------------------------------------------------------------------ union of local experts (decode)
// One CTA: flag the local experts any slot selected, prefix-count them into the sorted union, then
// map every slot to its union index (-1: expert not local).
__global__ void __launch_bounds__(1024) union_kernel(const int32_t* __restrict__ sel, int M, int topk, int expert_lo,
                                                     int E, int32_t* __restrict__ union_ids,
                                                     int32_t* __restrict__ n_union, int32_t* __restrict__ slot_map,
                                                     const EpSync w) {
  __shared__ int flag[1024];
  __shared__ int idx[1024];
  const int tid = threadIdx.x;
  // peer exchange: the selections arrive from the other ranks (a wait that gave up leaves the union
  // empty, and the status word reports it)
  if (w.flags && !ep_sync_wait(w)) M = 0;
  for (int e = tid; e < E; e += 1024) flag[e] = 0;
  __syncthreads();
  for (int i = tid; i < M * topk; i += 1024) {
    const int le = sel[i] - expert_lo;
    if (le >= 0 && le < E) flag[le] = 1;
  }
  __syncthreads();
  if (tid == 0) {
    int u = 0;
    for (int e = 0; e < E; ++e) {
      idx[e] = flag[e] ? u : -1;
      if (flag[e]) union_ids[u++] = e;
    }
    *n_union = u;
  }
  __syncthreads();
  for (int i = tid; i < M * topk; i += 1024) {
    const int le = sel[i] - expert_lo;
    slot_map[i] = (le >= 0 && le < E) ? idx[le] : -1;
  }
}

int union_launch(const int32_t* sel, int M, int topk, int expert_lo, int E, int32_t* union_ids, int32_t* n_union,
                 int32_t* slot_map, cudaStream_t s, const EpSync* w) {
  if (E <= 0 || E > 1024) return set_error(EINVAL_, "union: E must be 1..1024");
  union_kernel<<<1, 1024, 0, s>>>(sel, M, topk, expert_lo, E, union_ids, n_union, slot_map, w ? *w : EpSync());
  return set_cuda_error(cudaGetLastError(), "union_kernel");
}

// ------------------------------------------------------------------ slot gather / EP combine
__global__ void gather_slots_kernel(const int32_t* __restrict__ index, int M, int topk, int64_t H,
                                    const uint16_t* __restrict__ rows, int64_t row_mul, int64_t row_add,
                                    uint16_t* __restrict__ y_slots) {
  const int64_t hv = H / 8;
  const int64_t total = static_cast<int64_t>(M) * topk * hv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t ms = i / hv, v = i - ms * hv;
    const int m = static_cast<int>(ms / topk);
    const int ix = index[ms];
    if (ix < 0) continue;
    const int64_t r = static_cast<int64_t>(ix) * row_mul + static_cast<int64_t>(m) * row_add;
    reinterpret_cast<uint4*>(y_slots + ms * H)[v] = __ldg(reinterpret_cast<const uint4*>(rows + r * H) + v);
  }
}

int gather_slots_launch(const int32_t* index, int M, int topk, int64_t H, const uint16_t* rows, int64_t row_mul,
                        int64_t row_add, uint16_t* y_slots, cudaStream_t s) {
  if (H % 8) return set_error(EINVAL_, "gather_slots: H % 8 != 0");
  const int64_t total = static_cast<int64_t>(M) * topk * (H / 8);
  int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  if (blocks <= 0) return OK;
  gather_slots_kernel<<<blocks, 256, 0, s>>>(index, M, topk, H, rows, row_mul, row_add, y_slots);
  return set_cuda_error(cudaGetLastError(), "gather_slots_kernel");
}

__global__ void combine_pieces_kernel(const int32_t* __restrict__ sel, const uint16_t* __restrict__ sel_w, int M,
                                      int topk, int64_t H, int epp, const uint16_t* __restrict__ pieces,
                                      const uint16_t* __restrict__ shared, uint16_t* __restrict__ out,
                                      const EpSync w) {
  const int64_t hv = H / 8;
  // peer exchange: the pieces arrive from the other ranks (a wait that gave up skips the combine; the
  // status word reports it)
  const int64_t total = (w.flags && !ep_sync_wait(w)) ? 0 : static_cast<int64_t>(M) * hv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / hv);
    const int64_t v = i - static_cast<int64_t>(m) * hv;
    float facc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) facc[j] = 0.f;
    for (int s = 0; s < topk; ++s) {
      const int e = sel[m * topk + s];
      const float wv = bf16_bits_to_f32(sel_w[m * topk + s]);
      const int64_t row = (static_cast<int64_t>(e / epp) * M + m) * topk + s;
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(pieces + row * H) + v);
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        facc[2 * j] = __fadd_rn(facc[2 * j], __fmul_rn(wv, bf16_bits_to_f32(w4[j] & 0xFFFFu)));
        facc[2 * j + 1] = __fadd_rn(facc[2 * j + 1], __fmul_rn(wv, bf16_bits_to_f32(w4[j] >> 16)));
      }
    }
    if (shared) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(shared + static_cast<int64_t>(m) * H) + v);
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        facc[2 * j] = __fadd_rn(facc[2 * j], bf16_bits_to_f32(w4[j] & 0xFFFFu));
        facc[2 * j + 1] = __fadd_rn(facc[2 * j + 1], bf16_bits_to_f32(w4[j] >> 16));
      }
    }
    uint4 o;
    o.x = bf16_rne_bits(facc[0]) | (static_cast<uint32_t>(bf16_rne_bits(facc[1])) << 16);
    o.y = bf16_rne_bits(facc[2]) | (static_cast<uint32_t>(bf16_rne_bits(facc[3])) << 16);
    o.z = bf16_rne_bits(facc[4]) | (static_cast<uint32_t>(bf16_rne_bits(facc[5])) << 16);
    o.w = bf16_rne_bits(facc[6]) | (static_cast<uint32_t>(bf16_rne_bits(facc[7])) << 16);
    reinterpret_cast<uint4*>(out + static_cast<int64_t>(m) * H)[v] = o;
  }
  ep_sync_bump(w);
}

int combine_pieces_launch(const int32_t* sel, const uint16_t* sel_w, int M, int topk, int64_t H, int epp,
                          const uint16_t* pieces, const uint16_t* shared, uint16_t* out, cudaStream_t s, EpSync w) {
  if (H % 8 || epp <= 0) return set_error(EINVAL_, "combine_pieces: bad arguments");
  const int64_t total = static_cast<int64_t>(M) * (H / 8);
  int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  if (blocks <= 0) {
    if (!w.bump_arrive) return OK;
    blocks = 1;  // the layer call still ends here
  }
  combine_pieces_kernel<<<blocks, 256, 0, s>>>(sel, sel_w, M, topk, H, epp, pieces, shared, out, w);
  return set_cuda_error(cudaGetLastError(), "combine_pieces_kernel");
}

// ------------------------------------------------------------------ activations
// out[i] = bf16 glm sigmoid (kind 0) or glm silu (kind 1) of bf16 x[i]
__global__ void act_kernel(int kind, const uint16_t* __restrict__ x, int64_t n, uint16_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = bf16_bits_to_f32(x[i]);
    out[i] = bf16_rne_bits(kind == 0 ? glm_sigmoid_bf(v) : glm_silu_bf(v));
  }
}

int act_launch(int kind, const void* x, int64_t n, void* out, cudaStream_t s) {
  if (n <= 0) return OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 8192) blocks = 8192;
  act_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(kind, static_cast<const uint16_t*>(x), n,
                                                      static_cast<uint16_t*>(out));
  return set_cuda_error(cudaGetLastError(), "act_kernel");
}

}  // namespace aipu
