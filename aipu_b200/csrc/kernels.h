// Launch prototypes and parameter blocks of the exact kernels and the decode GEMV.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace aipu {

struct GemvParams;

struct RouterParams {
  int wt;                  // WT_F32: dense router [K, E]; WT_Q4K/Q6K/Q80/F16: GGUF rows [E, K]
  const uint8_t* w;
  const float* bias;       // [E] fp32, selection only (nullable)
  const uint16_t* x;       // bf16 [M, K]
  int M, K, E, topk;
  float scale;             // renormalisation scale (the reference uses 2.5)
  float neg_zero;          // -0.0f, set by the launcher (the packed product's addend)
  int tpw;                 // router_many_kernel: tokens per compute warp (1..8), set by the launcher
  uint16_t* gate;          // bf16 [M, E] sigmoid gates (scratch and output)
  uint16_t* logits;        // bf16 [M, E] (nullable)
  int32_t* sel;            // [M, topk] selected experts, slot order
  uint16_t* sel_w;         // bf16 [M, topk] routing weights
  int32_t* union_ids;      // [<= M*topk] sorted union of selected experts (nullable)
  int32_t* n_union;        // [1]
  int32_t* slot_map;       // [M, topk] index of sel[m, s] in union_ids
  int* counters;           // [token blocks + 1] arrival counters, zero between launches
  int* status;             // device status word
  alignas(64) CUtensorMap wmap;  // fp32 router: 2-D tiled map over W [K rows, E cols], box 128 x 32
};

struct CombineParams {
  int M, H, topk;
  const int32_t* slot_map;  // [M, topk]
  const uint16_t* sel_w;    // bf16 [M, topk]
  const uint16_t* y_union;  // bf16 [U, M, H] (decode) or [positions, H] (rows_are_positions)
  const uint16_t* y_shared; // bf16 [M, H] (nullable)
  uint16_t* out;            // bf16 [M, H]
  int rows_are_positions;   // 1: slot_map holds the row of y_union directly
  const int32_t* shared_rows; // [M] row of y_union holding the shared expert's output (nullable)
};

// prefill token permutation (kernels.cu): segment e (expert e; segment E = the shared expert over
// all tokens, when present) holds the tokens that selected e in ascending token order, starting at a
// multiple of 8 positions; the pad positions after a segment hold token -1. Also the position of
// every (token, slot), the shared-expert position of every token, and the tile list.
struct PermParams {
  const int32_t* sel;      // [T, topk] global expert ids
  int T, topk, E, nt;      // tokens, slots, local experts, tokens per tile
  int expert_lo;           // global id of local expert 0: sel - expert_lo outside [0, E) is not local
  int with_shared;         // 1: add segment E with tokens [shared_t0, shared_t0 + shared_n)
  int shared_t0, shared_n;
  int32_t* perm_tok;       // [positions] token of each position (-1: pad)
  int32_t* pos_of;         // [T, topk] position of each (token, slot), -1 for a non-local expert
  int32_t* shared_pos;     // [shared_n] position of each shared-segment token (with_shared)
  int4* tiles;             // (segment, first position, tokens, 0)
  int32_t* n_tiles;        // [1]
  int32_t* n_pos;          // [1] positions used (padded)
};
int perm_launch(const PermParams& p, cudaStream_t s);

// Union of the local experts selected by M tokens (sorted) and the index of each (token, slot) in
// it, -1 when the slot's expert is not local (global id - expert_lo outside [0, E)).
struct EpSync;
int union_launch(const int32_t* sel, int M, int topk, int expert_lo, int E, int32_t* union_ids, int32_t* n_union,
                 int32_t* slot_map, cudaStream_t s, const EpSync* w = nullptr);
// y_slots[m, s, :] = rows[index[m * topk + s]] (bf16 rows of H) for index >= 0; row index
// r_of(i) = index * row_mul + m * row_add (decode: union-major [U, M, H] rows: row_mul = M, row_add = 1)
int gather_slots_launch(const int32_t* index, int M, int topk, int64_t H, const uint16_t* rows, int64_t row_mul,
                        int64_t row_add, uint16_t* y_slots, cudaStream_t s);
// Expert-parallel combine: out[m] = bf16( sum_s sel_w[m,s] * pieces[owner(sel[m,s])][m, s] + shared[m] )
// in slot order, owner(e) = e / experts_per_piece; pieces [P, M, topk, H] bf16.
// expert-parallel exchange over peer memory (ep.cu)
constexpr int EP_MAX_RANKS = 8;
struct EpParams {
  int G, rank, Mmax, H, T;
  uint8_t* peers[EP_MAX_RANKS];  // every rank's symmetric buffer (this rank's own included)
  int64_t off_flags, off_in_sel, off_in_x, off_out;
  uint32_t* seq;                 // device sequence number of the last completed layer call (local);
                                 // seq[1], seq[2]: arrival counters of the return and combine kernels
  int* status;
};
// Arrival wait folded into a consuming kernel (peer exchange): before reading, the kernel waits
// (bounded) until flags[0..n) reach *seq + 1, the current layer call's sequence number. bump_arrive
// (nullable): the kernel's CTAs count their exits there, and the last one advances *seq, ending the
// layer call (every CTA read *seq before).
struct EpSync {
  const uint32_t* flags = nullptr;
  int n = 0;
  uint32_t* seq = nullptr;
  int* status = nullptr;
  uint32_t* bump_arrive = nullptr;
};
int ep_dispatch_launch(const EpParams& p, const uint16_t* x, const int32_t* sel, int M, cudaStream_t s);
int ep_return_launch(const EpParams& p, const int32_t* slot_map, const uint16_t* rows, int M, int Gtok,
                     cudaStream_t s);
EpSync ep_sync(const EpParams& p, int which, bool bump);
int combine_pieces_launch(const int32_t* sel, const uint16_t* sel_w, int M, int topk, int64_t H,
                          int experts_per_piece, const uint16_t* pieces, const uint16_t* shared, uint16_t* out,
                          cudaStream_t s, EpSync w = EpSync());
// upper bound of the positions perm_kernel uses
inline int64_t perm_max_positions(int64_t T, int topk, int E, int with_shared) {
  return T * topk + (with_shared ? T : 0) + 8 * static_cast<int64_t>(E + 1);
}
inline int64_t perm_max_tiles(int64_t T, int topk, int E, int with_shared, int nt) {
  return (T * topk + nt - 1) / nt + E + (with_shared ? (T + nt - 1) / nt : 0);
}

// prefill GEMM on tcgen05 (tc_gemm.cu): persistent, items = (tile of <= nt tokens, row tile), nt 64 or 128
struct TcParams {
  int wt;                  // WT_Q4K or WT_Q6K
  int swiglu;              // 1: 64 gate + 64 up rows per item; y = h = bf16(silu(g) * u)
  int use_tmap;            // set by tc_gemm_launch
  int shared_id;           // segment id that uses the shared-expert weights ws (-1: none)
  const uint8_t* w[2];     // routed weights (gate/down, up), expert e at w + e * expert_stride
  const uint8_t* ws[2];    // shared-expert weights (gate/down, up)
  int64_t row_bytes;
  int64_t expert_stride;
  int N, K, M;             // output rows per matrix, reduction length, tokens (dense mode)
  const uint8_t* xt;       // prescaled activations in the tiled operand layout (prescale_tiled)
  const int* xshift;       // [positions] power-of-two prescale
  const int4* tiles;       // per tile (segment, first position, tokens, 0) (nullable: dense tiles over M)
  const int* tile_count;   // device number of tiles
  uint16_t* y;             // bf16 [positions, N]
  int* status;
  alignas(64) CUtensorMap wmap[2];
  alignas(64) CUtensorMap smap[2];
};
int tc_gemm_launch(TcParams& p, int nt, int n_experts, int max_tiles, int num_sms, cudaStream_t s, bool pdl);
size_t xt_bytes(int64_t R, int64_t K);
// builds the device's bf16 SiLU table used by the prefill SwiGLU epilogue (synchronises `s`)
int silu_table_init(cudaStream_t s);
int prescale_tiled_launch(const uint16_t* x, int R, int K, const int* rows, int rows_mask, int n_pos_max,
                          const int* n_pos_dev, uint8_t* xt, int* shift, cudaStream_t s, bool pdl);

int dequant_launch(int wt, const void* w, int64_t nrows, int64_t K, void* out, int out_bf16, cudaStream_t s);
// exact GEMM (sequential fp32 chains), optionally over groups (experts): group g uses weights
// w + group_ids[g] * w_group_stride, activations x + g * x_group_stride, output y + g * y_group_stride
struct StrictParams {
  int wt;
  const uint8_t* w;
  int64_t w_group_stride;
  const int* group_ids;     // nullable: identity
  const int* n_groups_dev;  // nullable: all launched groups are live
  int N, K, M;
  const void* x;
  int xt;
  int64_t x_group_stride;   // elements
  uint16_t* y;              // bf16 (nullable)
  float* y_f32;             // fp32 accumulators (nullable)
  int64_t y_group_stride;   // elements
};
int strict_gemm_grouped_launch(const StrictParams& p, int n_groups, cudaStream_t s);
int swiglu_elem_launch(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* h, cudaStream_t s);
int strict_gemm_launch(int wt, const void* w, int N, int K, const void* x, int xt, int M, uint16_t* y, float* y_f32,
                       cudaStream_t s);
int router_launch(const RouterParams& p, cudaStream_t s, bool pdl);
// bf16 GEMV under the reference's bf16 dot contract (lmhead.cu): y[m, v] = dot7(x[m], w[v])
int bf16_dot7_launch(const uint16_t* w, int64_t V, int64_t K, const uint16_t* x, int64_t M, uint16_t* y, int num_sms,
                     cudaStream_t s, bool pdl);
int router_grid_ctas(const RouterParams& p);  // CTAs of the launch router_launch makes
int router_smem_bytes(const RouterParams& p); // its dynamic shared memory per CTA
int combine_launch(const CombineParams& p, cudaStream_t s, bool pdl);
// min_smem: dynamic shared memory of at least this many bytes per CTA (keeps CTAs off SMs whose
// remaining shared memory is less, e.g. SMs running a concurrent latency-bound kernel)
int gemv_launch(int wt, int xt, int epi, GemvParams p, int num_sms, cudaStream_t stream, bool pdl, int min_smem = 0);
int gemv_partials_floats(int num_sms);
int act_launch(int kind, const void* x, int64_t n, void* out, cudaStream_t s);
int wait_selftest_launch(int* status, cudaStream_t s);

// Bit-exact sequential-chain GEMV (chain.cu): every output is the reference's sequential fp32 chain
// over k (tools/q4k_ref.py:86-92), computed for many rows at once. Groups (experts) g use weights
// w + group_ids[g] * expert_stride; the tokens of group g are the x rows m with some slot
// slot_map[m * topk + s] == g (all M rows when slot_map is null). x rows of group g start at
// x + g * x_group_stride (elements; 0 = shared rows); outputs y[g * y_group_stride + m * N + n].
enum ChainEpi : int { CHAIN_STORE = 0, CHAIN_SWIGLU = 1 };
struct ChainParams {
  const uint8_t* w0;         // rows (CHAIN_SWIGLU: gate rows)
  const uint8_t* w1;         // up rows (CHAIN_SWIGLU)
  int64_t row_bytes, expert_stride;
  const int* group_ids;      // nullable: group g = expert g
  const int* n_groups_dev;   // nullable: n_groups groups
  int n_groups, n_experts;
  int N, K;
  const void* x;             // activations (bf16, or fp32 when x_f32)
  int x_f32;
  int64_t x_group_stride;
  int M;                     // token rows
  const int32_t* slot_map;   // [M, topk] group index of each (token, slot), -1 none (nullable)
  int topk;
  // tile mode (many tokens, tiles != null): the token lists of perm_kernel with 8 tokens per tile --
  // item rows come from tile t = (expert, first position p0, tokens c): tokens perm_tok[p0 .. p0 + c),
  // x row = perm_tok[p0 + j] (or p0 + j when x_by_pos), output row y[(p0 + j) * N + n]
  const int4* tiles;
  const int* n_tiles_dev;
  int max_tiles;
  const int32_t* perm_tok;
  int x_by_pos;
  uint16_t* y;               // bf16 out (CHAIN_SWIGLU: h = bf16(silu(bf16 g) * bf16 u))
  float* y_f32;              // fp32 accumulators (CHAIN_STORE, nullable)
  int64_t y_group_stride;
  int* status;
  // set by chain_launch
  float neg_zero;            // -0.0f (the addend that forms exact products; see chain.cu)
  int tiles_per_group, nstages, stage_bytes, w_bytes, mt;
  alignas(64) CUtensorMap tmap0;
  alignas(64) CUtensorMap tmap1;
};
// Returns OK, an error, or CHAIN_UNSUPPORTED (shape/type the kernel does not take: use the generic
// strict kernel).
constexpr int CHAIN_UNSUPPORTED = 1;
int chain_launch(int wt, int epi, ChainParams p, int num_sms, cudaStream_t s, bool pdl);
bool chain_supported(int wt, int64_t K, int64_t row_bytes);

}  // namespace aipu
