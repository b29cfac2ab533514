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
};

// prefill token permutation (kernels.cu): per-expert token lists in token order, the position of
// every (token, slot), and the tile list of the grouped tensor-core GEMM
struct PermParams {
  const int32_t* sel;      // [T, topk]
  int T, topk, E, nt;      // tokens, slots, experts, tokens per tile
  int32_t* perm_tok;       // [T*topk] token of each position
  int32_t* pos_of;         // [T, topk] position of each (token, slot)
  int4* tiles;             // (expert, first position, tokens, 0)
  int32_t* n_tiles;        // [1]
};
int perm_launch(const PermParams& p, cudaStream_t s);

// prefill GEMM on tcgen05 (tc_gemm.cu)
struct TcParams {
  int wt;                  // WT_Q4K or WT_Q6K
  int swiglu;              // 1: A rows 0..63 gate rows, 64..127 up rows; y = h = bf16(silu(g) * u)
  const uint8_t* w0;       // weights (gate rows for swiglu), expert e at w0 + e * expert_stride
  const uint8_t* w1;       // up rows (swiglu)
  int64_t row_bytes;
  int64_t expert_stride;
  int N, K, M;             // output rows per matrix, reduction length, tokens (dense mode)
  const __half* xh;        // prescaled fp16 activations [rows, K]
  const int* xshift;       // [rows] power-of-two prescale
  const __half* sx;        // [rows, K/256, 16] sub-block sums (Q4_K)
  const float* sxsb;       // [rows, K/256] super-block sums (Q4_K)
  const int* x_rows;       // position -> activation row (nullable: identity)
  const int4* tiles;       // per tile (group, first position, tokens, 0) (nullable: dense tiles over M)
  const int* tile_count;   // device number of tiles (nullable)
  const int* group_ids;    // group -> expert (nullable: identity)
  uint16_t* y;             // bf16 [positions, N]
  int* status;
};
int tc_gemm_launch(const TcParams& p, int nt, int max_tiles, cudaStream_t s, bool pdl);
int prescale_launch(const uint16_t* x, int R, int K, const int* rows, const int* n_rows_dev, __half* xh, int* shift,
                    __half* sx, float* sxsb, cudaStream_t s, bool pdl);

int dequant_launch(int wt, const void* w, int64_t nrows, int64_t K, void* out, int out_bf16, cudaStream_t s);
int strict_gemm_launch(int wt, const void* w, int N, int K, const void* x, int xt, int M, uint16_t* y, float* y_f32,
                       cudaStream_t s);
int router_launch(const RouterParams& p, cudaStream_t s, bool pdl);
int combine_launch(const CombineParams& p, cudaStream_t s, bool pdl);
int gemv_launch(int wt, int xt, int epi, GemvParams p, int num_sms, cudaStream_t stream, bool pdl);
int gemv_partials_floats(int num_sms);
int act_launch(int kind, const void* x, int64_t n, void* out, cudaStream_t s);

}  // namespace aipu
