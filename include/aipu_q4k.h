/* aipu_q4k.h -- C ABI of the B200 (sm_100a) k-quant dequant-GEMM and MoE library.
 *
 * Every function returns an int status (AIPU_OK = 0, negative on error) and never throws; the
 * text of the last error on the calling thread is available from aipu_last_error(). All device
 * pointers are caller-owned CUDA device memory; `stream` is a cudaStream_t (NULL = legacy default
 * stream). Calls are asynchronous on `stream` and do not synchronise.
 *
 * Weight layout: GGUF/ggml blocks, one weight row (= one output column of the contraction) is a
 * contiguous run of blocks along K, rows stored back to back:
 *   Q4_K 144 B / 256 weights, Q6_K 210 B / 256, Q8_0 34 B / 32, F16 2 B, F32 4 B.
 * Weight buffers must start on a 16-byte boundary and stay readable up to the next 16-byte boundary
 * after their last byte (the bulk copies move whole 16-byte chunks).
 *
 * Numeric contract (Wick-Lim/AIPU tools/q4k_ref.py:67-92): weights dequantised exactly as ggml,
 * products accumulated in fp32, output rounded to bf16 (round to nearest even).
 *   AIPU_MODE_FAST   tensor-core dot products, within 1 bf16 ulp of the sequential reference
 *   AIPU_MODE_STRICT sequential fp32 chain in K order, bit-identical to the reference
 */
#ifndef AIPU_Q4K_H
#define AIPU_Q4K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AIPU_OK 0
#define AIPU_EINVAL (-1)   /* bad shape, type or pointer */
#define AIPU_ECUDA (-2)    /* a CUDA runtime call failed */
#define AIPU_ETIMEOUT (-3) /* a bounded device-side wait gave up (device status word set) */
#define AIPU_ENCCL (-4)    /* an NCCL call failed */
#define AIPU_ENOMEM (-5)   /* workspace allocation failed */

/* weight types; values match the reference's w_type selector (src/glm_matmul_q4k.v:76-92) */
#define AIPU_Q4_K 0
#define AIPU_Q6_K 1
#define AIPU_Q8_0 2
#define AIPU_F16 3
#define AIPU_F32 4

/* activation / output dtypes */
#define AIPU_DT_F32 0
#define AIPU_DT_BF16 1

#define AIPU_MODE_FAST 0
#define AIPU_MODE_STRICT 1

typedef struct aipu_ctx aipu_ctx;

/* library version (major*10000 + minor*100 + patch) */
int aipu_version(void);
/* text of the last error raised on this thread ("" if none) */
const char* aipu_last_error(void);
/* bytes of one weight row of K weights of type `wtype` (0 if K is not a multiple of the block) */
int64_t aipu_row_bytes(int wtype, int64_t K);

/* A context owns the per-device workspace (stream-K partials and counters, MoE scratch) and a side
 * stream. One context per (device, concurrently used stream). The first MoE call sizes its scratch
 * (cudaMalloc), so make it once before capturing a CUDA graph. */
int aipu_ctx_create(aipu_ctx** ctx, int device);
int aipu_ctx_destroy(aipu_ctx* ctx);
/* Context flags.
 * AIPU_FLAG_PDL: launch the fast GEMM with programmatic dependent launch, so its weight stream
 * starts while the previous kernel on the stream is still running (activations are read only after
 * that kernel completes). Set it only when no kernel just before the GEMM writes the weights. */
#define AIPU_FLAG_PDL 1
/* AIPU_FLAG_STRICT: aipu_swiglu_expert and aipu_moe_layer run the bit-exact path: every GEMM as
 * the reference's sequential fp32 chain in K order (tools/q4k_ref.py:86-92), the SwiGLU product
 * and the combine in the reference's op order, so outputs equal tools/glm_model_q4k_ref.py
 * swiglu_expert / the decoder block's MoE branch bit for bit (slower: no tensor cores). */
#define AIPU_FLAG_STRICT 2
/* AIPU_FLAG_TC_DECODE: run the SwiGLU experts of the decode MoE path (aipu_moe_layer with few tokens,
 * aipu_moe_experts, aipu_swiglu_expert, aipu_ep_moe_layer) on the tensor-core GEMV (each GEMM within
 * 1 bf16 ulp, the layer not bit-exact) instead of the default bit-exact chain kernel. */
#define AIPU_FLAG_TC_DECODE 4
/* AIPU_FLAG_FAST_DOWN: on the default decode path, keep the bit-exact chains for gate/up (so the
 * SwiGLU product h equals the reference's bit for bit) and run the down projection on the integer-
 * engine GEMV (within 1 bf16 ulp of the sequential sum; the layer output is not bit-exact). Ignored
 * with AIPU_FLAG_TC_DECODE. */
#define AIPU_FLAG_FAST_DOWN 8
int aipu_ctx_set_flags(aipu_ctx* ctx, int flags);
/* device status word of the context (0 = no bounded wait ever gave up); resets it to 0. Bit 1: a
 * wait for data gave up, bit 2: a wait for a free buffer gave up, bit 4: bad arguments seen on the
 * device. */
int aipu_ctx_status(aipu_ctx* ctx, int* status);
/* Limit of every bounded device-side wait of kernels launched with this context, in SM clock cycles
 * (<= 0 restores the default of 4e9 cycles, about 2 s). When a wait reaches it, the kernel sets the
 * status word, drains its copies in flight and returns; the context stays usable. No counterpart in
 * the reference (its RTL waits are cycle-exact by construction). */
int aipu_ctx_set_wait_limit(aipu_ctx* ctx, int64_t cycles);
/* Failure-detection self-test: launches one bounded wait on a barrier that nothing releases, so it
 * runs out at the context's wait limit and sets the status word (read it with aipu_ctx_status). It
 * exercises the same give-up path as a lost peer or a stalled copy, without faulting the GPU. No
 * counterpart in the reference. */
int aipu_selftest_wait(aipu_ctx* ctx, void* stream);

/* Exact dequantisation of `nrows` rows of K weights to fp32 (out_dtype AIPU_DT_F32) or bf16
 * (AIPU_DT_BF16, RNE of the exact fp32). Bit-identical to the reference.
 * Replaces: tools/q4k_ref.py:39-65 dequantize_block_q4_K / dequantize_row_q4_K,
 *           tools/q4k_ref.py:105-124 dequantize_block_q6_K, tools/q4k_ref.py:126-129
 *           dequantize_block_q8_0, and the ggml dequant CLI tools/dequant_dump.c:11-33. */
int aipu_q4k_dequant(int wtype, const void* w, int64_t nrows, int64_t K, void* out, int out_dtype, void* stream);

/* Elementwise glm activation on bf16 values: kind 0 = sigmoid, 1 = SiLU (x * sigmoid(x)), bf16 out.
 * Degree-5 Horner exp, Quake-rsqrt^2 reciprocal, +-16 clamp; bit-identical to the reference.
 * Replaces: tools/glm_model_q4k_ref.py:293-299 glm_sigmoid / glm_silu (src/glm_act.v). */
int aipu_act_eval(int kind, const void* x, int64_t n, void* out, void* stream);

/* y[M, N] (bf16) = x[M, K] (fp32 or bf16, row-major) x W[N rows, K]^T.
 * FAST mode: K a multiple of 256, any M (internally blocks of 8 bf16 / 4 fp32 tokens), any N.
 * STRICT mode: any K that is a whole number of blocks; y_f32 (nullable) also receives the fp32
 * accumulator before rounding.
 * Replaces: tools/q4k_ref.py:86-92 matmul_q4k_col, tools/glm_model_q4k_ref.py:470-472
 *           matmul_q4k, and the GEMM core src/glm_matmul_q4k.v:50-288 (PE_M token rows). */
int aipu_q4k_gemm(aipu_ctx* ctx, int wtype, const void* w, int64_t N, int64_t K, const void* x, int x_dtype,
                  int64_t M, void* y, float* y_f32, int mode, void* stream);

/* Allocation-free fast GEMM, for callers that cannot call cudaMalloc: hosts whose allocator has
 * already reserved the device memory (a serving engine that owns all of HBM through its own pool),
 * plug-ins that must not create or keep a context object, and latency-critical paths where the
 * device-wide synchronisation of cudaMalloc/cudaFree is unacceptable. Same inputs, outputs and
 * numerics as aipu_q4k_gemm in AIPU_MODE_FAST (x_dtype AIPU_DT_F32 or AIPU_DT_BF16; wtype Q4_K,
 * Q6_K, Q8_0 or F16; K a multiple of 256), but its scratch (stream-K partial sums, arrival
 * counters and a status word, about 2.5 MiB) is a static array inside the library, held by every
 * GPU that loads the library until the process exits. Limit: N <= 65536 rows (larger N is
 * rejected with AIPU_EINVAL). The first call on a device looks up the array's device address
 * (guarded by a lock; make that first call before any stream capture). All calls share the one
 * array: calls that overlap on the GPU (different streams, or other threads) race and corrupt each
 * other; serialise them. The call is asynchronous, so its return code cannot report a bounded
 * device wait that gave up (its outputs are then left partly unwritten): the kernel records that in
 * the array's status word, which aipu_q4k_gemm_noalloc_status reads. No counterpart in the
 * reference. */
int aipu_q4k_gemm_noalloc(int wtype, const void* w, int64_t N, int64_t K, const void* x, int x_dtype, int64_t M,
                          void* y, void* stream);
/* Status word of aipu_q4k_gemm_noalloc on the current device (0 = no bounded wait gave up since the
 * last read), read synchronously and reset to 0; allocates nothing. No counterpart in the reference. */
int aipu_q4k_gemm_noalloc_status(int* status);

/* Prefill GEMM on the 5th-generation tensor cores (tcgen05 MMA, fp32 accumulators in TMEM):
 * y[M, N] (bf16) = x[M, K] (bf16, 16-byte aligned) x W[N rows, K]^T for Q4_K or Q6_K weights and many
 * token rows. Weights are dequantised in shared memory to exact fp16 operands (Q4_K: 1024 + sc*q;
 * Q6_K: two exact halves of sc*q), tokens are prescaled to fp16 by a power of two; fp32
 * accumulation per super-block, scales applied in the epilogue. Within 1 bf16 ulp of the sequential
 * reference (same bar as AIPU_MODE_FAST). The context grows a scratch buffer for the prescaled rows.
 * Replaces: tools/q4k_ref.py:86-92 matmul_q4k_col over many activation rows (the prefill use of
 *           src/glm_matmul_q4k.v). */
int aipu_q4k_gemm_tc(aipu_ctx* ctx, int wtype, const void* w, int64_t N, int64_t K, const void* x, int64_t M, void* y,
                     void* stream);

/* bf16 GEMV under the reference's bf16 dot-product contract (the LM head): y[m, v] (bf16) =
 * bf16((fl(p0 + p1) + fl(p2 + p3)) + (fl(p4 + p5) + fl(p6 + 0))) where p_l is the sequential fp32 sum
 * of fl(x[m, k] * w[v, k]) over k = l, l + 7, ... (bit-exact). w: V rows of K bf16 (16-byte
 * aligned, K % 8 == 0, K <= 14336); x: M rows of K bf16; y: [M, V] bf16.
 * Replaces: tools/glm_model_q4k_ref.py:474-486 matmul_bf16_dot (LM head use at :826). */
int aipu_bf16_dot_gemv(aipu_ctx* ctx, const void* w, int64_t V, int64_t K, const void* x, int64_t M, void* y,
                       void* stream);

/* Grouped fast GEMM: n_mats independent matrices of N rows x K (matrix g at w + g * mat_stride
 * bytes) applied to the same activations x[M, K] in ONE launch; y[g, M, N] (bf16). This is the
 * decode pattern of several projections or experts fed by the same token rows (e.g. all experts of
 * a layer on one token, or fused Q/K/V-style projections), and amortises the launch and the
 * activation staging over all matrices. Same numerics as AIPU_MODE_FAST.
 * Replaces: a loop of tools/q4k_ref.py:86-92 matmul_q4k_col over several weight matrices. */
int aipu_q4k_gemm_grouped(aipu_ctx* ctx, int wtype, const void* w, int64_t n_mats, int64_t mat_stride, int64_t N,
                          int64_t K, const void* x, int x_dtype, int64_t M, void* y, void* stream);

/* MoE router on M bf16 token rows x[M, K]:
 *   logits = bf16(sequential fp32 x . w_e) for every expert e  (strict, bit-exact)
 *   gate   = bf16 glm sigmoid(logits)
 *   select top-`topk` by gate (+ bias[e] in fp32 when bias != NULL; selection only), lower expert
 *   index wins ties; weights = bf16(gate_i * rsqrt(s)^2 * scale), s = balanced sum of the winners.
 * router_wtype AIPU_F32: w is fp32 [K, E] (x @ W); otherwise GGUF rows [E, K].
 * Outputs: sel int32 [M, topk] (slot 0 = largest), sel_w bf16 [M, topk], gate bf16 [M, E]
 * (nullable), logits bf16 [M, E] (nullable).
 * Replaces: tools/glm_model_q4k_ref.py:663-681 moe_router (src/moe_router_q4k.v,
 *           src/topk_select.v). The bias is an extension (absent in the reference). */
int aipu_moe_router(aipu_ctx* ctx, int router_wtype, const void* w, const float* bias, const void* x, int64_t M,
                    int64_t K, int64_t E, int topk, float scale, int32_t* sel, void* sel_w, void* gate, void* logits,
                    void* stream);

/* Weights of one MoE layer. Routed experts: gate/up [E][F rows][row bytes of H] and
 * down [E][H rows][row bytes of F], experts back to back (stride = rows * row bytes). */
typedef struct aipu_moe_weights {
  int64_t hidden;        /* H */
  int64_t ffn;           /* F */
  int64_t n_experts;     /* E */
  int32_t topk;
  float scale;           /* routing-weight scale (2.5 in the reference) */
  int32_t router_wtype;  /* AIPU_F32 ([H, E]) or a GGUF type ([E, H]) */
  const void* router_w;
  const float* router_bias; /* nullable */
  int32_t gate_wtype, up_wtype, down_wtype;
  const void* gate_w;
  const void* up_w;
  const void* down_w;
  const void* shared_gate_w; /* nullable: no shared expert */
  const void* shared_up_w;
  const void* shared_down_w;
} aipu_moe_weights;

/* y[M, H] (bf16) = MoE branch of the decoder block on bf16 token rows x[M, H]:
 * router (strict) -> per selected expert SwiGLU y_e = (silu(x Wg) * (x Wu)) Wd with bf16 rounding
 * at each stage -> facc = sum over slots (slot order) of w_slot * y_e, + y_shared -> bf16.
 * Each expert in the union of the M tokens' selections is streamed once for all M rows.
 * Optional outputs (nullable): sel [M, topk], sel_w bf16 [M, topk].
 * Replaces: tools/glm_model_q4k_ref.py:797-809 (decoder_block MoE branch) with
 *           swiglu_expert :702-708 (src/glm_decoder_block_q4k.v, src/swiglu_expert_q4k.v). */
int aipu_moe_layer(aipu_ctx* ctx, const aipu_moe_weights* wts, const void* x, int64_t M, void* y, int32_t* sel,
                   void* sel_w, void* stream);

/* One SwiGLU expert on bf16 rows x[M, H]: y[M, H] = bf16 rows of (silu(x Wg) * (x Wu)) Wd.
 * h (nullable, bf16 [M, F]) receives the hidden activation.
 * Replaces: tools/glm_model_q4k_ref.py:702-708 swiglu_expert (src/swiglu_expert_q4k.v). */
int aipu_swiglu_expert(aipu_ctx* ctx, int gate_wtype, const void* gate_w, int up_wtype, const void* up_w,
                       int down_wtype, const void* down_w, int64_t H, int64_t F, const void* x, int64_t M, void* h,
                       void* y, void* stream);

/* Expert-parallel pieces. A rank holds the routed experts [expert_lo, expert_lo + W->n_experts)
 * (W's gate/up/down point at them, back to back) and the replicated shared expert; router fields of
 * W are unused. For tokens x[M, H] (bf16) and their global selections sel[M, topk]:
 *   aipu_moe_experts: y_slots[m, s, :] = SwiGLU expert sel[m, s] of x[m] for every slot whose expert
 *     is local (other slots are left untouched); y_shared[i, :] = shared expert of token
 *     shared_t0 + i for i < shared_n (y_shared may be NULL). Many tokens use the tensor cores,
 *     AIPU_FLAG_STRICT the bit-exact chains.
 *   aipu_moe_combine: out[m] = bf16( sum_s sel_w[m, s] * pieces[sel[m, s] / experts_per_piece][m, s]
 *     + y_shared[m] ) in slot order, pieces [P, M, topk, H] bf16 (the y_slots of every rank, as an
 *     all-to-all returns them) -- the reference's combine order, so the layer equals the one-GPU one.
 * No counterpart function in the reference (its MoE runs on one device): the pieces are the
 * decoder-block MoE branch of tools/glm_model_q4k_ref.py:797-809 split at the expert loop. */
int aipu_moe_experts(aipu_ctx* ctx, const aipu_moe_weights* w_local, int64_t expert_lo, const void* x, int64_t M,
                     const int32_t* sel, void* y_slots, int64_t shared_t0, int64_t shared_n, void* y_shared,
                     void* stream);
int aipu_moe_combine(aipu_ctx* ctx, int64_t M, int64_t H, int topk, const int32_t* sel, const void* sel_w,
                     int64_t experts_per_piece, const void* pieces, const void* y_shared, void* out, void* stream);

/* Expert-parallel decode layer over NVLink peer memory (one process per GPU). Each rank creates an
 * endpoint (a symmetric buffer for max_tokens tokens per rank) and gets its CUDA IPC handle
 * (64 bytes); the caller exchanges the handles (e.g. an all-gather) and connects every rank to all
 * the others. aipu_ep_moe_layer then runs one MoE layer for this rank's M tokens (the same M on
 * every rank): route, store tokens and selections into every peer's inbox, the local experts on all
 * ranks' tokens, per-slot outputs stored into each owner's outbox, slot-order combine. Arrival is
 * signalled by sequence-numbered flags; every device wait is bounded (the context status word
 * reports an expired wait). w_local: this rank's experts [rank * E, (rank + 1) * E) plus the
 * replicated router (all experts) and shared expert. AIPU_FLAG_STRICT gives the one-GPU layer's
 * bits. No counterpart in the reference (its MoE runs on one device); same contract as
 * aipu_moe_layer (tools/glm_model_q4k_ref.py:797-809). */
typedef struct aipu_ep aipu_ep;
int aipu_ep_create(aipu_ctx* ctx, int world, int rank, int64_t max_tokens, int64_t hidden, int topk, aipu_ep** ep,
                   void* ipc_handle);
int aipu_ep_connect(aipu_ep* ep, const void* handles);
int aipu_ep_moe_layer(aipu_ep* ep, const aipu_moe_weights* w_local, int64_t expert_lo, const void* x, int64_t M,
                      void* y, void* stream);
int aipu_ep_destroy(aipu_ep* ep);

#ifdef __cplusplus
}
#endif
#endif /* AIPU_Q4K_H */
