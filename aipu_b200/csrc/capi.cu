// extern "C" entry points (include/aipu_q4k.h) and the per-device context.
#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cudaTypedefs.h>

#include "../../include/aipu_q4k.h"
#include "common.cuh"
#include "deq.cuh"
#include "gemv.cuh"
#include "kernels.h"
#include "launch.h"

namespace aipu {

static thread_local std::string g_err;

int set_error(int code, const char* msg) {
  g_err = msg ? msg : "";
  return code;
}
int set_cuda_error(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return OK;
  g_err = std::string(where) + ": " + cudaGetErrorString(e);
  return ECUDA_;
}
const char* last_error() { return g_err.c_str(); }

int launch_kernel(const void* kern, dim3 grid, dim3 block, int smem, cudaStream_t stream, bool pdl, void* arg0) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  void* args[1] = {arg0};
  return set_cuda_error(cudaLaunchKernelExC(&cfg, kern, args), "cudaLaunchKernelExC");
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides, const cuuint32_t* box) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &qr) !=
            cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !encode)
      return set_error(ECUDA_, "cuTensorMapEncodeTiled unavailable");
  }
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = encode(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ECUDA_, "tensor map encoding failed");
  return OK;
}

int set_smem_attr_once(const void* kern, int bytes, bool* done, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, what);
  if (dev < 0 || dev >= 64) return set_error(EINVAL_, "device index out of range (at most 64 devices)");
  if (done[dev]) return OK;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return set_cuda_error(e, what);
  done[dev] = true;
  return OK;
}

int num_sms_of_current_device() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

}  // namespace aipu

using namespace aipu;

// one stream-K workspace: partial sums per CTA and arrival counters per tile
struct Workspace {
  float* partials = nullptr;
  int* counters = nullptr;
  int max_tiles = 0;
  void* aux = nullptr;  // strict SwiGLU up-projection rows (grown on demand)
  size_t aux_bytes = 0;
};

struct aipu_ctx {
  int device = 0;
  int num_sms = 1;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  Workspace ws[2];  // [0] main stream, [1] side stream
  int* status = nullptr;
  int* router_counters = nullptr;  // [1024 + 1]
  // MoE scratch (grown on demand)
  void* moe = nullptr;
  size_t moe_bytes = 0;
  int flags = 0;  // AIPU_FLAG_*
  // prefill scratch (grown on demand)
  void* pre = nullptr;
  size_t pre_bytes = 0;
  void* rt = nullptr;     // router outputs of the many-token path
  size_t rt_bytes = 0;
  void* tmp = nullptr;    // gate rows of aipu_moe_router / h rows of aipu_swiglu_expert when the caller passes none
  size_t tmp_bytes = 0;
};

static int grow(void** buf, size_t* have, size_t need, const char* what) {
  if (need <= *have) return OK;
  cudaFree(*buf);
  *buf = nullptr;
  *have = 0;
  if (cudaMalloc(buf, need) != cudaSuccess) return set_error(ENOMEM_, what);
  *have = need;
  return OK;
}

static size_t al256x(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static const int kMaxTiles = 1 << 16;

static int ws_alloc(Workspace& w, int num_sms) {
  if (cudaMalloc(&w.partials, sizeof(float) * gemv_partials_floats(num_sms)) != cudaSuccess)
    return set_error(ENOMEM_, "cudaMalloc(partials)");
  if (cudaMalloc(&w.counters, sizeof(int) * kMaxTiles) != cudaSuccess) return set_error(ENOMEM_, "cudaMalloc(counters)");
  if (cudaMemset(w.counters, 0, sizeof(int) * kMaxTiles) != cudaSuccess) return set_error(ECUDA_, "cudaMemset");
  w.max_tiles = kMaxTiles;
  return OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

extern "C" {

int aipu_version(void) { return 100; }
const char* aipu_last_error(void) { return last_error(); }

int64_t aipu_row_bytes(int wtype, int64_t K) {
  if (K <= 0) return 0;
  if ((wtype == AIPU_Q4_K || wtype == AIPU_Q6_K) && K % 256) return 0;
  if (wtype == AIPU_Q8_0 && K % 32) return 0;
  if (wtype < 0 || wtype > 4) return 0;
  return row_bytes_of(wtype, K);
}

int aipu_ctx_create(aipu_ctx** out, int device) {
  if (!out) return set_error(EINVAL_, "ctx_create: null out pointer");
  *out = nullptr;
  DeviceGuard dg(device);
  aipu_ctx* c = new aipu_ctx();
  c->device = device;
  c->num_sms = num_sms_of_current_device();
  int rc = OK;
  if ((rc = ws_alloc(c->ws[0], c->num_sms)) || (rc = ws_alloc(c->ws[1], c->num_sms))) {
    aipu_ctx_destroy(c);
    return rc;
  }
  // status word + 64-bit bounded-wait limit (0 = default), see wait_limit() in common.cuh
  if (cudaMalloc(&c->status, 16) != cudaSuccess || cudaMemset(c->status, 0, 16) != cudaSuccess ||
      cudaMalloc(&c->router_counters, sizeof(int) * 1040) != cudaSuccess ||
      cudaMemset(c->router_counters, 0, sizeof(int) * 1040) != cudaSuccess) {
    aipu_ctx_destroy(c);
    return set_error(ENOMEM_, "ctx_create: cudaMalloc");
  }
  if (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming) != cudaSuccess) {
    aipu_ctx_destroy(c);
    return set_error(ECUDA_, "ctx_create: stream/event");
  }
  if (int trc = silu_table_init(c->side)) {
    aipu_ctx_destroy(c);
    return trc;
  }
  *out = c;
  return OK;
}

int aipu_ctx_destroy(aipu_ctx* c) {
  if (!c) return OK;
  DeviceGuard dg(c->device);
  for (auto& w : c->ws) {
    cudaFree(w.partials);
    cudaFree(w.counters);
    cudaFree(w.aux);
  }
  cudaFree(c->tmp);
  cudaFree(c->status);
  cudaFree(c->router_counters);
  cudaFree(c->moe);
  cudaFree(c->pre);
  cudaFree(c->rt);
  if (c->side) cudaStreamDestroy(c->side);
  if (c->ev_fork) cudaEventDestroy(c->ev_fork);
  if (c->ev_join) cudaEventDestroy(c->ev_join);
  delete c;
  return OK;
}

int aipu_ctx_set_flags(aipu_ctx* c, int flags) {
  if (!c || (flags & ~(AIPU_FLAG_PDL | AIPU_FLAG_STRICT | AIPU_FLAG_TC_DECODE | AIPU_FLAG_FAST_DOWN))) return set_error(EINVAL_, "ctx_set_flags: bad arguments");
  c->flags = flags;
  return OK;
}

int aipu_ctx_status(aipu_ctx* c, int* status) {
  if (!c || !status) return set_error(EINVAL_, "ctx_status: null pointer");
  DeviceGuard dg(c->device);
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, c->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_cuda_error(e, "ctx_status");
  cudaMemset(c->status, 0, sizeof(int));
  *status = v;
  return OK;
}

int aipu_ctx_set_wait_limit(aipu_ctx* c, int64_t cycles) {
  if (!c) return set_error(EINVAL_, "ctx_set_wait_limit: null context");
  DeviceGuard dg(c->device);
  const long long v = cycles > 0 ? static_cast<long long>(cycles) : 0;
  return set_cuda_error(cudaMemcpy(reinterpret_cast<char*>(c->status) + 8, &v, sizeof(v), cudaMemcpyHostToDevice),
                        "ctx_set_wait_limit");
}

int aipu_selftest_wait(aipu_ctx* c, void* stream) {
  if (!c) return set_error(EINVAL_, "selftest_wait: null context");
  DeviceGuard dg(c->device);
  return wait_selftest_launch(c->status, static_cast<cudaStream_t>(stream));
}

int aipu_q4k_dequant(int wtype, const void* w, int64_t nrows, int64_t K, void* out, int out_dtype, void* stream) {
  if (!w || !out || nrows < 0 || aipu_row_bytes(wtype, K) == 0 || (out_dtype != AIPU_DT_F32 && out_dtype != AIPU_DT_BF16))
    return set_error(EINVAL_, "dequant: bad arguments");
  return dequant_launch(wtype, w, nrows, K, out, out_dtype == AIPU_DT_BF16, static_cast<cudaStream_t>(stream));
}

int aipu_act_eval(int kind, const void* x, int64_t n, void* out, void* stream) {
  if (!x || !out || n < 0 || (kind != 0 && kind != 1)) return set_error(EINVAL_, "act_eval: bad arguments");
  return act_launch(kind, x, n, out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// fast GEMM on one stream-K workspace, splitting M into blocks the kernel takes
static int gemm_fast(aipu_ctx* c, Workspace& ws, int wtype, const void* w, int64_t N, int64_t K, const void* x,
                     int xt, int64_t M, void* y, cudaStream_t s, bool pdl) {
  const int mb = (xt == AIPU_DT_F32) ? 4 : 8;
  const int esz = (xt == AIPU_DT_F32) ? 4 : 2;
  if ((N + 15) / 16 > ws.max_tiles) return set_error(EINVAL_, "gemm: N too large for the workspace");
  for (int64_t m0 = 0; m0 < M; m0 += mb) {
    GemvParams p = {};
    p.w0 = static_cast<const uint8_t*>(w);
    p.row_bytes = row_bytes_of(wtype, K);
    p.n_groups = 1;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.x = static_cast<const uint8_t*>(x) + m0 * K * esz;
    p.M = static_cast<int>(std::min<int64_t>(mb, M - m0));
    p.y = static_cast<uint16_t*>(y) + m0 * N;
    p.partials = ws.partials;
    p.counters = ws.counters;
    p.status = c->status;
    int rc = gemv_launch(wtype, xt == AIPU_DT_F32 ? XT_F32 : XT_BF16, EPI_STORE, p, c->num_sms, s, pdl);
    if (rc) return rc;
  }
  return OK;
}

extern "C" int aipu_q4k_gemm(aipu_ctx* c, int wtype, const void* w, int64_t N, int64_t K, const void* x, int x_dtype,
                             int64_t M, void* y, float* y_f32, int mode, void* stream) {
  if (!c || !w || !x || (!y && !y_f32) || N <= 0 || M <= 0 || aipu_row_bytes(wtype, K) == 0 ||
      (x_dtype != AIPU_DT_F32 && x_dtype != AIPU_DT_BF16) || N > INT32_MAX || K > INT32_MAX)
    return set_error(EINVAL_, "gemm: bad arguments");
  if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0) return set_error(EINVAL_, "gemm: weights must be 16-byte aligned");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int xt = x_dtype == AIPU_DT_F32 ? XT_F32 : XT_BF16;
  if (mode == AIPU_MODE_STRICT || wtype == AIPU_F32 || y_f32) {
    if (wtype != AIPU_F32 && chain_supported(wtype, K, row_bytes_of(wtype, K))) {
      ChainParams p = {};
      p.w0 = static_cast<const uint8_t*>(w);
      p.row_bytes = row_bytes_of(wtype, K);
      p.n_groups = 1;
      p.N = static_cast<int>(N);
      p.K = static_cast<int>(K);
      p.x = x;
      p.x_f32 = (xt == XT_F32) ? 1 : 0;
      p.M = static_cast<int>(std::min<int64_t>(M, INT32_MAX));
      p.y = static_cast<uint16_t*>(y);
      p.y_f32 = y_f32;
      p.status = c->status;
      const int rc = chain_launch(wtype, CHAIN_STORE, p, c->num_sms, s, (c->flags & AIPU_FLAG_PDL) != 0);
      if (rc != CHAIN_UNSUPPORTED) return rc;
    }
    return strict_gemm_launch(wtype, w, static_cast<int>(N), static_cast<int>(K), x, xt, static_cast<int>(M),
                              static_cast<uint16_t*>(y), y_f32, s);
  }
  if (mode != AIPU_MODE_FAST) return set_error(EINVAL_, "gemm: unknown mode");
  if (K % 256) return set_error(EINVAL_, "gemm: fast mode needs K to be a multiple of 256");
  return gemm_fast(c, c->ws[0], wtype, w, N, K, x, x_dtype, M, y, s, (c->flags & AIPU_FLAG_PDL) != 0);
}

extern "C" int aipu_q4k_gemm_grouped(aipu_ctx* c, int wtype, const void* w, int64_t n_mats, int64_t mat_stride,
                                     int64_t N, int64_t K, const void* x, int x_dtype, int64_t M, void* y,
                                     void* stream) {
  if (!c || !w || !x || !y || n_mats <= 0 || N <= 0 || M <= 0 || K % 256 || aipu_row_bytes(wtype, K) == 0 ||
      wtype == AIPU_F32 || (x_dtype != AIPU_DT_F32 && x_dtype != AIPU_DT_BF16) || N > INT32_MAX || K > INT32_MAX ||
      mat_stride < N * aipu_row_bytes(wtype, K) || (mat_stride & 15) || (reinterpret_cast<uintptr_t>(w) & 15u))
    return set_error(EINVAL_, "gemm_grouped: bad arguments");
  if (n_mats * ((N + 15) / 16) > c->ws[0].max_tiles) return set_error(EINVAL_, "gemm_grouped: too many tiles");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mb = (x_dtype == AIPU_DT_F32) ? 4 : 8;
  const int esz = (x_dtype == AIPU_DT_F32) ? 4 : 2;
  for (int64_t m0 = 0; m0 < M; m0 += mb) {
    GemvParams p = {};
    p.w0 = static_cast<const uint8_t*>(w);
    p.row_bytes = row_bytes_of(wtype, K);
    p.expert_stride = mat_stride;
    p.n_experts = static_cast<int>(n_mats);
    p.n_groups = static_cast<int>(n_mats);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.x = static_cast<const uint8_t*>(x) + m0 * K * esz;
    p.x_group_stride = 0;
    p.M = static_cast<int>(std::min<int64_t>(mb, M - m0));
    p.y = static_cast<uint16_t*>(y) + m0 * N;
    p.y_group_stride = M * N;
    p.partials = c->ws[0].partials;
    p.counters = c->ws[0].counters;
    p.status = c->status;
    int rc = gemv_launch(wtype, x_dtype == AIPU_DT_F32 ? XT_F32 : XT_BF16, EPI_STORE, p, c->num_sms, s,
                         (c->flags & AIPU_FLAG_PDL) != 0);
    if (rc) return rc;
  }
  return OK;
}

extern "C" int aipu_moe_router(aipu_ctx* c, int wt, const void* w, const float* bias, const void* x, int64_t M,
                               int64_t K, int64_t E, int topk, float scale, int32_t* sel, void* sel_w, void* gate,
                               void* logits, void* stream) {
  if (!c || !w || !x || !sel || !sel_w || M <= 0 || M > 1024 || E <= 0 || E > 1024 || topk <= 0 || topk > 16 ||
      topk > E || (wt != AIPU_F32 && aipu_row_bytes(wt, K) == 0) || K <= 0)
    return set_error(EINVAL_, "router: bad arguments");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint16_t* gbuf = static_cast<uint16_t*>(gate);
  if (!gbuf) {
    // context workspace, grown on demand (make a first call before capturing a CUDA graph)
    const int grc = grow(&c->tmp, &c->tmp_bytes, sizeof(uint16_t) * M * E, "router: gate scratch");
    if (grc) return grc;
    gbuf = static_cast<uint16_t*>(c->tmp);
  }
  RouterParams p = {};
  p.wt = wt;
  p.w = static_cast<const uint8_t*>(w);
  p.bias = bias;
  p.x = static_cast<const uint16_t*>(x);
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.E = static_cast<int>(E);
  p.topk = topk;
  p.scale = scale;
  p.gate = gbuf;
  p.logits = static_cast<uint16_t*>(logits);
  p.sel = sel;
  p.sel_w = static_cast<uint16_t*>(sel_w);
  p.counters = c->router_counters;
  p.status = c->status;
  return router_launch(p, s, false);
}

// ------------------------------------------------------------------ MoE decode layer
struct MoeScratch {
  uint16_t* gate;     // [M, E]
  int32_t* sel;       // [M, T]
  uint16_t* sel_w;    // [M, T]
  int32_t* union_ids; // [U]
  int32_t* n_union;   // [1]
  int32_t* slot_map;  // [M, T]
  uint16_t* h;        // [U, M, F]
  uint16_t* y;        // [U, M, H]
  uint16_t* h_sh;     // [M, F]
  uint16_t* y_sh;     // [M, H]
};

static size_t al256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static int moe_scratch(aipu_ctx* c, int64_t M, int64_t E, int T, int64_t H, int64_t F, MoeScratch& sc) {
  const int64_t U = std::min<int64_t>(E, M * T);
  size_t sz[10] = {al256(2 * M * E), al256(4 * M * T), al256(2 * M * T), al256(4 * U), al256(4),
                   al256(4 * M * T), al256(2 * U * M * F), al256(2 * U * M * H), al256(2 * M * F), al256(2 * M * H)};
  size_t total = 0;
  for (size_t v : sz) total += v;
  if (total > c->moe_bytes) {
    cudaFree(c->moe);
    c->moe = nullptr;
    c->moe_bytes = 0;
    if (cudaMalloc(&c->moe, total) != cudaSuccess) return set_error(ENOMEM_, "moe: scratch allocation");
    c->moe_bytes = total;
  }
  uint8_t* b = static_cast<uint8_t*>(c->moe);
  void* ptr[10];
  for (int i = 0; i < 10; ++i) {
    ptr[i] = b;
    b += sz[i];
  }
  sc.gate = static_cast<uint16_t*>(ptr[0]);
  sc.sel = static_cast<int32_t*>(ptr[1]);
  sc.sel_w = static_cast<uint16_t*>(ptr[2]);
  sc.union_ids = static_cast<int32_t*>(ptr[3]);
  sc.n_union = static_cast<int32_t*>(ptr[4]);
  sc.slot_map = static_cast<int32_t*>(ptr[5]);
  sc.h = static_cast<uint16_t*>(ptr[6]);
  sc.y = static_cast<uint16_t*>(ptr[7]);
  sc.h_sh = static_cast<uint16_t*>(ptr[8]);
  sc.y_sh = static_cast<uint16_t*>(ptr[9]);
  return OK;
}

// SwiGLU on groups of experts: h[g] = bf16(silu(x Wg_e) * (x Wu_e)), y[g] = h[g] Wd_e
// shared memory of one SM (bytes): two CTAs whose shared memory adds up to more never share an SM
static const int kSmemPerSm = 233472;

static int swiglu_groups(aipu_ctx* c, Workspace& ws, int gwt, const void* gw, const void* uw, int dwt, const void* dw,
                         int64_t H, int64_t F, int n_experts, const int* group_ids, const int* n_groups_dev,
                         int n_groups, const int32_t* slot_map, int topk,
                         const void* x, int64_t M, uint16_t* h, uint16_t* y, cudaStream_t s, bool pdl,
                         int num_sms = 0, int min_smem = 0) {
  if (num_sms <= 0) num_sms = c->num_sms;
  const int64_t gstride = F * row_bytes_of(gwt, H), dstride = H * row_bytes_of(dwt, F);
  if (!(c->flags & AIPU_FLAG_TC_DECODE) && chain_supported(gwt, H, row_bytes_of(gwt, H)) &&
      chain_supported(dwt, F, row_bytes_of(dwt, F)) && gwt == WT_Q4K && (!slot_map || M <= 32)) {
    // the bit-exact sequential chains (tools/glm_model_q4k_ref.py:702-708 op for op), each expert on
    // the tokens that selected it: gate/up with the SwiGLU product fused, then the down projection
    ChainParams g = {};
    g.w0 = static_cast<const uint8_t*>(gw);
    g.w1 = static_cast<const uint8_t*>(uw);
    g.row_bytes = row_bytes_of(gwt, H);
    g.expert_stride = gstride;
    g.group_ids = group_ids;
    g.n_groups_dev = n_groups_dev;
    g.n_groups = n_groups;
    g.n_experts = n_experts;
    g.N = static_cast<int>(F);
    g.K = static_cast<int>(H);
    g.x = static_cast<const uint16_t*>(x);
    g.x_group_stride = 0;
    g.M = static_cast<int>(M);
    g.slot_map = slot_map;
    g.topk = topk;
    g.y = h;
    g.y_group_stride = M * F;
    g.status = c->status;
    int rc = chain_launch(gwt, CHAIN_SWIGLU, g, num_sms, s, pdl);
    if (rc == OK && (c->flags & AIPU_FLAG_FAST_DOWN)) {
      // h bit-exact from the chains; the down projection on the GEMV (1-ulp bar). Rows of tokens that
      // did not select an expert are computed from unwritten h and never read by the combine.
      for (int64_t m0 = 0; m0 < M; m0 += 8) {
        GemvParams q = {};
        q.w0 = static_cast<const uint8_t*>(dw);
        q.row_bytes = row_bytes_of(dwt, F);
        q.expert_stride = dstride;
        q.group_ids = group_ids;
        q.n_experts = n_experts;
        q.n_groups_dev = n_groups_dev;
        q.n_groups = n_groups;
        q.N = static_cast<int>(H);
        q.K = static_cast<int>(F);
        q.x = h + m0 * F;
        q.x_group_stride = M * F;
        q.M = static_cast<int>(std::min<int64_t>(8, M - m0));
        q.y = y + m0 * H;
        q.y_group_stride = M * H;
        q.partials = ws.partials;
        q.counters = ws.counters;
        q.status = c->status;
        rc = gemv_launch(dwt, XT_BF16, EPI_STORE, q, num_sms, s, pdl, min_smem);
        if (rc) return rc;
      }
      return OK;
    }
    if (rc == OK) {
      ChainParams d = g;
      d.w0 = static_cast<const uint8_t*>(dw);
      d.w1 = nullptr;
      d.row_bytes = row_bytes_of(dwt, F);
      d.expert_stride = dstride;
      d.N = static_cast<int>(H);
      d.K = static_cast<int>(F);
      d.x = h;
      d.x_group_stride = M * F;
      d.y = y;
      d.y_group_stride = M * H;
      rc = chain_launch(dwt, CHAIN_STORE, d, num_sms, s, true);
      if (rc == CHAIN_UNSUPPORTED) rc = set_error(EINVAL_, "swiglu: down projection not supported by the chain kernel");
      return rc;
    }
    if (rc != CHAIN_UNSUPPORTED) return rc;
  }
  if (c->flags & AIPU_FLAG_STRICT) {
    // bit-exact chains (tools/glm_model_q4k_ref.py:702-708): gate into h, up into a temporary,
    // h = bf16(silu(gate) * up) in place, then the down projection of h
    const int64_t n = static_cast<int64_t>(n_groups) * M * F;
    // up-projection rows in the workspace of this stream (grown on demand, before any capture)
    const int grc = grow(&ws.aux, &ws.aux_bytes, 2 * n, "swiglu (strict): scratch");
    if (grc) return grc;
    uint16_t* up = static_cast<uint16_t*>(ws.aux);
    StrictParams p = {};
    p.wt = gwt;
    p.w = static_cast<const uint8_t*>(gw);
    p.w_group_stride = gstride;
    p.group_ids = group_ids;
    p.n_groups_dev = n_groups_dev;
    p.N = static_cast<int>(F);
    p.K = static_cast<int>(H);
    p.M = static_cast<int>(M);
    p.x = x;
    p.xt = XT_BF16;
    p.y = h;
    p.y_group_stride = M * F;
    int rc = strict_gemm_grouped_launch(p, n_groups, s);
    if (!rc) {
      p.w = static_cast<const uint8_t*>(uw);
      p.y = up;
      rc = strict_gemm_grouped_launch(p, n_groups, s);
    }
    if (!rc) rc = swiglu_elem_launch(h, up, n, h, s);
    if (!rc) {
      StrictParams q = p;
      q.wt = dwt;
      q.w = static_cast<const uint8_t*>(dw);
      q.w_group_stride = dstride;
      q.N = static_cast<int>(H);
      q.K = static_cast<int>(F);
      q.x = h;
      q.x_group_stride = M * F;
      q.y = y;
      q.y_group_stride = M * H;
      rc = strict_gemm_grouped_launch(q, n_groups, s);
    }
    return rc;
  }
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    const int mb = static_cast<int>(std::min<int64_t>(8, M - m0));
    GemvParams p = {};
    p.w0 = static_cast<const uint8_t*>(gw);
    p.w1 = static_cast<const uint8_t*>(uw);
    p.row_bytes = row_bytes_of(gwt, H);
    p.expert_stride = gstride;
    p.group_ids = group_ids;
    p.n_experts = n_experts;
    p.n_groups_dev = n_groups_dev;
    p.n_groups = n_groups;
    p.N = static_cast<int>(F);
    p.K = static_cast<int>(H);
    p.x = static_cast<const uint16_t*>(x) + m0 * H;
    p.x_group_stride = 0;
    p.M = mb;
    p.y = h + m0 * F;
    p.y_group_stride = M * F;
    p.partials = ws.partials;
    p.counters = ws.counters;
    p.status = c->status;
    int rc = gemv_launch(gwt, XT_BF16, EPI_SWIGLU, p, num_sms, s, pdl, min_smem);
    if (rc) return rc;
    GemvParams q = p;
    q.w0 = static_cast<const uint8_t*>(dw);
    q.w1 = nullptr;
    q.row_bytes = row_bytes_of(dwt, F);
    q.expert_stride = dstride;
    q.N = static_cast<int>(H);
    q.K = static_cast<int>(F);
    q.x = h + m0 * F;
    q.x_group_stride = M * F;
    q.y = y + m0 * H;
    q.y_group_stride = M * H;
    // the group list was complete before the gate/up launch began (its producers do not trigger
    // their dependents early), so the down projection may read it and prefetch weights while the
    // gate/up launch drains
    q.ids_ready = 1;
    rc = gemv_launch(dwt, XT_BF16, EPI_STORE, q, num_sms, s, pdl, min_smem);
    if (rc) return rc;
  }
  return OK;
}

// ------------------------------------------------------------------ MoE prefill (many tokens)
// Expert computation of the many-token path on the tensor cores, for given selections: per-segment
// token lists (local experts of [expert_lo, expert_lo + E); segment E = the shared expert over tokens
// [shared_t0, shared_t0 + shared_n)) -> tiled prescale of the permuted tokens -> SwiGLU gate/up on
// tcgen05 -> tiled prescale of h -> down projection on tcgen05. Outputs (in c->pre): y_perm rows by
// position, pos_of[M * T] (-1: expert not local), shared_pos[shared_n].
struct TcExperts {
  uint16_t* y_perm;
  int32_t* pos_of;
  int32_t* shared_pos;
  uint8_t* aux;  // caller scratch after the expert buffers
};
static int moe_experts_tc(aipu_ctx* c, const aipu_moe_weights* W, const void* x, int64_t M, const int32_t* sel,
                          int64_t expert_lo, int64_t shared_t0, int64_t shared_n, size_t aux_bytes, TcExperts& out,
                          cudaStream_t s) {
  const int64_t H = W->hidden, F = W->ffn, E = W->n_experts;
  const int T = W->topk;
  // tokens per tile: top-8 of 256 experts gives ~64 tokens per expert at 2048 tokens, spread around
  // that; a 128-token tile takes most experts whole (one dequantisation of each weight tile), and
  // the MMA width follows the tile's tokens
  const int nt = 128;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w && shared_n > 0;
  const int64_t Pmax = M * T + (shared ? shared_n : 0) + 8 * (E + 1);
  const int64_t max_tiles = (M * T + nt - 1) / nt + E + (shared ? (shared_n + nt - 1) / nt : 0);
  size_t sz[12] = {al256x(4 * M * T),         al256x(4 * std::max<int64_t>(shared_n, 1)), al256x(4 * Pmax),
                   al256x(16 * max_tiles),    al256x(16),                                 al256x(xt_bytes(Pmax, H)),
                   al256x(4 * Pmax),          al256x(2 * Pmax * F),                       al256x(xt_bytes(Pmax, F)),
                   al256x(2 * Pmax * H),      al256x(4 * Pmax),                           al256x(aux_bytes)};
  size_t total = 0;
  for (size_t v : sz) total += v;
  int rc = grow(&c->pre, &c->pre_bytes, total, "moe: tensor-core scratch");
  if (rc) return rc;
  uint8_t* b = static_cast<uint8_t*>(c->pre);
  void* ptr[12];
  for (int i = 0; i < 12; ++i) {
    ptr[i] = b;
    b += sz[i];
  }
  int32_t* pos_of = static_cast<int32_t*>(ptr[0]);
  int32_t* shared_pos = static_cast<int32_t*>(ptr[1]);
  int32_t* perm_tok = static_cast<int32_t*>(ptr[2]);
  int4* tiles = static_cast<int4*>(ptr[3]);
  int32_t* counts = static_cast<int32_t*>(ptr[4]);  // [0] tiles, [1] positions
  uint8_t* xt = static_cast<uint8_t*>(ptr[5]);
  int* xshift = static_cast<int*>(ptr[6]);
  uint16_t* h_perm = static_cast<uint16_t*>(ptr[7]);
  uint8_t* ht = static_cast<uint8_t*>(ptr[8]);
  uint16_t* y_perm = static_cast<uint16_t*>(ptr[9]);
  int* hshift = static_cast<int*>(ptr[10]);
  out.y_perm = y_perm;
  out.pos_of = pos_of;
  out.shared_pos = shared_pos;
  out.aux = static_cast<uint8_t*>(ptr[11]);

  PermParams pp = {};
  pp.sel = sel;
  pp.T = static_cast<int>(M);
  pp.topk = T;
  pp.E = static_cast<int>(E);
  pp.nt = nt;
  pp.expert_lo = static_cast<int>(expert_lo);
  pp.with_shared = shared ? 1 : 0;
  pp.shared_t0 = static_cast<int>(shared_t0);
  pp.shared_n = shared ? static_cast<int>(shared_n) : 0;
  pp.perm_tok = perm_tok;
  pp.pos_of = pos_of;
  pp.shared_pos = shared_pos;
  pp.tiles = tiles;
  pp.n_tiles = counts;
  pp.n_pos = counts + 1;
  if ((rc = perm_launch(pp, s))) return rc;
  if ((rc = prescale_tiled_launch(static_cast<const uint16_t*>(x), static_cast<int>(M), static_cast<int>(H), perm_tok,
                                  0, static_cast<int>(Pmax), counts + 1, xt, xshift, s, true)))
    return rc;
  TcParams g = {};
  g.wt = W->gate_wtype;
  g.swiglu = 1;
  g.shared_id = shared ? static_cast<int>(E) : -1;
  g.w[0] = static_cast<const uint8_t*>(W->gate_w);
  g.w[1] = static_cast<const uint8_t*>(W->up_w);
  g.ws[0] = static_cast<const uint8_t*>(W->shared_gate_w);
  g.ws[1] = static_cast<const uint8_t*>(W->shared_up_w);
  g.row_bytes = row_bytes_of(W->gate_wtype, H);
  g.expert_stride = F * g.row_bytes;
  g.N = static_cast<int>(F);
  g.K = static_cast<int>(H);
  g.M = static_cast<int>(M);
  g.xt = xt;
  g.xshift = xshift;
  g.tiles = tiles;
  g.tile_count = counts;
  g.y = h_perm;
  g.status = c->status;
  if ((rc = tc_gemm_launch(g, nt, static_cast<int>(E), static_cast<int>(max_tiles), c->num_sms, s, true))) return rc;
  if ((rc = prescale_tiled_launch(h_perm, static_cast<int>(Pmax), static_cast<int>(F), perm_tok, 1,
                                  static_cast<int>(Pmax), counts + 1, ht, hshift, s, true)))
    return rc;
  TcParams dn = {};
  dn.wt = W->down_wtype;
  dn.swiglu = 0;
  dn.shared_id = g.shared_id;
  dn.w[0] = static_cast<const uint8_t*>(W->down_w);
  dn.ws[0] = static_cast<const uint8_t*>(W->shared_down_w);
  dn.row_bytes = row_bytes_of(W->down_wtype, F);
  dn.expert_stride = H * dn.row_bytes;
  dn.N = static_cast<int>(H);
  dn.K = static_cast<int>(F);
  dn.M = static_cast<int>(M);
  dn.xt = ht;
  dn.xshift = hshift;
  dn.tiles = tiles;
  dn.tile_count = counts;
  dn.y = y_perm;
  dn.status = c->status;
  return tc_gemm_launch(dn, nt, static_cast<int>(E), static_cast<int>(max_tiles), c->num_sms, s, true);
}

// Many-token MoE layer on one GPU: router -> moe_experts_tc (all experts, shared over all tokens) ->
// slot-order combine straight from the position-ordered rows (reference: glm_model_q4k_ref.py:663-809).
static int moe_prefill(aipu_ctx* c, const aipu_moe_weights* W, const void* x, int64_t M, void* y, int32_t* sel_out,
                       void* sel_w_out, cudaStream_t s) {
  const int64_t H = W->hidden, E = W->n_experts;
  const int T = W->topk;
  const int64_t P = M * T;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w;
  // router outputs live in the caller-scratch tail of the tensor-core scratch
  const size_t aux = al256x(2 * M * E) + al256x(4 * P) + al256x(2 * P);
  TcExperts te = {};
  // router outputs in their own context buffer (the expert pass may grow the tensor-core scratch)
  int rc = grow(&c->rt, &c->rt_bytes, aux, "moe_prefill: router scratch");
  if (rc) return rc;
  uint16_t* gate = static_cast<uint16_t*>(c->rt);
  int32_t* sel = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(gate) + al256x(2 * M * E));
  uint16_t* sel_w = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(sel) + al256x(4 * P));
  RouterParams rp = {};
  rp.wt = W->router_wtype;
  rp.w = static_cast<const uint8_t*>(W->router_w);
  rp.bias = W->router_bias;
  rp.x = static_cast<const uint16_t*>(x);
  rp.M = static_cast<int>(M);
  rp.K = static_cast<int>(H);
  rp.E = static_cast<int>(E);
  rp.topk = T;
  rp.scale = W->scale;
  rp.gate = gate;
  rp.sel = sel;
  rp.sel_w = sel_w;
  rp.counters = c->router_counters;
  rp.status = c->status;
  rc = router_launch(rp, s, false);
  if (!rc) rc = moe_experts_tc(c, W, x, M, sel, 0, 0, shared ? M : 0, 0, te, s);
  if (!rc) {
    CombineParams cp = {};
    cp.M = static_cast<int>(M);
    cp.H = static_cast<int>(H);
    cp.topk = T;
    cp.slot_map = te.pos_of;
    cp.sel_w = sel_w;
    cp.y_union = te.y_perm;
    cp.shared_rows = shared ? te.shared_pos : nullptr;
    cp.out = static_cast<uint16_t*>(y);
    cp.rows_are_positions = 1;
    rc = combine_launch(cp, s, true);
  }
  if (!rc && sel_out)
    rc = set_cuda_error(cudaMemcpyAsync(sel_out, sel, 4 * P, cudaMemcpyDeviceToDevice, s), "copy sel");
  if (!rc && sel_w_out)
    rc = set_cuda_error(cudaMemcpyAsync(sel_w_out, sel_w, 2 * P, cudaMemcpyDeviceToDevice, s), "copy sel_w");
  return rc;
}

// Many-token MoE experts, bit-exact: the tokens of every local expert (perm_kernel lists, 8 tokens per
// tile) run through the chain kernel -- gate/up with the SwiGLU product, then down, rows by position --
// and the shared expert over tokens [shared_t0, shared_t0 + shared_n) as dense chains. Outputs (in
// c->pre): y_perm rows by position, pos_of[M * T] (-1: expert not local), y_sh [shared_n, H].
struct ExactExperts {
  uint16_t* y_perm;
  int32_t* pos_of;
  uint16_t* y_sh;
};
static int moe_experts_exact(aipu_ctx* c, const aipu_moe_weights* W, const void* x, int64_t M, const int32_t* sel,
                             int64_t expert_lo, int64_t shared_t0, int64_t shared_n, ExactExperts& out, cudaStream_t s) {
  const int64_t H = W->hidden, F = W->ffn, E = W->n_experts;
  const int T = W->topk;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w && shared_n > 0;
  const int64_t Pmax = perm_max_positions(M, T, static_cast<int>(E), 0);
  const int64_t max_tiles = perm_max_tiles(M, T, static_cast<int>(E), 0, 8);
  const int64_t Sn = shared ? shared_n : 0;
  size_t sz[8] = {al256x(4 * M * T), al256x(4 * Pmax), al256x(16 * max_tiles), al256x(16), al256x(2 * Pmax * F),
                  al256x(2 * Pmax * H), al256x(2 * std::max<int64_t>(Sn, 1) * F), al256x(2 * std::max<int64_t>(Sn, 1) * H)};
  size_t total = 0;
  for (size_t v : sz) total += v;
  int rc = grow(&c->pre, &c->pre_bytes, total, "moe (exact): scratch");
  if (rc) return rc;
  uint8_t* b = static_cast<uint8_t*>(c->pre);
  void* ptr[8];
  for (int i = 0; i < 8; ++i) {
    ptr[i] = b;
    b += sz[i];
  }
  out.pos_of = static_cast<int32_t*>(ptr[0]);
  int32_t* perm_tok = static_cast<int32_t*>(ptr[1]);
  int4* tiles = static_cast<int4*>(ptr[2]);
  int32_t* counts = static_cast<int32_t*>(ptr[3]);
  uint16_t* h_perm = static_cast<uint16_t*>(ptr[4]);
  out.y_perm = static_cast<uint16_t*>(ptr[5]);
  uint16_t* h_sh = static_cast<uint16_t*>(ptr[6]);
  out.y_sh = static_cast<uint16_t*>(ptr[7]);
  PermParams pp = {};
  pp.sel = sel;
  pp.T = static_cast<int>(M);
  pp.topk = T;
  pp.E = static_cast<int>(E);
  pp.nt = 8;
  pp.expert_lo = static_cast<int>(expert_lo);
  pp.perm_tok = perm_tok;
  pp.pos_of = out.pos_of;
  pp.tiles = tiles;
  pp.n_tiles = counts;
  pp.n_pos = counts + 1;
  if ((rc = perm_launch(pp, s))) return rc;
  ChainParams g = {};
  g.w0 = static_cast<const uint8_t*>(W->gate_w);
  g.w1 = static_cast<const uint8_t*>(W->up_w);
  g.row_bytes = row_bytes_of(W->gate_wtype, H);
  g.expert_stride = F * g.row_bytes;
  g.n_experts = static_cast<int>(E);
  g.N = static_cast<int>(F);
  g.K = static_cast<int>(H);
  g.x = x;
  g.M = static_cast<int>(M);
  g.tiles = tiles;
  g.n_tiles_dev = counts;
  g.max_tiles = static_cast<int>(max_tiles);
  g.perm_tok = perm_tok;
  g.y = h_perm;
  g.status = c->status;
  if ((rc = chain_launch(W->gate_wtype, CHAIN_SWIGLU, g, c->num_sms, s, true)))
    return rc == CHAIN_UNSUPPORTED ? set_error(EINVAL_, "moe (exact): gate/up type or shape not supported") : rc;
  ChainParams d = g;
  d.w0 = static_cast<const uint8_t*>(W->down_w);
  d.w1 = nullptr;
  d.row_bytes = row_bytes_of(W->down_wtype, F);
  d.expert_stride = H * d.row_bytes;
  d.N = static_cast<int>(H);
  d.K = static_cast<int>(F);
  d.x = h_perm;
  d.x_by_pos = 1;
  d.M = static_cast<int>(Pmax);
  d.y = out.y_perm;
  if ((rc = chain_launch(W->down_wtype, CHAIN_STORE, d, c->num_sms, s, true)))
    return rc == CHAIN_UNSUPPORTED ? set_error(EINVAL_, "moe (exact): down type or shape not supported") : rc;
  if (shared) {
    ChainParams sg = {};
    sg.w0 = static_cast<const uint8_t*>(W->shared_gate_w);
    sg.w1 = static_cast<const uint8_t*>(W->shared_up_w);
    sg.row_bytes = g.row_bytes;
    sg.n_groups = 1;
    sg.N = static_cast<int>(F);
    sg.K = static_cast<int>(H);
    sg.x = static_cast<const uint16_t*>(x) + shared_t0 * H;
    sg.M = static_cast<int>(Sn);
    sg.y = h_sh;
    sg.status = c->status;
    if ((rc = chain_launch(W->gate_wtype, CHAIN_SWIGLU, sg, c->num_sms, s, true))) return rc;
    ChainParams sd = sg;
    sd.w0 = static_cast<const uint8_t*>(W->shared_down_w);
    sd.w1 = nullptr;
    sd.row_bytes = d.row_bytes;
    sd.N = static_cast<int>(H);
    sd.K = static_cast<int>(F);
    sd.x = h_sh;
    sd.y = out.y_sh;
    if ((rc = chain_launch(W->down_wtype, CHAIN_STORE, sd, c->num_sms, s, true))) return rc;
  }
  return OK;
}

// Many-token MoE layer, bit-exact: router -> moe_experts_exact -> slot-order combine from positions.
static int moe_exact_many(aipu_ctx* c, const aipu_moe_weights* W, const void* x, int64_t M, void* y, int32_t* sel_out,
                          void* sel_w_out, cudaStream_t s) {
  const int64_t E = W->n_experts;
  const int T = W->topk;
  const int64_t P = M * T;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w;
  const size_t aux = al256x(2 * M * E) + al256x(4 * P) + al256x(2 * P);
  int rc = grow(&c->rt, &c->rt_bytes, aux, "moe (exact): router scratch");
  if (rc) return rc;
  uint16_t* gate = static_cast<uint16_t*>(c->rt);
  int32_t* sel = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(gate) + al256x(2 * M * E));
  uint16_t* sel_w = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(sel) + al256x(4 * P));
  RouterParams rp = {};
  rp.wt = W->router_wtype;
  rp.w = static_cast<const uint8_t*>(W->router_w);
  rp.bias = W->router_bias;
  rp.x = static_cast<const uint16_t*>(x);
  rp.M = static_cast<int>(M);
  rp.K = static_cast<int>(W->hidden);
  rp.E = static_cast<int>(E);
  rp.topk = T;
  rp.scale = W->scale;
  rp.gate = gate;
  rp.sel = sel;
  rp.sel_w = sel_w;
  rp.counters = c->router_counters;
  rp.status = c->status;
  if ((rc = router_launch(rp, s, false))) return rc;
  ExactExperts ex = {};
  if ((rc = moe_experts_exact(c, W, x, M, sel, 0, 0, shared ? M : 0, ex, s))) return rc;
  CombineParams cp = {};
  cp.M = static_cast<int>(M);
  cp.H = static_cast<int>(W->hidden);
  cp.topk = T;
  cp.slot_map = ex.pos_of;
  cp.sel_w = sel_w;
  cp.y_union = ex.y_perm;
  cp.y_shared = shared ? ex.y_sh : nullptr;
  cp.out = static_cast<uint16_t*>(y);
  cp.rows_are_positions = 1;
  if ((rc = combine_launch(cp, s, true))) return rc;
  if (sel_out && (rc = set_cuda_error(cudaMemcpyAsync(sel_out, sel, 4 * P, cudaMemcpyDeviceToDevice, s), "copy sel")))
    return rc;
  if (sel_w_out &&
      (rc = set_cuda_error(cudaMemcpyAsync(sel_w_out, sel_w, 2 * P, cudaMemcpyDeviceToDevice, s), "copy sel_w")))
    return rc;
  return OK;
}

static bool exact_many_ok(const aipu_moe_weights* W, const void* x) {
  return W->gate_wtype == AIPU_Q4_K && chain_supported(W->gate_wtype, W->hidden, row_bytes_of(W->gate_wtype, W->hidden)) &&
         chain_supported(W->down_wtype, W->ffn, row_bytes_of(W->down_wtype, W->ffn)) &&
         (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (W->n_experts * W->ffn * row_bytes_of(W->gate_wtype, W->hidden)) > 0;
}

static const int64_t kPrefillMinTokens = 64;

extern "C" int aipu_moe_layer(aipu_ctx* c, const aipu_moe_weights* W, const void* x, int64_t M, void* y,
                              int32_t* sel_out, void* sel_w_out, void* stream) {
  if (!c || !W || !x || !y || M <= 0 || M > 8192) return set_error(EINVAL_, "moe_layer: bad arguments");
  const int64_t H = W->hidden, F = W->ffn, E = W->n_experts;
  const int T = W->topk;
  if (H % 256 || F % 256 || E <= 0 || E > 1024 || T <= 0 || T > 16 || T > E || !W->gate_w || !W->up_w ||
      !W->down_w || !W->router_w || W->gate_wtype != W->up_wtype || W->gate_wtype == AIPU_F32 ||
      W->down_wtype == AIPU_F32)
    return set_error(EINVAL_, "moe_layer: bad weights descriptor");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // many tokens: the tensor-core path (SwiGLU gate/up in Q4_K, down in Q4_K or Q6_K)
  const bool strict = (c->flags & AIPU_FLAG_STRICT) != 0;
  if (!strict && M >= kPrefillMinTokens && W->gate_wtype == AIPU_Q4_K &&
      (W->down_wtype == AIPU_Q4_K || W->down_wtype == AIPU_Q6_K) && (reinterpret_cast<uintptr_t>(x) & 15u) == 0)
    return moe_prefill(c, W, x, M, y, sel_out, sel_w_out, s);
  // more tokens than the decode union path takes (its per-expert token masks hold 32 tokens): the
  // bit-exact chains over per-expert token lists
  if (M > 32 && !(c->flags & AIPU_FLAG_TC_DECODE) && exact_many_ok(W, x))
    return moe_exact_many(c, W, x, M, y, sel_out, sel_w_out, s);
  if (M > 1024)
    return set_error(EINVAL_, strict ? "moe_layer (strict): at most 1024 tokens per call"
                                     : "moe_layer: more than 1024 tokens need Q4_K gate/up and Q4_K/Q6_K down");
  MoeScratch sc = {};
  int rc = moe_scratch(c, M, E, T, H, F, sc);
  if (rc) return rc;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w;
  // the shared expert runs on the side stream beside the (serial, latency-bound) router: the fork
  // point is recorded before the router, the side launches are submitted after it, on the SMs the
  // router leaves free and with enough shared memory that they cannot share an SM with it (a
  // co-resident GEMV would take issue slots from the router's dependent add chains)
  if (shared && (rc = set_cuda_error(cudaEventRecord(c->ev_fork, s), "eventRecord"))) return rc;
  RouterParams rp = {};
  rp.wt = W->router_wtype;
  rp.w = static_cast<const uint8_t*>(W->router_w);
  rp.bias = W->router_bias;
  rp.x = static_cast<const uint16_t*>(x);
  rp.M = static_cast<int>(M);
  rp.K = static_cast<int>(H);
  rp.E = static_cast<int>(E);
  rp.topk = T;
  rp.scale = W->scale;
  rp.gate = sc.gate;
  rp.sel = sc.sel;
  rp.sel_w = sc.sel_w;
  rp.union_ids = sc.union_ids;
  rp.n_union = sc.n_union;
  rp.slot_map = sc.slot_map;
  rp.counters = c->router_counters;
  rp.status = c->status;
  if ((rc = router_launch(rp, s, false))) return rc;
  if (shared) {
    const int router_ctas = router_grid_ctas(rp);
    const int side_sms = std::max(1, c->num_sms - router_ctas);
    if ((rc = set_cuda_error(cudaStreamWaitEvent(c->side, c->ev_fork, 0), "streamWaitEvent"))) return rc;
    rc = swiglu_groups(c, c->ws[1], W->gate_wtype, W->shared_gate_w, W->shared_up_w, W->down_wtype, W->shared_down_w,
                       H, F, 1, nullptr, nullptr, 1, nullptr, 0, x, M, sc.h_sh, sc.y_sh, c->side, false, side_sms,
                       kSmemPerSm - router_smem_bytes(rp));
    if (rc) return rc;
    if ((rc = set_cuda_error(cudaEventRecord(c->ev_join, c->side), "eventRecord"))) return rc;
  }
  const int Umax = static_cast<int>(std::min<int64_t>(E, M * T));
  rc = swiglu_groups(c, c->ws[0], W->gate_wtype, W->gate_w, W->up_w, W->down_wtype, W->down_w, H, F, static_cast<int>(E), sc.union_ids,
                     sc.n_union, Umax, sc.slot_map, T, x, M, sc.h, sc.y, s, true);
  if (rc) return rc;
  if (shared && (rc = set_cuda_error(cudaStreamWaitEvent(s, c->ev_join, 0), "streamWaitEvent"))) return rc;
  CombineParams cp = {};
  cp.M = static_cast<int>(M);
  cp.H = static_cast<int>(H);
  cp.topk = T;
  cp.slot_map = sc.slot_map;
  cp.sel_w = sc.sel_w;
  cp.y_union = sc.y;
  cp.y_shared = shared ? sc.y_sh : nullptr;
  cp.out = static_cast<uint16_t*>(y);
  if ((rc = combine_launch(cp, s, true))) return rc;
  if (sel_out && (rc = set_cuda_error(cudaMemcpyAsync(sel_out, sc.sel, 4 * M * T, cudaMemcpyDeviceToDevice, s), "copy sel")))
    return rc;
  if (sel_w_out &&
      (rc = set_cuda_error(cudaMemcpyAsync(sel_w_out, sc.sel_w, 2 * M * T, cudaMemcpyDeviceToDevice, s), "copy sel_w")))
    return rc;
  return OK;
}

// ------------------------------------------------------------------ expert-parallel pieces
extern "C" int aipu_moe_experts(aipu_ctx* c, const aipu_moe_weights* W, int64_t expert_lo, const void* x, int64_t M,
                                const int32_t* sel, void* y_slots, int64_t shared_t0, int64_t shared_n,
                                void* y_shared, void* stream) {
  if (!c || !W || !x || !sel || !y_slots || M <= 0 || M > 65536 || expert_lo < 0)
    return set_error(EINVAL_, "moe_experts: bad arguments");
  const int64_t H = W->hidden, F = W->ffn, E = W->n_experts;
  const int T = W->topk;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w && y_shared && shared_n > 0;
  if (H % 256 || F % 256 || E <= 0 || E > 1024 || T <= 0 || T > 16 || !W->gate_w || !W->up_w || !W->down_w ||
      W->gate_wtype != W->up_wtype || W->gate_wtype == AIPU_F32 || W->down_wtype == AIPU_F32 ||
      (shared && (shared_t0 < 0 || shared_t0 + shared_n > M)))
    return set_error(EINVAL_, "moe_experts: bad weights descriptor or shared token range");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool strict = (c->flags & AIPU_FLAG_STRICT) != 0;
  int rc;
  if (!strict && M >= kPrefillMinTokens && W->gate_wtype == AIPU_Q4_K &&
      (W->down_wtype == AIPU_Q4_K || W->down_wtype == AIPU_Q6_K) && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    TcExperts te = {};
    rc = moe_experts_tc(c, W, x, M, sel, expert_lo, shared_t0, shared ? shared_n : 0, 0, te, s);
    if (!rc)
      rc = gather_slots_launch(te.pos_of, static_cast<int>(M), T, H, te.y_perm, 1, 0,
                               static_cast<uint16_t*>(y_slots), s);
    if (!rc && shared)
      rc = gather_slots_launch(te.shared_pos, static_cast<int>(shared_n), 1, H, te.y_perm, 1, 0,
                               static_cast<uint16_t*>(y_shared), s);
    return rc;
  }
  if (M > 1024) return set_error(EINVAL_, "moe_experts: more than 1024 tokens need the tensor-core path");
  MoeScratch sc = {};
  if ((rc = moe_scratch(c, M, E, T, H, F, sc))) return rc;
  if ((rc = union_launch(sel, static_cast<int>(M), T, static_cast<int>(expert_lo), static_cast<int>(E), sc.union_ids,
                         sc.n_union, sc.slot_map, s)))
    return rc;
  const int Umax = static_cast<int>(std::min<int64_t>(E, M * T));
  rc = swiglu_groups(c, c->ws[0], W->gate_wtype, W->gate_w, W->up_w, W->down_wtype, W->down_w, H, F,
                     static_cast<int>(E), sc.union_ids, sc.n_union, Umax, sc.slot_map, T, x, M, sc.h, sc.y, s, false);
  if (!rc)
    rc = gather_slots_launch(sc.slot_map, static_cast<int>(M), T, H, sc.y, M, 1, static_cast<uint16_t*>(y_slots), s);
  if (!rc && shared)
    rc = swiglu_groups(c, c->ws[0], W->gate_wtype, W->shared_gate_w, W->shared_up_w, W->down_wtype, W->shared_down_w,
                       H, F, 1, nullptr, nullptr, 1, nullptr, 0, static_cast<const uint16_t*>(x) + shared_t0 * H, shared_n,
                       sc.h_sh, static_cast<uint16_t*>(y_shared), s, false);
  return rc;
}

extern "C" int aipu_moe_combine(aipu_ctx* c, int64_t M, int64_t H, int topk, const int32_t* sel, const void* sel_w,
                                int64_t experts_per_piece, const void* pieces, const void* y_shared, void* out,
                                void* stream) {
  if (!c || !sel || !sel_w || !pieces || !out || M <= 0 || H <= 0 || H % 8 || topk <= 0 || experts_per_piece <= 0)
    return set_error(EINVAL_, "moe_combine: bad arguments");
  DeviceGuard dg(c->device);
  return combine_pieces_launch(sel, static_cast<const uint16_t*>(sel_w), static_cast<int>(M), topk, H,
                               static_cast<int>(experts_per_piece), static_cast<const uint16_t*>(pieces),
                               static_cast<const uint16_t*>(y_shared), static_cast<uint16_t*>(out),
                               static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ expert parallel over peer memory
struct aipu_ep {
  aipu_ctx* ctx = nullptr;
  EpParams p = {};
  void* buf = nullptr;   // this rank's symmetric buffer
  size_t bytes = 0;
  bool mapped[EP_MAX_RANKS] = {};
  uint32_t* seq = nullptr;
  void* loc = nullptr;   // local scratch: sel, sel_w, y_shared
  int64_t E_local = 0;
};

extern "C" int aipu_ep_create(aipu_ctx* c, int world, int rank, int64_t max_tokens, int64_t hidden, int topk,
                              aipu_ep** out, void* ipc_handle) {
  if (!c || !out || !ipc_handle || world < 1 || world > EP_MAX_RANKS || rank < 0 || rank >= world ||
      max_tokens <= 0 || max_tokens > 64 || hidden <= 0 || hidden % 256 || topk <= 0 || topk > 16)
    return set_error(EINVAL_, "ep_create: bad arguments (world <= 8, tokens per rank <= 64)");
  DeviceGuard dg(c->device);
  aipu_ep* e = new aipu_ep();
  e->ctx = c;
  EpParams& p = e->p;
  p.G = world;
  p.rank = rank;
  p.Mmax = static_cast<int>(max_tokens);
  p.H = static_cast<int>(hidden);
  p.T = topk;
  const int64_t G = world, M = max_tokens, H = hidden, T = topk;
  p.off_flags = 0;
  p.off_in_sel = 256;
  p.off_in_x = al256x(p.off_in_sel + 4 * G * M * T);
  p.off_out = al256x(p.off_in_x + 2 * G * M * H);
  e->bytes = al256x(p.off_out + 2 * G * M * T * H);
  if (cudaMalloc(&e->buf, e->bytes) != cudaSuccess || cudaMemset(e->buf, 0, e->bytes) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void**>(&e->seq), 256) != cudaSuccess || cudaMemset(e->seq, 0, 256) != cudaSuccess ||
      cudaMalloc(&e->loc, al256x(4 * M * T) + al256x(2 * M * T) + al256x(2 * M * H)) != cudaSuccess) {
    cudaFree(e->buf);
    cudaFree(e->seq);
    delete e;
    return set_error(ENOMEM_, "ep_create: allocation");
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, e->buf) != cudaSuccess) {
    cudaFree(e->buf);
    cudaFree(e->seq);
    cudaFree(e->loc);
    delete e;
    return set_error(ECUDA_, "ep_create: cudaIpcGetMemHandle");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  p.peers[rank] = static_cast<uint8_t*>(e->buf);
  p.seq = e->seq;
  p.status = c->status;
  *out = e;
  return OK;
}

extern "C" int aipu_ep_connect(aipu_ep* e, const void* handles) {
  if (!e || !handles) return set_error(EINVAL_, "ep_connect: bad arguments");
  DeviceGuard dg(e->ctx->device);
  for (int q = 0; q < e->p.G; ++q) {
    if (q == e->p.rank || e->mapped[q]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(handles) + q * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return set_error(ECUDA_, "ep_connect: cudaIpcOpenMemHandle (peer access over NVLink required)");
    e->p.peers[q] = static_cast<uint8_t*>(ptr);
    e->mapped[q] = true;
  }
  return OK;
}

extern "C" int aipu_ep_destroy(aipu_ep* e) {
  if (!e) return OK;
  DeviceGuard dg(e->ctx->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < e->p.G; ++q)
    if (e->mapped[q]) cudaIpcCloseMemHandle(e->p.peers[q]);
  cudaFree(e->buf);
  cudaFree(e->seq);
  cudaFree(e->loc);
  delete e;
  return OK;
}

// One decode MoE layer with the routed experts sharded over the ranks (every rank calls it with the
// same M): route the local tokens; store tokens and selections into every peer's inbox (peer stores,
// released flags); shared expert on the local tokens; once every rank's tokens arrived, the local
// experts on all of them (grouped GEMV, or the exact chains in strict mode) and their per-slot
// outputs stored straight into each owner's outbox; once every piece arrived, the slot-order combine.
extern "C" int aipu_ep_moe_layer(aipu_ep* e, const aipu_moe_weights* W, int64_t expert_lo, const void* x, int64_t M,
                                 void* y, void* stream) {
  if (!e || !W || !x || !y || M <= 0 || M > e->p.Mmax || W->hidden != e->p.H || W->topk != e->p.T ||
      !W->router_w || (reinterpret_cast<uintptr_t>(x) & 15u))
    return set_error(EINVAL_, "ep_moe_layer: bad arguments");
  aipu_ctx* c = e->ctx;
  const int64_t H = W->hidden, F = W->ffn, El = W->n_experts;
  const int T = W->topk, G = e->p.G;
  const int64_t Et = El * G;
  const bool shared = W->shared_gate_w && W->shared_up_w && W->shared_down_w;
  if (H % 256 || F % 256 || El <= 0 || Et > 1024 || W->gate_wtype != W->up_wtype || W->gate_wtype == AIPU_F32 ||
      W->down_wtype == AIPU_F32 || expert_lo != static_cast<int64_t>(e->p.rank) * El)
    return set_error(EINVAL_, "ep_moe_layer: bad weights descriptor (rank r holds experts [r*E, (r+1)*E))");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t Gtok = G * M;
  int32_t* sel = static_cast<int32_t*>(e->loc);
  uint16_t* sel_w = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(e->loc) + al256x(4 * e->p.Mmax * T));
  uint16_t* y_sh = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(e->loc) + al256x(4 * e->p.Mmax * T) +
                                               al256x(2 * e->p.Mmax * T));
  MoeScratch sc = {};
  int rc = moe_scratch(c, Gtok, El, T, H, F, sc);
  if (rc) return rc;
  // the shared expert runs on the side stream beside the router and the exchange (as in
  // aipu_moe_layer: forked before the router, on the SMs the router leaves free), joined before the
  // combine
  if (shared && (rc = set_cuda_error(cudaEventRecord(c->ev_fork, s), "eventRecord"))) return rc;
  // 1. route the local tokens (all experts of the layer)
  RouterParams rp = {};
  rp.wt = W->router_wtype;
  rp.w = static_cast<const uint8_t*>(W->router_w);
  rp.bias = W->router_bias;
  rp.x = static_cast<const uint16_t*>(x);
  rp.M = static_cast<int>(M);
  rp.K = static_cast<int>(H);
  rp.E = static_cast<int>(Et);
  rp.topk = T;
  rp.scale = W->scale;
  rp.gate = sc.gate;
  rp.sel = sel;
  rp.sel_w = sel_w;
  rp.counters = c->router_counters;
  rp.status = c->status;
  if ((rc = router_launch(rp, s, false))) return rc;
  // 2. shared expert on the local tokens (side stream)
  if (shared) {
    const int router_ctas = router_grid_ctas(rp);
    const int side_sms = std::max(1, c->num_sms - router_ctas);
    if ((rc = set_cuda_error(cudaStreamWaitEvent(c->side, c->ev_fork, 0), "streamWaitEvent"))) return rc;
    rc = swiglu_groups(c, c->ws[1], W->gate_wtype, W->shared_gate_w, W->shared_up_w, W->down_wtype, W->shared_down_w,
                       H, F, 1, nullptr, nullptr, 1, nullptr, 0, x, M, sc.h_sh, y_sh, c->side, false, side_sms,
                       kSmemPerSm - router_smem_bytes(rp));
    if (rc) return rc;
    if ((rc = set_cuda_error(cudaEventRecord(c->ev_join, c->side), "eventRecord"))) return rc;
  }
  // 3. dispatch
  if ((rc = ep_dispatch_launch(e->p, static_cast<const uint16_t*>(x), sel, static_cast<int>(M), s))) return rc;
  // 4. every rank's tokens: local experts
  const uint8_t* inbox = static_cast<const uint8_t*>(e->buf);
  const int32_t* in_sel = reinterpret_cast<const int32_t*>(inbox + e->p.off_in_sel);
  const uint16_t* in_x = reinterpret_cast<const uint16_t*>(inbox + e->p.off_in_x);
  // the union kernel waits for every rank's tokens (dispatch flags) before reading the inbox
  const EpSync wait_in = ep_sync(e->p, 0, false);
  if ((rc = union_launch(in_sel, static_cast<int>(Gtok), T, static_cast<int>(expert_lo), static_cast<int>(El),
                         sc.union_ids, sc.n_union, sc.slot_map, s, &wait_in)))
    return rc;
  const int Umax = static_cast<int>(std::min<int64_t>(El, Gtok * T));
  if ((rc = swiglu_groups(c, c->ws[0], W->gate_wtype, W->gate_w, W->up_w, W->down_wtype, W->down_w, H, F,
                          static_cast<int>(El), sc.union_ids, sc.n_union, Umax, sc.slot_map, T, in_x, Gtok, sc.h, sc.y,
                          s, false)))
    return rc;
  // 5. per-slot outputs into the owners' outboxes
  if ((rc = ep_return_launch(e->p, sc.slot_map, sc.y, static_cast<int>(M), static_cast<int>(Gtok), s))) return rc;
  if (shared && (rc = set_cuda_error(cudaStreamWaitEvent(s, c->ev_join, 0), "streamWaitEvent"))) return rc;
  // 6. slot-order combine of this rank's tokens: waits for every rank's returned pieces (return flags)
  // and ends the layer call (advances the sequence number)
  return combine_pieces_launch(sel, sel_w, static_cast<int>(M), T, H, static_cast<int>(El),
                               reinterpret_cast<const uint16_t*>(inbox + e->p.off_out), shared ? y_sh : nullptr,
                               static_cast<uint16_t*>(y), s, ep_sync(e->p, 1, true));
}

extern "C" int aipu_swiglu_expert(aipu_ctx* c, int gwt, const void* gw, int uwt, const void* uw, int dwt,
                                  const void* dw, int64_t H, int64_t F, const void* x, int64_t M, void* h, void* y,
                                  void* stream) {
  if (!c || !gw || !uw || !dw || !x || !y || M <= 0 || H % 256 || F % 256 || gwt != uwt || gwt == AIPU_F32 ||
      dwt == AIPU_F32)
    return set_error(EINVAL_, "swiglu_expert: bad arguments");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint16_t* hb = static_cast<uint16_t*>(h);
  if (!hb) {
    const int grc = grow(&c->tmp, &c->tmp_bytes, 2 * M * F, "swiglu: scratch");
    if (grc) return grc;
    hb = static_cast<uint16_t*>(c->tmp);
  }
  return swiglu_groups(c, c->ws[0], gwt, gw, uw, dwt, dw, H, F, 1, nullptr, nullptr, 1, nullptr, 0, x, M, hb,
                       static_cast<uint16_t*>(y), s, false);
}

extern "C" int aipu_bf16_dot_gemv(aipu_ctx* c, const void* w, int64_t V, int64_t K, const void* x, int64_t M,
                                  void* y, void* stream) {
  if (!c || !w || !x || !y || V <= 0 || K <= 0 || M <= 0) return set_error(EINVAL_, "bf16_dot_gemv: bad arguments");
  DeviceGuard dg(c->device);
  return bf16_dot7_launch(static_cast<const uint16_t*>(w), V, K, static_cast<const uint16_t*>(x), M,
                          static_cast<uint16_t*>(y), c->num_sms, static_cast<cudaStream_t>(stream),
                          (c->flags & AIPU_FLAG_PDL) != 0);
}

extern "C" int aipu_q4k_gemm_tc(aipu_ctx* c, int wtype, const void* w, int64_t N, int64_t K, const void* x, int64_t M,
                                void* y, void* stream) {
  if (!c || !w || !x || !y || N <= 0 || M <= 0 || K <= 0 || K % 256 || (wtype != AIPU_Q4_K && wtype != AIPU_Q6_K) ||
      N > INT32_MAX || M > (1 << 24) || (reinterpret_cast<uintptr_t>(x) & 15u))
    return set_error(EINVAL_, "gemm_tc: bad arguments (Q4_K/Q6_K, K % 256 == 0, 16-byte aligned bf16 x)");
  DeviceGuard dg(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t xb = al256x(xt_bytes(M, K));
  int rc = grow(&c->pre, &c->pre_bytes, xb + al256x(4 * M), "gemm_tc: scratch");
  if (rc) return rc;
  uint8_t* xt = static_cast<uint8_t*>(c->pre);
  int* shift = reinterpret_cast<int*>(xt + xb);
  const int rpad = static_cast<int>((M + 7) & ~7LL);
  rc = prescale_tiled_launch(static_cast<const uint16_t*>(x), static_cast<int>(M), static_cast<int>(K), nullptr, 0,
                             rpad, nullptr, xt, shift, s, false);
  if (rc) return rc;
  TcParams p = {};
  p.wt = wtype;
  p.shared_id = -1;
  p.w[0] = static_cast<const uint8_t*>(w);
  p.row_bytes = row_bytes_of(wtype, K);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.M = static_cast<int>(M);
  p.xt = xt;
  p.xshift = shift;
  p.y = static_cast<uint16_t*>(y);
  p.status = c->status;
  return tc_gemm_launch(p, 128, 1, static_cast<int>((M + 127) / 128), c->num_sms, s, true);
}
