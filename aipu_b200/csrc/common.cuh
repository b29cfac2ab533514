// Shared device helpers for the sm_100a k-quant kernels.
//
// Numerics rules for every kernel in this library (they are what makes the dequant bit-exact
// to the reference's numpy golden, tools/q4k_ref.py):
//   * fp32 products and sums that the contract rounds separately are written with
//     __fmul_rn / __fadd_rn / __fsub_rn, which the compiler never contracts into an FMA;
//   * nothing is built with --use_fast_math or -ftz=true (subnormal fp16 scales stay exact);
//   * fp16 -> fp32 uses __half2float (exact, subnormals included).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace aipu {

// weight types (values match the reference's w_type selector, src/glm_matmul_q4k.v:76-92)
enum WType : int { WT_Q4K = 0, WT_Q6K = 1, WT_Q80 = 2, WT_F16 = 3, WT_F32 = 4 };
enum XType : int { XT_F32 = 0, XT_BF16 = 1 };

// device status word bits (written by kernels that hit a bounded wait limit or bad input)
enum : int { ST_OK = 0, ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_BAD_ARGS = 4 };

// Bytes of one "unit" = 256 consecutive weights of one row, per type.
__host__ __device__ constexpr int unit_bytes(int wt) {
  return wt == WT_Q4K ? 144 : wt == WT_Q6K ? 210 : wt == WT_Q80 ? 272 : wt == WT_F16 ? 512 : 1024;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier + bulk copy (TMA)
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Every bounded wait's limit in SM clock cycles. The device status word passed to the kernels is the
// first int of a 16-byte block whose 64-bit word at byte 8 holds the wait limit set for the context
// (aipu_ctx_set_wait_limit; 0 = the default of 4e9 cycles, about 2 s). Read only once a wait has
// lasted kWaitGrace cycles: a wait that ends sooner never stalls on that global load (limits below
// the grace act as the grace).
constexpr long long kDefaultWaitCycles = 4000000000LL;
constexpr long long kWaitGrace = 65536;
__device__ __forceinline__ long long wait_limit(const int* status) {
  if (!status) return kDefaultWaitCycles;
  const long long v = *reinterpret_cast<const volatile long long*>(status + 2);
  return v > 0 ? v : kDefaultWaitCycles;
}

// Bounded wait: gives up after the context's wait limit (or `limit_cycles` when positive), sets the
// status bit and returns false. No wait in this library can spin forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status, int bit,
                                                  long long limit_cycles = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  long long limit = limit_cycles;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    const long long el = clock64() - t0;
    if (el > kWaitGrace) {
      if (limit <= 0) limit = wait_limit(status);
      if (el > limit) {
        if (status) atomicOr(status, bit);
        return false;
      }
    }
  }
  return true;
}

// Shared-memory progress counters between two warps of a CTA (cheaper than an mbarrier round trip
// when the waiting warp is on the critical path). Writer: its lanes' shared stores, __syncwarp, then
// one lane publishes with st.release; reader: every lane polls with ld.acquire.
__device__ __forceinline__ uint32_t ld_acquire_cta_shared(const uint32_t* f) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(f)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta_shared(uint32_t* f, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(f)), "r"(v) : "memory");
}
// Warp-uniform bounded wait until *f >= target (wrapping compare). Returns the value seen (>= target),
// or target - 1 after `limit_cycles` (status bit set).
__device__ __forceinline__ uint32_t warp_wait_counter(const uint32_t* f, uint32_t target, int* status, int bit,
                                                      long long limit_cycles = 0) {
  // every lane acquires; the value returned is the warp minimum (each lane saw at least that much)
  uint32_t v = ld_acquire_cta_shared(f) - target;
  if (__all_sync(0xffffffffu, static_cast<int32_t>(v) >= 0)) return __reduce_min_sync(0xffffffffu, v) + target;
  long long limit = limit_cycles;
  const long long t0 = clock64();
  while (true) {
    v = ld_acquire_cta_shared(f) - target;
    if (__all_sync(0xffffffffu, static_cast<int32_t>(v) >= 0)) return __reduce_min_sync(0xffffffffu, v) + target;
    const long long el = clock64() - t0;
    if (el > kWaitGrace && limit <= 0) limit = wait_limit(status);
    if (__any_sync(0xffffffffu, el > kWaitGrace && el > limit)) {
      if (status && (threadIdx.x & 31) == 0) atomicOr(status, bit);
      return target - 1u;
    }
  }
}

// 1-D bulk copy global -> shared, completion counted on an mbarrier (the untiled TMA path).
// dst, src 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load (tensor map in kernel-parameter space), completion on an mbarrier. No multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ programmatic dependent launch
// atomic add with release (this thread's and, through a preceding barrier, its CTA's writes) and
// acquire (the writes released by earlier adders) at GPU scope; returns the old value
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ named barriers
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ warp MMA (dot-product engine)
// D[16x8] += A[16x16] * B[16x8], fp16 inputs, fp32 accumulate. Used as an exact-product dot
// engine for the HBM-bound decode GEMV (the operands are exact small integers and fp16 x).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  // (a & mask) | orv in one LOP3
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2_bits(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ------------------------------------------------------------------ numeric helpers
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}
// fp32 -> bf16 RNE on the low 16 bits; inf/NaN truncate (reference q4k_ref.py:76-84).
__device__ __forceinline__ uint16_t bf16_rne_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>(u >> 16);
  uint32_t lsb = (u >> 16) & 1u;
  return static_cast<uint16_t>((u + 0x7FFFu + lsb) >> 16);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ float bf16_round_f(float x) { return bf16_bits_to_f32(bf16_rne_bits(x)); }

// exact power-of-two scale 2^e for |e| <= 126
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

}  // namespace aipu
