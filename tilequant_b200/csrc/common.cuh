// Shared device/host helpers for the TileQuant B200 kernels (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tilequant_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tilequant_b200 kernels are written for sm_100a (B200) only"
#endif

namespace tq {

// Upper bound of any device-side wait loop (mbarrier / cluster flag polls).  A wait
// that reaches it records TQ_ERR_TIMEOUT in the error word and gives up instead of
// hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ float h2f(uint16_t h, int dtype) {
  if (dtype == TQ_DTYPE_BF16) return __uint_as_float(((uint32_t)h) << 16);
  return __half2float(__ushort_as_half(h));
}

// Round an f32 to the 16-bit activation type and back (the value `t.to(dtype)` holds).
__device__ __forceinline__ float round16(float f, int dtype) {
  if (dtype == TQ_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(f));
  return __half2float(__float2half_rn(f));
}

__device__ __forceinline__ uint16_t f2h(float f, int dtype) {
  if (dtype == TQ_DTYPE_BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  return __half_as_ushort(__float2half_rn(f));
}

// q = clamp(rint(v / s), -127, 127) with the IEEE round-to-nearest f32 quotient
// (quant_utils.py:113-115, quantize_activation.py:70-71).
__device__ __forceinline__ int quant_code(float v, float s) {
  float q = rintf(__fdiv_rn(v, s));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return (int)q;
}

// Same result as quant_code, faster: v * r (r = 1/s rounded) is within 2^-15 of the
// correctly rounded quotient for |v / s| <= 256, so its nearest integer is the
// quotient's unless the product sits within 2^-14 of a half-integer; only those
// rare elements take the exact IEEE division.
__device__ __forceinline__ int quant_code_fast(float v, float s, float r) {
  float t = v * r;
  float k = rintf(t);
  float d = fabsf(t - k);
  if (fabsf(t) >= 256.0f || d > 0.5f - 6.103515625e-05f) k = rintf(__fdiv_rn(v, s));
  k = fminf(fmaxf(k, -127.0f), 127.0f);
  return (int)k;
}

// Maximum over the CTA (every thread gets it); `red` holds 32 floats of shared memory.
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// Activation tile scale from its absmax: the quotient rounded to the 16-bit type, 1 for
// an all-zero tile (quant_utils.py:41-74).
template <int XT>
__device__ __forceinline__ float scale_from_absmax(float amax) {
  return amax > 0.0f ? round16(__fdiv_rn(amax, 127.0f), XT) : 1.0f;
}

__device__ __forceinline__ void report(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records TQ_ERR_TIMEOUT) when
// the phase did not complete within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  report(err, TQ_ERR_TIMEOUT);
  return false;
}

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait that lets the waiting warp sleep instead of spinning: a few plain polls,
// then polls that suspend the thread until the phase completes or `kSleepNs` passes,
// so waiting warps take almost no issue slots from the warps doing the work.  Gives up
// (TQ_ERR_TIMEOUT) after about two seconds.
constexpr uint32_t kSleepNs = 20000;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err) {
#pragma unroll 1
  for (int i = 0; i < 4; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
#pragma unroll 1
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_sleep(bar, parity, kSleepNs)) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  report(err, TQ_ERR_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte async copy with zero fill of the bytes past `src_bytes` (0..16).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int XT>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  if constexpr (XT == TQ_DTYPE_BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

}  // namespace tq

// ----------------------------------------------------------- host helpers

#define TQ_CUDA_TRY(expr)                                   \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return tq_set_cuda_error(_e);    \
  } while (0)

// Check the launch just issued and count it.
#define TQ_LAUNCHED()                                       \
  do {                                                      \
    cudaError_t _e = cudaGetLastError();                    \
    if (_e != cudaSuccess) return tq_set_cuda_error(_e);    \
    tq_count_launch();                                      \
  } while (0)

int tq_set_cuda_error(cudaError_t e);
void tq_count_launch(int n = 1);
int tq_set_error(int code, const char* msg);
int tq_sm_count();
