// g4_common.cuh -- sm_100a building blocks shared by the gemma4.kt B200 kernels:
// mbarrier + cp.async.bulk (TMA, non-tensor, one CTA) staging, bounded
// waits that report a timeout instead of hanging, and GGML block constants.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4 {

// GGML type ids (GGMLType.kt:16-46)
enum GgmlType : int {
  F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_1 = 7, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14, BF16 = 30, MXFP4 = 39
};

// Error bits written to the context's device status word.
enum DevErr : unsigned { ERR_TIMEOUT_FULL = 1u, ERR_TIMEOUT_EMPTY = 2u, ERR_TIMEOUT_DRAIN = 4u,
                         ERR_BAD_ARG = 8u };

__host__ __device__ constexpr int block_size(int t) {
  return (t == Q8_0 || t == Q4_0 || t == Q4_1 || t == Q5_1 || t == MXFP4) ? 32
         : (t == Q4_K || t == Q5_K || t == Q6_K)                          ? 256
                                                                          : 1;
}
__host__ __device__ constexpr int type_size(int t) {
  return t == F32 ? 4 : t == F16 ? 2 : t == BF16 ? 2 : t == Q8_0 ? 34 : t == Q4_K ? 144 : t == Q6_K ? 210
       : t == Q4_0 ? 18 : t == Q4_1 ? 20 : t == Q5_1 ? 24 : t == Q5_K ? 176 : t == MXFP4 ? 17 : 0;
}

// A bounded wait gives up after this many nanoseconds of %globaltimer.  Far
// above any legitimate stall: only a logic error can reach it.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy (cp.async, L2 only); completion by commit groups.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// the caller records an error) if it has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// 1-D bulk copy global -> shared (cp.async.bulk into this CTA).  dst, src and
// bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: wait for the grids this one depends on
// (no-op when launched without the attribute), and let the next grid launch.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void record_error(unsigned* status, unsigned bits) {
  if (status) atomicOr(status, bits);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint32_t lds32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint16_t lds16(const void* p) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)));
  return v;
}

// 16 bytes from a shared address that is only 2-byte aligned.
__device__ __forceinline__ void lds16B_unaligned(const uint8_t* p, uint32_t w[4]) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  uint32_t sh = (uint32_t)(a & 3u) * 8u;
  uint32_t r0 = lds32(base), r1 = lds32(base + 4), r2 = lds32(base + 8), r3 = lds32(base + 12);
  if (sh == 0) {
    w[0] = r0; w[1] = r1; w[2] = r2; w[3] = r3;
    return;
  }
  uint32_t r4 = lds32(base + 16);
  w[0] = __funnelshift_r(r0, r1, sh);
  w[1] = __funnelshift_r(r1, r2, sh);
  w[2] = __funnelshift_r(r2, r3, sh);
  w[3] = __funnelshift_r(r3, r4, sh);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the CTA, the same fixed order in every CTA; red holds >= 33 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < nw ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// Llama.gelu (Llama.kt:23-25): double precision, rounded to float.
__device__ __forceinline__ float gelu_ref(float x) {
  double xd = (double)x;
  double inner = 0.7978845608028654 * (xd + 0.044715 * (xd * xd * xd));
  return (float)(0.5 * xd * (1.0 + tanh(inner)));
}

// rmsnorm's scale (Llama.kt:28-31): ss / size + eps in float, 1/sqrt in double.
__device__ __forceinline__ float rms_scale(float ss, int size, float eps) {
  ss = __fdiv_rn(ss, (float)size);
  ss = __fadd_rn(ss, eps);
  return (float)(1.0 / sqrt((double)ss));
}

}  // namespace g4
