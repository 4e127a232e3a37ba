// common.cuh — device helpers shared by the kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "engine.h"
#include "exact_math.cuh"

namespace yar {

// Programmatic dependent launch: a kernel launched with the programmatic-serialization
// attribute may start while its predecessor is still running; everything before
// pdl_wait() must not read the predecessor's outputs (weights and old KV are fine).
// Without the attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16-byte streaming load of data read once per step (weights): no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg16(const void *p) {
  return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// SiLU with FP32 opmath, x / (1 + exp(-x)), then one rounding by the caller.
__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + expf(-x)); }

// RMSNorm scale rounded to BF16 (modeling_yue2.py:132: rsqrt(mean + eps).to(bf16)).
__device__ __forceinline__ float rms_scale_bf16(float sum_sq, int n, float eps) {
  const float var = sum_sq / float(n);
  return rbf(1.0f / sqrtf(var + eps));
}

}  // namespace yar
