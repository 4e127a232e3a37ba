// exact_math.cuh — arithmetic whose bits must not depend on the compiler or the device.
//
// The sampler's draw contract (Philox uniform, yexp, sequential FP32 sums) must give the
// same bits on the GPU and in the CPU restatement used by the parity tests. Every
// operation here is a single IEEE float32 operation written with the _rn intrinsics on
// the device (nvcc would otherwise contract a*b+c into an FMA) and compiled with
// -ffp-contract=off on the host.
#pragma once
#include <cstdint>
#include <cmath>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__)
#define YAR_HD __host__ __device__ __forceinline__
#else
#define YAR_HD inline
#endif

namespace yar {

YAR_HD float f_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  volatile float r = a * b;
  return r;
#endif
}
YAR_HD float f_add(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  volatile float r = a + b;
  return r;
#endif
}
YAR_HD float f_sub(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  volatile float r = a - b;
  return r;
#endif
}
YAR_HD float f_div(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  volatile float r = a / b;
  return r;
#endif
}
YAR_HD float f_rint(float a) {
#if defined(__CUDA_ARCH__)
  return rintf(a);
#else
  return std::nearbyint(a);
#endif
}
YAR_HD float bits_to_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}
YAR_HD uint32_t f32_to_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}

// BF16 <-> FP32 on raw bits (round to nearest, ties to even; NaN kept quiet).
YAR_HD uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
    return uint16_t((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
YAR_HD float bf16_bits_to_f32(uint16_t b) { return bits_to_f32(uint32_t(b) << 16); }
YAR_HD float round_bf16(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

// exp(x) for x <= 0: Cody–Waite reduction x = n*ln2 + r with ln 2 split into a
// short high part (n*LN2_HI is exact for |n| < 2^7) and a low part, then the degree-7
// Taylor polynomial of e^r in Horner form, then scaling by 2^n. Arguments below -87
// (and NaN / -inf) flush to zero, which keeps 2^n a normal number.
constexpr float kLn2Hi = 0.693145751953125f;
constexpr float kLn2Lo = 1.428606765330187e-06f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kExpFlush = -87.0f;

YAR_HD float yexp(float x) {
  if (!(x >= kExpFlush)) return 0.0f;
  const float n = f_rint(f_mul(x, kLog2e));
  const float r = f_sub(f_sub(x, f_mul(n, kLn2Hi)), f_mul(n, kLn2Lo));
  float p = float(1.0 / 5040.0);
  p = f_add(f_mul(p, r), float(1.0 / 720.0));
  p = f_add(f_mul(p, r), float(1.0 / 120.0));
  p = f_add(f_mul(p, r), float(1.0 / 24.0));
  p = f_add(f_mul(p, r), float(1.0 / 6.0));
  p = f_add(f_mul(p, r), 0.5f);
  p = f_add(f_mul(p, r), 1.0f);
  p = f_add(f_mul(p, r), 1.0f);
  const int ni = int(n);
  return f_mul(p, bits_to_f32(uint32_t(ni + 127) << 23));
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as
// 1, 2, 3", SC'11): multipliers, Weyl key increments and round structure as published.
struct Philox4 {
  uint32_t v[4];
};
YAR_HD void mulhilo32(uint32_t a, uint32_t b, uint32_t &hi, uint32_t &lo) {
#if defined(__CUDA_ARCH__)
  hi = __umulhi(a, b);
  lo = a * b;
#else
  const uint64_t p = uint64_t(a) * uint64_t(b);
  hi = uint32_t(p >> 32);
  lo = uint32_t(p);
#endif
}
YAR_HD Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                             uint32_t k1) {
  for (int round = 0; round < 10; ++round) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(0xD2511F53u, c0, hi0, lo0);
    mulhilo32(0xCD9E8D57u, c2, hi1, lo1);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    if (round < 9) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
  }
  return Philox4{{c0, c1, c2, c3}};
}
// The per-step FP32 uniform in [0, 1): top 24 bits of word 0 of Philox((step, stream,
// 0, 0), (seed_lo, seed_hi)) times 2^-24.
YAR_HD float step_uniform(uint64_t seed, uint32_t step, uint32_t stream) {
  const Philox4 r = philox4x32_10(step, stream, 0u, 0u, uint32_t(seed), uint32_t(seed >> 32));
  return float(r.v[0] >> 8) * (1.0f / 16777216.0f);
}

// Order-preserving map of FP32 to uint32 (ascending keys <=> ascending floats).
YAR_HD uint32_t f32_order_key(float f) {
  const uint32_t u = f32_to_bits(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
YAR_HD float f32_from_order_key(uint32_t k) {
  return bits_to_f32((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

}  // namespace yar
