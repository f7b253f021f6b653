// Shared definitions for the llmq kernels (sm_100a).
//
// Float arithmetic follows the reference's operation order exactly, so the
// library is compiled with -fmad=false: every a*b+c the reference writes as
// two operations stays two roundings, and fmaf() is used where the reference
// calls .fma. exp and tanh are this library's own (Cody-Waite reduction plus
// Taylor polynomials, IEEE add/mul/fma/div only), so they give the same bits
// wherever they run.
#pragma once

#include <climits>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#define LLMQ_HD __host__ __device__ __forceinline__

namespace llmq {

LLMQ_HD float bits_to_float(uint32_t b) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  __builtin_memcpy(&f, &b, 4);
  return f;
#endif
}

LLMQ_HD uint32_t float_to_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t b;
  __builtin_memcpy(&b, &f, 4);
  return b;
#endif
}

// IEEE binary16 bits -> float (exact).
LLMQ_HD float half_bits_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (exp == 0x1F) return bits_to_float(sign | 0x7F800000u | (man << 13));
  if (exp == 0) {
    if (man == 0) return bits_to_float(sign);
    // subnormal: man * 2^-24, exact in float
    float f = (float)man * bits_to_float(0x33800000u);  // 2^-24
    return (sign ? -f : f);
  }
  return bits_to_float(sign | ((exp + 112u) << 23) | (man << 13));
}

LLMQ_HD float pow2i(int k) { return bits_to_float((uint32_t)(k + 127) << 23); }

// e^x: k = rint(x log2 e); r = x - k ln2 with ln2 split in a high and a low
// part (Cody and Waite); e^r by its Taylor series through r^7; times 2^k,
// in two steps when the result is subnormal so that it rounds once.
LLMQ_HD float lm_expf(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return bits_to_float(0x7F800000u);
  if (x < -103.972084f) return 0.0f;
  float k = rintf(x * 1.44269502f);
  float r = fmaf(-k, 0.693145751953125f, x);
  r = fmaf(-k, 1.42860677e-06f, r);
  float p = (float)(1.0 / 5040.0);
  p = fmaf(p, r, (float)(1.0 / 720.0));
  p = fmaf(p, r, (float)(1.0 / 120.0));
  p = fmaf(p, r, (float)(1.0 / 24.0));
  p = fmaf(p, r, (float)(1.0 / 6.0));
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ki = (int)k;
  if (ki > 127) return (p * pow2i(127)) * 2.0f;
  if (ki < -125) return (p * pow2i(ki + 24)) * pow2i(-24);
  return p * pow2i(ki);
}

// tanh: the odd Taylor polynomial through a^15 below 0.5, otherwise
// 1 - 2 / (e^(2a) + 1), and 1 beyond 9.
LLMQ_HD float lm_tanhf(float x) {
  float a = fabsf(x);
  float t;
  if (a != a) return x;
  if (a < 0.5f) {
    float z = a * a;
    float p = (float)(-929569.0 / 638512875.0);
    p = fmaf(p, z, (float)(21844.0 / 6081075.0));
    p = fmaf(p, z, (float)(-1382.0 / 155925.0));
    p = fmaf(p, z, (float)(62.0 / 2835.0));
    p = fmaf(p, z, (float)(-17.0 / 315.0));
    p = fmaf(p, z, (float)(2.0 / 15.0));
    p = fmaf(p, z, (float)(-1.0 / 3.0));
    t = fmaf(a * z, p, a);
  } else if (a > 9.0f) {
    t = 1.0f;
  } else {
    float e = lm_expf(2.0f * a);
    t = 1.0f - 2.0f / (e + 1.0f);
  }
  return copysignf(t, x);
}

// GELU-tanh in the order of kernels.mojo:43-45 (store_out) and :277-279
// (finish): 0.5 * r * (1 + tanh(s * (r + 0.044715 * r * r * r))).
LLMQ_HD float gelu(float r) {
  const float s = 0.7978845608028654f;
  float inner = r + ((0.044715f * r) * r) * r;
  return (0.5f * r) * (1.0f + lm_tanhf(s * inner));
}

// round(x), halfway cases away from zero (Mojo's `round`), as an int, for
// |x| < 2^31: the nearest-even integer from one rounding instruction, then
// exact ties moved away from zero (x - rint(x) is exact here, and x +- 0.5
// is an exact integer at a tie).
__device__ __forceinline__ int round_away(float x) {
  float r = rintf(x);
  float d = x - r;
  if (fabsf(d) == 0.5f) r = x + copysignf(0.5f, x);
  return (int)r;
}

// s16 x u8 pair products: c + a.lo16*b.byte0 + a.hi16*b.byte1 (lo) or with
// bytes 2 and 3 (hi). Exact int32 arithmetic (wraps mod 2^32).
__device__ __forceinline__ int dp2a_lo_su(int a, unsigned b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_su(int a, unsigned b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Packed float pairs: the f32x2 operations of sm_100 are two independent
// IEEE operations, each rounded to nearest once, the same as their scalar
// forms, at one instruction per pair.
__device__ __forceinline__ unsigned long long f2_bits(int a, int b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_pair(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(unsigned long long v, float &a, float &b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}


}  // namespace llmq
