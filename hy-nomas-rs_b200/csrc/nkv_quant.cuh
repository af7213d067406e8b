// nkv_quant.cuh — per-value INT8 code arithmetic of quantize_one
// (cache/int8.rs:65-81), shared by the commit kernels and the fused K/V
// projection epilogue.  The derivation (Markstein quotient, half-away-from-
// zero rounding by the 1.5 * 2^23 constant) is described where the commit
// kernels use it (kernels_commit.cu).
#pragma once
#include <cfloat>
#include <cstdint>

#include "nkv_device.cuh"

namespace nkv {

// round_half_away(x / s) + 128 as a byte, with an IEEE division: the path
// for scales outside [FLT_MIN, 1e37].
__device__ __forceinline__ uint32_t quant_exact(float x, float s) {
  float t = roundf(__fdiv_rn(x, s));
  t = dev::cmin(dev::cmax(t, -127.0f), 127.0f);
  t = __fadd_rn(__fmul_rn(t, 1.0f), 128.0f);
  t = dev::cmin(dev::cmax(t, 0.0f), 255.0f);
  return dev::as_u8(t);
}

// Code of one value: the f32 M + round_half_away(RN(x / s)) with
// M = 1.5 * 2^23, whose binade has unit spacing, so the low byte of the bit
// pattern is the rounded quotient mod 256 (pack4 turns it into the code by
// XOR 0x80); valid for s in [FLT_MIN, 1e37] with r = RN(1/s) and
// |x / s| < 128.
//  * RN(|x| / s) without a divide: q0 = RN(|x| r), the residual
//    e = |x| - s q0 exact by an FMA, q1 = RN(q0 + e r) (Markstein) wherever
//    the quotient is normal (a subnormal quotient rounds to 0 either way);
//  * round half away from zero of q1 >= 0 is floor(RN(q1 + C)) with
//    C = 0.5 - 2^-25 (true for every f32 in [0, 128]);
//  the two identities and the resulting code byte are checked on the device
//  for every bf16 value and row peak (tests/test_gpu_quant_identities.py);
//    adding M with round-toward-zero takes the floor and leaves n in the low
//    bits, and M + sign(x) n (an exact FMA) puts the sign back.
__device__ __forceinline__ uint32_t code_bits(float x, float s, float r) {
  const float M = 12582912.0f;  // 1.5 * 2^23
  const float ax = fabsf(x);
  const float q0 = __fmul_rn(ax, r);
  const float e = __fmaf_rn(-q0, s, ax);
  const float q1 = __fmaf_rn(e, r, q0);                          // RN(|x| / s)
  const float z = __fadd_rz(__fadd_rn(q1, 0.49999997f), M);      // M + n
  const float n = __fadd_rn(z, -M);                              // n, exact
  return __float_as_uint(__fmaf_rn(copysignf(1.0f, x), n, M));   // M + sign(x) n, exact
}

// code_bits of two values at once on packed f32x2 operations: the same
// roundings lane by lane (every step is a single add, multiply or fused
// multiply-add, so nothing can be contracted across steps).
__device__ __forceinline__ uint2 code_bits2(float2 x, float s, float r) {
  const float2 M = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const float2 C = make_float2(0.49999997f, 0.49999997f);
  const float2 s2 = make_float2(s, s), r2 = make_float2(r, r);
  const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 q0 = __fmul2_rn(ax, r2);
  const float2 e = __ffma2_rn(make_float2(-q0.x, -q0.y), s2, ax);
  const float2 q1 = __ffma2_rn(e, r2, q0);                        // RN(|x| / s)
  const float2 z = __fadd2_rz(__fadd2_rn(q1, C), M);              // M + n
  const float2 n = __fadd2_rn(z, make_float2(-M.x, -M.y));        // n, exact
  const float2 o = __ffma2_rn(make_float2(copysignf(1.0f, x.x), copysignf(1.0f, x.y)), n, M);
  return make_uint2(__float_as_uint(o.x), __float_as_uint(o.y));
}

__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410) ^ 0x80808080u;
}

// Lane-wise max(|a|, |b|) of two bf16 pairs (the sign bit is the XOR of the
// operands' and is masked off by the caller); a NaN lane yields a NaN, so
// one instruction per pair serves both the peak and the non-finite scan.
__device__ __forceinline__ uint32_t maxabs_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

}  // namespace nkv
