// nkv_device.cuh — device-side numerics shared by the cache kernels.
//
// The reference rounds through candle 0.11.1 and half 2.7.1; these helpers
// reproduce those conversions bit for bit with integer operations instead of
// the hardware converters (whose NaN payload handling differs from half's).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "nkv_kernels.h"

namespace nkv {
namespace dev {

// f32 -> bf16 bits, round to nearest even; a NaN keeps its top payload bits
// and gets the quiet bit (half's f32_to_bf16).
__device__ __forceinline__ uint32_t bf16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (u >> 16) | 0x40u;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
// Two f32 -> packed bf16 pair (a in the low half) by the hardware converter:
// round to nearest even, equal to bf16_bits for every non-NaN input (checked
// over all 2^32 patterns by tests/cuda/convert_check.cu); only NaN payloads
// differ, so callers use it where no input can be NaN.
__device__ __forceinline__ uint32_t bf16x2_bits_nonnan(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// The same for IEEE binary16 (equal to f16_bits for every non-NaN input).
__device__ __forceinline__ uint32_t f16x2_bits_nonnan(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// bf16 bits -> f32 (half's bf16_to_f32: NaN gets the quiet bit).
__device__ __forceinline__ float bf16_value(uint32_t b) {
  b &= 0xFFFFu;
  if ((b & 0x7FFFu) > 0x7F80u) b |= 0x40u;
  return __uint_as_float(b << 16);
}

// f32 -> IEEE binary16 bits, round to nearest even; NaN as x86 F16C / half.
__device__ __forceinline__ uint32_t f16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u)
    return ((u >> 16) & 0x8000u) | 0x7C00u | 0x0200u | ((u & 0x007FFFFFu) >> 13);
  return __half_as_ushort(__float2half_rn(x));
}
// binary16 bits -> f32 (exact; NaN gets the quiet bit).
__device__ __forceinline__ float f16_value(uint32_t h) {
  h &= 0xFFFFu;
  uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  if (exp == 0x1Fu) return __uint_as_float(sign | 0x7F800000u | (man ? (0x00400000u | (man << 13)) : 0u));
  return __half2float(__ushort_as_half((unsigned short)h));
}

// Round an f32 to the value set of dtype DT (candle to_dtype), as f32.
template <int DT>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (DT == BF16) return bf16_value(bf16_bits(x));
  else if constexpr (DT == F16) return f16_value(f16_bits(x));
  else return x;
}

// Element i of a raw buffer of dtype DT, as f32.
template <int DT>
__device__ __forceinline__ float load_elem(const void* p, uint64_t i) {
  if constexpr (DT == F32) return __ldg(static_cast<const float*>(p) + i);
  else if constexpr (DT == BF16) return bf16_value(__ldg(static_cast<const unsigned short*>(p) + i));
  else return f16_value(__ldg(static_cast<const unsigned short*>(p) + i));
}

// Store an f32 that is already in the value set of DT (or is to be rounded).
template <int DT>
__device__ __forceinline__ void store_elem(void* p, uint64_t i, float v) {
  if constexpr (DT == F32) static_cast<float*>(p)[i] = v;
  else if constexpr (DT == BF16) static_cast<unsigned short*>(p)[i] = (unsigned short)bf16_bits(v);
  else static_cast<unsigned short*>(p)[i] = (unsigned short)f16_bits(v);
}

// 8 consecutive elements starting at element i (i multiple of 8, buffer
// 16-byte aligned) as f32.
template <int DT>
__device__ __forceinline__ void load8(const void* p, uint64_t i, float (&x)[8]) {
  if constexpr (DT == F32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    float4 a = __ldg(q), b = __ldg(q + 1);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  } else {
    uint4 w = __ldg(reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(p) + i));
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (DT == BF16) {
        x[2 * j] = bf16_value(ws[j] & 0xFFFFu);
        x[2 * j + 1] = bf16_value(ws[j] >> 16);
      } else {
        x[2 * j] = f16_value(ws[j] & 0xFFFFu);
        x[2 * j + 1] = f16_value(ws[j] >> 16);
      }
    }
  }
}

// candle's maximum / minimum (a < b ? b : a, a > b ? b : a): a NaN first
// operand survives, unlike fmaxf / fminf.
__device__ __forceinline__ float cmax(float a, float b) { return a < b ? b : a; }
__device__ __forceinline__ float cmin(float a, float b) { return a > b ? b : a; }

// Rust `v as u8` for f32: saturating, NaN -> 0.
__device__ __forceinline__ uint32_t as_u8(float v) {
  if (!(v == v) || v <= 0.0f) return 0u;
  if (v >= 255.0f) return 255u;
  return (uint32_t)v;
}

// SplitMix64 finalizer (tensor_utils.rs:75-81 without the state step).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace dev
}  // namespace nkv
