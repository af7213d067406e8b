// Exhaustive checks of the two shortcuts the INT8 quantizer takes instead of
// quantize_one's IEEE division and round (cache/int8.rs:65-81), over their
// whole domains, with the device functions the product uses (nkv_quant.cuh):
//
//  1. Markstein quotient.  For every finite bf16 peak p > 0 whose scale
//     s = RN(RN(p * RN(1/127)) + 0) lies in [FLT_MIN, 1e37] (the fast path's
//     range) and every bf16 x with |x| <= p (a value of that row):
//     q1 = fma(|x| - s q0, r, q0) with q0 = RN(|x| r), r = RN(1/s), against
//     RN(|x| / s); the pairs where they differ are counted by the magnitude of
//     the quotient (>= 1/2, [2^-24, 1/2), normal below 2^-24, subnormal), and
//     so are those off by more than one ulp.
//  2. Round half away from zero.  For every f32 q in [0, 128]:
//     floor(RN(q + (0.5 - 2^-25))), taken as RZ(RN(q + C) + 1.5*2^23) - 1.5*2^23,
//     equals roundf(q).
//  3. The whole code.  For the pairs of (1), the scalar code_bits and both
//     lanes of the packed code_bits2 give the byte quant_exact (the IEEE
//     division path) gives.
//
// Built and run by tests/test_gpu_quant_identities.py; prints the pair
// counts and the mismatch counts.
#include <cfloat>
#include <cstdio>

#include "nkv_quant.cuh"

__global__ void check_pairs(unsigned long long* out) {
  // out: [0] pairs checked, [1] quotient mismatches at quotients >= 1/2,
  // [2] scalar code mismatches, [3] packed code mismatches, [4] fast-path
  // peaks, [7] quotient mismatches in [2^-24, 1/2), [8] ... normal below
  // 2^-24, [9] ... subnormal, [10] quotients off by more than one ulp
  unsigned long long pairs = 0, bad_q = 0, bad_c = 0, bad_c2 = 0, peaks = 0, q_mid = 0, q_small = 0, q_sub = 0,
                     q_far = 0;
  const float inv127 = (float)(1.0 / 127.0);
  for (uint32_t pb = 1 + blockIdx.x; pb < 0x7F80u; pb += gridDim.x) {
    const float p = __uint_as_float(pb << 16);
    const float s = __fadd_rn(__fmul_rn(p, inv127), 0.0f);
    if (!(s >= FLT_MIN && s <= 1e37f)) continue;
    if (threadIdx.x == 0) ++peaks;
    const float r = __frcp_rn(s);
    for (uint32_t xb = threadIdx.x; xb <= 0x7F80u; xb += blockDim.x) {
      if ((xb << 16) > (pb << 16)) break;  // |x| > p
      const float ax = __uint_as_float(xb << 16);
      // (1) the corrected quotient against the IEEE division
      const float q0 = __fmul_rn(ax, r);
      const float e = __fmaf_rn(-q0, s, ax);
      const float q1 = __fmaf_rn(e, r, q0);
      const float qx = __fdiv_rn(ax, s);
      if (__float_as_uint(q1) != __float_as_uint(qx)) {
        if (qx >= 0.5f) ++bad_q;
        else if (qx >= 0x1p-24f) ++q_mid;
        else if (qx >= FLT_MIN) ++q_small;
        else ++q_sub;
        const int32_t dist = (int32_t)__float_as_uint(q1) - (int32_t)__float_as_uint(qx);
        q_far += dist > 1 || dist < -1;
      }
      // (3) the code of +x and -x, scalar and packed, against quant_exact
      for (int sg = 0; sg < 2; ++sg) {
        const float x = sg ? -ax : ax;
        const uint32_t want = nkv::quant_exact(x, s);
        const uint32_t got = (nkv::code_bits(x, s, r) & 0xFFu) ^ 0x80u;
        bad_c += got != want;
        ++pairs;
      }
      const uint2 c2 = nkv::code_bits2(make_float2(ax, -ax), s, r);
      bad_c2 += ((c2.x & 0xFFu) ^ 0x80u) != nkv::quant_exact(ax, s);
      bad_c2 += ((c2.y & 0xFFu) ^ 0x80u) != nkv::quant_exact(-ax, s);
    }
  }
  atomicAdd(out + 0, pairs);
  if (bad_q) atomicAdd(out + 1, bad_q);
  if (bad_c) atomicAdd(out + 2, bad_c);
  if (bad_c2) atomicAdd(out + 3, bad_c2);
  if (peaks) atomicAdd(out + 4, peaks);
  if (q_mid) atomicAdd(out + 7, q_mid);
  if (q_small) atomicAdd(out + 8, q_small);
  if (q_sub) atomicAdd(out + 9, q_sub);
  if (q_far) atomicAdd(out + 10, q_far);
}

__global__ void check_rounding(unsigned long long* out) {
  // out: [5] values checked, [6] mismatches
  const float M = 12582912.0f;  // 1.5 * 2^23
  unsigned long long n_checked = 0, bad = 0;
  const uint32_t last = 0x43000000u;  // 128.0f
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= last; i += stride) {
    const float q = __uint_as_float((uint32_t)i);
    const float z = __fadd_rz(__fadd_rn(q, 0.49999997f), M);
    const float n = __fadd_rn(z, -M);
    bad += __float_as_uint(n) != __float_as_uint(roundf(q));
    ++n_checked;
  }
  atomicAdd(out + 5, n_checked);
  if (bad) atomicAdd(out + 6, bad);
}

int main() {
  unsigned long long* d = nullptr;
  if (cudaMalloc(&d, 16 * sizeof(unsigned long long)) != cudaSuccess) return 2;
  if (cudaMemset(d, 0, 16 * sizeof(unsigned long long)) != cudaSuccess) return 2;
  check_pairs<<<148 * 8, 256>>>(d);
  check_rounding<<<148 * 16, 256>>>(d);
  unsigned long long h[16];
  if (cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
  cudaFree(d);
  printf("pairs %llu quotient_mismatches_ge_half %llu code_mismatches %llu packed_code_mismatches %llu "
         "fast_peaks %llu rounding_values %llu rounding_mismatches %llu quotient_mismatches_mid %llu "
         "quotient_mismatches_small_normal %llu quotient_mismatches_subnormal %llu quotient_off_by_more_than_1ulp "
         "%llu\n",
         h[0], h[1], h[2], h[3], h[4], h[5], h[6], h[7], h[8], h[9], h[10]);
  return 0;
}
