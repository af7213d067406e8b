// Exhaustive check that the hardware pair converters used on the
// no-NaN fast paths (dev::bf16x2_bits_nonnan, dev::f16x2_bits_nonnan) give
// the same bits as the library's reference-exact integer conversions
// (dev::bf16_bits, dev::f16_bits) for every non-NaN f32 bit pattern.
// Built and run by tests/test_gpu_kernels.py; prints the mismatch counts.
#include <cstdio>

#include "nkv_device.cuh"

__global__ void check(unsigned long long* bad) {
  unsigned long long nb = 0, nh = 0;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
    const uint32_t u = (uint32_t)i;
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) continue;  // NaN
    const float x = __uint_as_float(u);
    const float y = __uint_as_float(u ^ 0x80000000u);  // the second lane sees the negated value
    const uint32_t pb = nkv::dev::bf16x2_bits_nonnan(x, y);
    nb += (pb & 0xFFFFu) != (nkv::dev::bf16_bits(x) & 0xFFFFu);
    nb += (pb >> 16) != (nkv::dev::bf16_bits(y) & 0xFFFFu);
    const uint32_t ph = nkv::dev::f16x2_bits_nonnan(x, y);
    nh += (ph & 0xFFFFu) != (nkv::dev::f16_bits(x) & 0xFFFFu);
    nh += (ph >> 16) != (nkv::dev::f16_bits(y) & 0xFFFFu);
  }
  if (nb) atomicAdd(bad, nb);
  if (nh) atomicAdd(bad + 1, nh);
}

int main() {
  unsigned long long* d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(unsigned long long)) != cudaSuccess) return 2;
  cudaMemset(d, 0, 2 * sizeof(unsigned long long));
  check<<<148 * 16, 256>>>(d);
  unsigned long long h[2] = {~0ull, ~0ull};
  if (cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
  cudaFree(d);
  printf("bf16_mismatches %llu f16_mismatches %llu\n", h[0], h[1]);
  return 0;
}
