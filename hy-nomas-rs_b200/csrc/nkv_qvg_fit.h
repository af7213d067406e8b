// nkv_qvg_fit.h — host-side QVG codebook fit (cache/qvg.rs:130-167, 351-442).
#pragma once

#include <cstddef>
#include <cstdint>

namespace nkv {

// fit_head_codebooks: mat is n x D f32, out is stages x E x D f32.
void qvg_fit_head(const float* mat, size_t n, size_t D, int stages, int E, uint64_t seed, float* out);

// QvgCodec::fit for one layer: k, v are (L, H, D) f32 host arrays; out is
// [2][H][stages][E][D]; `threads` host threads share the 2*H head fits.
void qvg_fit_layer(const float* k, const float* v, size_t L, size_t H, size_t D, int stages, int E, uint64_t seed,
                   float* out, int threads);

}  // namespace nkv
