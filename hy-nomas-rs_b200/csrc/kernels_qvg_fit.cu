// kernels_qvg_fit.cu — the one-time QVG codebook fit on the device:
// QvgCodec::fit / fit_head_codebooks / farthest_point_init
// (cache/qvg.rs:130-167, 351-442), bit-identical to the reference.
//
// One CTA per (layer, side, head) fit.  Each fit owns a residual matrix
// (n tokens x D, f32) in scratch, initialised from the committed K or V and
// updated after every stage with r -= cb[nearest] (f32, one rounding), as the
// reference does.  Every floating-point sum keeps the reference's order:
//   * per-token squared distances: one thread per token, sequential f64 in d
//     (farthest-point distances, nearest entry with strict < so ties keep the
//     lower index; the reference's early exit cannot change the argmin);
//   * Lloyd sums sum_i r_id over the tokens of one entry: one thread per d,
//     sequential f64 in token order (each (entry, d) sum is independent);
//   * the farthest-point total sum_i dmin_i and the weighted pick scan
//     pick -= dmin_i: thread 0, sequential in token order, with the seeded
//     SplitMix64 stream (seed + head, both sides, tensor_utils.rs:65-95).
// Counts per entry are integers (order free).
#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"

namespace nkv {

namespace {

constexpr int FT = 256;  // threads per fit

struct SplitMix64 {
  uint64_t state;
  __device__ uint64_t next() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  // 53 random bits scaled by 2^-53: both steps exact
  __device__ double uniform() { return __dmul_rn(__ull2double_rn(next() >> 11), 1.0 / 9007199254740992.0); }
};

// Index of the entry of cb (E x D) nearest to row x (qvg.rs:303-321).
__device__ int nearest_row(const float* cb, int E, int D, const float* x) {
  int best = 0;
  double best_d = __longlong_as_double(0x7FF0000000000000ll);  // +inf
  for (int e = 0; e < E; ++e) {
    const float* c = cb + (size_t)e * D;
    double acc = 0.0;
    for (int d = 0; d < D; ++d) {
      const double diff = __dsub_rn((double)x[d], (double)c[d]);
      acc = __dadd_rn(acc, __dmul_rn(diff, diff));
      if (acc >= best_d) break;
    }
    if (acc < best_d) {
      best_d = acc;
      best = e;
    }
  }
  return best;
}

}  // namespace

template <int IN_DT>
__global__ void __launch_bounds__(FT) k_qvg_fit(const QvgFitTask* __restrict__ tasks, uint64_t n, int H, int D,
                                                 int stages, int E) {
  extern __shared__ int fit_counts[];  // [E]
  __shared__ uint64_t s_idx;
  __shared__ int s_jitter;
  const QvgFitTask T = tasks[blockIdx.x];
  const int t = threadIdx.x;
  float* res = T.res;  // n x D

  // ---- residual = the committed K or V of this head, as f32
  for (uint64_t j = t; j < n * (uint64_t)D; j += FT) {
    const uint64_t i = j / D, d = j % D;
    res[j] = dev::load_elem<IN_DT>(T.x, (i * H + T.h) * (uint64_t)D + d);
  }
  __syncthreads();
  SplitMix64 rng{T.seed};  // advanced by thread 0 only

  for (int s = 0; s < stages; ++s) {
    float* cb = T.out + (size_t)s * E * D;
    if (n == 0) {  // no rows: zero codebooks (the reference fits nothing)
      for (int j = t; j < E * D; j += FT) cb[j] = 0.0f;
      __syncthreads();
      continue;
    }
    // ---- farthest_point_init (qvg.rs:396-442)
    if (t == 0) s_idx = (uint64_t)(rng.uniform() * (double)n) % n;
    for (uint64_t i = t; i < n; i += FT) T.dmin[i] = __longlong_as_double(0x7FF0000000000000ll);
    __syncthreads();
    for (int d = t; d < D; d += FT) cb[d] = res[s_idx * D + d];
    __syncthreads();
    for (int have = 1; have < E; ++have) {
      const float* last = cb + (size_t)(have - 1) * D;
      for (uint64_t i = t; i < n; i += FT) {
        const float* r = res + i * D;
        double dd = 0.0;
        for (int d = 0; d < D; ++d) {
          const double diff = __dsub_rn((double)r[d], (double)last[d]);
          dd = __dadd_rn(dd, __dmul_rn(diff, diff));
        }
        if (dd < T.dmin[i]) T.dmin[i] = dd;
      }
      __syncthreads();
      if (t == 0) {
        double total = 0.0;
        for (uint64_t i = 0; i < n; ++i) total = __dadd_rn(total, T.dmin[i]);
        if (total <= 1e-12) {
          s_jitter = 1;  // every row coincides with an entry: jitter a copy of the first
        } else {
          s_jitter = 0;
          double pick = __dmul_rn(rng.uniform(), total);
          uint64_t idx = n - 1;
          for (uint64_t i = 0; i < n; ++i) {
            pick = __dsub_rn(pick, T.dmin[i]);
            if (pick <= 0.0) {
              idx = i;
              break;
            }
          }
          s_idx = idx;
        }
      }
      __syncthreads();
      float* dst = cb + (size_t)have * D;
      if (s_jitter) {
        for (int d = t; d < D; d += FT) dst[d] = d == 0 ? __fadd_rn(cb[0], __fmul_rn((float)have, 1e-3f)) : cb[d];
      } else {
        for (int d = t; d < D; d += FT) dst[d] = res[s_idx * D + d];
      }
      __syncthreads();
    }
    // ---- two Lloyd iterations (qvg.rs:365-385)
    for (int it = 0; it < 2; ++it) {
      for (int c = t; c < E; c += FT) fit_counts[c] = 0;
      __syncthreads();
      for (uint64_t i = t; i < n; i += FT) {
        const int c = nearest_row(cb, E, D, res + i * D);
        T.codes[i] = (uint8_t)c;
        atomicAdd(&fit_counts[c], 1);
      }
      __syncthreads();
      for (int d = t; d < D; d += FT) {
        for (int c = 0; c < E; ++c) T.sums[(size_t)c * D + d] = 0.0;
        for (uint64_t i = 0; i < n; ++i) {
          double* sc = T.sums + (size_t)T.codes[i] * D + d;
          *sc = __dadd_rn(*sc, (double)res[i * D + d]);
        }
      }
      __syncthreads();
      for (int j = t; j < E * D; j += FT) {
        const int c = j / D;
        if (fit_counts[c] > 0) cb[j] = __double2float_rn(__ddiv_rn(T.sums[j], (double)fit_counts[c]));
      }
      __syncthreads();
    }
    // ---- subtract each row's nearest entry (qvg.rs:386-392)
    if (s + 1 < stages) {
      for (uint64_t i = t; i < n; i += FT) {
        float* r = res + i * D;
        const float* c = cb + (size_t)nearest_row(cb, E, D, r) * D;
        for (int d = 0; d < D; ++d) r[d] = __fsub_rn(r[d], c[d]);
      }
      __syncthreads();
    }
  }
}

size_t qvg_fit_scratch_bytes(uint64_t n, int D, int E) {
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  return up(n * (size_t)D * 4) + up(n * 8) + up((size_t)E * D * 8) + up(n);
}

cudaError_t launch_qvg_fit(const QvgFitTask* tasks_dev, int n_tasks, int in_dtype, uint64_t n, int H, int D,
                           int stages, int E, cudaStream_t s) {
  if (n_tasks == 0) return cudaSuccess;
  const size_t smem = (size_t)E * sizeof(int);
  switch (in_dtype) {
    case F32: k_qvg_fit<F32><<<n_tasks, FT, smem, s>>>(tasks_dev, n, H, D, stages, E); break;
    case BF16: k_qvg_fit<BF16><<<n_tasks, FT, smem, s>>>(tasks_dev, n, H, D, stages, E); break;
    default: k_qvg_fit<F16><<<n_tasks, FT, smem, s>>>(tasks_dev, n, H, D, stages, E); break;
  }
  return cudaGetLastError();
}

}  // namespace nkv
