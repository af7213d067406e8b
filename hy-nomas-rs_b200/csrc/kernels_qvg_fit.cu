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
constexpr size_t kFitCountsBytes = 256 * sizeof(int);  // E <= 256 (8 bits per stage)
constexpr size_t kFitSharedSums = 40 * 1024;           // Lloyd sums in shared memory up to this size
constexpr size_t kFitSharedDmin = 96 * 1024;           // farthest-point distances likewise (n <= 12,288)

// Dynamic shared memory of one fit: counts, then the Lloyd sums and the
// farthest-point distances when each fits its budget (else global scratch).
__host__ __device__ size_t fit_smem_bytes(uint64_t n, int D, int E, size_t* sums_off, size_t* dmin_off) {
  size_t off = kFitCountsBytes;
  const size_t sums = (size_t)E * D * 8, dmin = (size_t)n * 8;
  *sums_off = sums <= kFitSharedSums ? off : 0;
  off += sums <= kFitSharedSums ? sums : 0;
  *dmin_off = dmin <= kFitSharedDmin ? off : 0;
  off += dmin <= kFitSharedDmin ? dmin : 0;
  return off;
}

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

// head_dim 128 (the default): a token's residual row lives in registers for
// a whole pass, loaded with 32 vector loads issued up front.
constexpr int RD = 128;
struct Row128 {
  float4 v[RD / 4];
};
__device__ __forceinline__ void load_row(const float* r, Row128& x) {
#pragma unroll
  for (int k = 0; k < RD / 4; ++k) x.v[k] = reinterpret_cast<const float4*>(r)[k];
}
// sequential f64 sum_d (x_d - c_d)^2 over float4 chunks [K0, K1), continuing
// acc (compile-time bounds keep the row in registers)
template <int K0, int K1>
__device__ __forceinline__ double dist_chunks(const Row128& x, const float* c, double acc) {
#pragma unroll
  for (int k = K0; k < K1; ++k) {
    const float4 c4 = reinterpret_cast<const float4*>(c)[k];
    double diff = __dsub_rn((double)x.v[k].x, (double)c4.x);
    acc = __dadd_rn(acc, __dmul_rn(diff, diff));
    diff = __dsub_rn((double)x.v[k].y, (double)c4.y);
    acc = __dadd_rn(acc, __dmul_rn(diff, diff));
    diff = __dsub_rn((double)x.v[k].z, (double)c4.z);
    acc = __dadd_rn(acc, __dmul_rn(diff, diff));
    diff = __dsub_rn((double)x.v[k].w, (double)c4.w);
    acc = __dadd_rn(acc, __dmul_rn(diff, diff));
  }
  return acc;
}
// nearest_row for a register row; the early exit is checked every 32 values
// (a partial sum already >= the best can only grow, so the argmin is the same)
__device__ __forceinline__ int nearest_row128(const float* cb, int E, const Row128& x) {
  int best = 0;
  double best_d = __longlong_as_double(0x7FF0000000000000ll);
  for (int e = 0; e < E; ++e) {
    const float* c = cb + (size_t)e * RD;
    double acc = dist_chunks<0, 8>(x, c, 0.0);
    if (!(acc >= best_d)) acc = dist_chunks<8, 16>(x, c, acc);
    if (!(acc >= best_d)) acc = dist_chunks<16, 24>(x, c, acc);
    if (!(acc >= best_d)) acc = dist_chunks<24, 32>(x, c, acc);
    if (acc < best_d) {
      best_d = acc;
      best = e;
    }
  }
  return best;
}

}  // namespace

template <int IN_DT>
__global__ void __launch_bounds__(FT, 1) k_qvg_fit(const QvgFitTask* __restrict__ tasks, uint64_t n, int H, int D,
                                                 int stages, int E) {
  // dynamic shared memory: [E] counts, then (when they fit) the [E][D] Lloyd
  // sums and the [n] farthest-point distances
  extern __shared__ __align__(16) unsigned char fit_smem[];
  size_t sums_off, dmin_off;
  fit_smem_bytes(n, D, E, &sums_off, &dmin_off);
  int* fit_counts = reinterpret_cast<int*>(fit_smem);
  __shared__ uint64_t s_idx;
  __shared__ int s_jitter;
  const QvgFitTask T = tasks[blockIdx.x];
  const int t = threadIdx.x;
  float* res = T.res;  // n x D
  double* sums = sums_off ? reinterpret_cast<double*>(fit_smem + sums_off) : T.sums;
  double* dmin = dmin_off ? reinterpret_cast<double*>(fit_smem + dmin_off) : T.dmin;

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
    for (uint64_t i = t; i < n; i += FT) dmin[i] = __longlong_as_double(0x7FF0000000000000ll);
    __syncthreads();
    for (int d = t; d < D; d += FT) cb[d] = res[s_idx * D + d];
    __syncthreads();
    for (int have = 1; have < E; ++have) {
      const float* last = cb + (size_t)(have - 1) * D;
      for (uint64_t i = t; i < n; i += FT) {
        const float* r = res + i * D;
        double dd = 0.0;
        if (D == RD) {
          Row128 x;
          load_row(r, x);
          dd = dist_chunks<0, RD / 4>(x, last, 0.0);
        } else {
          for (int d = 0; d < D; ++d) {
            const double diff = __dsub_rn((double)r[d], (double)last[d]);
            dd = __dadd_rn(dd, __dmul_rn(diff, diff));
          }
        }
        if (dd < dmin[i]) dmin[i] = dd;
      }
      __syncthreads();
      if (t == 0) {
        double total = 0.0;
#pragma unroll 4
        for (uint64_t i = 0; i < n; ++i) total = __dadd_rn(total, dmin[i]);
        if (total <= 1e-12) {
          s_jitter = 1;  // every row coincides with an entry: jitter a copy of the first
        } else {
          s_jitter = 0;
          double pick = __dmul_rn(rng.uniform(), total);
          uint64_t idx = n - 1, i = 0;
          bool found = false;
          // the reference's scan, four loads issued ahead of the dependent subtractions
          for (; i + 4 <= n && !found; i += 4) {
            const double d0 = dmin[i], d1 = dmin[i + 1], d2 = dmin[i + 2], d3 = dmin[i + 3];
            if ((pick = __dsub_rn(pick, d0)) <= 0.0) idx = i, found = true;
            else if ((pick = __dsub_rn(pick, d1)) <= 0.0) idx = i + 1, found = true;
            else if ((pick = __dsub_rn(pick, d2)) <= 0.0) idx = i + 2, found = true;
            else if ((pick = __dsub_rn(pick, d3)) <= 0.0) idx = i + 3, found = true;
          }
          for (; i < n && !found; ++i)
            if ((pick = __dsub_rn(pick, dmin[i])) <= 0.0) idx = i, found = true;
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
        int c;
        if (D == RD) {
          Row128 x;
          load_row(res + i * D, x);
          c = nearest_row128(cb, E, x);
        } else {
          c = nearest_row(cb, E, D, res + i * D);
        }
        T.codes[i] = (uint8_t)c;
        atomicAdd(&fit_counts[c], 1);
      }
      __syncthreads();
      for (int d = t; d < D; d += FT) {
        for (int c = 0; c < E; ++c) sums[(size_t)c * D + d] = 0.0;
        uint64_t i = 0;
        for (; i + 8 <= n; i += 8) {  // eight tokens' loads ahead of the in-order adds
          float rv[8];
          int cv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            cv[u] = T.codes[i + u];
            rv[u] = res[(i + u) * D + d];
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            double* sc = sums + (size_t)cv[u] * D + d;
            *sc = __dadd_rn(*sc, (double)rv[u]);
          }
        }
        for (; i < n; ++i) {
          double* sc = sums + (size_t)T.codes[i] * D + d;
          *sc = __dadd_rn(*sc, (double)res[i * D + d]);
        }
      }
      __syncthreads();
      for (int j = t; j < E * D; j += FT) {
        const int c = j / D;
        if (fit_counts[c] > 0) cb[j] = __double2float_rn(__ddiv_rn(sums[j], (double)fit_counts[c]));
      }
      __syncthreads();
    }
    // ---- subtract each row's nearest entry (qvg.rs:386-392)
    if (s + 1 < stages) {
      for (uint64_t i = t; i < n; i += FT) {
        float* r = res + i * D;
        if (D == RD) {
          Row128 x;
          load_row(r, x);
          const float4* c = reinterpret_cast<const float4*>(cb + (size_t)nearest_row128(cb, E, x) * RD);
#pragma unroll
          for (int k = 0; k < RD / 4; ++k) {
            const float4 c4 = c[k];
            reinterpret_cast<float4*>(r)[k] = make_float4(__fsub_rn(x.v[k].x, c4.x), __fsub_rn(x.v[k].y, c4.y),
                                                          __fsub_rn(x.v[k].z, c4.z), __fsub_rn(x.v[k].w, c4.w));
          }
        } else {
          const float* c = cb + (size_t)nearest_row(cb, E, D, r) * D;
          for (int d = 0; d < D; ++d) r[d] = __fsub_rn(r[d], c[d]);
        }
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
  size_t so, dof;
  const size_t smem = fit_smem_bytes(n, D, E, &so, &dof);
  cudaError_t e = cudaSuccess;
  switch (in_dtype) {
    case F32:
      e = cudaFuncSetAttribute(k_qvg_fit<F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) k_qvg_fit<F32><<<n_tasks, FT, smem, s>>>(tasks_dev, n, H, D, stages, E);
      break;
    case BF16:
      e = cudaFuncSetAttribute(k_qvg_fit<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) k_qvg_fit<BF16><<<n_tasks, FT, smem, s>>>(tasks_dev, n, H, D, stages, E);
      break;
    default:
      e = cudaFuncSetAttribute(k_qvg_fit<F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) k_qvg_fit<F16><<<n_tasks, FT, smem, s>>>(tasks_dev, n, H, D, stages, E);
      break;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace nkv
