// kernels_commit.cu — the commit side of the lifelong KV cache on sm_100a:
// INT8 quantize (cache/int8.rs:65-134), the FLOAT archive copy
// (cache/history.rs:243-247), QVG residual-VQ encode (cache/qvg.rs:173-256)
// and the synthetic K/V generator used by tests and benchmarks.
//
// Exactness: every f32 / f64 operation the reference rounds separately is
// written with an explicit round-to-nearest intrinsic, and the library is
// compiled with -fmad=false, so no multiply-add is contracted behind our
// back.  Explicit fma() is used only where the product is exact (f32 x f32
// in f64), where fused and unfused results are identical.
#include <cfloat>
#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"
#include "nkv_quant.cuh"

namespace nkv {

// ---------------------------------------------------------------------------
// INT8 quantize.  G threads per (token, head) row, 8 consecutive values per
// thread (16-byte loads for BF16/F16, 2 x 16 bytes for F32), shuffle absmax
// across the G lanes, coalesced 8-byte code stores and one f32 scale store
// per row.
//
// Per value the reference computes round_half_away(x / s) with an IEEE
// division.  The kernels get the same correctly rounded quotient without a
// divide: with r = RN(1/s) (one IEEE reciprocal per row), q0 = RN(x * r),
// the residual e = x - s * q0 computed exactly by an FMA, and
// q1 = RN(q0 + e * r), Markstein's theorem gives q1 = RN(x / s) whenever the
// quotient is in the normal range (a subnormal quotient rounds to 0 either
// way).  Round-half-away-from-zero of the quotient's magnitude is then
// floor(RN(q1 + (0.5 - 2^-25))), taken by a round-toward-zero add of the
// 1.5 * 2^23 magic constant (code_bits in nkv_quant.cuh).  Rows whose scale
// is subnormal (or above 1e37) take the IEEE division.
// ---------------------------------------------------------------------------
// The exact per-value path kept out of line: inlined, the compiler turns the
// rarely taken branch into predicated code that every thread issues.
__device__ __noinline__ uint2 quant8_exact(float4 lo, float4 hi, float s) {
  const float x[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  uint32_t b[8];
  for (int j = 0; j < 8; ++j) b[j] = quant_exact(x[j], s);
  return make_uint2(b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24), b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24));
}

// 16 bf16 values (8 words) of one row with scale s, exact path.
__device__ __noinline__ uint4 quant16_bf16_exact(uint4 w0, uint4 w1, float s) {
  const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  uint32_t out[4];
  for (int k = 0; k < 4; ++k) {
    uint32_t b[4];
    for (int e = 0; e < 4; ++e) {
      const uint32_t h = (ws[2 * k + e / 2] >> (16 * (e & 1))) & 0xFFFFu;
      b[e] = quant_exact(__uint_as_float(h << 16), s);
    }
    out[k] = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// 8 values of one row with scale s -> 8 packed code bytes.
__device__ __forceinline__ uint2 quant8(const float (&x)[8], float s) {
  if (!(s >= FLT_MIN && s <= 1e37f))
    return quant8_exact(make_float4(x[0], x[1], x[2], x[3]), make_float4(x[4], x[5], x[6], x[7]), s);
  const float r = __frcp_rn(s);
  uint32_t c[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) c[j] = code_bits(x[j], s, r);
  return make_uint2(pack4(c[0], c[1], c[2], c[3]), pack4(c[4], c[5], c[6], c[7]));
}

// R rows per thread and iteration: all R loads are issued before any of
// them is consumed, so each thread keeps R x 16 bytes in flight.
template <int IN_DT, int G, int R>
__global__ void __launch_bounds__(256) k_int8_quantize(const QuantJob* __restrict__ jobs, uint64_t rows,
                                                       uint64_t in_row_offset, uint32_t* __restrict__ flag) {
  constexpr int D = 8 * G;
  const QuantJob J = jobs[blockIdx.y >> 1];
  const int side = blockIdx.y & 1;
  const void* in = side ? J.v : J.k;
  uint8_t* q = side ? J.vq : J.kq;
  float* sc = side ? J.vs : J.ks;
  const int sub = threadIdx.x % G;
  const uint64_t rows_per_pass = blockDim.x / G;
  const float inv127 = (float)(1.0 / 127.0);
  bool bad = false;
  for (uint64_t base = (uint64_t)blockIdx.x * rows_per_pass * R; base < rows;
       base += (uint64_t)gridDim.x * rows_per_pass * R) {
    float x[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t row = base + r * rows_per_pass + threadIdx.x / G;
      if (row < rows) {
        dev::load8<IN_DT>(in, (in_row_offset + row) * D + sub * 8, x[r]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[r][j] = 0.0f;
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t row = base + r * rows_per_pass + threadIdx.x / G;
      if constexpr (IN_DT != BF16) {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[r][j] = dev::round_to<BF16>(x[r][j]);  // to_dtype(BF16), history.rs:249
      }
      float peak = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = fabsf(x[r][j]);
        bad |= !(a < FLT_MAX);  // x != x || |x| >= f32::MAX (int8.rs:99-117)
        peak = fmaxf(peak, a);
      }
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xFFFFFFFFu, peak, o));
      if (row >= rows) continue;
      // scale = where(peak > 0, peak * (f32)(1/127) + 0, 1)   (int8.rs:72)
      const float s = peak > 0.0f ? __fadd_rn(__fmul_rn(peak, inv127), 0.0f) : 1.0f;
      *reinterpret_cast<uint2*>(q + row * D + sub * 8) = quant8(x[r], s);
      if (sub == 0) sc[row] = s;
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) {
    atomicOr(flag, 1u << side);
    if (J.flag) atomicOr(J.flag, 1u << side);
  }
}

// ---------------------------------------------------------------------------
// BF16 input, head_dim = 16 * G: the commit kernel of the 8B geometry.
// G threads per (token, head) row, 16 values (two 16-byte loads) per thread,
// R rows per thread in flight, branch-free per value (code_bits above):
//  * |x| max runs on the raw 16-bit patterns (max.u16x2 on |bits|): for
//    non-negative bf16 the integer order is the float order, and inf / NaN
//    patterns (>= 0x7F80) sort above every finite value, so the same max
//    also answers the reference's non-finite scan (no finite bf16 reaches
//    f32::MAX, int8.rs:110-116);
//  * the rounded quotient is placed in the low byte of M + f (M = 1.5 * 2^23)
//    and an XOR with 0x80 makes it (f + 128) mod 256.  |x / s| < 127.5 for
//    every value of the row (x <= peak, s = peak * (1 + O(2^-23)) / 127), so
//    the reference's clamp to [-127, 127] never binds.
// ---------------------------------------------------------------------------
template <int G, int R, int V>
__global__ void __launch_bounds__(256) k_int8_quantize_bf16(const QuantJob* __restrict__ jobs, uint64_t rows,
                                                            uint64_t in_row_offset, uint32_t* __restrict__ flag) {
  // G threads per row, V bf16 values per thread (V = 16 or 32)
  constexpr int D = V * G;
  constexpr int NW = V / 8;  // 16-byte loads per thread and row
  const QuantJob J = jobs[blockIdx.y >> 1];
  const int side = blockIdx.y & 1;
  const uint4* in = reinterpret_cast<const uint4*>(side ? J.v : J.k);
  uint4* q = reinterpret_cast<uint4*>(side ? J.vq : J.kq);
  float* sc = side ? J.vs : J.ks;
  const int sub = threadIdx.x % G;
  const uint64_t rows_per_pass = blockDim.x / G;
  const float inv127 = (float)(1.0 / 127.0);
  uint32_t worst = 0;  // max |bits| seen: >= 0x7F80 means inf / NaN
  for (uint64_t base = (uint64_t)blockIdx.x * rows_per_pass * R; base < rows;
       base += (uint64_t)gridDim.x * rows_per_pass * R) {
    uint4 w[R][NW];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t row = base + r * rows_per_pass + threadIdx.x / G;
      if (row < rows) {
        const uint4* p = in + ((in_row_offset + row) * D + sub * V) / 8;
#pragma unroll
        for (int k = 0; k < NW; ++k) w[r][k] = __ldg(p + k);
      } else {
#pragma unroll
        for (int k = 0; k < NW; ++k) w[r][k] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t row = base + r * rows_per_pass + threadIdx.x / G;
      uint32_t ws[V / 2];
#pragma unroll
      for (int k = 0; k < NW; ++k) {
        ws[4 * k] = w[r][k].x, ws[4 * k + 1] = w[r][k].y, ws[4 * k + 2] = w[r][k].z, ws[4 * k + 3] = w[r][k].w;
      }
      uint32_t m2 = 0;
#pragma unroll
      for (int j = 0; j < V / 2; ++j) m2 = maxabs_bf16x2(m2, ws[j]);
      m2 &= 0x7FFF7FFFu;
      uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
      worst = max(worst, m);
      if (row >= rows) continue;
      const float peak = __uint_as_float(m << 16);
      // scale = where(peak > 0, peak * (f32)(1/127) + 0, 1)   (int8.rs:72)
      const float s = peak > 0.0f ? __fadd_rn(__fmul_rn(peak, inv127), 0.0f) : 1.0f;
      uint4* qo = q + (row * D + sub * V) / 16;
      if (s >= FLT_MIN && s <= 1e37f) {
        const float rc = __frcp_rn(s);
#pragma unroll
        for (int k = 0; k < V / 16; ++k) {
          uint32_t c[16];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint2 cc = code_bits2(
                make_float2(__uint_as_float(ws[8 * k + j] << 16), __uint_as_float(ws[8 * k + j] & 0xFFFF0000u)), s,
                rc);
            c[2 * j] = cc.x;
            c[2 * j + 1] = cc.y;
          }
          qo[k] = make_uint4(pack4(c[0], c[1], c[2], c[3]), pack4(c[4], c[5], c[6], c[7]),
                             pack4(c[8], c[9], c[10], c[11]), pack4(c[12], c[13], c[14], c[15]));
        }
      } else {
#pragma unroll
        for (int k = 0; k < V / 16; ++k) qo[k] = quant16_bf16_exact(w[r][2 * k], w[r][2 * k + 1], s);
      }
      if (sub == 0) sc[row] = s;
    }
  }
  const bool bad = worst >= 0x7F80u;
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) {
    atomicOr(flag, 1u << side);
    if (J.flag) atomicOr(J.flag, 1u << side);
  }
}

// Generic shape: one warp per row, any D, any alignment, exact division.
template <int IN_DT>
__global__ void __launch_bounds__(256) k_int8_quantize_generic(const QuantJob* __restrict__ jobs, uint64_t rows,
                                                               uint64_t in_row_offset, int64_t D,
                                                               uint32_t* __restrict__ flag) {
  const QuantJob J = jobs[blockIdx.y >> 1];
  const int side = blockIdx.y & 1;
  const void* in = side ? J.v : J.k;
  uint8_t* q = side ? J.vq : J.kq;
  float* sc = side ? J.vs : J.ks;
  const int lane = threadIdx.x & 31;
  const uint64_t warps = blockDim.x / 32;
  const float inv127 = (float)(1.0 / 127.0);
  bool bad = false;
  for (uint64_t row = (uint64_t)blockIdx.x * warps + threadIdx.x / 32; row < rows; row += (uint64_t)gridDim.x * warps) {
    const uint64_t ib = (in_row_offset + row) * (uint64_t)D;
    float peak = 0.0f;
    for (int64_t d = lane; d < D; d += 32) {
      const float a = fabsf(dev::round_to<BF16>(dev::load_elem<IN_DT>(in, ib + d)));
      bad |= !(a < FLT_MAX);
      peak = fmaxf(peak, a);
    }
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xFFFFFFFFu, peak, o));
    const float s = peak > 0.0f ? __fadd_rn(__fmul_rn(peak, inv127), 0.0f) : 1.0f;
    for (int64_t d = lane; d < D; d += 32)
      q[row * D + d] = (uint8_t)quant_exact(dev::round_to<BF16>(dev::load_elem<IN_DT>(in, ib + d)), s);
    if (lane == 0) sc[row] = s;
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) {
    atomicOr(flag, 1u << side);
    if (J.flag) atomicOr(J.flag, 1u << side);
  }
}

template <int IN_DT>
static cudaError_t quantize_dispatch(const QuantJob* jobs, int n_jobs, uint64_t rows, uint64_t off, int64_t D,
                                     bool vec_ok, uint32_t* flag, cudaStream_t s) {
  if (rows == 0 || n_jobs == 0) return cudaSuccess;
  const int threads = 256;
  auto grid_for = [&](uint64_t rows_per_cta) {
    uint64_t need = (rows + rows_per_cta - 1) / rows_per_cta;
    uint64_t cap = 148ull * 16;  // enough CTAs to fill every SM several times
    return dim3((unsigned)(need < cap ? need : cap), (unsigned)(2 * n_jobs));
  };
  if constexpr (IN_DT == BF16) {
    constexpr int R2 = 2;
    if (vec_ok) {
      switch (D) {
        case 16: k_int8_quantize_bf16<1, R2, 16><<<grid_for(threads / 1 * R2), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
        case 32: k_int8_quantize_bf16<2, R2, 16><<<grid_for(threads / 2 * R2), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
        case 64: k_int8_quantize_bf16<2, R2, 32><<<grid_for(threads / 2 * R2), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
        case 128: k_int8_quantize_bf16<4, R2, 32><<<grid_for(threads / 4 * R2), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
        case 256: k_int8_quantize_bf16<8, R2, 32><<<grid_for(threads / 8 * R2), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
        default: break;
      }
    }
  }
  constexpr int R = 4;
  if (vec_ok) {
    switch (D) {
      case 16: k_int8_quantize<IN_DT, 2, R><<<grid_for(threads / 2 * R), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
      case 32: k_int8_quantize<IN_DT, 4, R><<<grid_for(threads / 4 * R), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
      case 64: k_int8_quantize<IN_DT, 8, R><<<grid_for(threads / 8 * R), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
      case 128: k_int8_quantize<IN_DT, 16, R><<<grid_for(threads / 16 * R), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
      case 256: k_int8_quantize<IN_DT, 32, R><<<grid_for(threads / 32 * R), threads, 0, s>>>(jobs, rows, off, flag); return cudaGetLastError();
      default: break;
    }
  }
  k_int8_quantize_generic<IN_DT><<<grid_for(threads / 32), threads, 0, s>>>(jobs, rows, off, D, flag);
  return cudaGetLastError();
}

cudaError_t launch_int8_quantize(const QuantJob* jobs_dev, int n_jobs, uint64_t rows, uint64_t in_row_offset,
                                 int64_t D, int in_dtype, bool aligned16, uint32_t* flag, cudaStream_t s) {
  // The vector path loads 16-byte chunks: every buffer must be 16-byte
  // aligned (checked by the caller) and D a multiple of 8 keeps rows aligned.
  const bool vec_ok = aligned16 && (D % 8) == 0;
  switch (in_dtype) {
    case F32: return quantize_dispatch<F32>(jobs_dev, n_jobs, rows, in_row_offset, D, vec_ok, flag, s);
    case BF16: return quantize_dispatch<BF16>(jobs_dev, n_jobs, rows, in_row_offset, D, vec_ok, flag, s);
    default: return quantize_dispatch<F16>(jobs_dev, n_jobs, rows, in_row_offset, D, vec_ok, flag, s);
  }
}

// ---------------------------------------------------------------------------
// FLOAT archive: `to_dtype(model)` copy of each layer's K / V.
// ---------------------------------------------------------------------------
template <int IN_DT, int OUT_DT>
__global__ void __launch_bounds__(256) k_convert(const ConvertJob* __restrict__ jobs, uint64_t n) {
  const ConvertJob J = jobs[blockIdx.y];
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const float v = dev::load_elem<IN_DT>(J.src, i);
    if constexpr (IN_DT == OUT_DT) {
      if constexpr (OUT_DT == F32) static_cast<float*>(J.dst)[i] = v;
      else static_cast<unsigned short*>(J.dst)[i] = static_cast<const unsigned short*>(J.src)[i];
    } else {
      dev::store_elem<OUT_DT>(J.dst, i, v);
    }
  }
}

template <int IN_DT>
static cudaError_t convert_out(const ConvertJob* jobs, int n_jobs, uint64_t n, int out_dt, cudaStream_t s) {
  uint64_t need = (n + 255) / 256;
  dim3 grid((unsigned)(need < 148ull * 32 ? need : 148ull * 32), (unsigned)n_jobs);
  switch (out_dt) {
    case F32: k_convert<IN_DT, F32><<<grid, 256, 0, s>>>(jobs, n); break;
    case BF16: k_convert<IN_DT, BF16><<<grid, 256, 0, s>>>(jobs, n); break;
    default: k_convert<IN_DT, F16><<<grid, 256, 0, s>>>(jobs, n); break;
  }
  return cudaGetLastError();
}

__global__ void k_flag_reduce(uint32_t* flags, int n) {
  uint32_t any = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) any |= flags[1 + i];
  for (int o = 16; o > 0; o >>= 1) any |= __shfl_xor_sync(0xFFFFFFFFu, any, o);
  if (threadIdx.x == 0 && any) atomicOr(flags, any);
}

cudaError_t launch_flag_reduce(uint32_t* flags, int n, cudaStream_t s) {
  k_flag_reduce<<<1, 32, 0, s>>>(flags, n);
  return cudaGetLastError();
}

cudaError_t launch_convert(const ConvertJob* jobs_dev, int n_jobs, uint64_t n, int in_dtype, int out_dtype,
                           cudaStream_t s) {
  if (n == 0 || n_jobs == 0) return cudaSuccess;
  switch (in_dtype) {
    case F32: return convert_out<F32>(jobs_dev, n_jobs, n, out_dtype, s);
    case BF16: return convert_out<BF16>(jobs_dev, n_jobs, n, out_dtype, s);
    default: return convert_out<F16>(jobs_dev, n_jobs, n, out_dtype, s);
  }
}

// ---------------------------------------------------------------------------
// QVG encode (cache/qvg.rs:173-256).  One CTA per (head, 64-token block,
// layer x side), one thread per token of the block.  The block's residual
// rows live in shared memory; per stage every thread finds its nearest
// codeword with the reference's sequential f64 distance (ties to the lower
// index), then one thread forms alpha = num / den from the per-token f64
// inner sums in token order, and every thread subtracts alpha * e in f32.
// ---------------------------------------------------------------------------
template <int IN_DT>
__global__ void __launch_bounds__(256) k_qvg_encode(const QvgEncodeJob* __restrict__ jobs, uint64_t L, int H, int D,
                                                    uint64_t tokens, int stages, int bits, int block) {
  extern __shared__ unsigned char smem_raw[];
  const QvgEncodeJob J = jobs[blockIdx.z];
  const int h = blockIdx.x;
  const uint64_t blk = blockIdx.y;
  const uint64_t start = blk * (uint64_t)block;
  const int n = (int)((tokens - start) < (uint64_t)block ? (tokens - start) : (uint64_t)block);
  const int E = 1 << bits;
  const int ld = D + 1;
  const uint64_t n_blocks = (tokens + block - 1) / block;
  const int bpt = (stages * bits + 7) / 8;

  float* res = reinterpret_cast<float*>(smem_raw);  // [block][D + 1]
  size_t res_words = (size_t)block * ld;
  res_words += res_words & 1;
  double* inner = reinterpret_cast<double*>(res + res_words);              // [block]
  double* ee = inner + block;                                              // [E]
  uint64_t* packed = reinterpret_cast<uint64_t*>(ee + E);                  // [block]
  int* code_s = reinterpret_cast<int*>(packed + block);                    // [block]
  float* alpha_s = reinterpret_cast<float*>(code_s + block);               // [1]

  for (int e = threadIdx.x; e < n * D; e += blockDim.x) {
    const int t = e / D, d = e % D;
    res[t * ld + d] = dev::load_elem<IN_DT>(J.x, ((start + t) * (uint64_t)H + h) * (uint64_t)D + d);
  }
  for (int t = threadIdx.x; t < n; t += blockDim.x) packed[t] = 0;
  __syncthreads();

  for (int s = 0; s < stages; ++s) {
    const float* cbs = J.cb + ((size_t)h * stages + s) * E * D;
    // sum_d e_d^2 per entry, sequential in d (the den inner sum, qvg.rs:228)
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      double acc = 0.0;
      for (int d = 0; d < D; ++d) {
        const double v = (double)__ldg(cbs + (size_t)e * D + d);
        acc = fma(v, v, acc);  // exact product: fused == unfused
      }
      ee[e] = acc;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float* r = res + (size_t)i * ld;
      // nearest (qvg.rs:303-321)
      int best = 0;
      double best_d = __longlong_as_double(0x7FF0000000000000ll);
      for (int e = 0; e < E; ++e) {
        const float* ce = cbs + (size_t)e * D;
        double dist = 0.0;
        for (int d = 0; d < D; ++d) {
          const double diff = __dsub_rn((double)r[d], (double)__ldg(ce + d));
          dist = __dadd_rn(dist, __dmul_rn(diff, diff));
          if (dist >= best_d) break;
        }
        if (dist < best_d) {
          best_d = dist;
          best = e;
        }
      }
      const float* ce = cbs + (size_t)best * D;
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc = fma((double)r[d], (double)__ldg(ce + d), acc);  // qvg.rs:223-227
      inner[i] = acc;
      code_s[i] = best;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double num = 0.0, den = 0.0;
      for (int t = 0; t < n; ++t) {
        num = __dadd_rn(num, inner[t]);
        den = __dadd_rn(den, ee[code_s[t]]);
      }
      const float alpha = den > 1e-12 ? __double2float_rn(__ddiv_rn(num, den)) : 1.0f;  // qvg.rs:230
      *alpha_s = alpha;
      J.scales[((size_t)h * n_blocks + blk) * stages + s] = alpha;
    }
    __syncthreads();
    const float alpha = *alpha_s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float* r = res + (size_t)i * ld;
      const int best = code_s[i];
      const float* ce = cbs + (size_t)best * D;
      for (int d = 0; d < D; ++d) r[d] = __fsub_rn(r[d], __fmul_rn(alpha, __ldg(ce + d)));  // qvg.rs:232-237
      packed[i] |= (uint64_t)best << (s * bits);  // pack_bits, LSB first (qvg.rs:238-244)
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    uint8_t* out = J.codes + ((start + i) * (uint64_t)H + h) * bpt;
    for (int b = 0; b < bpt; ++b) out[b] = (uint8_t)(packed[i] >> (8 * b));
  }
}

static size_t qvg_encode_smem(int D, int block, int E) {
  size_t res = (size_t)block * (D + 1);
  res += res & 1;
  return res * 4 + (size_t)block * 8 + (size_t)E * 8 + (size_t)block * 8 + (size_t)block * 4 + 16;
}

cudaError_t launch_qvg_encode(const QvgEncodeJob* jobs_dev, int n_jobs, int in_dtype, uint64_t L, int H, int D,
                              uint64_t tokens, int stages, int bits, int block, bool aligned16, cudaStream_t s) {
  if (tokens == 0 || n_jobs == 0 || H == 0) return cudaSuccess;
  cudaError_t fast_err = cudaSuccess;
  if (launch_qvg_encode_d128(jobs_dev, n_jobs, in_dtype, H, D, tokens, stages, bits, block, aligned16, s, &fast_err))
    return fast_err;
  const int E = 1 << bits;
  const size_t smem = qvg_encode_smem(D, block, E);
  const uint64_t n_blocks = (tokens + block - 1) / block;
  dim3 grid((unsigned)H, (unsigned)n_blocks, (unsigned)n_jobs);
  const int threads = block >= 256 ? 256 : ((block + 31) / 32) * 32;
  cudaError_t err;
  switch (in_dtype) {
    case F32:
      err = cudaFuncSetAttribute(k_qvg_encode<F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      k_qvg_encode<F32><<<grid, threads, smem, s>>>(jobs_dev, L, H, D, tokens, stages, bits, block);
      break;
    case BF16:
      err = cudaFuncSetAttribute(k_qvg_encode<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      k_qvg_encode<BF16><<<grid, threads, smem, s>>>(jobs_dev, L, H, D, tokens, stages, bits, block);
      break;
    default:
      err = cudaFuncSetAttribute(k_qvg_encode<F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      k_qvg_encode<F16><<<grid, threads, smem, s>>>(jobs_dev, L, H, D, tokens, stages, bits, block);
      break;
  }
  return cudaGetLastError();
}

size_t qvg_encode_smem_bytes(int D, int block, int bits) { return qvg_encode_smem(D, block, 1 << bits); }

// ---------------------------------------------------------------------------
// Synthetic K/V: counter-based, so any element can be regenerated on the CPU
// (tests/ reproduce it with numpy).
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) k_synth_fill(void* dst, uint64_t n, int HD, uint64_t key, uint64_t offset,
                                                    const float* __restrict__ table,
                                                    const float* __restrict__ chan_scale) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t u = dev::mix64(key + (i + offset + 1) * 0x9E3779B97F4A7C15ull);
    float v = __ldg(table + (u >> 48));
    if (chan_scale) v = __fmul_rn(v, __ldg(chan_scale + (i % (uint64_t)HD)));
    dev::store_elem<DT>(dst, i, v);
  }
}

cudaError_t launch_synth_fill(void* dst, int dtype, uint64_t rows, int H, int D, uint64_t key,
                              uint64_t index_offset, const float* table, const float* chan_scale, cudaStream_t s) {
  const uint64_t n = rows * (uint64_t)H * (uint64_t)D;
  if (n == 0) return cudaSuccess;
  uint64_t need = (n + 255) / 256;
  unsigned grid = (unsigned)(need < 148ull * 64 ? need : 148ull * 64);
  switch (dtype) {
    case F32: k_synth_fill<F32><<<grid, 256, 0, s>>>(dst, n, H * D, key, index_offset, table, chan_scale); break;
    case BF16: k_synth_fill<BF16><<<grid, 256, 0, s>>>(dst, n, H * D, key, index_offset, table, chan_scale); break;
    default: k_synth_fill<F16><<<grid, 256, 0, s>>>(dst, n, H * D, key, index_offset, table, chan_scale); break;
  }
  return cudaGetLastError();
}

}  // namespace nkv
