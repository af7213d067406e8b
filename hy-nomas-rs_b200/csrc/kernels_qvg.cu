// kernels_qvg.cu — QVG encode for the reference's default codec shape
// (4 entries per stage, head_dim 128, 64-token blocks, up to 4 stages):
// QvgCodec::encode (cache/qvg.rs:173-256) restated bit for bit with far less
// double-precision work than the literal algorithm.
//
// Per (token, stage) the reference
//   1. picks c = argmin_i D_i, D_i the sequential f64 sum of (r_d - e_id)^2
//      (nearest, qvg.rs:303-321; ties to the lower index),
//   2. adds the sequential f64 dot r . e_c to the block's numerator and the
//      sequential f64 e_c . e_c to its denominator (qvg.rs:220-229),
//   3. after alpha = f32(num / den) updates r_d -= f32(alpha * e_cd).
//
// Step 1 is screened in f32: with u_i = e_i - e_0, the exact distance
// differences are T_i - T_0 = (|e_i|^2 - |e_0|^2) - 2 r.u_i, and the f32 dots
// carry a rigorous error bound (gamma_n |r||u_i| plus the rounding of u_i).
// When the chosen entry beats every other by more than those bounds plus the
// reference's own f64 rounding (<= 1.5e-14 T), the reference's sequential
// f64 argmin is certainly the same entry; otherwise (near ties, duplicate
// codewords, NaN) the reference's sequential f64 distances are computed
// exactly.
//
// Step 2 is certified instead of replayed.  Products of f32 values are exact
// in f64, so any f64 evaluation differs from the reference's only in the
// order of its additions.  The kernel sums in a parallel order and bounds
// both its own error and the reference's sequential one:
//   |num_kernel - num_ref| <= (gamma_24 + gamma_127 + gamma_63) S <= 3e-14 S,
//   S = sum |r_d e_cd| <= sum_t |r_t| |e_c|   (Cauchy-Schwarz),
//   |den_kernel - den_ref| <= (gamma_6 + gamma_63) den <= 1e-14 den
// (the per-token e_c . e_c sums are the reference's own values).  With
// directed-rounding interval division the reference's alpha =
// f32(f64(num / den)) lies between f32(lo) and f32(hi); when those agree it is
// known exactly (rounding is monotone).  Otherwise (a quotient within ~1e-13
// of an f32 rounding boundary, non-finite values, den near the 1e-12 cut)
// the block replays the reference's sequential sums.
//
// Step 3 is two f32 roundings as in the reference: warp 0 builds the stage's
// table -f32(alpha * e_c) with scalar multiplies, and each thread adds its
// table row with packed f32x2 adds (no multiply in the thread's data flow,
// so nothing can be contracted into one rounding).
//
// Layout: one CTA of 256 threads per (layer x side, head, group of blocks);
// four threads per token of the current 64-token block, thread q of a token
// holding its residual's float4 chunks 4k + q (k = 0..7) in registers, so
// a quarter warp reads 64 contiguous bytes of every table row.  Quad
// shuffles give all four threads of a token bit-identical sums (IEEE
// addition commutes), hence identical decisions.
#include <cfloat>
#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"

namespace nkv {

namespace {

constexpr int QD = 128;                // head_dim
constexpr int QE = 4;                  // codewords per stage (2 bits)
constexpr int QB = 64;                 // tokens per block
constexpr int QSMAX = 4;               // stages
constexpr int QT = 4;                  // threads per token
constexpr int QC = QD / 4 / QT;        // float4 chunks per thread
constexpr int QTHREADS = QB * QT;      // 256
constexpr int QWARPS = QTHREADS / 32;  // 8
constexpr unsigned FULL = 0xFFFFFFFFu;

struct QvgSmem {
  float u[QSMAX][3][QD];          // e_i - e_0 rounded to f32, i = 1..3
  float e32[QSMAX][QE][QD];       // codewords
  double e64[QSMAX][QE][QD + 2];  // codewords as f64 (rows padded 16 bytes)
  double ee[QSMAX][QE];           // sequential f64 sum of e_d^2 (the den inner sum)
  float enorm[QSMAX][QE];         // upper bounds of |e_i|
  float unorm[QSMAX][3];          // upper bounds of |e_i - e_0|
  float nP[QE][QD];               // -f32(alpha * e_c) of the current stage
  float fbr[QWARPS][QD];          // one token's residual for a warp's exact paths
  double part[QWARPS][3];         // per-warp numerator, S bound, denominator
  double inner[QB];               // exact path: the reference's per-token inner sums
  double dv[QB];                  // exact path: per-token denominator terms
  int cert;
};

// Chunk k of thread q covers dims 16 k + 4 q .. 16 k + 4 q + 3.
__device__ __forceinline__ int chunk_dim(int k, int q) { return 16 * k + 4 * q; }

template <int DT>
__device__ __forceinline__ float4 load4(const void* p, uint64_t i) {  // i: multiple of 4
  if constexpr (DT == F32) {
    return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
  } else {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(static_cast<const unsigned short*>(p) + i));
    if constexpr (DT == BF16)
      return make_float4(dev::bf16_value(w.x), dev::bf16_value(w.x >> 16), dev::bf16_value(w.y),
                         dev::bf16_value(w.y >> 16));
    else
      return make_float4(dev::f16_value(w.x), dev::f16_value(w.x >> 16), dev::f16_value(w.y),
                         dev::f16_value(w.y >> 16));
  }
}

// The reference's alpha (qvg.rs:230) when num_ref / den_ref is pinned by the
// bounds above; false when it is not.
__device__ __forceinline__ bool certify_alpha(double num, double S, double den, float* alpha) {
  if (!(isfinite(num) && isfinite(S) && isfinite(den))) return false;
  const double bn = __dmul_ru(3.0e-14, __dmul_ru(S, 1.000001));
  const double bd = __dmul_ru(1.0e-14, den);
  const double dlo = __dsub_rd(den, bd), dhi = __dadd_ru(den, bd);
  if (dhi <= 1e-12) {
    *alpha = 1.0f;
    return true;
  }
  if (!(dlo > 1e-12)) return false;
  const double nlo = __dsub_rd(num, bn), nhi = __dadd_ru(num, bn);
  const double lo = fmin(__ddiv_rd(nlo, dlo), __ddiv_rd(nlo, dhi));
  const double hi = fmax(__ddiv_ru(nhi, dlo), __ddiv_ru(nhi, dhi));
  const float alo = __double2float_rn(lo), ahi = __double2float_rn(hi);
  *alpha = alo;
  return __float_as_uint(alo) == __float_as_uint(ahi);
}

__device__ __forceinline__ float quad_sum(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(FULL, v, 1));
  return __fadd_rn(v, __shfl_xor_sync(FULL, v, 2));
}
__device__ __forceinline__ double quad_sum(double v) {
  v = __dadd_rn(v, __shfl_xor_sync(FULL, v, 1));
  return __dadd_rn(v, __shfl_xor_sync(FULL, v, 2));
}
// Sum over the warp's 8 tokens (lanes of one token hold equal values).
__device__ __forceinline__ double tokens_sum(double v) {
  v = __dadd_rn(v, __shfl_xor_sync(FULL, v, 4));
  v = __dadd_rn(v, __shfl_xor_sync(FULL, v, 8));
  return __dadd_rn(v, __shfl_xor_sync(FULL, v, 16));
}

// Warp 0: the stage's -f32(alpha * e) rows (one rounding per product, as the
// reference's alpha * e[d], qvg.rs:232-237).
__device__ __forceinline__ void build_table(QvgSmem& sm, int s, float alpha, int lane) {
  for (int i = lane; i < QE * QD; i += 32) sm.nP[i / QD][i % QD] = __fmul_rn(-alpha, sm.e32[s][i / QD][i % QD]);
}

}  // namespace

template <int IN_DT>
__global__ void __launch_bounds__(QTHREADS, 3) k_qvg_encode_d128(const QvgEncodeJob* __restrict__ jobs, int H,
                                                               uint64_t tokens, int stages) {
  __shared__ __align__(16) QvgSmem sm;
  const QvgEncodeJob J = jobs[blockIdx.z];
  const int h = blockIdx.x;
  const int t = threadIdx.x, ti = t / QT, q = t % QT, lane = t & 31, warp = t >> 5;
  const uint64_t n_blocks = (tokens + QB - 1) / QB;

  // ---- codebooks of this (side, head), all stages
  const float* cbh = J.cb + (size_t)h * stages * QE * QD;
  for (int i = t; i < stages * QE * QD; i += QTHREADS) {
    const int s = i / (QE * QD), e = (i / QD) % QE, d = i % QD;
    const float v = __ldg(cbh + i);
    sm.e32[s][e][d] = v;
    sm.e64[s][e][d] = (double)v;
  }
  __syncthreads();
  for (int i = t; i < stages * 3 * QD; i += QTHREADS) {
    const int s = i / (3 * QD), j = (i / QD) % 3, d = i % QD;
    sm.u[s][j][d] = __fsub_rn(sm.e32[s][j + 1][d], sm.e32[s][0][d]);
  }
  for (int i = t; i < stages * QE; i += QTHREADS) {
    const int s = i / QE, e = i % QE;
    double acc = 0.0;
    for (int d = 0; d < QD; ++d) acc = fma(sm.e64[s][e][d], sm.e64[s][e][d], acc);  // exact products
    sm.ee[s][e] = acc;
    sm.enorm[s][e] = (float)(sqrt(acc) * (1.0 + 1e-6));
  }
  __syncthreads();
  for (int i = t; i < stages * 3; i += QTHREADS) {
    const int s = i / 3, j = i % 3;
    double acc = 0.0;
    for (int d = 0; d < QD; ++d) acc = fma((double)sm.u[s][j][d], (double)sm.u[s][j][d], acc);
    sm.unorm[s][j] = (float)(sqrt(acc) * (1.0 + 1e-6));
  }
  __syncthreads();

  for (uint64_t blk = blockIdx.y; blk < n_blocks; blk += gridDim.y) {
    const uint64_t start = blk * QB;
    const int n = (int)((tokens - start) < (uint64_t)QB ? (tokens - start) : (uint64_t)QB);
    const bool active = ti < n;
    float4 rv[QC];
    if (active) {
      const uint64_t base = ((start + ti) * (uint64_t)H + h) * QD;
#pragma unroll
      for (int k = 0; k < QC; ++k) rv[k] = load4<IN_DT>(J.x, base + chunk_dim(k, q));
    } else {
#pragma unroll
      for (int k = 0; k < QC; ++k) rv[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    uint32_t packed = 0;
    for (int s = 0; s < stages; ++s) {
      // ---- f32 screen of the nearest codeword
      float2 g1 = make_float2(0.0f, 0.0f), g2 = g1, g3 = g1, rr2 = g1;
#pragma unroll
      for (int k = 0; k < QC; ++k) {
        const int d0 = chunk_dim(k, q);
        const float4 u1 = *reinterpret_cast<const float4*>(&sm.u[s][0][d0]);
        const float4 u2 = *reinterpret_cast<const float4*>(&sm.u[s][1][d0]);
        const float4 u3 = *reinterpret_cast<const float4*>(&sm.u[s][2][d0]);
        const float2 ra = make_float2(rv[k].x, rv[k].y), rb = make_float2(rv[k].z, rv[k].w);
        g1 = __ffma2_rn(ra, make_float2(u1.x, u1.y), g1);
        g2 = __ffma2_rn(ra, make_float2(u2.x, u2.y), g2);
        g3 = __ffma2_rn(ra, make_float2(u3.x, u3.y), g3);
        rr2 = __ffma2_rn(ra, ra, rr2);
        g1 = __ffma2_rn(rb, make_float2(u1.z, u1.w), g1);
        g2 = __ffma2_rn(rb, make_float2(u2.z, u2.w), g2);
        g3 = __ffma2_rn(rb, make_float2(u3.z, u3.w), g3);
        rr2 = __ffma2_rn(rb, rb, rr2);
      }
      const float G1 = quad_sum(__fadd_rn(g1.x, g1.y)), G2 = quad_sum(__fadd_rn(g2.x, g2.y));
      const float G3 = quad_sum(__fadd_rn(g3.x, g3.y)), RR = quad_sum(__fadd_rn(rr2.x, rr2.y));
      const double rn = sqrt((double)RR) * (1.0 + 2e-5);  // >= |r|
      const double G[4] = {0.0, (double)G1, (double)G2, (double)G3};
      // S_j ~ T_j - T_0 with error <= E_j (S_0 = E_0 = 0 exactly)
      double S[4], E[4];
      S[0] = 0.0;
      E[0] = 0.0;
#pragma unroll
      for (int j = 1; j < 4; ++j) {
        const double ru = rn * (double)sm.unorm[s][j - 1];
        S[j] = (sm.ee[s][j] - sm.ee[s][0]) - 2.0 * G[j];
        E[j] = 1.6e-5 * ru + 2e-14 * (sm.ee[s][j] + sm.ee[s][0]) + 4e-15 * ru;
      }
      int c = 0;
      double Sc = 0.0, Ec = 0.0;
#pragma unroll
      for (int j = 1; j < 4; ++j)
        if (S[j] < Sc) {
          c = j;
          Sc = S[j];
          Ec = E[j];
        }
      const double ac = rn + (double)sm.enorm[s][c];
      bool sure = true;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const double aj = rn + (double)sm.enorm[s][j];
        const double tol = E[j] + Ec + 1.6e-14 * (aj * aj + ac * ac);
        sure &= (j == c) || ((S[j] - Sc) > tol);
      }
      if (!active) {
        c = 0;
        sure = true;
      }
      // ---- nearest() exactly as the reference (qvg.rs:303-321) where the
      // screen is not conclusive: one token at a time through smem, sequential
      // f64 squared distances, strict < so the lower index wins ties
      for (unsigned need = __ballot_sync(FULL, !sure && q == 0); need; need &= need - 1) {
        const int tl = __ffs(need) - 1;  // lane of the token's first thread
        if ((lane & ~(QT - 1)) == tl) {
#pragma unroll
          for (int k = 0; k < QC; ++k) *reinterpret_cast<float4*>(&sm.fbr[warp][chunk_dim(k, q)]) = rv[k];
        }
        __syncwarp();
        int ce = 0;
        if (lane == tl) {
          double best_d = __longlong_as_double(0x7FF0000000000000ll);
          for (int i = 0; i < QE; ++i) {
            const double* ei = sm.e64[s][i];
            double dist = 0.0;
            for (int d = 0; d < QD; ++d) {
              const double diff = __dsub_rn((double)sm.fbr[warp][d], ei[d]);
              dist = __dadd_rn(dist, __dmul_rn(diff, diff));
            }
            if (dist < best_d) {
              best_d = dist;
              ce = i;
            }
          }
        }
        ce = __shfl_sync(FULL, ce, tl);
        if ((lane & ~(QT - 1)) == tl) c = ce;
        __syncwarp();
      }
      // ---- numerator: this thread's 32 exact products, parallel order
      const double* ec = sm.e64[s][c];
      double a0 = 0.0, a1 = 0.0;
#pragma unroll
      for (int k = 0; k < QC; ++k) {
        const int d0 = chunk_dim(k, q);
        const double2 e01 = *reinterpret_cast<const double2*>(&ec[d0]);
        const double2 e23 = *reinterpret_cast<const double2*>(&ec[d0 + 2]);
        a0 = fma((double)rv[k].x, e01.x, a0);
        a1 = fma((double)rv[k].y, e01.y, a1);
        a0 = fma((double)rv[k].z, e23.x, a0);
        a1 = fma((double)rv[k].w, e23.y, a1);
      }
      double in = quad_sum(__dadd_rn(a0, a1));
      double sb = rn * (double)sm.enorm[s][c];  // >= sum_d |r_d e_cd|
      double dvv = sm.ee[s][c];
      if (!active) in = sb = dvv = 0.0;
      in = tokens_sum(in);
      sb = tokens_sum(sb);
      dvv = tokens_sum(dvv);
      if (lane == 0) {
        sm.part[warp][0] = in;
        sm.part[warp][1] = sb;
        sm.part[warp][2] = dvv;
      }
      __syncthreads();
      if (warp == 0) {
        float alpha = 0.0f;
        int cert = 0;
        if (lane == 0) {
          double v[3];
#pragma unroll
          for (int m = 0; m < 3; ++m)
            v[m] = __dadd_rn(__dadd_rn(__dadd_rn(sm.part[0][m], sm.part[1][m]), __dadd_rn(sm.part[2][m], sm.part[3][m])),
                             __dadd_rn(__dadd_rn(sm.part[4][m], sm.part[5][m]), __dadd_rn(sm.part[6][m], sm.part[7][m])));
          cert = certify_alpha(v[0], v[1], v[2], &alpha);
          sm.cert = cert;
          if (cert) J.scales[((size_t)h * n_blocks + blk) * stages + s] = alpha;
        }
        cert = __shfl_sync(FULL, cert, 0);
        alpha = __shfl_sync(FULL, alpha, 0);
        if (cert) build_table(sm, s, alpha, lane);
      }
      __syncthreads();
      if (!sm.cert) {  // uniform over the CTA
        // the reference's sums: inner sums sequential in d (qvg.rs:223-227),
        // one token at a time per warp
        for (int tk = 0; tk < 32 / QT; ++tk) {
          const int tl = tk * QT, tok = warp * (32 / QT) + tk;
          if ((lane & ~(QT - 1)) == tl) {
#pragma unroll
            for (int k = 0; k < QC; ++k) *reinterpret_cast<float4*>(&sm.fbr[warp][chunk_dim(k, q)]) = rv[k];
          }
          __syncwarp();
          if (lane == tl) {
            double acc = 0.0;
            if (tok < n)
              for (int d = 0; d < QD; ++d) acc = fma((double)sm.fbr[warp][d], ec[d], acc);
            sm.inner[tok] = acc;
            sm.dv[tok] = tok < n ? sm.ee[s][c] : 0.0;
          }
          __syncwarp();
        }
        __syncthreads();
        if (warp == 0) {
          float alpha = 0.0f;
          if (lane == 0) {
            // token order; idle tokens add +0, which leaves a sum started at +0 unchanged
            double num = 0.0, den = 0.0;
            for (int i = 0; i < QB; ++i) {
              num = __dadd_rn(num, sm.inner[i]);
              den = __dadd_rn(den, sm.dv[i]);
            }
            alpha = den > 1e-12 ? __double2float_rn(__ddiv_rn(num, den)) : 1.0f;  // qvg.rs:230
            J.scales[((size_t)h * n_blocks + blk) * stages + s] = alpha;
          }
          alpha = __shfl_sync(FULL, alpha, 0);
          build_table(sm, s, alpha, lane);
        }
        __syncthreads();
      }
      // ---- r + (-f32(alpha * e)): the second rounding
#pragma unroll
      for (int k = 0; k < QC; ++k) {
        const float4 np = *reinterpret_cast<const float4*>(&sm.nP[c][chunk_dim(k, q)]);
        const float2 lo = __fadd2_rn(make_float2(rv[k].x, rv[k].y), make_float2(np.x, np.y));
        const float2 hi = __fadd2_rn(make_float2(rv[k].z, rv[k].w), make_float2(np.z, np.w));
        rv[k] = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      packed |= (uint32_t)c << (2 * s);
    }
    if (active && q == 0) J.codes[(start + ti) * (uint64_t)H + h] = (uint8_t)packed;
  }
}

// Launches the d128 kernel when the codec has the reference's default shape
// (2 bits, block 64, <= 4 stages, head_dim 128) and the inputs are 16-byte
// aligned; returns false otherwise (the caller then uses k_qvg_encode).
bool launch_qvg_encode_d128(const QvgEncodeJob* jobs_dev, int n_jobs, int in_dtype, int H, int D, uint64_t tokens,
                            int stages, int bits, int block, bool aligned16, cudaStream_t s, cudaError_t* err) {
  if (D != QD || bits != 2 || block != QB || stages < 1 || stages > QSMAX || !aligned16) return false;
  const uint64_t n_blocks = (tokens + QB - 1) / QB;
  // enough CTAs to fill the GPU several times; each loops over its blocks so
  // the codebook tables are built once per CTA
  uint64_t per = (uint64_t)H * (uint64_t)n_jobs;
  uint64_t gy = (148ull * 8 + per - 1) / per;
  if (gy > n_blocks) gy = n_blocks;
  if (gy < 1) gy = 1;
  dim3 grid((unsigned)H, (unsigned)gy, (unsigned)n_jobs);
  switch (in_dtype) {
    case F32: k_qvg_encode_d128<F32><<<grid, QTHREADS, 0, s>>>(jobs_dev, H, tokens, stages); break;
    case BF16: k_qvg_encode_d128<BF16><<<grid, QTHREADS, 0, s>>>(jobs_dev, H, tokens, stages); break;
    default: k_qvg_encode_d128<F16><<<grid, QTHREADS, 0, s>>>(jobs_dev, H, tokens, stages); break;
  }
  *err = cudaGetLastError();
  return true;
}

}  // namespace nkv
