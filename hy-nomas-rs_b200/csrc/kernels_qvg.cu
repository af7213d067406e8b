// kernels_qvg.cu — QVG encode for the reference's default codec shape
// (4 entries per stage, head_dim 128, 64-token blocks, up to 4 stages):
// QvgCodec::encode (cache/qvg.rs:173-256) restated bit for bit with far less
// double-precision work than the literal algorithm.
//
// Per (token, stage) the reference
//   1. picks c = argmin_i D_i, D_i the sequential f64 sum of (r_d - e_id)^2
//      (nearest, qvg.rs:303-321; ties to the lower index),
//   2. adds the sequential f64 dot r . e_c to the block's numerator
//      (qvg.rs:220-229),
//   3. after alpha = f32(num / den) updates r_d -= f32(alpha * e_cd).
// Here step 1 is screened in f32: with u_i = e_i - e_0, the exact distance
// differences are T_i - T_0 = (|e_i|^2 - |e_0|^2) - 2 r.u_i, and the f32 dots
// carry a rigorous error bound (gamma_128 |r||u_i| plus the rounding of u_i).
// When the chosen entry beats every other by more than those bounds plus the
// reference's own f64 rounding (<= 1.5e-14 T), the reference's sequential
// f64 argmin is certainly the same entry; otherwise (near ties, duplicate
// codewords, NaN) the thread computes the reference's sequential f64
// distances exactly.  Step 2 is the reference's computation itself: products
// of f32 values are exact in f64, so the FMA chain in d order reproduces its
// rounding.  Step 3 is two f32 roundings, as in the reference: warp 0 builds
// the stage's table -f32(alpha * e_c) with scalar multiplies, and each token
// adds its row with packed f32x2 adds (no multiply in the thread's data flow,
// so nothing can be contracted into one rounding).
//
// One CTA of 64 threads per (layer x side, head, group of blocks); thread t
// owns token t of the current block, its residual in registers.
#include <cfloat>
#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"

namespace nkv {

namespace {

constexpr int QD = 128;    // head_dim
constexpr int QE = 4;      // codewords per stage (2 bits)
constexpr int QB = 64;     // tokens per block
constexpr int QSMAX = 4;   // stages

struct QvgSmem {
  float u[QSMAX][3][QD];           // e_i - e_0 rounded to f32, i = 1..3
  float e32[QSMAX][QE][QD + 4];    // codewords (rows padded against bank conflicts)
  double e64[QSMAX][QE][QD + 1];   // codewords as f64
  double ee[QSMAX][QE];            // sequential f64 sum of e_d^2 (the den inner sum)
  float enorm[QSMAX][QE];          // upper bounds of |e_i|
  float unorm[QSMAX][3];           // upper bounds of |e_i - e_0|
  double inner[QB];                // per-token numerator inner sums (+0 for idle threads)
  double dv[QB];                   // per-token denominator inner sums (+0 for idle threads)
  float nP[QE][QD + 4];            // -f32(alpha * e_c) of the current stage (rows padded)
};

}  // namespace

template <int IN_DT>
__global__ void __launch_bounds__(QB, 6) k_qvg_encode_d128(const QvgEncodeJob* __restrict__ jobs, int H,
                                                        uint64_t tokens, int stages) {
  __shared__ QvgSmem sm;
  const QvgEncodeJob J = jobs[blockIdx.z];
  const int h = blockIdx.x;
  const int t = threadIdx.x;
  const uint64_t n_blocks = (tokens + QB - 1) / QB;

  // ---- codebooks of this (side, head), all stages
  const float* cbh = J.cb + (size_t)h * stages * QE * QD;
  for (int i = t; i < stages * QE * QD; i += QB) {
    const int s = i / (QE * QD), e = (i / QD) % QE, d = i % QD;
    const float v = __ldg(cbh + i);
    sm.e32[s][e][d] = v;
    sm.e64[s][e][d] = (double)v;
  }
  __syncthreads();
  for (int i = t; i < stages * 3 * QD; i += QB) {
    const int s = i / (3 * QD), j = (i / QD) % 3, d = i % QD;
    sm.u[s][j][d] = __fsub_rn(sm.e32[s][j + 1][d], sm.e32[s][0][d]);
  }
  for (int i = t; i < stages * QE; i += QB) {
    const int s = i / QE, e = i % QE;
    double acc = 0.0;
    for (int d = 0; d < QD; ++d) acc = fma(sm.e64[s][e][d], sm.e64[s][e][d], acc);  // exact products
    sm.ee[s][e] = acc;
    sm.enorm[s][e] = (float)(sqrt(acc) * (1.0 + 1e-6));
  }
  __syncthreads();
  for (int i = t; i < stages * 3; i += QB) {
    const int s = i / 3, j = i % 3;
    double acc = 0.0;
    for (int d = 0; d < QD; ++d) acc = fma((double)sm.u[s][j][d], (double)sm.u[s][j][d], acc);
    sm.unorm[s][j] = (float)(sqrt(acc) * (1.0 + 1e-6));
  }
  __syncthreads();

  for (uint64_t blk = blockIdx.y; blk < n_blocks; blk += gridDim.y) {
    const uint64_t start = blk * QB;
    const int n = (int)((tokens - start) < (uint64_t)QB ? (tokens - start) : (uint64_t)QB);
    const bool active = t < n;
    float2 r[QD / 2];
    if (active) {
      const uint64_t base = ((start + t) * (uint64_t)H + h) * QD;
#pragma unroll
      for (int k = 0; k < QD / 8; ++k) {
        float x[8];
        dev::load8<IN_DT>(J.x, base + 8 * k, x);
#pragma unroll
        for (int j = 0; j < 4; ++j) r[4 * k + j] = make_float2(x[2 * j], x[2 * j + 1]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < QD / 2; ++k) r[k] = make_float2(0.0f, 0.0f);
    }
    uint32_t packed = 0;
    for (int s = 0; s < stages; ++s) {
      int c = 0;
      double acc = 0.0;
      if (active) {
        // ---- f32 screen of the nearest codeword
        float2 g1 = make_float2(0.0f, 0.0f), g2 = g1, g3 = g1, rr2 = g1;
#pragma unroll
        for (int k = 0; k < QD / 4; ++k) {
          const float4 u1 = *reinterpret_cast<const float4*>(&sm.u[s][0][4 * k]);
          const float4 u2 = *reinterpret_cast<const float4*>(&sm.u[s][1][4 * k]);
          const float4 u3 = *reinterpret_cast<const float4*>(&sm.u[s][2][4 * k]);
          const float2 ra = r[2 * k], rb = r[2 * k + 1];
          g1 = __ffma2_rn(ra, make_float2(u1.x, u1.y), g1);
          g2 = __ffma2_rn(ra, make_float2(u2.x, u2.y), g2);
          g3 = __ffma2_rn(ra, make_float2(u3.x, u3.y), g3);
          rr2 = __ffma2_rn(ra, ra, rr2);
          g1 = __ffma2_rn(rb, make_float2(u1.z, u1.w), g1);
          g2 = __ffma2_rn(rb, make_float2(u2.z, u2.w), g2);
          g3 = __ffma2_rn(rb, make_float2(u3.z, u3.w), g3);
          rr2 = __ffma2_rn(rb, rb, rr2);
        }
        const double rn = sqrt((double)__fadd_rn(rr2.x, rr2.y)) * (1.0 + 2e-5);  // >= |r|
        const double G[4] = {0.0, (double)__fadd_rn(g1.x, g1.y), (double)__fadd_rn(g2.x, g2.y),
                             (double)__fadd_rn(g3.x, g3.y)};
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
        if (!sure) {
          // nearest() exactly as the reference (qvg.rs:303-321): sequential f64
          // squared distances, strict < so the lower index wins ties
          double best_d = __longlong_as_double(0x7FF0000000000000ll);
          c = 0;
#pragma unroll 1
          for (int i = 0; i < QE; ++i) {
            const double* ei = sm.e64[s][i];
            double dist = 0.0;
#pragma unroll
            for (int k = 0; k < QD / 2; ++k) {
              double diff = __dsub_rn((double)r[k].x, ei[2 * k]);
              dist = __dadd_rn(dist, __dmul_rn(diff, diff));
              diff = __dsub_rn((double)r[k].y, ei[2 * k + 1]);
              dist = __dadd_rn(dist, __dmul_rn(diff, diff));
            }
            if (dist < best_d) {
              best_d = dist;
              c = i;
            }
          }
        }
        // ---- numerator inner sum of the chosen codeword, in the reference's order
        const double* ec = sm.e64[s][c];
#pragma unroll
        for (int k = 0; k < QD / 2; ++k) {
          acc = fma((double)r[k].x, ec[2 * k], acc);
          acc = fma((double)r[k].y, ec[2 * k + 1], acc);
        }
      }
      sm.inner[t] = acc;                    // +0 for idle threads
      sm.dv[t] = active ? sm.ee[s][c] : 0.0;
      __syncthreads();
      if (t < 32) {
        // warp 0: alpha = f32(num / den) of the block's sums in token order
        // (qvg.rs:220-230); idle tokens add +0, which leaves a sum started at
        // +0 unchanged.  The sums are first taken as a 64-term tree (depth 6)
        // across the warp: a tree and the sequential order differ by at most
        // (gamma_6 + gamma_63) sum|x| <= 2^-46 sum|x| (u = 2^-53), so the
        // reference's quotient lies in an interval computed with outward
        // rounding; when both ends round to the same f32 (and den > 1e-12 is
        // certain either way) that is the reference's alpha.  Otherwise (a
        // numerator interval around 0, non-finite terms, an f32 rounding
        // boundary inside the interval) lane 0 takes the sequential sums.
        const double n0 = sm.inner[2 * t], n1 = sm.inner[2 * t + 1];
        const double d0 = sm.dv[2 * t], d1 = sm.dv[2 * t + 1];
        double tn = __dadd_rn(n0, n1), an = __dadd_rn(fabs(n0), fabs(n1)), td = __dadd_rn(d0, d1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          tn = __dadd_rn(tn, __shfl_xor_sync(0xFFFFFFFFu, tn, o));
          an = __dadd_rn(an, __shfl_xor_sync(0xFFFFFFFFu, an, o));
          td = __dadd_rn(td, __shfl_xor_sync(0xFFFFFFFFu, td, o));
        }
        float alpha = 0.0f;
        if (t == 0) {
          const double kTreeVsSeq = 0x1p-46;  // >= (gamma_6 + gamma_63) / (1 - gamma_6)
          const double dn = __dmul_ru(an, kTreeVsSeq), dd = __dmul_ru(td, kTreeVsSeq);  // den terms are >= 0
          const double nlo = __dsub_rd(tn, dn), nhi = __dadd_ru(tn, dn);
          const double dlo = __dsub_rd(td, dd), dhi = __dadd_ru(td, dd);
          bool sure = isfinite(nlo) && isfinite(nhi) && isfinite(dlo) && isfinite(dhi);
          if (sure && dhi <= 1e-12) {
            alpha = 1.0f;  // den <= 1e-12 for certain
          } else if (sure && dlo > 1e-12 && (nlo > 0.0 || nhi < 0.0)) {
            const double qlo = nlo > 0.0 ? __ddiv_rd(nlo, dhi) : __ddiv_rd(nlo, dlo);
            const double qhi = nlo > 0.0 ? __ddiv_ru(nhi, dlo) : __ddiv_ru(nhi, dhi);
            const float alo = __double2float_rn(qlo), ahi = __double2float_rn(qhi);
            sure = alo == ahi;
            alpha = alo;
          } else {
            sure = false;
          }
          if (!sure) {
            double num = 0.0, den = 0.0;
#pragma unroll 1
            for (int i = 0; i < QB; ++i) {
              num = __dadd_rn(num, sm.inner[i]);
              den = __dadd_rn(den, sm.dv[i]);
            }
            alpha = den > 1e-12 ? __double2float_rn(__ddiv_rn(num, den)) : 1.0f;  // qvg.rs:230
          }
          J.scales[((size_t)h * n_blocks + blk) * stages + s] = alpha;
        }
        alpha = __shfl_sync(0xFFFFFFFFu, alpha, 0);
        // the stage's -f32(alpha * e) rows: one rounding per product, as the
        // reference's alpha * e[d] (qvg.rs:232-237)
#pragma unroll
        for (int i = t; i < QE * QD; i += 32) sm.nP[i / QD][i % QD] = __fmul_rn(-alpha, sm.e32[s][i / QD][i % QD]);
      }
      __syncthreads();
      if (active) {
        // r + (-f32(alpha * e)): the second rounding.  The table comes from
        // memory, so no multiply can be fused into these packed adds.
        const float* np = sm.nP[c];
#pragma unroll
        for (int k = 0; k < QD / 4; ++k) {
          const float4 q = *reinterpret_cast<const float4*>(&np[4 * k]);
          r[2 * k] = __fadd2_rn(r[2 * k], make_float2(q.x, q.y));
          r[2 * k + 1] = __fadd2_rn(r[2 * k + 1], make_float2(q.z, q.w));
        }
        packed |= (uint32_t)c << (2 * s);
      }
    }
    if (active) J.codes[(start + t) * (uint64_t)H + h] = (uint8_t)packed;
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
  uint64_t gy = (148ull * 40 + per - 1) / per;
  if (gy > n_blocks) gy = n_blocks;
  if (gy < 1) gy = 1;
  dim3 grid((unsigned)H, (unsigned)gy, (unsigned)n_jobs);
  switch (in_dtype) {
    case F32: k_qvg_encode_d128<F32><<<grid, QB, 0, s>>>(jobs_dev, H, tokens, stages); break;
    case BF16: k_qvg_encode_d128<BF16><<<grid, QB, 0, s>>>(jobs_dev, H, tokens, stages); break;
    default: k_qvg_encode_d128<F16><<<grid, QB, 0, s>>>(jobs_dev, H, tokens, stages); break;
  }
  *err = cudaGetLastError();
  return true;
}

}  // namespace nkv
