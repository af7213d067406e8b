// kernels_gather.cu — the rebuild side of the lifelong KV cache on sm_100a.
//
// HistoryCache::rebuild (cache/history.rs:341-446) decodes every represented
// archived segment in full and index_selects the sampled frames' token runs
// plus the text block.  Here the host turns the selection into a list of
// contiguous token runs and one kernel gathers exactly those tokens from the
// archive, decoding on the fly:
//   RUN_FLOAT     : copy (archive already holds the model dtype),
//   RUN_INT8      : (u8 - 128) * scale, then to_dtype(model)  (int8.rs:139-155),
//   RUN_QVG_VIDEO : sum_s alpha_s * cb_s[code_s] in f32 from +0, then
//                   to_dtype(model)                           (qvg.rs:259-300).
// Only selected tokens are read; every output byte is written once.
//
// Work decomposition: one CTA per (tile, layer, side).  A tile is <= 32
// tokens of one run; each thread handles 16-value chunks (one 16-byte code
// load, 32 or 64 bytes of stores), 4 chunks in flight.
#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"

namespace nkv {

namespace {

// 16 dequantized values (u8 code - 128) * s as f32.  (f32(q) + (-128)) is
// exact; the product rounds once, like candle's broadcast_mul.
__device__ __forceinline__ void dequant16(const uint4 w, float s, float (&o)[16]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // 0x4B0000bb = 2^23 + byte; minus (2^23 + 128) = byte - 128 exactly
      const float f = __uint_as_float(__byte_perm(ws[j], 0x4B00u, 0x5440u + k));
      o[4 * j + k] = __fmul_rn(__fadd_rn(f, -8388736.0f), s);
    }
  }
}

// Store 16 f32 values rounded to OUT_DT at element offset `i` (16-aligned).
// NONNAN: no value is NaN (dequantized INT8), so the hardware pair
// converters give the reference's bits.
template <int OUT_DT, bool NONNAN>
__device__ __forceinline__ void store16(void* out, uint64_t i, const float (&v)[16]) {
  if constexpr (OUT_DT == F32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + i);
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if constexpr (NONNAN && OUT_DT == BF16) {
        w[j] = dev::bf16x2_bits_nonnan(v[2 * j], v[2 * j + 1]);
      } else if constexpr (NONNAN) {
        w[j] = dev::f16x2_bits_nonnan(v[2 * j], v[2 * j + 1]);
      } else if constexpr (OUT_DT == BF16) {
        w[j] = (dev::bf16_bits(v[2 * j]) & 0xFFFFu) | (dev::bf16_bits(v[2 * j + 1]) << 16);
      } else {
        w[j] = (dev::f16_bits(v[2 * j]) & 0xFFFFu) | (dev::f16_bits(v[2 * j + 1]) << 16);
      }
    }
    uint4* p = reinterpret_cast<uint4*>(static_cast<unsigned short*>(out) + i);
    p[0] = make_uint4(w[0], w[1], w[2], w[3]);
    p[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

}  // namespace

constexpr int kGatherThreads = 256;

template <int OUT_DT>
__global__ void __launch_bounds__(kGatherThreads) k_gather(const GatherArgs a) {
  if (a.abort_flag && *a.abort_flag) return;
  const GatherTile tile = a.tiles[blockIdx.x];
  const int layer = blockIdx.y;
  const int side = blockIdx.z;
  const GatherRun& run = a.runs[tile.run];
  const int H = a.H, D = a.D;
  const int64_t HD = (int64_t)H * D;
  const unsigned char* base = run.src + (int64_t)layer * run.layer_stride;
  const int64_t off_data = side ? run.off[1] : run.off[0];
  const int64_t off_scale = side ? run.off[3] : run.off[2];
  void* const* outs = run.out_set ? (side ? a.out2_v : a.out2_k) : (side ? a.out_v : a.out_k);
  void* out_base = outs[layer];
  const int64_t out_tok = (int64_t)tile.b * (run.out_set ? a.out2_L : a.out_L) + run.dst_tok + tile.tok0;
  const int64_t src_tok = (int64_t)tile.b * run.src_L + run.src_tok + tile.tok0;
  // Chunk arithmetic in 32 bits: a tile holds at most 32 tokens.
  const int chunks_per_tok = (int)(HD / 16);
  const int chunks_per_head = D / 16;
  const int n_chunks = tile.ntok * chunks_per_tok;
  constexpr int U = 4;

  if (run.kind == RUN_INT8) {
    const uint8_t* codes = base + off_data + src_tok * HD;
    const float* scales = reinterpret_cast<const float*>(base + off_scale) + src_tok * H;
    for (int c0 = threadIdx.x; c0 < n_chunks; c0 += kGatherThreads * U) {
      uint4 w[U];
      float s[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * kGatherThreads;
        if (c < n_chunks) {
          w[u] = __ldg(reinterpret_cast<const uint4*>(codes) + c);
          const int t = c / chunks_per_tok;
          const int h = (c - t * chunks_per_tok) / chunks_per_head;
          s[u] = __ldg(scales + t * H + h);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * kGatherThreads;
        if (c < n_chunks) {
          float v[16];
          dequant16(w[u], s[u], v);
          store16<OUT_DT, true>(out_base, (uint64_t)(out_tok * HD + (int64_t)c * 16), v);
        }
      }
    }
  } else if (run.kind == RUN_FLOAT) {
    const size_t esz = OUT_DT == F32 ? 4 : 2;
    const uint4* src = reinterpret_cast<const uint4*>(base + off_data + src_tok * HD * esz);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<unsigned char*>(out_base) + out_tok * HD * esz);
    const int64_t n16 = (int64_t)tile.ntok * HD * esz / 16;
    for (int64_t c0 = threadIdx.x; c0 < n16; c0 += (int64_t)kGatherThreads * U) {
      uint4 w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + (int64_t)u * kGatherThreads;
        if (c < n16) w[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + (int64_t)u * kGatherThreads;
        if (c < n16) dst[c] = w[u];
      }
    }
  } else {  // RUN_QVG_VIDEO
    const int stages = a.stages, bits = a.bits, E = 1 << bits;
    const int bpt = (stages * bits + 7) / 8;
    const uint8_t* codes = base + off_data;
    const float* scales = reinterpret_cast<const float*>(base + off_scale);
    const float* cb = a.cb + (int64_t)layer * a.cb_layer_stride + (int64_t)side * H * stages * E * D;
    const uint32_t mask = (1u << bits) - 1u;
    for (int c = threadIdx.x; c < n_chunks; c += kGatherThreads) {
      const int t = c / chunks_per_tok;
      const int w = c - t * chunks_per_tok;
      const int h = w / chunks_per_head;
      const int d0 = (w - h * chunks_per_head) * 16;
      const int64_t tok = src_tok + t;  // batch is 1 for QVG
      const uint8_t* cp = codes + (tok * H + h) * bpt;
      uint64_t packed = 0;
      for (int b = 0; b < bpt; ++b) packed |= (uint64_t)__ldg(cp + b) << (8 * b);
      const int64_t blk = tok / a.block;
      const float* al = scales + ((int64_t)h * run.n_blocks + blk) * stages;
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.0f;
      for (int s = 0; s < stages; ++s) {
        const uint32_t code = (uint32_t)(packed >> (s * bits)) & mask;
        const float alpha = __ldg(al + s);
        const float4* e = reinterpret_cast<const float4*>(cb + (((int64_t)h * stages + s) * E + code) * D + d0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 q = __ldg(e + j);
          v[4 * j] = __fadd_rn(v[4 * j], __fmul_rn(alpha, q.x));
          v[4 * j + 1] = __fadd_rn(v[4 * j + 1], __fmul_rn(alpha, q.y));
          v[4 * j + 2] = __fadd_rn(v[4 * j + 2], __fmul_rn(alpha, q.z));
          v[4 * j + 3] = __fadd_rn(v[4 * j + 3], __fmul_rn(alpha, q.w));
        }
      }
      store16<OUT_DT, false>(out_base, (uint64_t)(out_tok * HD + (int64_t)c * 16), v);
    }
  }
}

// Any shape (head_dim not a multiple of 16, or unaligned tensors): one
// thread per output element, same arithmetic.
template <int OUT_DT>
__global__ void __launch_bounds__(kGatherThreads) k_gather_generic(const GatherArgs a) {
  if (a.abort_flag && *a.abort_flag) return;
  const GatherTile tile = a.tiles[blockIdx.x];
  const int layer = blockIdx.y;
  const int side = blockIdx.z;
  const GatherRun& run = a.runs[tile.run];
  const int H = a.H, D = a.D;
  const int64_t HD = (int64_t)H * D;
  const unsigned char* base = run.src + (int64_t)layer * run.layer_stride;
  const int64_t off_data = side ? run.off[1] : run.off[0];
  const int64_t off_scale = side ? run.off[3] : run.off[2];
  void* const* outs = run.out_set ? (side ? a.out2_v : a.out2_k) : (side ? a.out_v : a.out_k);
  void* out_base = outs[layer];
  const int64_t out_tok = (int64_t)tile.b * (run.out_set ? a.out2_L : a.out_L) + run.dst_tok + tile.tok0;
  const int64_t src_tok = (int64_t)tile.b * run.src_L + run.src_tok + tile.tok0;
  const int64_t n = (int64_t)tile.ntok * HD;
  for (int64_t i = threadIdx.x; i < n; i += kGatherThreads) {
    const int64_t t = i / HD;
    const int64_t rem = i - t * HD;
    const int h = (int)(rem / D);
    const int d = (int)(rem - (int64_t)h * D);
    float v;
    if (run.kind == RUN_INT8) {
      const uint8_t q = base[off_data + (src_tok + t) * HD + rem];
      const float sc = reinterpret_cast<const float*>(base + off_scale)[(src_tok + t) * H + h];
      v = __fmul_rn(__fadd_rn((float)q, -128.0f), sc);
    } else if (run.kind == RUN_FLOAT) {
      const int64_t j = (src_tok + t) * HD + rem;
      if constexpr (OUT_DT == F32) v = reinterpret_cast<const float*>(base + off_data)[j];
      else {
        reinterpret_cast<unsigned short*>(out_base)[(out_tok + t) * HD + rem] =
            reinterpret_cast<const unsigned short*>(base + off_data)[j];
        continue;
      }
    } else {
      const int stages = a.stages, bits = a.bits, E = 1 << bits, bpt = (stages * bits + 7) / 8;
      const int64_t tok = src_tok + t;
      const uint8_t* cp = base + off_data + (tok * H + h) * bpt;
      uint64_t packed = 0;
      for (int b = 0; b < bpt; ++b) packed |= (uint64_t)cp[b] << (8 * b);
      const float* al = reinterpret_cast<const float*>(base + off_scale) +
                        ((int64_t)h * run.n_blocks + tok / a.block) * stages;
      const float* cb = a.cb + (int64_t)layer * a.cb_layer_stride + (int64_t)side * H * stages * E * D;
      v = 0.0f;
      for (int s = 0; s < stages; ++s) {
        const uint32_t code = (uint32_t)(packed >> (s * bits)) & ((1u << bits) - 1u);
        v = __fadd_rn(v, __fmul_rn(al[s], cb[(((int64_t)h * stages + s) * E + code) * D + d]));
      }
    }
    dev::store_elem<OUT_DT>(out_base, (uint64_t)((out_tok + t) * HD + rem), v);
  }
}

// ---------------------------------------------------------------------------
// Table-driven QVG video decode (qvg.rs:259-300) for the default codec
// (4 stages x 2 bits, head_dim 128).  Inside one 64-token payload block the
// alphas are fixed, so per (block, head) the reference's decode
//   out = (((+0 + a0 e0[c0]) + a1 e1[c1]) + a2 e2[c2]) + a3 e3[c3]
// (every product and sum rounded to f32, in this order) takes its first two
// steps from a 16-row table Q01[c0][c1] = RN(RN(+0 + RN(a0 e0[c0])) + RN(a1 e1[c1])),
// the third from P2[c2] = RN(a2 e2[c2]) and the last from P3[c3] =
// RN(a3 e3[c3]).  The tables are built with the same f32 operations, so
// every output is bit-identical.  Q01 and P2 live in shared memory; P3 lives
// in registers: warp w always serves head w % 4 and lane l always columns
// 4l..4l+3, so its 4 x 4 P3 values are fixed and three selects pick the row.
// Per value that is 8 bytes of shared-memory reads (the kernel's limit)
// instead of 16 bytes of codebook rows through L1.
//
// CTA: one tile (<= 64 tokens of one block) x kQvgHeads heads x (layer, side);
// warp w decodes tokens w / 4, w / 4 + 2, ... of head w % 4, one 128-value
// row per warp instruction.
// ---------------------------------------------------------------------------
namespace {

constexpr int kQvgHeads = 4;
constexpr int kQvgThreads = 256;
constexpr int kQD = 128;
static_assert(kQvgThreads == 2 * kQvgHeads * 32, "two warps per head");

struct QvgTables {
  float q01[kQvgHeads][16][kQD];              // 32 KB
  float p2[kQvgHeads][4][kQD];                // 8 KB
  uint8_t code[kQvgTileTokens * kQvgHeads];   // the tile's packed codes, [token][head slot]
};  // 40.25 KB (dynamic shared memory)

__device__ __forceinline__ bool finite_f32(float v) { return (__float_as_uint(v) & 0x7FFFFFFFu) < 0x7F800000u; }

// FAST: no value can be NaN, so the hardware pair converters give the same
// bits as the integer rounding.
template <int OUT_DT, bool FAST>
__device__ __forceinline__ void store4(void* out, uint64_t i, float a, float b, float c, float d) {
  if constexpr (OUT_DT == F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + i) = make_float4(a, b, c, d);
  } else if constexpr (FAST) {
    uint32_t w0, w1;
    if constexpr (OUT_DT == BF16) {
      w0 = dev::bf16x2_bits_nonnan(a, b);
      w1 = dev::bf16x2_bits_nonnan(c, d);
    } else {
      w0 = dev::f16x2_bits_nonnan(a, b);
      w1 = dev::f16x2_bits_nonnan(c, d);
    }
    *reinterpret_cast<uint2*>(static_cast<unsigned short*>(out) + i) = make_uint2(w0, w1);
  } else {
    uint32_t w0, w1;
    if constexpr (OUT_DT == BF16) {
      w0 = (dev::bf16_bits(a) & 0xFFFFu) | (dev::bf16_bits(b) << 16);
      w1 = (dev::bf16_bits(c) & 0xFFFFu) | (dev::bf16_bits(d) << 16);
    } else {
      w0 = (dev::f16_bits(a) & 0xFFFFu) | (dev::f16_bits(b) << 16);
      w1 = (dev::f16_bits(c) & 0xFFFFu) | (dev::f16_bits(d) << 16);
    }
    *reinterpret_cast<uint2*>(static_cast<unsigned short*>(out) + i) = make_uint2(w0, w1);
  }
}

// P3 row c of this lane's 4 columns, by three selects (no local memory).
__device__ __forceinline__ float4 pick4(const float4 (&p)[4], uint32_t c) {
  const bool b0 = c & 1u, b1 = c & 2u;
  const float4 lo = b0 ? p[1] : p[0];
  const float4 hi = b0 ? p[3] : p[2];
  return b1 ? hi : lo;
}

// One output row: the 4 values of this lane for the token whose code is `code`.
template <int OUT_DT, bool FAST>
__device__ __forceinline__ void decode4(void* out, uint64_t o, const QvgTables& T, const float4 (&p3)[4], int hh,
                                        int d, uint32_t code) {
  const float4 x = *reinterpret_cast<const float4*>(&T.q01[hh][(code & 3u) * 4 + ((code >> 2) & 3u)][d]);
  const float4 y = *reinterpret_cast<const float4*>(&T.p2[hh][(code >> 4) & 3u][d]);
  const float4 z = pick4(p3, code >> 6);
  // (Q01 + P2) + P3, each add rounded: packed adds of table values (no
  // multiply anywhere in this data flow, so nothing can be contracted)
  const float2 lo = __fadd2_rn(__fadd2_rn(make_float2(x.x, x.y), make_float2(y.x, y.y)), make_float2(z.x, z.y));
  const float2 hi = __fadd2_rn(__fadd2_rn(make_float2(x.z, x.w), make_float2(y.z, y.w)), make_float2(z.z, z.w));
  store4<OUT_DT, FAST>(out, o, lo.x, lo.y, hi.x, hi.y);
}

template <int OUT_DT, bool FAST>
__device__ __forceinline__ void decode_rows(void* out, const QvgTables& T, const float4 (&p3)[4], int ntok,
                                            int64_t dst0, int H, int h, int hh, int tpar, int lane) {
  const int d = 4 * lane;
  const uint64_t step = (uint64_t)2 * H * kQD;  // two tokens on
  uint64_t o = ((uint64_t)(dst0 + tpar) * H + h) * kQD + d;
  int t = tpar;
  // two tokens per iteration (this warp's tokens are tpar, tpar + 2, ...)
  for (; t + 2 < ntok; t += 4, o += 2 * step) {
    const uint32_t c0 = T.code[t * kQvgHeads + hh], c1 = T.code[(t + 2) * kQvgHeads + hh];  // stage s: bits 2s, 2s+1
    decode4<OUT_DT, FAST>(out, o, T, p3, hh, d, c0);
    decode4<OUT_DT, FAST>(out, o + step, T, p3, hh, d, c1);
  }
  if (t < ntok) decode4<OUT_DT, FAST>(out, o, T, p3, hh, d, T.code[t * kQvgHeads + hh]);
}

}  // namespace

template <int OUT_DT>
__global__ void __launch_bounds__(kQvgThreads) k_gather_qvg(const GatherArgs a) {
  if (a.abort_flag && *a.abort_flag) return;
  extern __shared__ __align__(16) unsigned char qvg_smem[];
  QvgTables& T = *reinterpret_cast<QvgTables*>(qvg_smem);
  const GatherQvgTile tile = a.qtiles[blockIdx.x];
  const int layer = (int)(blockIdx.z >> 1), side = (int)(blockIdx.z & 1);
  const int H = a.H;
  const int h0 = (int)blockIdx.y * kQvgHeads;
  const int nh = min(kQvgHeads, H - h0);
  const GatherRun& run = a.runs[tile.run];
  const unsigned char* base = run.src + (int64_t)layer * run.layer_stride;
  const uint8_t* codes = base + (side ? run.off[1] : run.off[0]);
  const float* scales = reinterpret_cast<const float*>(base + (side ? run.off[3] : run.off[2]));
  const float* cb = a.cb + (int64_t)layer * a.cb_layer_stride + (int64_t)side * H * 16 * kQD;
  const int64_t src0 = run.src_tok + tile.tok0;
  uint32_t nonfinite = 0;  // any table entry inf or NaN

  // ---- the tile's codes, kQvgHeads slots per token (slots >= nh unused)
  for (int i = threadIdx.x; i < tile.ntok * kQvgHeads; i += kQvgThreads) {
    const int t = i / kQvgHeads, hh = i % kQvgHeads;
    if (hh < nh) T.code[i] = __ldg(codes + (src0 + t) * H + h0 + hh);
  }

  // ---- this lane's P3 values: head w % 4, columns 4 lane .. 4 lane + 3
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hh = warp % kQvgHeads, tpar = warp / kQvgHeads;
  float4 p3[4];
  if (hh < nh) {
    const int h = h0 + hh;
    const float a3 = __ldg(scales + ((int64_t)h * run.n_blocks + tile.blk) * 4 + 3);
    const float4* e3 = reinterpret_cast<const float4*>(cb + ((int64_t)h * 16 + 12) * kQD) + lane;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 e = __ldg(e3 + c * (kQD / 4));
      p3[c] = make_float4(__fmul_rn(a3, e.x), __fmul_rn(a3, e.y), __fmul_rn(a3, e.z), __fmul_rn(a3, e.w));
      nonfinite |= !(finite_f32(p3[c].x) && finite_f32(p3[c].y) && finite_f32(p3[c].z) && finite_f32(p3[c].w));
    }
  }

  // ---- Q01 and P2 in shared memory, thread per (head, d): <= 2 items each,
  // all loads issued before any use
  static_assert(kQvgHeads * kQD <= 2 * kQvgThreads, "two table items per thread");
  float ev[2][12], av[2][3];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = threadIdx.x + k * kQvgThreads;
    if (i < nh * kQD) {
      const int ih = i / kQD, d = i % kQD, h = h0 + ih;
      const float* al = scales + ((int64_t)h * run.n_blocks + tile.blk) * 4;
      const float* e = cb + (int64_t)h * 16 * kQD + d;  // [stage][entry][d]
#pragma unroll
      for (int s2 = 0; s2 < 3; ++s2) av[k][s2] = __ldg(al + s2);
#pragma unroll
      for (int r = 0; r < 12; ++r) ev[k][r] = __ldg(e + r * kQD);
    }
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = threadIdx.x + k * kQvgThreads;
    if (i < nh * kQD) {
      const int ih = i / kQD, d = i % kQD;
      float p0[4], p1[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        p0[c] = __fadd_rn(0.0f, __fmul_rn(av[k][0], ev[k][c]));  // out = +0, out += a0 e0
        p1[c] = __fmul_rn(av[k][1], ev[k][4 + c]);
        const float v2 = __fmul_rn(av[k][2], ev[k][8 + c]);
        T.p2[ih][c][d] = v2;
        nonfinite |= !finite_f32(v2);
      }
#pragma unroll
      for (int c0 = 0; c0 < 4; ++c0)
#pragma unroll
        for (int c1 = 0; c1 < 4; ++c1) {
          const float q = __fadd_rn(p0[c0], p1[c1]);
          T.q01[ih][c0 * 4 + c1][d] = q;
          nonfinite |= !finite_f32(q);
        }
    }
  }
  // With every table entry finite no output is NaN (finite sums can only
  // overflow to +-inf), so the hardware converters are exact.
  const bool all_finite = __syncthreads_and(nonfinite == 0) != 0;
  if (hh >= nh) return;
  void* const* outs = run.out_set ? (side ? a.out2_v : a.out2_k) : (side ? a.out_v : a.out_k);
  void* out = outs[layer];
  const int64_t dst0 = run.dst_tok + tile.tok0;  // batch 1
  if (all_finite) decode_rows<OUT_DT, true>(out, T, p3, tile.ntok, dst0, H, h0 + hh, hh, tpar, lane);
  else decode_rows<OUT_DT, false>(out, T, p3, tile.ntok, dst0, H, h0 + hh, hh, tpar, lane);
}

cudaError_t launch_gather(const GatherArgs& a, bool vector_ok, cudaStream_t s) {
  if (a.n_layers == 0) return cudaSuccess;
  if (a.n_qtiles > 0) {
    if (!vector_ok || a.D != kQD || a.n_layers > 32767) return cudaErrorInvalidValue;
    dim3 qgrid((unsigned)a.n_qtiles, (unsigned)((a.H + kQvgHeads - 1) / kQvgHeads), (unsigned)(2 * a.n_layers));
    const int smem = (int)sizeof(QvgTables);
    // above the 48 KB default: opt in (set on every launch, so it holds on
    // whichever device is current)
    auto prep = [&](const void* fn, int) -> cudaError_t {
      return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    };
    cudaError_t e = cudaSuccess;
    switch (a.out_dtype) {
      case F32:
        if ((e = prep((const void*)k_gather_qvg<F32>, 0)) == cudaSuccess)
          k_gather_qvg<F32><<<qgrid, kQvgThreads, smem, s>>>(a);
        break;
      case BF16:
        if ((e = prep((const void*)k_gather_qvg<BF16>, 1)) == cudaSuccess)
          k_gather_qvg<BF16><<<qgrid, kQvgThreads, smem, s>>>(a);
        break;
      default:
        if ((e = prep((const void*)k_gather_qvg<F16>, 2)) == cudaSuccess)
          k_gather_qvg<F16><<<qgrid, kQvgThreads, smem, s>>>(a);
        break;
    }
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (a.n_tiles == 0) return cudaSuccess;
  dim3 grid((unsigned)a.n_tiles, (unsigned)a.n_layers, 2);
  const bool vec = vector_ok && (a.D % 16) == 0;
  switch (a.out_dtype) {
    case F32:
      if (vec) k_gather<F32><<<grid, kGatherThreads, 0, s>>>(a);
      else k_gather_generic<F32><<<grid, kGatherThreads, 0, s>>>(a);
      break;
    case BF16:
      if (vec) k_gather<BF16><<<grid, kGatherThreads, 0, s>>>(a);
      else k_gather_generic<BF16><<<grid, kGatherThreads, 0, s>>>(a);
      break;
    default:
      if (vec) k_gather<F16><<<grid, kGatherThreads, 0, s>>>(a);
      else k_gather_generic<F16><<<grid, kGatherThreads, 0, s>>>(a);
      break;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Standalone dequantize (int8.rs:139-155) and QVG decode (qvg.rs:259-300),
// element per thread: used by the C-ABI kernel entry points and tests.
// ---------------------------------------------------------------------------
template <int OUT_DT>
__global__ void __launch_bounds__(256) k_dequantize(const uint8_t* __restrict__ q, const float* __restrict__ scales,
                                                    uint64_t n, int64_t D, void* out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const float sg = __fadd_rn(__fmul_rn((float)q[i], 1.0f), -128.0f);
    dev::store_elem<OUT_DT>(out, i, __fmul_rn(sg, __ldg(scales + i / (uint64_t)D)));
  }
}

cudaError_t launch_int8_dequantize(const uint8_t* q, const float* scales, uint64_t rows, int64_t D, int out_dtype,
                                   void* out, cudaStream_t s) {
  const uint64_t n = rows * (uint64_t)D;
  if (n == 0) return cudaSuccess;
  const uint64_t need = (n + 255) / 256;
  const unsigned grid = (unsigned)(need < 148ull * 32 ? need : 148ull * 32);
  switch (out_dtype) {
    case F32: k_dequantize<F32><<<grid, 256, 0, s>>>(q, scales, n, D, out); break;
    case BF16: k_dequantize<BF16><<<grid, 256, 0, s>>>(q, scales, n, D, out); break;
    default: k_dequantize<F16><<<grid, 256, 0, s>>>(q, scales, n, D, out); break;
  }
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_qvg_decode(const float* __restrict__ cb, const uint8_t* __restrict__ codes,
                                                    const float* __restrict__ scales, uint64_t tokens, int H, int D,
                                                    int stages, int bits, int block, float* __restrict__ out) {
  const int E = 1 << bits, bpt = (stages * bits + 7) / 8;
  const uint64_t n_blocks = (tokens + block - 1) / block;
  const uint64_t n = tokens * (uint64_t)H * D;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t th = i / D;
    const int d = (int)(i - th * D);
    const uint64_t tok = th / H;
    const int h = (int)(th - tok * H);
    uint64_t packed = 0;
    for (int b = 0; b < bpt; ++b) packed |= (uint64_t)codes[th * bpt + b] << (8 * b);
    float acc = 0.0f;
    for (int s = 0; s < stages; ++s) {
      const uint32_t code = (uint32_t)(packed >> (s * bits)) & ((1u << bits) - 1u);
      const float alpha = scales[((uint64_t)h * n_blocks + tok / block) * stages + s];
      acc = __fadd_rn(acc, __fmul_rn(alpha, cb[(((uint64_t)h * stages + s) * E + code) * D + d]));
    }
    out[i] = acc;
  }
}

cudaError_t launch_qvg_decode(const float* cb_side, const uint8_t* codes, const float* scales, uint64_t tokens,
                              int H, int D, int stages, int bits, int block, float* out, cudaStream_t s) {
  const uint64_t n = tokens * (uint64_t)H * D;
  if (n == 0) return cudaSuccess;
  const uint64_t need = (n + 255) / 256;
  const unsigned grid = (unsigned)(need < 148ull * 32 ? need : 148ull * 32);
  k_qvg_decode<<<grid, 256, 0, s>>>(cb_side, codes, scales, tokens, H, D, stages, bits, block, out);
  return cudaGetLastError();
}

}  // namespace nkv
