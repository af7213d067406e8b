// kernels_attn.cu — attention of the current queries over the archived
// history, reading the INT8 archive directly (the fused dequant-in-attention
// consumer of the working set).
//
// The reference concatenates the rebuilt history working set with the
// current segment's K / V and runs softmax(Q K^T / sqrt(D) + mask) V
// (modules/attention.rs:143-189, fed by model/dit.rs:355); every current
// token sees every history token (masks.rs: "history tokens are keys-only"),
// so the history part is unmasked.  This kernel computes that part without
// the materialised BF16 working set: for each 128-key tile of the history
// (the rebuild's run table, each tile inside one archived segment) it
// dequantizes the INT8 codes into shared memory exactly as the rebuild does
// (int8.rs:139-155: (code - 128) * scale in f32, rounded to bf16), and runs
//   S = Q K^T            tcgen05.mma kind::f16, bf16 operands, f32 in TMEM
//   online softmax       f32, one query row per thread
//   O_tile = P V         tcgen05.mma, P rounded to bf16 (the reference rounds
//                        its probabilities to the value dtype as well)
// and returns O (normalised, f32) and the row log-sum-exp, so a caller merges
// it with the masked current-segment part in the usual split-KV way.
//
// Shared-memory tiles are 128-byte-swizzled: a 128 x 128 bf16 tile is two
// halves of 64 columns, each 16 rows-groups of 8 rows x 128 bytes (1024-byte
// atoms) with the 16-byte chunk index XORed with the row in the atom.  Q, K
// and P are K-major operands of that layout; V, stored the same way (key
// rows, dims contiguous), is the MN-major operand of P V (its two halves are
// the 64-dim blocks, LBO 16 KB apart; key groups of 8 rows, SBO 1024 bytes).
//
// Every wait on an mbarrier gives up after 1 s of %globaltimer: the CTA then
// sets bit 0 of the caller's status word, frees its TMEM and returns.
#include <cuda_runtime.h>

#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"

namespace nkv {
namespace {

constexpr int AQ = 128;                    // queries per half (TMEM lanes)
constexpr int kHalves = 2;                 // query halves per CTA, sharing every K / V tile
constexpr int AK = 128;                    // keys per tile
constexpr int AD = 128;                    // head_dim
constexpr int kAttnThreads = 256;
constexpr int HALF_BYTES = 128 * 128;      // 128 rows x 64 bf16
constexpr int TILE_BYTES = 2 * HALF_BYTES; // 32 KB
// Q (two halves), K (two buffers), V, P (two halves); barriers; alignment.
constexpr int kAttnSmem = 7 * TILE_BYTES + 128 + 1024;
constexpr uint64_t kAttnWaitNs = 1000000000ull;

// S: f32 accumulate, bf16 A and B, both K-major, N = 128, M = 128.
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(AK >> 3) << 17) | (uint32_t(AQ >> 4) << 24);
// O: as S but B (V) MN-major, N = head_dim.
constexpr uint32_t kIdescO =
    (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (uint32_t(AD >> 3) << 17) | (uint32_t(AQ >> 4) << 24);

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `parity`; false when it ran out.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  if (bar_try(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (bar_try(bar, parity)) return true;
    if (gtimer() - t0 > kAttnWaitNs) return false;
  }
}

// Byte offset of 16-byte chunk `c` (0..15 across the 128 columns) of row
// `r` in a swizzled 128 x 128 bf16 tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return uint32_t((c >> 3) * HALF_BYTES + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// K-major SW128 descriptor (rows of 128 bytes, 8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// MN-major SW128 descriptor: 64-element MN blocks LBO = 16 KB apart, 8-row K
// groups SBO = 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {
  return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(HALF_BYTES >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane, waited for.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Store 32 f32 columns to this thread's TMEM lane, waited for.
__device__ __forceinline__ void tmem_store32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// The rebuild's dequantization (int8.rs:139-155) of 8 codes into 4 bf16
// pairs: RN((code - 128) * s) rounded to bf16.  code - 128 is exact as
// (2^23 + code) - (2^23 + 128), with 2^23 + code assembled by one byte
// permute; the product is the reference's one rounding; the values are
// finite, where the hardware pair conversion is the library's round to
// nearest even.
__device__ __forceinline__ uint4 dequant8(uint2 codes, float s) {
  uint32_t w[4];
  const uint32_t c[2] = {codes.x, codes.y};
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  const float2 s2 = make_float2(s, s);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t word = c[j >> 1];
    const uint32_t i0 = uint32_t((j & 1) * 2);
    // bytes [0x4B, 0, 0, code]: 0x4B0000xx = 2^23 + code
    const float a = __uint_as_float(__byte_perm(word, 0x4Bu, 0x4550u | i0));
    const float b = __uint_as_float(__byte_perm(word, 0x4Bu, 0x4550u | (i0 + 1)));
    const float2 v = __fmul2_rn(__fadd2_rn(make_float2(a, b), bias), s2);
    w[j] = dev::bf16x2_bits_nonnan(v.x, v.y);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace

// One CTA per (256-query tile, head): two halves of 128 queries share each
// dequantized K / V tile.  Warp w runs the softmax of half w / 4, rows
// 32 (w % 4) + lane (its TMEM lane quadrant); thread j dequantizes key row
// j % 128 of the next K tile (j < 128) or of the current V tile (j >= 128),
// from codes loaded one iteration ahead.  Per tile t:
//   1. thread 0 issues S_h = Q_h K_t^T for both halves (after P V of t - 1 in
//      the tensor pipe);
//   2. wait for P V of t - 1 (it read V and P);
//   3. dequantize K_{t+1} (second K buffer) and V_t; load the next codes;
//   4. wait for S; softmax, lazy rescale of O_h, P_h to shared memory;
//   5. thread 0 issues O_h += P_h V_t.
__global__ void __launch_bounds__(kAttnThreads, 1) k_attend_int8(const AttnArgs a) {
  extern __shared__ unsigned char attn_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(attn_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = base;                   // halves at 0 / TILE_BYTES
  unsigned char* Kb = base + 2 * TILE_BYTES;  // buffers at 0 / TILE_BYTES
  unsigned char* Vs = base + 4 * TILE_BYTES;
  unsigned char* Ps = base + 5 * TILE_BYTES;  // halves at 0 / TILE_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 7 * TILE_BYTES);  // [0] S done, [1] P V done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile uint32_t* abort_flag = tslot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hf = warp >> 2;                   // the softmax half of this warp
  const int row = (warp & 3) * 32 + lane;     // its query row in the half
  const int h = blockIdx.y, H = a.H;
  const int64_t q0 = int64_t(blockIdx.x) * (kHalves * AQ);
  const uint32_t barS = smem_addr(&bars[0]), barO = smem_addr(&bars[1]);
  const int n = a.n_tiles;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tslot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(barS) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(barO) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_flag = 0u;
  }
  // the two query halves (zero rows past the end): thread j loads row j
  {
    const int64_t q = q0 + tid;
    unsigned char* Qh = Qs + (tid >> 7) * TILE_BYTES;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (q < a.Lq) v = __ldg(reinterpret_cast<const uint4*>(a.q + (q * H + h) * AD) + c);
      *reinterpret_cast<uint4*>(Qh + swz(tid & 127, c)) = v;
    }
  }
  // this thread's dequantization job: key row kr of K (tid < 128) or V
  const int kr = tid & 127;
  const bool is_v = tid >= 128;
  uint4 codes[8];
  float scale = 0.0f;
  bool have = false;  // the registers hold the codes of the next job
  // the descriptor of the job after that, fetched a job ahead so the code
  // loads never wait for it
  AttnKeyTile nextT{};
  bool next_ok = false;
  auto fetch_desc = [&](int tile) {
    next_ok = tile < n;
    if (next_ok) nextT = a.tiles[tile];
  };
  auto load_job = [&]() {  // the codes of the job whose descriptor is prefetched
    have = next_ok && kr < nextT.ntok;
    if (!have) return;
    const int64_t r = int64_t(kr) * H + h;
    const uint4* src = reinterpret_cast<const uint4*>((is_v ? nextT.v_codes : nextT.k_codes) + r * AD);
#pragma unroll
    for (int c = 0; c < 8; ++c) codes[c] = __ldg(src + c);
    scale = __ldg((is_v ? nextT.v_scales : nextT.k_scales) + r);
  };
  auto store_job = [&](unsigned char* tile_base) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
      if (have) {
        lo = dequant8(make_uint2(codes[c].x, codes[c].y), scale);
        hi = dequant8(make_uint2(codes[c].z, codes[c].w), scale);
      }
      *reinterpret_cast<uint4*>(tile_base + swz(kr, 2 * c)) = lo;
      *reinterpret_cast<uint4*>(tile_base + swz(kr, 2 * c + 1)) = hi;
    }
  };
  // prologue: K_0 into buffer 0; next jobs: K_1 (rows < 128) and V_0
  fetch_desc(0);
  load_job();
  if (!is_v) {
    store_job(Kb);
    fetch_desc(1);
    load_job();
    fetch_desc(2);
  } else {
    fetch_desc(1);
  }
  fence_async_smem();
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_q = uint32_t((warp & 3) * 32) << 16;
  const uint32_t s_cols = tmem + lane_q + uint32_t(hf * 128);        // S_hf
  const uint32_t o_cols = tmem + lane_q + uint32_t(256 + hf * 128);  // O_hf

  float m = -INFINITY, l = 0.0f;
  bool ok = true;
  for (int t = 0; t < n; ++t) {
    const int ntok = a.tiles[t].ntok;
    // 1. S_h = Q_h K_t^T
    if (tid == 0) {
      const uint32_t kaddr = smem_addr(Kb + (t & 1) * TILE_BYTES);
#pragma unroll
      for (int hh = 0; hh < kHalves; ++hh)
#pragma unroll
        for (int kk = 0; kk < AD / 16; ++kk) {
          const uint32_t off = uint32_t((kk >> 2) * HALF_BYTES + (kk & 3) * 32);
          mma_f16(tmem + uint32_t(hh * 128), desc_k(smem_addr(Qs + hh * TILE_BYTES) + off), desc_k(kaddr + off),
                  kIdescS, kk > 0 ? 1u : 0u);
        }
      mma_commit(barS);
    }
    // 2. P V of the previous tile has read V and P
    if (t > 0 && !bar_wait(barO, uint32_t(t - 1) & 1u)) *abort_flag = 1u;
    tc_after();
    // 3. dequantize K_{t+1} / V_t, load the codes of K_{t+2} / V_{t+1}
    if (is_v) {
      store_job(Vs);
      load_job();  // V_{t+1}
      fetch_desc(t + 2);
    } else if (t + 1 < n) {
      store_job(Kb + ((t + 1) & 1) * TILE_BYTES);
      load_job();  // K_{t+2}
      fetch_desc(t + 3);
    }
    fence_async_smem();
    // 4. softmax of this thread's row of half hf (base-2 logits)
    if (!bar_wait(barS, uint32_t(t) & 1u)) *abort_flag = 1u;
    tc_after();
    float mt = -INFINITY;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      float sv[32];
      tmem_load32(s_cols + ch * 32, sv);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (ch * 32 + j < ntok) mt = fmaxf(mt, sv[j] * a.scale_log2);
    }
    const bool move = mt > m + 8.0f;
    const float mn = move ? mt : m;
    const float alpha = move ? exp2f(m - mn) : 1.0f;  // 0 on the first tile
    if (t > 0 && __any_sync(0xFFFFFFFFu, move)) {
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        float ov[32];
        tmem_load32(o_cols + ch * 32, ov);
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] *= alpha;
        tmem_store32(o_cols + ch * 32, ov);
      }
    }
    float lsum = 0.0f;
    unsigned char* Ph = Ps + hf * TILE_BYTES;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      float sv[32];
      tmem_load32(s_cols + ch * 32, sv);
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int k0 = ch * 32 + 2 * j;
        const float p0 = k0 < ntok ? fast_exp2(__fmaf_rn(sv[2 * j], a.scale_log2, -mn)) : 0.0f;
        const float p1 = k0 + 1 < ntok ? fast_exp2(__fmaf_rn(sv[2 * j + 1], a.scale_log2, -mn)) : 0.0f;
        lsum += p0 + p1;
        w[j] = dev::bf16x2_bits_nonnan(p0, p1);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(Ph + swz(row, ch * 4 + q)) =
            make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
    l = l * alpha + lsum;
    m = mn;
    fence_async_smem();
    tc_before();
    __syncthreads();
    tc_after();
    if (*abort_flag) {
      ok = false;
      break;
    }
    // 5. O_h += P_h V_t
    if (tid == 0) {
      const uint32_t vaddr = smem_addr(Vs);
#pragma unroll
      for (int hh = 0; hh < kHalves; ++hh)
#pragma unroll
        for (int kk = 0; kk < AK / 16; ++kk) {
          const uint32_t aoff = uint32_t((kk >> 2) * HALF_BYTES + (kk & 3) * 32);
          mma_f16(tmem + uint32_t(256 + hh * 128), desc_k(smem_addr(Ps + hh * TILE_BYTES) + aoff),
                  desc_mn(vaddr + uint32_t(kk * 2 * 1024)), kIdescO, (t > 0 || kk > 0) ? 1u : 0u);
        }
      mma_commit(barO);
    }
  }

  if (ok && n > 0) {
    if (!bar_wait(barO, uint32_t(n - 1) & 1u)) ok = false;
    tc_after();
  }
  if (ok && n > 0) {
    const int64_t q = q0 + hf * AQ + row;
    const float inv = 1.0f / l;
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      float ov[32];
      tmem_load32(o_cols + ch * 32, ov);
      if (q < a.Lq) {
        float4* out = reinterpret_cast<float4*>(a.out + (q * H + h) * AD + ch * 32);
#pragma unroll
        for (int d = 0; d < 8; ++d)
          out[d] = make_float4(ov[4 * d] * inv, ov[4 * d + 1] * inv, ov[4 * d + 2] * inv, ov[4 * d + 3] * inv);
      }
    }
    if (q < a.Lq) a.lse[int64_t(h) * a.Lq + q] = (m + log2f(l)) * 0.69314718055994531f;
  } else if (!ok && tid == 0) {
    atomicOr(a.status, 1u);
  }
  tc_before();
  __syncthreads();
  tc_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

cudaError_t launch_attend_int8(const AttnArgs& a, cudaStream_t s) {
  if (a.Lq <= 0 || a.H <= 0 || a.n_tiles <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k_attend_int8, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(unsigned((a.Lq + kHalves * AQ - 1) / (kHalves * AQ)), unsigned(a.H));
  k_attend_int8<<<grid, kAttnThreads, kAttnSmem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace nkv
