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

constexpr int AQ = 128;                    // queries per CTA (TMEM lanes)
constexpr int AK = 128;                    // keys per tile
constexpr int AD = 128;                    // head_dim
constexpr int kAttnThreads = 128;
constexpr int HALF_BYTES = 128 * 128;      // 128 rows x 64 bf16
constexpr int TILE_BYTES = 2 * HALF_BYTES; // 32 KB
constexpr int kAttnSmem = 4 * TILE_BYTES + 2 * AK * 4 + 64 + 1024;
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

// The rebuild's dequantization (int8.rs:139-155) of 8 codes into 4 bf16 pairs.
__device__ __forceinline__ uint4 dequant8(uint2 codes, float s) {
  uint32_t w[4];
  const uint32_t c[2] = {codes.x, codes.y};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t word = c[j >> 1];
    const int sh = (j & 1) * 16;
    const float a = __fmul_rn(__fadd_rn(__fmul_rn((float)((word >> sh) & 0xFFu), 1.0f), -128.0f), s);
    const float b = __fmul_rn(__fadd_rn(__fmul_rn((float)((word >> (sh + 8)) & 0xFFu), 1.0f), -128.0f), s);
    w[j] = (dev::bf16_bits(a) & 0xFFFFu) | (dev::bf16_bits(b) << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace

// One CTA per (128-query tile, head).  Thread t owns query row t (TMEM lane
// t) for the softmax and key row t of each tile for the dequantization.
__global__ void __launch_bounds__(kAttnThreads, 1) k_attend_int8(const AttnArgs a) {
  extern __shared__ unsigned char attn_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(attn_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = base;
  unsigned char* Ks = base + TILE_BYTES;
  unsigned char* Vs = base + 2 * TILE_BYTES;
  unsigned char* Ps = base + 3 * TILE_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + 4 * TILE_BYTES + 2 * AK * 4);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile uint32_t* abort_flag = tslot + 1;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int h = blockIdx.y, H = a.H;
  const int64_t q0 = int64_t(blockIdx.x) * AQ;
  const uint32_t bar_a = smem_addr(bar);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_addr(tslot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_flag = 0u;
  }
  // the query tile (zero rows past the end)
  {
    const int64_t q = q0 + tid;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (q < a.Lq) v = __ldg(reinterpret_cast<const uint4*>(a.q + (q * H + h) * AD) + c);
      *reinterpret_cast<uint4*>(Qs + swz(tid, c)) = v;
    }
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);

  // O accumulates in TMEM columns [128, 256) across the tiles.  Each row
  // keeps the base-2 maximum m its exponentials are taken against and moves
  // it only when a tile's maximum exceeds it by more than 8 (the unscaled
  // terms then stay below 2^8); a warp with such a row rescales its O rows.
  float m = -INFINITY, l = 0.0f;
  uint32_t phase = 0;
  bool ok = true;

  for (int t = 0; t < a.n_tiles; ++t) {
    const AttnKeyTile T = a.tiles[t];
    // ---- K and V rows of the tile, dequantized as the rebuild does
    {
      const bool valid = tid < T.ntok;
      const int64_t row = int64_t(tid) * H + h;
      const float sk = valid ? __ldg(T.k_scales + row) : 0.0f;
      const float sv = valid ? __ldg(T.v_scales + row) : 0.0f;
      const uint2* kc = reinterpret_cast<const uint2*>(T.k_codes + row * AD);
      const uint2* vc = reinterpret_cast<const uint2*>(T.v_codes + row * AD);
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        uint4 kb = make_uint4(0u, 0u, 0u, 0u), vb = kb;
        if (valid) {
          kb = dequant8(__ldg(kc + c), sk);
          vb = dequant8(__ldg(vc + c), sv);
        }
        *reinterpret_cast<uint4*>(Ks + swz(tid, c)) = kb;
        *reinterpret_cast<uint4*>(Vs + swz(tid, c)) = vb;
      }
    }
    fence_async_smem();
    tc_before();
    __syncthreads();
    tc_after();
    // ---- S = Q K^T into TMEM columns [0, 128)
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < AD / 16; ++kk) {
        const uint32_t off = uint32_t((kk >> 2) * HALF_BYTES + (kk & 3) * 32);
        mma_f16(tmem, desc_k(smem_addr(Qs) + off), desc_k(smem_addr(Ks) + off), kIdescS, kk > 0 ? 1u : 0u);
      }
      mma_commit(bar_a);
    }
    if (!bar_wait(bar_a, phase)) *abort_flag = 1u;
    phase ^= 1u;
    tc_after();
    __syncthreads();
    if (*abort_flag) {
      ok = false;
      break;
    }
    // ---- online softmax of this thread's row (base-2 logits)
    float mt = -INFINITY;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      float s[32];
      tmem_load32(lane_base + ch * 32, s);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (ch * 32 + j < T.ntok) mt = fmaxf(mt, s[j] * a.scale_log2);
    }
    const bool move = mt > m + 8.0f;
    const float mn = move ? mt : m;
    const float alpha = move ? exp2f(m - mn) : 1.0f;  // 0 on the first tile
    if (t > 0 && __any_sync(0xFFFFFFFFu, move)) {
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        float ov[32];
        tmem_load32(lane_base + 128 + ch * 32, ov);
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] *= alpha;
        tmem_store32(lane_base + 128 + ch * 32, ov);
      }
    }
    float lsum = 0.0f;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      float s[32];
      tmem_load32(lane_base + ch * 32, s);
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int k0 = ch * 32 + 2 * j;
        const float p0 = k0 < T.ntok ? exp2f(s[2 * j] * a.scale_log2 - mn) : 0.0f;
        const float p1 = k0 + 1 < T.ntok ? exp2f(s[2 * j + 1] * a.scale_log2 - mn) : 0.0f;
        lsum += p0 + p1;
        w[j] = dev::bf16x2_bits_nonnan(p0, p1);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(Ps + swz(tid, ch * 4 + q)) =
            make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
    l = l * alpha + lsum;
    m = mn;
    fence_async_smem();
    tc_before();
    __syncthreads();
    tc_after();
    // ---- O += P V into TMEM columns [128, 256)
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < AK / 16; ++kk) {
        const uint32_t aoff = uint32_t((kk >> 2) * HALF_BYTES + (kk & 3) * 32);
        mma_f16(tmem + 128, desc_k(smem_addr(Ps) + aoff), desc_mn(smem_addr(Vs) + uint32_t(kk * 2 * 1024)),
                kIdescO, (t > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(bar_a);
    }
    if (!bar_wait(bar_a, phase)) *abort_flag = 1u;
    phase ^= 1u;
    tc_after();
    __syncthreads();
    if (*abort_flag) {
      ok = false;
      break;
    }
  }

  if (ok) {
    const int64_t q = q0 + tid;
    const float inv = 1.0f / l;
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      float ov[32];
      tmem_load32(lane_base + 128 + ch * 32, ov);
      if (q < a.Lq) {
        float4* out = reinterpret_cast<float4*>(a.out + (q * H + h) * AD + ch * 32);
#pragma unroll
        for (int d = 0; d < 8; ++d)
          out[d] = make_float4(ov[4 * d] * inv, ov[4 * d + 1] * inv, ov[4 * d + 2] * inv, ov[4 * d + 3] * inv);
      }
    }
    if (q < a.Lq) a.lse[int64_t(h) * a.Lq + q] = (m + log2f(l)) * 0.69314718055994531f;
  } else if (tid == 0) {
    atomicOr(a.status, 1u);
  }
  tc_before();
  __syncthreads();
  tc_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
}

cudaError_t launch_attend_int8(const AttnArgs& a, cudaStream_t s) {
  if (a.Lq <= 0 || a.H <= 0 || a.n_tiles <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k_attend_int8, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(unsigned((a.Lq + AQ - 1) / AQ), unsigned(a.H));
  k_attend_int8<<<grid, kAttnThreads, kAttnSmem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace nkv
