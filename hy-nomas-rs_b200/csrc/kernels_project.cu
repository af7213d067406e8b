// kernels_project.cu — the commit producer fused into the K/V projection on
// sm_100a: tcgen05 tensor cores fed by TMA, with the reference's whole
// per-(token, head) chain from the projection to the INT8 archive codes in
// the epilogue.
//
// Reference chain for one layer's captured K / V (batch 1):
//   k = Lin_k(x)             modules/mod.rs:122-142 (bf16 GEMM, then + bias in bf16)
//   k = RmsNorm_k(k)         modules/attention.rs:117-122, modules/norm.rs:55-65
//   k = apply_rotary(k)      modules/attention.rs:144, rope.rs:257-306
//   v = Lin_v(x)             modules/attention.rs:116
//   quantize_kv_pair(k, v)   cache/int8.rs:85-134 (the commit's archive step)
// The bf16 K / V are still written (the attention of the capturing pass
// reads them, attention.rs:145-147), but the commit no longer reads them
// back: the codes and scales come out of the same epilogue.
//
// Kernel shape: persistent CTA pairs (clusters of 2, one CTA per SM, 320
// threads each) computing 256-token x 256-column tiles with the two-SM form
// of the tensor-core MMA (tcgen05.mma.cta_group::2, M=256 N=256 K=16): CTA r
// of a pair holds token rows 128r..128r+127 of A and rows 128r..128r+127 of
// the tile's 256 weight rows, so each SM streams a third less operand data
// from L2 than a 128 x 256 single-SM tile would;
//  * warp 0, one thread per CTA: TMA producer.  Its CTA's 128 x 64 slices of
//    x and of W_k or W_v per stage, 128-byte swizzled, into a 4-stage ring
//    (32 KB per stage); the loads complete on the pair leader's barrier
//    (plain per-CTA loads);
//  * warp 1: allocates 512 TMEM columns per CTA (two 128 x 256 f32
//    accumulators, the CTA's half of a tile); in the leader, one thread
//    issues the MMAs, frees each stage of both CTAs with tcgen05.commit and
//    hands a finished accumulator to both CTAs' epilogues;
//  * warps 2-9: the epilogue.  Warp w reads TMEM lanes 32*(w%4)..+31 of
//    head (w-2)/4's 128 columns, so thread l owns token row 32*(w%4)+l of
//    the tile for one head, 128 values in its registers: bias, RMS norm,
//    rotary pairs, |x| max and codes need no cross-thread exchange.  Two
//    epilogue warps per SM sub-partition hide each other's latency; while
//    they run, the MMA warp fills the other accumulator with the next tile.
//
// Every wait is bounded (kWaitNs on %globaltimer); a wait that runs out sets
// kProjectTimeoutBit in the status word and the CTA's abort flag, every role
// leaves its loop, and the CTA frees its TMEM after a bounded drain.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cfloat>
#include <cstdint>
#include <map>
#include <mutex>

#include "nkv_device.cuh"
#include "nkv_kernels.h"
#include "nkv_quant.cuh"

namespace nkv {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int PAIR_M = 2 * BM;          // tokens per pair tile
constexpr int B_ROWS = BN / 2;          // weight rows each CTA of a pair loads
constexpr int A_BYTES = BM * BK * 2;      // 16 KB
constexpr int B_BYTES = B_ROWS * BK * 2;  // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
// Warp 0 TMA, warp 1 MMA, warps 2-3 idle (they complete the first warpgroup
// for the register split), warps 4-11 the epilogue: two per SM
// sub-partition, warps 4-7 head 0 and 8-11 head 1 of a tile.
constexpr int kEpiWarps = 8, kEpiFirst = 4;
constexpr int kThreads = 32 * (kEpiFirst + kEpiWarps);
// Registers per thread after the split (setmaxnreg, per warpgroup): the
// launch gives 384 x 168; the first warpgroup 128 x 88 + the epilogue
// 256 x 208 = 64,512, exactly the launch's total.
constexpr int kRegsLaunch = 168, kRegsCtl = 88, kRegsEpi = 208;
static_assert(kRegsCtl * 128 + kRegsEpi * 32 * kEpiWarps <= kRegsLaunch * kThreads,
              "register split exceeds the launch's registers");
// Epilogue constants staged in shared memory ahead of each tile (cp.async,
// overlapping the tile's main loop): the tile's 128 token rows of the rotary
// cos / sin tables (the head-0 warp of a lane quadrant copies cos, the head-1
// warp sin, for the quadrant's 32 rows), rows padded to 68 floats so the 32
// lanes' 16-byte reads of one column fall in distinct bank groups; and per
// epilogue warp its head's 128 bias values and the 128 gain values, widened
// to f32 so the epilogue adds and multiplies them as packed f32x2 pairs.
constexpr int ROPE_PITCH = 68;
constexpr int ROPE_BYTES = BM * ROPE_PITCH * 4;  // one table
constexpr int WARP_CONST_BYTES = (128 + 128) * 4;
constexpr int kSmemBytes = STAGES * STAGE_BYTES + 2 * ROPE_BYTES + kEpiWarps * WARP_CONST_BYTES +
                           1024 /* barriers */ + 1024 /* alignment */;
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s per wait

// tcgen05 instruction descriptor: f32 accumulate (bits 4-5 = 1), A and B
// bf16 (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at
// bit 17, M >> 4 at bit 24 (M = 256: the CTA pair's rows).
constexpr uint32_t kIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(PAIR_M >> 4) << 24);

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Arrive on a barrier given by its shared::cluster address (own or peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// The shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
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

// Wait for the phase of parity `parity` to complete; false when the CTA was
// aborted or the wait ran out (which aborts the CTA and sets *err).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                          uint32_t* err) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) {
      *abort_flag = 1u;
      atomicOr(err, kProjectTimeoutBit);
      return false;
    }
  }
}

// 2-D tiled TMA load (a plain per-CTA load) into this CTA's shared memory,
// completing on `bar`, a shared::cluster barrier address of the CTA pair
// (the leader's full barrier).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile whose
// rows are 128 bytes (64 bf16): start address >> 4 in bits 0-13, leading
// byte offset 1 (unused for swizzled K-major), stride byte offset 1024 >> 4
// (eight rows) in bits 32-45, descriptor version 1 (bit 46), layout
// SWIZZLE_128B = 2 in bits 61-63.  Tiles start on 1024-byte boundaries, so
// the base offset field stays 0; stepping K by 16 elements adds 32 bytes to
// the start address.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// One M=256 N=256 K=16 MMA of the CTA pair, issued by the leader: A and B
// descriptors address the same offsets in both CTAs' shared memory.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate));
}

// Arrive on `bar` (shared::cluster address, own or peer CTA) once the pair's
// MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// One lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xFFFFFFFF;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r));
  return r != 0;
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// tcgen05.wait::ld, with the 32 registers of one load threaded through it
// so no use of them is scheduled ahead of the wait.
__device__ __forceinline__ void tmem_wait32(float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Values travel through the epilogue as packed bf16 pairs (element 2j in the
// low half of word j): every stage of the chain ends in a bf16 rounding, a
// rotary (re, im) pair is exactly one word, and 128 values take 64 registers.
// The hardware pair conversion is the integer round-to-nearest-even for
// every non-NaN input; a NaN stays a NaN (its payload is not the
// reference's, which only matters for rows the non-finite check rejects).
__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) { return dev::bf16x2_bits_nonnan(lo, hi); }

// The values of one (token row, head): w holds bf16(accumulator) of the
// row's 128 values and leaves with the K / V the reference commits.  bias:
// this head's 128 bias values or null; gain: the 128 RMS-norm gains or null;
// rope_c / rope_s: this row's 64 cos / sin values or null (all in shared
// memory).
__device__ __forceinline__ void finish_values(uint32_t (&w)[64], const KvProjectParams& p, int side,
                                              const float* bias, const float* gain, const float* rope_c,
                                              const float* rope_s) {
  // Lin::fwd (modules/mod.rs:135-138): the GEMM's bf16 result plus the bias,
  // added in f32 (a packed f32x2 add: two independent roundings) and rounded
  // to bf16
  if (bias) {
    const float4* b4 = reinterpret_cast<const float4*>(bias);
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const float4 b = b4[q];
      uint32_t& x0 = w[2 * q];
      uint32_t& x1 = w[2 * q + 1];
      const float2 v0 = __fadd2_rn(make_float2(lo_f(x0), hi_f(x0)), make_float2(b.x, b.y));
      const float2 v1 = __fadd2_rn(make_float2(lo_f(x1), hi_f(x1)), make_float2(b.z, b.w));
      x0 = pack_rn(v0.x, v0.y);
      x1 = pack_rn(v1.x, v1.y);
    }
  }
  if (side == 0 && p.qk_norm) {
    // RmsNorm (norm.rs:55-65): f32 mean of squares over the head dim, four
    // interleaved partial sums (d mod 4) added as (s0 + s1) + (s2 + s3);
    // 1/sqrt(var + eps) as an IEEE square root and division.  The squares
    // stay scalar multiplies and adds (a packed multiply feeding a packed
    // add could be contracted into one rounding); the scaling below is
    // multiplies only, so it runs on packed pairs.
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float a = lo_f(w[j]), b = hi_f(w[j]);
      s[(2 * j) & 3] = __fadd_rn(s[(2 * j) & 3], __fmul_rn(a, a));
      s[(2 * j + 1) & 3] = __fadd_rn(s[(2 * j + 1) & 3], __fmul_rn(b, b));
    }
    const float ss = __fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3]));
    const float var = __fmul_rn(ss, 0.0078125f);  // / 128, exact
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
    const float2 inv2 = make_float2(inv, inv);
    if (gain) {
      const float4* g4 = reinterpret_cast<const float4*>(gain);
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const float4 g = g4[q];
        uint32_t& x0 = w[2 * q];
        uint32_t& x1 = w[2 * q + 1];
        const float2 v0 = __fmul2_rn(__fmul2_rn(make_float2(lo_f(x0), hi_f(x0)), inv2), make_float2(g.x, g.y));
        const float2 v1 = __fmul2_rn(__fmul2_rn(make_float2(lo_f(x1), hi_f(x1)), inv2), make_float2(g.z, g.w));
        x0 = pack_rn(v0.x, v0.y);
        x1 = pack_rn(v1.x, v1.y);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float2 v = __fmul2_rn(make_float2(lo_f(w[j]), hi_f(w[j])), inv2);
        w[j] = pack_rn(v.x, v.y);
      }
    }
  }
  if (side == 0 && rope_c) {
    // apply_rotary (rope.rs:269-305): interleaved (re, im) pairs, products
    // and sums rounded separately in f32, then bf16
    const float4* c4 = reinterpret_cast<const float4*>(rope_c);
    const float4* s4 = reinterpret_cast<const float4*>(rope_s);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const float4 c = c4[q], sn = s4[q];
      const float cs[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t& x = w[4 * q + j];
        const float xr = lo_f(x), xi = hi_f(x);
        x = pack_rn(__fsub_rn(__fmul_rn(xr, cs[j]), __fmul_rn(xi, ss[j])),
                    __fadd_rn(__fmul_rn(xi, cs[j]), __fmul_rn(xr, ss[j])));
      }
    }
  }
}

// The archive row of one (token row, head): quantize_one (int8.rs:65-81) of
// the 128 values in w, codes written as 128 bytes to `stage` (shared
// memory), the scale returned; `bad` gets the non-finite check.
__device__ __forceinline__ float quantize_row(const uint32_t (&w)[64], uint8_t* stage, bool& bad) {
  // |x| max on the bf16 patterns: NaN-propagating, and inf / NaN patterns
  // (>= 0x7F80) sort above every finite one, so the same max answers the
  // non-finite scan (x != x || |x| >= f32::MAX, int8.rs:99-117; no finite
  // bf16 reaches f32::MAX)
  uint32_t m = w[0] & 0x7FFF7FFFu;
#pragma unroll
  for (int j = 1; j < 64; ++j) m = maxabs_bf16x2(m, w[j]) & 0x7FFF7FFFu;
  const uint32_t pk = max(m & 0xFFFFu, m >> 16);
  bad |= pk >= 0x7F80u;
  const float peak = __uint_as_float(pk << 16);
  const float inv127 = (float)(1.0 / 127.0);
  const float s = peak > 0.0f ? __fadd_rn(__fmul_rn(peak, inv127), 0.0f) : 1.0f;
  uint4* qo = reinterpret_cast<uint4*>(stage);
  if (s >= FLT_MIN && s <= 1e37f) {
    const float r = __frcp_rn(s);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t c[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t a = w[8 * k + 2 * j], b = w[8 * k + 2 * j + 1];
        const uint2 ca = code_bits2(make_float2(lo_f(a), hi_f(a)), s, r);
        const uint2 cb = code_bits2(make_float2(lo_f(b), hi_f(b)), s, r);
        c[j] = pack4(ca.x, ca.y, cb.x, cb.y);
      }
      qo[k] = make_uint4(c[0], c[1], c[2], c[3]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t c[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t a = w[8 * k + 2 * j], b = w[8 * k + 2 * j + 1];
        c[j] = quant_exact(lo_f(a), s) | (quant_exact(hi_f(a), s) << 8) | (quant_exact(lo_f(b), s) << 16) |
               (quant_exact(hi_f(b), s) << 24);
      }
      qo[k] = make_uint4(c[0], c[1], c[2], c[3]);
    }
  }
  return s;
}

// The archive row of token row `row` (rows [lo, hi) of x go to archive rows
// dst..), or -1 when the row is not committed.
__device__ __forceinline__ int64_t archive_row(const KvProjectParams& p, int64_t row) {
  int64_t dst = -1;
#pragma unroll
  for (int i = 0; i < 2; ++i)
    if (i < p.n_ranges && row >= p.range_lo[i] && row < p.range_hi[i]) dst = row - p.range_lo[i] + p.range_dst[i];
  return row < p.M ? dst : -1;
}

__global__ void __launch_bounds__(kThreads, 1)
    k_kv_project(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wk,
                 const __grid_constant__ CUtensorMap tm_wv, const KvProjectParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* rope_cos_s = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES);
  float* rope_sin_s = rope_cos_s + BM * ROPE_PITCH;
  uint16_t* warp_consts = reinterpret_cast<uint16_t*>(smem + STAGES * STAGE_BYTES + 2 * ROPE_BYTES);
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + 2 * ROPE_BYTES + kEpiWarps * WARP_CONST_BYTES);
  // bars: full[STAGES] (leader), empty[STAGES], tfull[2], tempty[2] (leader)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = the pair's leader
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int dim = p.H * 128;
  const int n_half = dim / BN;  // N tiles per side
  const int tiles_m = int((p.M + PAIR_M - 1) / PAIR_M);
  const int n_tiles = tiles_m * 2 * n_half;
  const int kb_count = dim / BK;

  const uint32_t smem_base = smem_u32(smem);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + 2 + b); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);   // the leader's producer arms it for both CTAs' bytes
      mbar_init(empty_bar(s), 1);  // one commit from the leader's MMA thread
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < kEpiFirst) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));
   if (warp == 0) {
    // ---------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < n_tiles && !*abort_flag; t += n_pairs) {
        const int tm = t % tiles_m, tn = t / tiles_m;
        const int side = tn / n_half, n0 = (tn % n_half) * BN + int(rank) * B_ROWS;
        const int m0 = tm * PAIR_M + int(rank) * BM;
        const CUtensorMap* wmap = side ? &tm_wv : &tm_wk;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.err)) break;
          const uint32_t a_dst = smem_base + stage * STAGE_BYTES;
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (rank == 0) mbar_expect_tx(full_bar(stage), 2 * STAGE_BYTES);
          tma_load_2d_pair(a_dst, &tm_x, kb * BK, m0, leader_full);
          tma_load_2d_pair(a_dst + A_BYTES, wmap, kb * BK, n0, leader_full);
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer (leader)
    // The whole warp runs the schedule, so the descriptors are warp-uniform;
    // lane 0 waits (its outcome is the warp's) and one elected lane issues
    // each stage's MMAs and commits.
    if (rank == 0) {
      auto wait = [&](uint32_t bar, uint32_t parity) {
        int r = 1;
        if (lane == 0) r = mbar_wait(bar, parity, abort_flag, p.err) ? 1 : 0;
        r = __shfl_sync(0xFFFFFFFFu, r, 0);
        tc_fence_after();
        return r != 0;
      };
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t acc_phase = 0;
      for (int t = pair; t < n_tiles; t += n_pairs) {
        if (__shfl_sync(0xFFFFFFFFu, int(*abort_flag), 0)) break;
        if (!wait(tempty_bar(buf), acc_phase ^ 1u)) break;
        const uint32_t d_tmem = tmem_base + uint32_t(buf * BN);
        bool ok = true;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!wait(full_bar(stage), phase)) {
            ok = false;
            break;
          }
          const uint32_t a_addr = smem_base + stage * STAGE_BYTES;
          const uint64_t adesc = smem_desc(a_addr), bdesc = smem_desc(a_addr + A_BYTES);
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)  // +32 bytes per K step = +2 in the address field
              umma_bf16_pair(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), (kb | k) != 0 ? 1u : 0u);
            umma_commit_pair(map_to_rank(empty_bar(stage), 0));
            umma_commit_pair(map_to_rank(empty_bar(stage), 1));
          }
          __syncwarp();
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        if (elect_one()) {
          umma_commit_pair(map_to_rank(tfull_bar(buf), 0));
          umma_commit_pair(map_to_rank(tfull_bar(buf), 1));
        }
        __syncwarp();
        if (++buf == 2) buf = 0, acc_phase ^= 1u;
      }
    }
   }
  } else {
    // ---------------------------------------------------- epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpi));
    const int quad = warp & 3, hh = (warp - kEpiFirst) >> 2;  // lane quadrant, head of the tile
    const int rit = quad * 32 + lane;                 // row in the tile
    const float* my_cos = rope_cos_s + rit * ROPE_PITCH;
    const float* my_sin = rope_sin_s + rit * ROPE_PITCH;
    float* my_table = (hh == 0 ? rope_cos_s : rope_sin_s) + rit * ROPE_PITCH;
    float* wc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(warp_consts) + (warp - kEpiFirst) * WARP_CONST_BYTES);
    // wc: [bias 128][gain 128] f32
    const uint32_t pair_bar = 1 + quad;  // named barrier of the two warps of a quadrant
    int buf = 0;
    uint32_t acc_phase = 0;
    bool bad = false;
    for (int t = pair; t < n_tiles; t += n_pairs) {
      const int tm = t % tiles_m, tn = t / tiles_m;
      const int side = tn / n_half, head = (tn % n_half) * (BN / 128) + hh;
      const int64_t row = int64_t(tm) * PAIR_M + int64_t(rank) * BM + rit;
      // stage this tile's constants while its main loop runs
      const uint16_t* bias_g = side ? p.bias_v : p.bias_k;
      const bool rope = side == 0 && p.rope_cos != nullptr;
      const bool gain = side == 0 && p.qk_norm && p.k_gain != nullptr;
      // lanes 0-15: 8 bias values each, lanes 16-31: 8 gain values each,
      // loaded now and widened into the warp's f32 constants after the wait
      uint4 cw = make_uint4(0, 0, 0, 0);
      const bool cw_bias = bias_g && lane < 16, cw_gain = gain && lane >= 16;
      if (cw_bias) cw = __ldg(reinterpret_cast<const uint4*>(bias_g + head * 128 + lane * 8));
      if (cw_gain) cw = __ldg(reinterpret_cast<const uint4*>(p.k_gain + (lane - 16) * 8));
      if (rope && row < p.M) {
        const float* src = (hh == 0 ? p.rope_cos : p.rope_sin) + row * 64;
#pragma unroll
        for (int q = 0; q < 16; ++q) cp_async16(my_table + 4 * q, src + 4 * q);
      }
      cp_async_commit();
      const bool ok = mbar_wait(tfull_bar(buf), acc_phase, abort_flag, p.err);
      cp_async_wait_all();
      if (cw_bias || cw_gain) {
        float4* dst = reinterpret_cast<float4*>(wc + (cw_bias ? lane * 8 : 128 + (lane - 16) * 8));
        dst[0] = make_float4(lo_f(cw.x), hi_f(cw.x), lo_f(cw.y), hi_f(cw.y));
        dst[1] = make_float4(lo_f(cw.z), hi_f(cw.z), lo_f(cw.w), hi_f(cw.w));
      }
      // both tables of the quadrant's rows and the warp's constants are in
      // place (a barrier even on abort, so the partner warp is never left
      // waiting)
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(buf * BN + hh * 128);
      uint32_t w[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float acc[32];
        tmem_ld32(taddr + uint32_t(c * 32), acc);
        tmem_wait32(acc);
#pragma unroll
        for (int j = 0; j < 16; ++j) w[c * 16 + j] = pack_rn(acc[2 * j], acc[2 * j + 1]);
      }
      // the accumulator is in registers: hand it back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(tempty_bar(buf), 0));  // the leader's barrier
      if (row < p.M)
        finish_values(w, p, side, bias_g ? wc : nullptr, gain ? wc + 128 : nullptr, rope ? my_cos : nullptr,
                      my_sin);
      // Stores go out as whole 128-byte lines: each thread parks its row in
      // the quadrant's rotary rows (free once both warps of the quadrant are
      // past the rotation; this warp takes the table it copied), then the
      // warp writes 2 rows x 256 bytes (K / V) or 4 rows x 128 bytes (codes)
      // per instruction.
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      const int64_t row0 = row - lane;  // the warp's first token row
      uint8_t* stage_base = reinterpret_cast<uint8_t*>((hh == 0 ? rope_cos_s : rope_sin_s) + quad * 32 * ROPE_PITCH);
      uint8_t* my_stage = stage_base + lane * ROPE_PITCH * 4;
      uint16_t* out = side ? p.v_out : p.k_out;
      if (out) {
        if (row < p.M) {
          uint4* st = reinterpret_cast<uint4*>(my_stage);
#pragma unroll
          for (int q = 0; q < 16; ++q) st[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
        __syncwarp();
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int u = i * 32 + lane, r = u >> 4, cu = u & 15;
          if (row0 + r < p.M)
            *reinterpret_cast<uint4*>(out + (row0 + r) * dim + head * 128 + cu * 8) =
                *reinterpret_cast<const uint4*>(stage_base + r * ROPE_PITCH * 4 + cu * 16);
        }
        __syncwarp();
      }
      uint8_t* codes = side ? p.v_codes : p.k_codes;
      if (codes) {
        const int64_t dst = archive_row(p, row);
        if (dst >= 0) {
          const float sc = quantize_row(w, my_stage, bad);
          (side ? p.v_scales : p.k_scales)[dst * p.H + head] = sc;
        }
        __syncwarp();
#pragma unroll 4
        for (int i = 0; i < 8; ++i) {
          const int u = i * 32 + lane, r = u >> 3, cu = u & 7;
          const int64_t d = archive_row(p, row0 + r);
          if (d >= 0)
            *reinterpret_cast<uint4*>(codes + d * dim + head * 128 + cu * 16) =
                *reinterpret_cast<const uint4*>(stage_base + r * ROPE_PITCH * 4 + cu * 16);
        }
      }
      if (__any_sync(0xFFFFFFFFu, bad)) {
        if (lane == 0) atomicOr(p.flag, 1u << side);
        bad = false;
      }
      // the quadrant's rotary / staging rows and the warp's constants are
      // free again
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      if (++buf == 2) buf = 0, acc_phase ^= 1u;
    }
  }

  cp_async_wait_all();  // an aborted epilogue may have copies in flight
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // copies or MMAs of an aborted pair may still be in flight: give them a
    // bounded 1 ms to land before the memory they target is released
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 1000000ull) {
    }
  }
  cluster_sync();  // no MMA or arrival of the pair targets this CTA any more
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// Row-major bf16 matrix of `rows` x `cols` as a 2-D tensor map with a
// (64 columns x box_rows) 128-byte-swizzled box.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {uint32_t(BK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// tokens and heads bounded so tile counts (<= 2^18 x 2^8) and TMA row
// coordinates stay well inside int32
bool kv_project_shape_ok(int64_t M, int H, int D) {
  return M > 0 && M <= (int64_t(1) << 26) && D == 128 && H > 0 && H <= 256 && (H * D) % BN == 0;
}

cudaError_t launch_kv_project(const void* x, const void* wk, const void* wv, const KvProjectParams& p,
                              cudaStream_t stream) {
  if (!kv_project_shape_ok(p.M, p.H, 128)) return cudaErrorInvalidValue;
  const uint64_t dim = uint64_t(p.H) * 128;
  CUtensorMap mx, mk, mv;
  if (!make_map(&mx, x, uint64_t(p.M), dim, BM) || !make_map(&mk, wk, dim, dim, B_ROWS) ||
      !make_map(&mv, wv, dim, dim, B_ROWS))
    return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // once per device: the shared-memory opt-in and the number of CTA pairs
  // that can be resident at once (the persistent grid)
  static std::mutex mu;
  static std::map<int, int> pairs_of_device;
  int max_pairs = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = pairs_of_device.find(dev);
    if (it == pairs_of_device.end()) {
      e = cudaFuncSetAttribute(k_kv_project, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return e;
      // the register split's increase waits for registers the launch must
      // hold: refuse a build whose launch count differs from the split's
      cudaFuncAttributes fa{};
      e = cudaFuncGetAttributes(&fa, k_kv_project);
      if (e != cudaSuccess) return e;
      if (fa.numRegs != kRegsLaunch) return cudaErrorInvalidConfiguration;
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      cfg.gridDim = dim3(2 * (sms / 2));
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, k_kv_project, &cfg);
      if (e != cudaSuccess) return e;
      if (clusters < 1) return cudaErrorInvalidConfiguration;
      it = pairs_of_device.emplace(dev, clusters).first;
    }
    max_pairs = it->second;
  }
  const int tiles = int((p.M + PAIR_M - 1) / PAIR_M) * int(2 * dim / BN);
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cfg.gridDim = dim3(2 * pairs);
  return cudaLaunchKernelEx(&cfg, k_kv_project, mx, mk, mv, p);
}

}  // namespace nkv
