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
// atoms) with the 16-byte chunk index XORed with the row in the atom.  Q and K
// are K-major operands of that layout; V, stored the same way (key rows, dims
// contiguous), is the MN-major operand of P V (its two halves are the 64-dim
// blocks, LBO 16 KB apart; key groups of 8 rows, SBO 1024 bytes); P is read
// from TMEM as the A operand of P V.
//
// The codes of a key tile come by TMA (one 3-D box per side from the
// archived record's tensor map) when the archive is in device memory, and by
// plain loads when it reaches the pinned host tier.  Units of (256 queries,
// head) beyond the last whole wave are split into key ranges whose partial
// rows k_attend_combine merges.
//
// Every wait on an mbarrier gives up after 1 s of %globaltimer: the CTA then
// sets bit 0 of the caller's status word, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "nkv_device.cuh"
#include "nkv_kernels.h"

namespace nkv {
namespace {

constexpr int AQ = 128;                    // queries per half (TMEM lanes)
constexpr int kHalves = 2;                 // query halves per CTA, sharing every K / V tile
constexpr int AK = 128;                    // keys per tile
constexpr int AD = 128;                    // head_dim
// warps 0-7 softmax (half = warp / 4), 8-11 dequantization, 12 MMA issue,
// 13-15 idle (they complete the fourth warpgroup for the register split)
constexpr int kSoftmaxWarps = 8, kDequantWarps = 4;
constexpr int kMmaWarp = kSoftmaxWarps + kDequantWarps;
constexpr int kAttnThreads = 512;
// Registers per thread after the split (setmaxnreg, per warpgroup): the
// launch gives 512 x 128; softmax 256 x 168 + dequantization 128 x 128 + MMA /
// idle 128 x 48 = 65,536, exactly the launch's total.
constexpr int kRegsLaunch = 128, kRegsSoftmax = 168, kRegsDequant = 128, kRegsOther = 48;
static_assert(kRegsSoftmax * 32 * kSoftmaxWarps + kRegsDequant * 32 * kDequantWarps + kRegsOther * 128 <=
                  kRegsLaunch * kAttnThreads,
              "register split exceeds the launch's registers");
constexpr int HALF_BYTES = 128 * 128;      // 128 rows x 64 bf16
constexpr int TILE_BYTES = 2 * HALF_BYTES; // 32 KB
// INT8 codes of one side of a key tile: 128 rows of 128 bytes.
constexpr int CODE_BYTES = AK * AD;
// Q (two halves), K and V (two buffers each), the K and V code stages of the
// TMA path; barriers; alignment: 230,656 of the 232,448 bytes a CTA may have.
constexpr int kAttnSmem = 6 * TILE_BYTES + 2 * CODE_BYTES + 256 + 1024;
static_assert(kAttnSmem <= 232448, "shared memory");
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

// Store 16 32-bit columns (32 packed bf16) to this thread's TMEM lane.
__device__ __forceinline__ void tmem_store16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// 32 consecutive f32 columns of this thread's TMEM lane, not waited for.
__device__ __forceinline__ void tmem_load32_async(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// The constant upper word of both descriptor forms: SBO 1024 bytes (bits
// 32-45), descriptor version 1 (bit 46), 128-byte swizzle (bits 61-63).
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
// Lower words: start address >> 4 (bits 0-13) and LBO (bits 16-29).  K-major
// form (Q, K, P): rows of 128 bytes, 8-row groups SBO = 1024 bytes apart, LBO
// unused (16 bytes).  MN-major form (V in P V): 64-element MN blocks LBO =
// 16 KB apart, 8-row K groups SBO = 1024 bytes apart.  Adding (byte offset >>
// 4) to a lower word moves the start address.
__device__ __forceinline__ uint32_t desc_k_lo(uint32_t addr) { return ((addr & 0x3FFFFu) >> 4) | (1u << 16); }
__device__ __forceinline__ uint32_t desc_mn_lo(uint32_t addr) {
  return ((addr & 0x3FFFFu) >> 4) | (uint32_t(HALF_BYTES >> 4) << 16);
}

// SS MMA from descriptor lower words plus a start-address offset (16-byte units).
__device__ __forceinline__ void mma_ss_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t off, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 al, bl;\n\t.reg .b64 da, db;\n\t"
      "add.u32 al, %1, %5;\n\tadd.u32 bl, %2, %5;\n\t"
      "mov.b64 da, {al, %6};\n\tmov.b64 db, {bl, %6};\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(acc), "r"(off), "n"(kDescHi));
}

// TS MMA (A from TMEM) with B from a descriptor lower word plus an offset.
__device__ __forceinline__ void mma_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t off,
                                          uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 bl;\n\t.reg .b64 db;\n\t"
      "add.u32 bl, %2, %5;\n\tmov.b64 db, {bl, %6};\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(acc), "r"(off), "n"(kDescHi));
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

__device__ __forceinline__ void tmem_load_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Threads 32 registers of an earlier unwaited TMEM load through an empty
// volatile statement placed after tmem_load_wait(), so no use of them is
// scheduled ahead of the wait.
__device__ __forceinline__ void tmem_regs_after_wait(float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}


// One head's 128 consecutive tokens of a record's code plane (a 3-D tensor
// map: bytes, head, token) into 16 KB of shared memory, 128-byte swizzled,
// completing on `bar`.  The innermost coordinate is 0 (16-byte aligned).
__device__ __forceinline__ void tma_codes(uint32_t dst, const TmaDesc* map, int h, int tok0, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(h), "r"(tok0), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace

// One CTA per (256-query tile, head): two halves of 128 queries share each
// dequantized K / V tile.  Warp roles:
//  * warps 0-7 (softmax): half w / 4, row 32 (w % 4) + lane of that half (its
//    TMEM lane quadrant).  Per tile: wait for S_h, take the row maximum, move
//    the row's reference maximum (and rescale its O_h row in TMEM) only when
//    the tile exceeds it by more than 8 (base 2), write the bf16 P_h row into
//    the first 64 columns of S_h (a packed pair per column), arrive on P_h;
//  * warps 8-11 (dequantization): thread j dequantizes key row j of K_t and of
//    V_t into the tile's buffer (two buffers each), codes loaded a tile ahead;
//  * warp 12, lane 0 (MMA issue), in the order
//      S_0(t) S_1(t) | PV_0(t) S_0(t+1) | PV_1(t) S_1(t+1) | ...
//    so one half's softmax runs while the tensor pipe serves the other half.
// TMEM: S_0 / P_0 columns [0, 128), S_1 / P_1 [128, 256), O_0 [256, 384),
// O_1 [384, 512).  An MMA reads P_h from TMEM (the A operand) and V from
// shared memory; MMAs run in issue order, so S_h(t+1) overwrites P_h(t) only
// after PV_h(t) read it, and S_h(t+1) completing implies PV_h(t) completed.
template <bool kTma>
__global__ void __launch_bounds__(kAttnThreads, 1) k_attend_int8(const AttnArgs a) {
  extern __shared__ unsigned char attn_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(attn_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = base;                   // halves at 0 / TILE_BYTES
  unsigned char* Kb = base + 2 * TILE_BYTES;  // buffers at 0 / TILE_BYTES
  unsigned char* Vb = base + 4 * TILE_BYTES;  // buffers at 0 / TILE_BYTES
  unsigned char* Cs = base + 6 * TILE_BYTES;  // TMA path: K codes, then V codes
  // barriers: 0-1 S full (half), 2-3 P full (half), 4-5 K full (buffer),
  // 6-7 V full, 8-9 K empty, 10-11 V empty, 12 O done; TMA path: 13 / 14 K /
  // V codes landed, 15 / 16 K / V codes read by every dequantization thread
  uint64_t* bars = reinterpret_cast<uint64_t*>(Cs + 2 * CODE_BYTES);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile uint32_t* abort_flag = tslot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The work item: units (256 queries, head), head-major, whole for the first
  // a.full_units CTAs; the remaining units split into a.parts key ranges each
  // (the last wave would otherwise hold only those units), whose partial
  // results a combine kernel merges.
  const int H = a.H;
  int unit = int(blockIdx.x), part = -1, tb = 0, n = a.n_tiles;
  if (unit >= a.full_units) {
    const int j = unit - a.full_units;
    unit = a.full_units + j / a.parts;
    part = j % a.parts;
    tb = int(int64_t(a.n_tiles) * part / a.parts);
    n = int(int64_t(a.n_tiles) * (part + 1) / a.parts) - tb;
  }
  const int h = unit / a.q_tiles;
  const int64_t q0 = int64_t(unit % a.q_tiles) * (kHalves * AQ);
  const AttnKeyTile* tiles = a.tiles + tb;  // this CTA's key tiles
  auto B = [&](int i) { return smem_addr(&bars[i]); };

  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tslot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(B(0 + i)) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(B(2 + i)), "r"(32 * kSoftmaxWarps / 2) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(B(4 + i)), "r"(32 * kDequantWarps) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(B(6 + i)), "r"(32 * kDequantWarps) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(B(8 + i)) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(B(10 + i)) : "memory");
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(B(12)) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(B(13)) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(B(14)) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(B(15)), "r"(32 * kDequantWarps) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(B(16)), "r"(32 * kDequantWarps) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_flag = 0u;
  }
  // the two query halves (zero rows past the end): softmax thread j loads row j
  if (warp < kSoftmaxWarps) {
    const int64_t q = q0 + tid;
    unsigned char* Qh = Qs + (tid >> 7) * TILE_BYTES;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (q < a.Lq) v = __ldg(reinterpret_cast<const uint4*>(a.q + (q * H + h) * AD) + c);
      *reinterpret_cast<uint4*>(Qh + swz(tid & 127, c)) = v;
    }
    fence_async_smem();
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;
  bool ok = true;
  auto fail = [&]() {
    *abort_flag = 1u;
    ok = false;
  };

  if (warp >= kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
    if (warp == kMmaWarp && n > 0) {
      // The whole warp runs the schedule, so the descriptors are warp-uniform;
      // one elected lane issues each batch of MMAs and its commits.  Lane 0
      // waits and its outcome is the warp's.
      const uint32_t dq0 = desc_k_lo(smem_addr(Qs)), dk0 = desc_k_lo(smem_addr(Kb)), dv0 = desc_mn_lo(smem_addr(Vb));
      constexpr uint32_t kTileLo = TILE_BYTES >> 4;  // the second half / buffer
      auto wait = [&](int i, uint32_t parity) {
        int r = 1;
        if (lane == 0) r = bar_wait(B(i), parity) ? 1 : 0;
        r = __shfl_sync(0xFFFFFFFFu, r, 0);
        if (!r) fail();
        tc_after();
        return r != 0;
      };
      // S_hh = Q_hh K_t^T, then the commits of `c0` / `c1` (-1: none)
      auto issue_s = [&](int t, int hh, int c0, int c1) {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < AD / 16; ++kk) {
            const uint32_t off = uint32_t(((kk >> 2) * HALF_BYTES + (kk & 3) * 32) >> 4);
            mma_ss_lo(tmem + uint32_t(hh * 128), dq0 + uint32_t(hh) * kTileLo, dk0 + uint32_t(t & 1) * kTileLo, off,
                      kIdescS, kk > 0 ? 1u : 0u);
          }
          if (c0 >= 0) mma_commit(B(c0));
          if (c1 >= 0) mma_commit(B(c1));
        }
        __syncwarp();
      };
      // O_hh += P_hh V_t (P_hh from TMEM), then the commit of `c0`
      auto issue_pv = [&](int t, int hh, int c0) {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < AK / 16; ++kk)
            mma_ts_lo(tmem + uint32_t(256 + hh * 128), tmem + uint32_t(hh * 128 + kk * 8),
                      dv0 + uint32_t(t & 1) * kTileLo, uint32_t(kk * 2 * 1024 >> 4), kIdescO,
                      (t > 0 || kk > 0) ? 1u : 0u);
          if (c0 >= 0) mma_commit(B(c0));
        }
        __syncwarp();
      };
      if (wait(4, 0)) {
        issue_s(0, 0, 0, -1);
        issue_s(0, 1, 1, 8);
      }
      for (int t = 0; t < n && ok; ++t) {
        if (__shfl_sync(0xFFFFFFFFu, int(*abort_flag), 0)) break;
        if (!wait(6 + (t & 1), uint32_t(t >> 1) & 1u) || !wait(2, uint32_t(t) & 1u)) break;
        issue_pv(t, 0, -1);
        if (t + 1 < n) {
          if (!wait(4 + ((t + 1) & 1), uint32_t((t + 1) >> 1) & 1u)) break;
          issue_s(t + 1, 0, 0, -1);
        }
        if (!wait(3, uint32_t(t) & 1u)) break;
        issue_pv(t, 1, 10 + (t & 1));
        if (t + 1 < n) issue_s(t + 1, 1, 1, 8 + ((t + 1) & 1));
      }
      if (elect_one()) mma_commit(B(12));
      __syncwarp();
    }
  } else if (warp >= kSoftmaxWarps) {
    // ---------------------------------------------------- dequantization
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsDequant));
    if constexpr (kTma) {
      // Thread j owns key row j of every tile.  One code stage per side:
      // thread 0 brings the next tile's codes (one TMA box per side: one
      // head's rows of 128 tokens) as soon as every thread has read the
      // current ones; the next tile's scales are loaded a tile ahead, tile
      // descriptors two tiles ahead.
      const int kr = tid - 32 * kSoftmaxWarps;  // key row 0..127
      const uint32_t kc_row = smem_addr(Cs) + uint32_t(kr) * 128u, vc_row = kc_row + uint32_t(CODE_BYTES);
      const uint32_t rsw = uint32_t(kr & 7);
      auto issue = [&](int side, const AttnKeyTile& T) {
        bar_expect_tx(B(13 + side), uint32_t(CODE_BYTES));
        tma_codes(smem_addr(Cs) + uint32_t(side * CODE_BYTES), a.maps + 2 * T.map + side, h, T.tok0, B(13 + side));
      };
      auto scales = [&](const AttnKeyTile& T, float& k, float& v) {
        if (kr < T.ntok) {
          k = __ldg(T.k_scales + int64_t(kr) * H + h);
          v = __ldg(T.v_scales + int64_t(kr) * H + h);
        }
      };
      // the rebuild's dequantization (int8.rs:139-155) of row kr of a code
      // stage into a swizzled bf16 tile, zeros for rows past the tile's end
      auto convert = [&](uint32_t src, float sc, bool hv, unsigned char* tile) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
          if (hv) {
            uint4 w;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                         : "r"(src + ((uint32_t(c) ^ rsw) << 4)));
            lo = dequant8(make_uint2(w.x, w.y), sc);
            hi = dequant8(make_uint2(w.z, w.w), sc);
          }
          *reinterpret_cast<uint4*>(tile + swz(kr, 2 * c)) = lo;
          *reinterpret_cast<uint4*>(tile + swz(kr, 2 * c + 1)) = hi;
        }
        fence_async_smem();
      };
      int k_issued = 0, v_issued = 0;  // tiles whose K / V codes were requested (thread 0)
      float ks = 0.0f, vs = 0.0f, ks1 = 0.0f, vs1 = 0.0f;
      AttnKeyTile d1{};
      int nt = 0;  // rows of tile t
      if (n > 0) {
        const AttnKeyTile d0 = tiles[0];
        nt = d0.ntok;
        if (tid == 32 * kSoftmaxWarps) {
          issue(0, d0);
          issue(1, d0);
          k_issued = v_issued = 1;
        }
        scales(d0, ks, vs);
      }
      if (n > 1) {
        d1 = tiles[1];
        scales(d1, ks1, vs1);
      }
      int t = 0;
      for (; t < n; ++t) {
        const int b = t & 1;
        const uint32_t ph = uint32_t(t) & 1u;
        const uint32_t pe = uint32_t((t >> 1) - 1) & 1u;  // the buffer's previous use, tile t - 2
        const bool hv = kr < nt;
        AttnKeyTile d2{};
        if (t + 2 < n) d2 = tiles[t + 2];
        // K_t into buffer b once its codes landed and S of tile t - 2 completed
        if (!bar_wait(B(13), ph) || (t >= 2 && !bar_wait(B(8 + b), pe))) {
          fail();
          break;
        }
        convert(kc_row, ks, hv, Kb + b * TILE_BYTES);
        bar_arrive(B(4 + b));
        bar_arrive(B(15));
        if (tid == 32 * kSoftmaxWarps && t + 1 < n) {
          if (!bar_wait(B(15), ph)) {
            fail();
            break;
          }
          issue(0, d1);
          k_issued = t + 2;
        }
        // V_t once its codes landed and P V of tile t - 2 completed
        if (!bar_wait(B(14), ph) || (t >= 2 && !bar_wait(B(10 + b), pe))) {
          fail();
          break;
        }
        convert(vc_row, vs, hv, Vb + b * TILE_BYTES);
        bar_arrive(B(6 + b));
        bar_arrive(B(16));
        if (tid == 32 * kSoftmaxWarps && t + 1 < n) {
          if (!bar_wait(B(16), ph)) {
            fail();
            break;
          }
          issue(1, d1);
          v_issued = t + 2;
        }
        ks = ks1;
        vs = vs1;
        if (t + 2 < n) scales(d2, ks1, vs1);
        nt = d1.ntok;
        d1 = d2;
        if (*abort_flag) break;
      }
      // no copy in flight when the CTA ends: on an early exit, wait (bounded)
      // for the boxes requested but not consumed
      if (tid == 32 * kSoftmaxWarps) {
        for (int u = t; u < k_issued; ++u) bar_wait(B(13), uint32_t(u) & 1u);
        for (int u = t; u < v_issued; ++u) bar_wait(B(14), uint32_t(u) & 1u);
      }
    } else {
    // Thread j owns key row j of every tile.  The K codes of tile t + 1 are
    // requested right after K_t is written and the V codes right after V_t,
    // so each load has the wait for the next buffer (about one tile of MMA
    // work) to land; tile descriptors are read two tiles ahead.
    const int kr = tid - 32 * kSoftmaxWarps;  // key row 0..127
    uint4 kc[8], vc[8];
    float ks = 0.0f, vs = 0.0f;
    bool khave = false, vhave = false;
    auto load_k = [&](const AttnKeyTile& T) {
      khave = kr < T.ntok;
      if (!khave) return;
      const int64_t r = int64_t(kr) * H + h;
      const uint4* k4 = reinterpret_cast<const uint4*>(T.k_codes + r * AD);
#pragma unroll
      for (int c = 0; c < 8; ++c) kc[c] = __ldg(k4 + c);
      ks = __ldg(T.k_scales + r);
    };
    auto load_v = [&](const AttnKeyTile& T) {
      vhave = kr < T.ntok;
      if (!vhave) return;
      const int64_t r = int64_t(kr) * H + h;
      const uint4* v4 = reinterpret_cast<const uint4*>(T.v_codes + r * AD);
#pragma unroll
      for (int c = 0; c < 8; ++c) vc[c] = __ldg(v4 + c);
      vs = __ldg(T.v_scales + r);
    };
    // the rebuild's dequantization (int8.rs:139-155) of row kr into a
    // swizzled bf16 tile, zeros for rows past the tile's end
    auto store = [&](unsigned char* tile, const uint4* w, float sc, bool hv) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
        if (hv) {
          lo = dequant8(make_uint2(w[c].x, w[c].y), sc);
          hi = dequant8(make_uint2(w[c].z, w[c].w), sc);
        }
        *reinterpret_cast<uint4*>(tile + swz(kr, 2 * c)) = lo;
        *reinterpret_cast<uint4*>(tile + swz(kr, 2 * c + 1)) = hi;
      }
      fence_async_smem();
    };
    AttnKeyTile d1{};  // descriptor of tile t + 1
    if (n > 0) {
      const AttnKeyTile d0 = tiles[0];
      load_k(d0);
      load_v(d0);
    }
    if (n > 1) d1 = tiles[1];
    for (int t = 0; t < n; ++t) {
      const int b = t & 1;
      const uint32_t pe = uint32_t((t >> 1) - 1) & 1u;  // the buffer's previous use, tile t - 2
      AttnKeyTile d2{};
      if (t + 2 < n) d2 = tiles[t + 2];
      // K_t into buffer b once S of tile t - 2 completed
      if (t >= 2 && !bar_wait(B(8 + b), pe)) {
        fail();
        break;
      }
      store(Kb + b * TILE_BYTES, kc, ks, khave);
      bar_arrive(B(4 + b));
      if (t + 1 < n) load_k(d1);
      // V_t into buffer b once P V of tile t - 2 completed
      if (t >= 2 && !bar_wait(B(10 + b), pe)) {
        fail();
        break;
      }
      store(Vb + b * TILE_BYTES, vc, vs, vhave);
      bar_arrive(B(6 + b));
      if (t + 1 < n) load_v(d1);
      d1 = d2;
      if (*abort_flag) break;
    }
    }
  } else {
    // ------------------------------------------------------------ softmax
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int hf = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_q = uint32_t((warp & 3) * 32) << 16;
    const uint32_t s_cols = tmem + lane_q + uint32_t(hf * 128);
    const uint32_t o_cols = tmem + lane_q + uint32_t(256 + hf * 128);
    float m = -INFINITY, l = 0.0f;
    for (int t = 0; t < n; ++t) {
      const int ntok = tiles[t].ntok;
      if (!bar_wait(B(hf), uint32_t(t) & 1u)) {
        fail();
        break;
      }
      tc_after();
      // the row's 128 scores in registers; keys past the tile's end at -inf
      float sv[AK];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) tmem_load32_async(s_cols + ch * 32, sv + ch * 32);
      tmem_load_wait();
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) tmem_regs_after_wait(sv + ch * 32);
      if (ntok < AK) {
#pragma unroll
        for (int j = 0; j < AK; ++j)
          if (j >= ntok) sv[j] = -INFINITY;
      }
      // row maximum of the raw scores (the scale is positive): eight chains
      // of three-input maxima
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = fmaxf(sv[c], sv[8 + c]);
#pragma unroll
      for (int j = 16; j < AK; j += 16)
#pragma unroll
        for (int c = 0; c < 8; ++c) mx[c] = max3(mx[c], sv[j + c], sv[j + 8 + c]);
      const float mt =
          max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) * a.scale_log2;
      const bool move = mt > m + 8.0f;
      const float mn = move ? mt : m;
      const float alpha = move ? exp2f(m - mn) : 1.0f;  // 0 on the first tile
      // P = 2^(s scale_log2 - mn) (masked keys give 0), packed bf16 pairs into
      // the first 64 columns of S_h; the row sum in eight f32 partials
      const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-mn, -mn);
      float2 ls[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                      make_float2(0.0f, 0.0f)};
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int k0 = ch * 32 + 2 * j;
          const float2 x = __ffma2_rn(make_float2(sv[k0], sv[k0 + 1]), sc2, nm2);
          const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          ls[j & 3] = __fadd2_rn(ls[j & 3], p);
          w[j] = dev::bf16x2_bits_nonnan(p.x, p.y);
        }
        tmem_store16(s_cols + ch * 16, w);
      }
      const float2 l01 = __fadd2_rn(ls[0], ls[1]), l23 = __fadd2_rn(ls[2], ls[3]);
      const float lsum = (l01.x + l01.y) + (l23.x + l23.y);
      if (t > 0 && __any_sync(0xFFFFFFFFu, move)) {
        // O_h's row rescaled; PV_h(t - 1) completed before S_h(t) did
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          float ov[32];
          tmem_load32(o_cols + ch * 32, ov);
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] *= alpha;
          tmem_store32(o_cols + ch * 32, ov);
        }
      }
      tmem_store_wait();
      l = l * alpha + lsum;
      m = mn;
      tc_before();
      bar_arrive(B(2 + hf));
      if (*abort_flag) break;
    }
    if (!*abort_flag && n > 0) {
      if (!bar_wait(B(12), 0)) fail();
      tc_after();
      if (ok) {
        const int64_t q = q0 + hf * AQ + row;
        // a part writes its unnormalised rows, running maximum and sum (base 2)
        const int64_t prow = int64_t((unit - a.full_units) * a.parts + part) * (kHalves * AQ) + hf * AQ + row;
        const float inv = part < 0 ? 1.0f / l : 1.0f;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          float ov[32];
          tmem_load32(o_cols + ch * 32, ov);
          if (q < a.Lq) {
            float4* out = reinterpret_cast<float4*>((part < 0 ? a.out + (q * H + h) * AD : a.part_o + prow * AD) +
                                                    ch * 32);
#pragma unroll
            for (int d = 0; d < 8; ++d)
              out[d] =
                  make_float4(ov[4 * d] * inv, ov[4 * d + 1] * inv, ov[4 * d + 2] * inv, ov[4 * d + 3] * inv);
          }
        }
        if (q < a.Lq) {
          if (part < 0)
            a.lse[int64_t(h) * a.Lq + q] = (m + log2f(l)) * 0.69314718055994531f;
          else
            reinterpret_cast<float2*>(a.part_ml)[prow] = make_float2(m, l);
        }
      }
    }
  }
  tc_before();
  __syncthreads();
  tc_after();
  if (*abort_flag && tid == 0) atomicOr(a.status, 1u);
  if (warp == kMmaWarp) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

static_assert(sizeof(CUtensorMap) == sizeof(TmaDesc) && alignof(CUtensorMap) <= alignof(TmaDesc), "TmaDesc");

bool make_codes_map(TmaDesc* m, const void* base, uint64_t tokens, int H) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  if (!enc) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  if (tokens == 0 || H <= 0 || (reinterpret_cast<uintptr_t>(base) & 15u)) return false;
  const cuuint64_t dims[3] = {uint64_t(AD), uint64_t(H), tokens};
  const cuuint64_t strides[2] = {uint64_t(AD), uint64_t(H) * AD};
  const cuuint32_t box[3] = {uint32_t(AD), 1u, uint32_t(AK)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return enc(reinterpret_cast<CUtensorMap*>(m), CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims,
             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The merge of a split unit's parts, one thread per query row: with M the
// largest part maximum, O = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p and
// lse = (M + log2 of that sum) ln 2.
__global__ void __launch_bounds__(kHalves * AQ) k_attend_combine(const AttnArgs a) {
  const int unit = a.full_units + int(blockIdx.x), r = int(threadIdx.x);
  const int h = unit / a.q_tiles;
  const int64_t q = int64_t(unit % a.q_tiles) * (kHalves * AQ) + r;
  if (q >= a.Lq) return;
  const int64_t row0 = int64_t(blockIdx.x) * a.parts * (kHalves * AQ) + r;  // part p: + p * 256
  const float2* ml = reinterpret_cast<const float2*>(a.part_ml);
  float M = -INFINITY;
  for (int p = 0; p < a.parts; ++p) M = fmaxf(M, ml[row0 + int64_t(p) * (kHalves * AQ)].x);
  float L = 0.0f;
  for (int p = 0; p < a.parts; ++p) {
    const float2 v = ml[row0 + int64_t(p) * (kHalves * AQ)];
    L += exp2f(v.x - M) * v.y;
  }
  const float inv = 1.0f / L;
  float4* out = reinterpret_cast<float4*>(a.out + (q * a.H + h) * AD);
  for (int d = 0; d < AD / 4; ++d) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int p = 0; p < a.parts; ++p) {
      const int64_t pr = row0 + int64_t(p) * (kHalves * AQ);
      const float w = exp2f(ml[pr].x - M) * inv;
      const float4 o = reinterpret_cast<const float4*>(a.part_o + pr * AD)[d];
      acc.x += w * o.x;
      acc.y += w * o.y;
      acc.z += w * o.z;
      acc.w += w * o.w;
    }
    out[d] = acc;
  }
  a.lse[int64_t(h) * a.Lq + q] = (M + log2f(L)) * 0.69314718055994531f;
}

int64_t attend_plan(int64_t q_len, int H, int n_tiles, int sms, AttnArgs* a) {
  const int64_t q_tiles = (q_len + kHalves * AQ - 1) / (kHalves * AQ);
  const int64_t units = q_tiles * H;
  a->q_tiles = int32_t(q_tiles);
  a->full_units = int32_t(units);
  a->parts = 1;
  const int64_t rem = sms > 0 ? units % sms : 0;
  if (rem == 0) return 0;
  const int64_t parts = std::min<int64_t>(sms / rem, n_tiles / 4);
  if (parts < 2) return 0;
  a->full_units = int32_t(units - rem);
  a->parts = int32_t(parts);
  return rem * parts * (kHalves * AQ);
}

template <bool kTma>
static cudaError_t launch_attend(const AttnArgs& a, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(k_attend_int8<kTma>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess) return e;
  // the register split's increase waits for registers the launch must hold:
  // refuse a build whose launch count differs from the split's
  cudaFuncAttributes fa{};
  e = cudaFuncGetAttributes(&fa, k_attend_int8<kTma>);
  if (e != cudaSuccess) return e;
  if (fa.numRegs != kRegsLaunch) return cudaErrorInvalidConfiguration;
  const int64_t units = int64_t(a.q_tiles) * a.H;
  const int64_t split = units - a.full_units;
  k_attend_int8<kTma><<<unsigned(a.full_units + split * a.parts), kAttnThreads, kAttnSmem, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess || split == 0) return e;
  k_attend_combine<<<unsigned(split), kHalves * AQ, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_attend_int8(const AttnArgs& a, cudaStream_t s) {
  if (a.Lq <= 0 || a.H <= 0 || a.n_tiles <= 0) return cudaSuccess;
  return a.maps ? launch_attend<true>(a, s) : launch_attend<false>(a, s);
}

}  // namespace nkv
