// nkv_kernels.h — launch interface between the bank (host C++) and the
// sm_100a kernels.  Plain structs of device pointers and sizes; every launch
// is asynchronous on the given stream.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace nkv {

enum DType : int { F32 = 0, BF16 = 1, F16 = 2 };

inline size_t dtype_size(int dt) { return dt == F32 ? 4 : 2; }

// ---------------------------------------------------------- INT8 commit ---
// One job per (layer): quantize `rows` rows of D values of k and v
// (cache/int8.rs:85-134 after the BF16 cast of history.rs:249-250).
struct QuantJob {
  const void* k;
  const void* v;
  uint8_t* kq;
  uint8_t* vq;
  float* ks;
  float* vs;
  uint32_t* flag;  // this job's non-finite bits (may be null)
};
// in_row_offset: rows of the input skipped before the first quantized row
// (QVG text tokens start after the video tokens).  A non-finite value sets
// bit 0 (k) / bit 1 (v) of *flag and of the job's own flag.
// aligned16: every k/v/kq/vq pointer of every job is 16-byte aligned.
cudaError_t launch_int8_quantize(const QuantJob* jobs_dev, int n_jobs, uint64_t rows, uint64_t in_row_offset,
                                 int64_t D, int in_dtype, bool aligned16, uint32_t* flag, cudaStream_t s);

// -------------------------------------------------------- FLOAT commit ---
// Archive copy `to_dtype(model)` (history.rs:243-247): n elements per job.
struct ConvertJob {
  const void* src;
  void* dst;
};
cudaError_t launch_convert(const ConvertJob* jobs_dev, int n_jobs, uint64_t n, int in_dtype, int out_dtype,
                           cudaStream_t s);

// ---------------------------------------------------------- QVG commit ---
// One job per (layer, side): encode the first `tokens` tokens of a
// (1, L, H, D) tensor with that side's codebooks [H][stages][E][D].
struct QvgEncodeJob {
  const void* x;
  uint8_t* codes;   // [tokens][H][bpt]
  float* scales;    // [H][n_blocks][stages]
  const float* cb;  // [H][stages][E][D]
};
// aligned16: every job's input is 16-byte aligned (enables the d128 kernel).
cudaError_t launch_qvg_encode(const QvgEncodeJob* jobs_dev, int n_jobs, int in_dtype, uint64_t L, int H, int D,
                              uint64_t tokens, int stages, int bits, int block, bool aligned16, cudaStream_t s);
// The specialised encoder of kernels_qvg.cu (2 bits, head_dim 128, block 64,
// <= 4 stages, aligned inputs); false when the shape does not qualify.
bool launch_qvg_encode_d128(const QvgEncodeJob* jobs_dev, int n_jobs, int in_dtype, int H, int D, uint64_t tokens,
                            int stages, int bits, int block, bool aligned16, cudaStream_t s, cudaError_t* err);
// Dynamic shared memory the encode kernel needs (the bank rejects configs
// above the per-CTA limit at creation).
size_t qvg_encode_smem_bytes(int D, int block, int bits);

// ------------------------------------------------------------ QVG fit ---
// One (layer, side, head) codebook fit (QvgCodec::fit, cache/qvg.rs:130-167,
// 351-442) on the first committed segment.  Scratch (per task, from
// qvg_fit_scratch_bytes): the residual rows, the farthest-point distances,
// the Lloyd sums and the per-token entry indices.
struct QvgFitTask {
  const void* x;    // (L, H, D) K or V of the segment, in_dtype
  float* out;       // [stages][E][D] codebooks of this (side, head)
  float* res;       // n x D
  double* dmin;     // n
  double* sums;     // E x D
  uint8_t* codes;   // n
  uint64_t seed;    // codebook_seed + head
  int32_t h;
};
size_t qvg_fit_scratch_bytes(uint64_t n, int D, int E);
cudaError_t launch_qvg_fit(const QvgFitTask* tasks_dev, int n_tasks, int in_dtype, uint64_t n, int H, int D,
                           int stages, int E, cudaStream_t s);

// -------------------------------------------------------------- gather ---
enum RunKind : int32_t { RUN_FLOAT = 0, RUN_INT8 = 1, RUN_QVG_VIDEO = 2 };

// A contiguous token range of one archived segment copied (and decoded) to
// a contiguous range of the output.  Component byte offsets are relative to
// the layer block `src + layer * layer_stride`:
//   RUN_FLOAT     : off[0] k values, off[1] v values (model dtype)
//   RUN_INT8      : off[0] k codes, off[1] v codes, off[2] k scales, off[3] v scales
//   RUN_QVG_VIDEO : off[0] k codes, off[1] v codes, off[2] k scales, off[3] v scales
struct GatherRun {
  const unsigned char* src;
  int64_t layer_stride;
  int64_t off[4];
  int64_t src_L;    // tokens per batch row of the source component
  int64_t src_tok;  // first source token
  int64_t dst_tok;  // first output token
  int64_t ntok;
  int32_t kind;
  int32_t n_blocks;  // QVG: blocks in the payload
  int32_t out_set;   // 0: out_k / out_v / out_L; 1: out2_k / out2_v / out2_L
  int32_t pad_;
};

// Work unit of one CTA: `ntok` tokens of run `run` for batch row `b`,
// starting `tok0` tokens into the run.
struct GatherTile {
  int32_t run;
  int32_t b;
  int32_t tok0;
  int32_t ntok;
};

// Work unit of the table-driven QVG decoder: `ntok` (<= kQvgTileTokens)
// video tokens of run `run` starting `tok0` tokens into it, all inside the
// payload block `blk` (so one alpha per head and stage); batch is 1.
struct GatherQvgTile {
  int32_t run;
  int32_t tok0;
  int32_t ntok;
  int32_t blk;
};
constexpr int kQvgTileTokens = 64;

// The table-driven decoder handles the reference's default codec shape:
// 4 stages of 2 bits (one code byte per token and head), head_dim 128.
inline bool qvg_gather_fast_ok(int H, int D, int stages, int bits) {
  return D == 128 && stages == 4 && bits == 2 && H >= 1;
}

struct GatherArgs {
  const GatherRun* runs;
  const GatherTile* tiles;
  int32_t n_tiles;
  const GatherQvgTile* qtiles;  // QVG video tiles for k_gather_qvg
  int32_t n_qtiles;
  int32_t n_layers;
  void* const* out_k;  // [n_layers] output bases (device array)
  void* const* out_v;
  int64_t out_L;  // tokens per batch row of the output
  // A second output set for runs with out_set == 1 (a segment decoded in the
  // same launch as the rebuild); unused otherwise.
  void* const* out2_k;
  void* const* out2_v;
  int64_t out2_L;
  int32_t H, D;
  int32_t out_dtype;
  // QVG
  const float* cb;          // layer 0 codebooks [2][H][stages][E][D]
  int64_t cb_layer_stride;  // floats between layers
  int32_t stages, bits, block;
  // When non-null and nonzero at kernel start the gather writes nothing: a
  // commit whose quantize found non-finite input leaves the working set as
  // it was (the host then rolls the commit back).
  const uint32_t* abort_flag;
};

// vector_ok: all run sources and outputs are 16-byte aligned (the kernel
// additionally needs head_dim % 16 == 0 for its vector path).  QVG video
// tiles (a.qtiles) need vector_ok (the host only builds them for aligned
// outputs); without it they are an argument error.
cudaError_t launch_gather(const GatherArgs& a, bool vector_ok, cudaStream_t s);

// ------------------------------------------------------- standalone ops ---
cudaError_t launch_int8_dequantize(const uint8_t* q, const float* scales, uint64_t rows, int64_t D, int out_dtype,
                                   void* out, cudaStream_t s);
cudaError_t launch_qvg_decode(const float* cb_side, const uint8_t* codes, const float* scales, uint64_t tokens,
                              int H, int D, int stages, int bits, int block, float* out, cudaStream_t s);
cudaError_t launch_synth_fill(void* dst, int dtype, uint64_t rows, int H, int D, uint64_t key,
                              uint64_t index_offset, const float* table, const float* chan_scale, cudaStream_t s);

// Fused K/V projection + commit producer (kernels_project.cu).  x is the
// (M, H*128) bf16 input of one layer, W_k / W_v the (H*128, H*128) bf16
// nn.Linear weights ([out][in]); every other pointer may be null where the
// comment says so.
struct KvProjectParams {
  int64_t M;                        // tokens
  int32_t H;                        // heads (head_dim is 128; H*128 % 256 == 0)
  int32_t qk_norm;                  // RmsNorm on K (attention.rs:120-122)
  float eps;                        // RmsNorm eps as f32
  const uint16_t* bias_k;           // (H*128) bf16 or null
  const uint16_t* bias_v;
  const uint16_t* k_gain;           // (128) bf16 RmsNorm gain or null (no gain)
  const float* rope_cos;            // (M, 64) f32 or null (no rotation)
  const float* rope_sin;
  uint16_t* k_out;                  // (M, H*128) bf16 or null
  uint16_t* v_out;
  uint8_t* k_codes;                 // INT8 archive rows or null (no codes)
  float* k_scales;
  uint8_t* v_codes;
  float* v_scales;
  int32_t n_ranges;                 // rows [lo, hi) of x -> archive rows dst.. (at most 2)
  int64_t range_lo[2], range_hi[2], range_dst[2];
  uint32_t* flag;                   // bit 0: non-finite K, bit 1: V, in a committed row
  uint32_t* err;                    // kProjectTimeoutBit is OR-ed in when a bounded wait ran out
};
constexpr uint32_t kProjectTimeoutBit = 0x80000000u;
bool kv_project_shape_ok(int64_t M, int H, int D);
// OR of flags[1..n] into flags[0] (a staged commit's per-layer status words
// into the word the rebuild gather aborts on)
cudaError_t launch_flag_reduce(uint32_t* flags, int n, cudaStream_t s);

// ------------------------------------------------- history attention ---
// A tile of <= 128 consecutive history keys inside one archived INT8
// segment: the addresses of its first token (head 0) in the archive.
// An encoded TMA descriptor (a CUtensorMap), opaque here.
struct alignas(64) TmaDesc {
  unsigned char bytes[128];
};
// The INT8 code plane of one archived record and layer, (tokens, H, 128)
// bytes at `base` (16-byte aligned, device memory), as a 3-D tensor map
// whose box is one head's 128-byte rows of 128 consecutive tokens,
// 128-byte swizzled; tokens past the end read as zeros.  False when the
// driver's encoder is unavailable or refuses the shape.
bool make_codes_map(TmaDesc* m, const void* base, uint64_t tokens, int H);

struct AttnKeyTile {
  const uint8_t* k_codes;  // the tile's first row (register path)
  const uint8_t* v_codes;
  const float* k_scales;  // the tile's first row
  const float* v_scales;
  int32_t tok0;  // the tile's first token in its record
  int32_t ntok;
  int32_t map;  // TMA path: the record's K / V code planes are maps[2 map] / maps[2 map + 1]
  int32_t pad_;
};
// Attention of q (Lq, H, 128) bf16 over the history keys of `tiles`, head
// by head: out (Lq, H, 128) f32 normalised, lse (H, Lq) f32 natural log;
// bit 0 of *status is set when a bounded wait ran out.
struct AttnArgs {
  const AttnKeyTile* tiles;
  int32_t n_tiles;
  int32_t H;
  const uint16_t* q;
  int64_t Lq;
  float scale_log2;  // softmax scale x log2(e)
  float* out;
  float* lse;
  uint32_t* status;
  const TmaDesc* maps;  // non-null: codes by TMA through these maps (device-memory archives)
  // the schedule (attend_plan): units of (256 queries, head), head-major; the
  // first full_units whole, the rest split into `parts` key ranges whose
  // partial rows go to part_o (f32, 128 per row) and part_ml ((max, sum) per
  // row, base 2), 256 rows per (unit, part)
  int32_t q_tiles;
  int32_t full_units;
  int32_t parts;
  float* part_o;
  float* part_ml;
};
// The schedule for q_len queries x H heads over n_tiles key tiles on `sms`
// SMs: units beyond the last whole wave are split into key ranges (at least
// four tiles each) so that the last wave fills the GPU.  Returns the partial
// rows the split needs (0: none).
int64_t attend_plan(int64_t q_len, int H, int n_tiles, int sms, AttnArgs* a);
cudaError_t launch_attend_int8(const AttnArgs& a, cudaStream_t s);
cudaError_t launch_kv_project(const void* x, const void* wk, const void* wv, const KvProjectParams& p,
                              cudaStream_t stream);

}  // namespace nkv
