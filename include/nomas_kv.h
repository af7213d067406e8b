/*
 * nomas_kv.h — C ABI of the B200-native lifelong KV cache.
 *
 * Drop-in for the `nomas-core` cache API of hy-nomas-rs (Rust crate
 * `nomas-core`, directory `src/cache/`).  One `nkv_bank` stands for one
 * `KvBank` (cache/mod.rs:225-320): a contiguous block of DiT layers, each
 * layer one `HistoryCache` (cache/history.rs:84-569), optionally wrapped in a
 * `PhaseSwappedCache` (cache/phase_swap.rs:27-161) when the config asks for
 * phase swap.  Every entry point below names the reference item it replaces.
 *
 * Conventions
 *  - Every function returns an `nkv_status`; on failure `nkv_last_error()`
 *    returns a thread-local message (the reference's `Error` Display text
 *    where one exists).
 *  - All device work of a bank is stream-ordered on the stream given to
 *    nkv_bank_create.  Device pointers passed in are borrowed: they must stay
 *    valid until the call's work on that stream has completed.  Pointers
 *    returned (working sets) are owned by the bank and stay valid until the
 *    next commit / rollback / park / destroy of that bank.
 *  - Calls on one bank are not thread-safe (the reference mutates through
 *    `&mut self`).  Different banks (e.g. one per GPU) are independent.
 *  - Tensors are dense row-major (B, L, H, D) exactly like the reference's
 *    candle tensors; B is the batch, L tokens, H heads, D head_dim.
 *
 * The library has no CPU fallback: every data-path operation runs a CUDA
 * kernel built for sm_100a, and a bank cannot be created without a device.
 */
#ifndef NOMAS_KV_H
#define NOMAS_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NKV_ABI_VERSION 1

/* Status codes.  One per reference `Error` kind the cache raises
 * (nomas-core/src/error.rs:7-46). */
typedef enum {
  NKV_OK = 0,
  NKV_ERR_GEOMETRY = 1,       /* Error::Geometry      (error.rs:34-36)   */
  NKV_ERR_CACHE_STATE = 2,    /* Error::CacheState    (error.rs:28-32)   */
  NKV_ERR_INVALID_CONFIG = 3, /* Error::InvalidConfig (error.rs:24-26)   */
  NKV_ERR_MSG = 4,            /* Error::Msg: non-finite K/V (int8.rs:99-117), sampler checks
                                 (uniform_history.rs:105-123)            */
  NKV_ERR_CUDA = 5,           /* device/runtime failure (the reference's Error::Candle slot) */
  NKV_ERR_ARGUMENT = 6        /* bad pointer / index across the C ABI (no reference kind) */
} nkv_status;

/* Model / input element types (config.rs DataType: F32, Bf16, F16). */
typedef enum { NKV_F32 = 0, NKV_BF16 = 1, NKV_F16 = 2 } nkv_dtype;

/* CacheStorage (config.rs:116-124). */
typedef enum { NKV_STORAGE_FLOAT = 0, NKV_STORAGE_INT8 = 1, NKV_STORAGE_QVG = 2 } nkv_storage;

/* HistorySampling (config.rs:55-67). */
typedef enum {
  NKV_SAMPLING_RECENT = 0,
  NKV_SAMPLING_UNIFORM = 1,
  NKV_SAMPLING_RECENT_MIX = 2,
  NKV_SAMPLING_TEMPORAL = 3 /* TemporalContext { gamma } */
} nkv_sampling;

/* QvgConfig (config.rs:89-112; defaults 4 stages, 2 bits, block 64, text as
 * INT8, seed 0x5EED0002 at config.rs:101-111). */
typedef struct {
  int32_t stages;
  int32_t bits_per_stage;
  int32_t block_size;
  int32_t text_as_int8; /* carried for completeness; like the reference, text is always INT8 */
  uint64_t codebook_seed;
} nkv_qvg_config;

/* CacheConfig (config.rs:142-174).  `capacity: Option<usize>` is
 * (has_capacity, capacity).  cache_at_step / cache_noise_sigma are pipeline
 * knobs the cache never reads and are not carried. */
typedef struct {
  int32_t storage;  /* nkv_storage */
  nkv_qvg_config qvg;
  int32_t sampling; /* nkv_sampling */
  double gamma;     /* TemporalContext gamma; ignored otherwise */
  int32_t has_capacity;
  uint64_t capacity;
  uint64_t past_frames;
  int32_t phase_swap;
} nkv_cache_config;

/* SegmentKv without its tensors (cache/mod.rs:100-118). */
typedef struct {
  uint64_t segment_index;
  uint64_t frame_start;
  uint64_t frame_count;
  uint64_t image_tokens;
  uint64_t text_tokens;
  int64_t action_start; /* -1 when the segment has no action tokens */
} nkv_segment_desc;

/* SegmentLayout (cache/mod.rs:61-75). */
typedef struct {
  uint64_t segment_index;
  uint64_t video_start;
  uint64_t video_end;
  uint64_t text_start;
  uint64_t text_end;
  int64_t action_start;
} nkv_segment_layout;

/* CacheMetrics (cache/mod.rs:133-151). */
typedef struct {
  uint64_t archived_segments;
  uint64_t archived_bytes;
  uint64_t encode_calls;
  uint64_t d2h_bytes;
  uint64_t h2d_bytes;
  uint64_t rebuilds;
  uint64_t evicted_tokens;
  uint64_t rollbacks;
} nkv_metrics;

/* The scalar accessors of LifetimeKvCache (cache/mod.rs:173-186). */
typedef struct {
  uint64_t valid_len;        /* valid_len()        mod.rs:174 */
  uint64_t capacity;         /* capacity()         mod.rs:177, UINT64_MAX when unbounded */
  uint64_t n_segments;       /* n_segments()       mod.rs:180 */
  uint64_t total_frames;     /* total_frames()     mod.rs:183 */
  uint64_t tokens_per_frame; /* tokens_per_frame() mod.rs:186 */
  int32_t parked;            /* PhaseSwappedCache::is_parked (phase_swap.rs:84-86) */
  int32_t storage;           /* storage_format()   mod.rs:156 */
  int32_t sampling;          /* sampling()         mod.rs:159 */
  int32_t qvg_fitted;        /* QvgCodec::is_fitted (qvg.rs:107-109) */
} nkv_cache_info_t;

/* Per-kernel device time collected while timing is enabled (no reference
 * counterpart; CUDA events on the bank's stream around each launch). */
typedef struct {
  uint64_t launches;
  double total_ms;
} nkv_kernel_stat;

enum {
  NKV_KERNEL_QUANTIZE = 0,      /* INT8 commit: quantize K/V + non-finite scan       */
  NKV_KERNEL_FLOAT_ARCHIVE = 1, /* FLOAT commit: dtype conversion into the archive   */
  NKV_KERNEL_QVG_ENCODE = 2,    /* QVG commit: residual VQ encode of video tokens    */
  NKV_KERNEL_GATHER = 3,        /* rebuild: gather + dequant/decode                  */
  NKV_KERNEL_SEGMENT_DECODE = 4, /* nkv_bank_decode_segment: the same gather kernel  */
  NKV_KERNEL_QVG_FIT = 5,       /* first QVG commit: device codebook fit             */
  NKV_KERNEL_ATTEND = 6,        /* nkv_bank_attend_history                          */
  NKV_KERNEL_COUNT = 7
};

typedef struct nkv_bank nkv_bank;

/* ---------------------------------------------------------------- misc -- */
const char* nkv_last_error(void);
int32_t nkv_abi_version(void);

/* ------------------------------------------------------------ the bank -- */

/* KvBank::new (cache/mod.rs:231-244) -> build_cache (mod.rs:208-222) ->
 * HistoryCache::new (history.rs:104-156), for layers
 * [layer_begin, layer_begin + n_layers) of the model on CUDA device `device`.
 * Config validation happens before any device call and returns
 * NKV_ERR_INVALID_CONFIG with the reference's messages.  `stream` is a
 * cudaStream_t (NULL = the legacy default stream). */
int nkv_bank_create(const nkv_cache_config* cfg, int32_t n_layers, int32_t layer_begin, int64_t batch,
                    int64_t heads, int64_t head_dim, int32_t dtype, int32_t device, void* stream,
                    nkv_bank** out);

/* Drop the bank and every device/pinned allocation it owns. */
int nkv_bank_destroy(nkv_bank* bank);

/* KvBank::commit (cache/mod.rs:257-268) -> HistoryCache::commit_segment
 * (history.rs:458-463): validate_segment (history.rs:168-238),
 * archive_segment (history.rs:241-305), rebuild (history.rs:341-446).
 * k_dev[i] / v_dev[i] are device pointers to the (B, L, H, D) K / V of local
 * layer i, L = image_tokens + text_tokens, element type `kv_dtype`.
 * Validation and non-finite errors leave every layer unchanged (the commit
 * is all-or-nothing across the bank).  Like the reference, a rebuild error
 * (working set over capacity) is reported after the segment was archived. */
int nkv_bank_commit(nkv_bank* bank, const nkv_segment_desc* seg, int32_t kv_dtype, const void* const* k_dev,
                    const void* const* v_dev);

/* KvBank::rollback (cache/mod.rs:276-281) -> HistoryCache::rollback_last_segment
 * (history.rs:507-528). */
int nkv_bank_rollback(nkv_bank* bank);

/* KvBank::park_all / unpark_all (cache/mod.rs:284-297) -> PhaseSwappedCache::park
 * / unpark (phase_swap.rs:42-81).  No-ops unless cfg.phase_swap (the trait's
 * default methods, mod.rs:196-203).  Park copies each layer's working set to
 * pinned host memory and frees its device memory; unpark restores it. */
int nkv_bank_park(nkv_bank* bank);
int nkv_bank_unpark(nkv_bank* bank);

/* KvBank::metrics (cache/mod.rs:305-319): max over layers for
 * archived_segments / rebuilds / evicted_tokens / rollbacks, sum otherwise. */
int nkv_bank_metrics(const nkv_bank* bank, nkv_metrics* out);

/* Wait for all of the bank's device work (no reference counterpart; the
 * reference's candle calls are synchronous). */
int nkv_bank_synchronize(nkv_bank* bank);

/* Pre-reserve device memory: `archive_bytes` for archived segments and a
 * working set of `working_tokens` tokens per layer, so later commits do not
 * allocate (no reference counterpart). */
int nkv_bank_reserve(nkv_bank* bank, uint64_t archive_bytes, uint64_t working_tokens);

/* Device bytes one archived segment of this geometry takes per layer
 * (allocation size, incl. alignment), for sizing nkv_bank_reserve. */
int nkv_bank_segment_bytes(const nkv_bank* bank, const nkv_segment_desc* seg, uint64_t* bytes_per_layer);

/* HistoryCache::decode_segment (history.rs:308-338) of archive position
 * `archive_pos` for every local layer, written as model-dtype (B, L_seg, H, D)
 * into the caller's device buffers k_out[i] / v_out[i]. */
int nkv_bank_decode_segment(nkv_bank* bank, uint64_t archive_pos, void* const* k_out, void* const* v_out);

/* The history part of the reference's attention (modules/attention.rs:
 * 143-189; every current token sees every history token, masks.rs) computed
 * straight from the INT8 archive, without the materialised BF16 working set:
 * softmax(q k^T * scale) v over this layer's working-set keys and values (the
 * same tokens, dequantized as the rebuild does), head by head.  q: (q_len, H,
 * 128) bf16 device; out: (q_len, H, 128) f32, normalised; lse: (H, q_len) f32,
 * the natural-log log-sum-exp of each row's scaled scores, for merging with
 * the current segment's (masked) part.  INT8 storage, head_dim 128, batch 1,
 * bf16 model dtype, a finite positive scale; CacheState while parked, with
 * an empty history or a working set that is not the archive's rebuild.  Runs
 * on the bank's stream
 * and returns after the kernel.  No reference counterpart as a separate
 * call. */
int nkv_bank_attend_history(nkv_bank* bank, int32_t layer, const void* q, uint64_t q_len, float scale, float* out,
                            float* lse);

/* Tiered archive (no reference counterpart; the reference's archive lives in
 * host memory of its own process).  Archive chunks allocated after this call
 * go to device memory while the bank's device archive chunks total at most
 * `device_bytes`, and to pinned host memory mapped into the device's address
 * space beyond it; the kernels read and write host slabs over the host link,
 * with the same results.  0 removes the limit.  Staged commits
 * (nkv_bank_stage_segment) are refused while a limit is set.  Reserve
 * (nkv_bank_reserve) after setting the limit to place the chunks up front. */
int nkv_bank_set_archive_device_limit(nkv_bank* bank, uint64_t device_bytes);
/* Bytes of the archived slabs (all local layers) in device / host memory. */
int nkv_bank_archive_usage(nkv_bank* bank, uint64_t* device_bytes, uint64_t* host_bytes);

/* nkv_bank_commit followed by nkv_bank_decode_segment of the segment it
 * archived (no reference counterpart as one call: commit_segment,
 * history.rs:458-463, then decode_segment, history.rs:308-338).  The new
 * segment's K/V as the archive holds them (INT8 dequantized, QVG decoded
 * plus the INT8 text, Float as stored), model dtype (B, L_seg, H, D), go to
 * k_out[i] / v_out[i] from the same gather launch that rebuilds the working
 * set.  Errors as nkv_bank_commit; when it fails the outputs are not
 * written. */
int nkv_bank_commit_decode(nkv_bank* bank, const nkv_segment_desc* seg, int32_t kv_dtype, const void* const* k_dev,
                           const void* const* v_dev, void* const* k_out, void* const* v_out);

/* Enable/disable per-kernel CUDA-event timing and read / reset the totals. */
int nkv_bank_set_timing(nkv_bank* bank, int32_t enable);
int nkv_bank_kernel_stats(nkv_bank* bank, nkv_kernel_stat* out /* [NKV_KERNEL_COUNT] */, int32_t reset);

/* Two-phase INT8 commit for a producer that writes the archive rows itself,
 * such as nkv_kv_project below (no reference counterpart: it splits
 * KvBank::commit, cache/mod.rs:257-268, around archive_segment's quantize,
 * history.rs:248-253, so the K/V need not be read back).
 *  - nkv_bank_stage_segment: validate_segment (history.rs:168-238) without
 *    the input-tensor checks, then reserve the segment's record; out[i] gets
 *    local layer i's INT8 planes — k_codes / v_codes (B, L, H, D) u8
 *    (int8 + 128), k_scales / v_scales (B, L, H) f32 — and its status word,
 *    into which the producer ORs bit 0 (non-finite K) / bit 1 (V).  INT8
 *    storage only (else NKV_ERR_INVALID_CONFIG); one staged segment at a
 *    time; commit, rollback, save and load are refused while one is pending.
 *  - nkv_bank_commit_staged: archive the staged record and rebuild, with
 *    nkv_bank_commit's semantics from the non-finite check on (a set status
 *    bit rejects the segment, NKV_ERR_MSG, and nothing changes).  Stage
 *    zeroes the status words on the bank's stream, so the producer's work
 *    must come after stage and before commit_staged in that stream's order
 *    (simplest: launch it on the bank's stream).
 *  - nkv_bank_discard_staged: drop it (waits for the bank's stream). */
typedef struct {
  uint8_t* k_codes;
  uint8_t* v_codes;
  float* k_scales;
  float* v_scales;
  uint32_t* status;
} nkv_staged_layer;
int nkv_bank_stage_segment(nkv_bank* bank, const nkv_segment_desc* seg, nkv_staged_layer* out /* [n_layers] */);
int nkv_bank_commit_staged(nkv_bank* bank);
int nkv_bank_discard_staged(nkv_bank* bank);

/* Archive persistence.  No counterpart in the reference, whose archive lives
 * in memory only.  nkv_bank_save writes the segment timeline, the counters,
 * the QVG codebooks and every archived payload of the bank's local layers to
 * `path`; it refuses (NKV_ERR_CACHE_STATE) while parked or while the working
 * set is not the rebuild of the archive (after a failed rebuild, or a commit
 * or rollback while parked).  nkv_bank_load restores such a file into a bank
 * created with the same configuration and geometry that has committed
 * nothing yet (else NKV_ERR_INVALID_CONFIG / NKV_ERR_CACHE_STATE), rebuilds
 * the working set on the device and restores the counters as saved.  A file
 * that is not a saved archive, or is truncated, is NKV_ERR_MSG and leaves the
 * bank fresh.  Files use the host's byte order. */
int nkv_bank_save(nkv_bank* bank, const char* path);
int nkv_bank_load(nkv_bank* bank, const char* path);

/* ----------------------------------------------------- one layer's cache -- */

/* LifetimeKvCache::working_set (cache/mod.rs:168; history.rs:465-481):
 * device pointers to the model-dtype (B, valid_len, H, D) K and V of local
 * layer `layer`.  NULL pointers with valid_len 0 when the set is empty.
 * NKV_ERR_CACHE_STATE while parked (phase_swap.rs:107-114). */
int nkv_cache_working_set(const nkv_bank* bank, int32_t layer, const void** k_dev, const void** v_dev,
                          uint64_t* valid_len);

/* LifetimeKvCache::working_layout (cache/mod.rs:171; phase_swap.rs:116-121).
 * Writes min(n, cap) entries; *n = number of segments in the layout. */
int nkv_cache_layout(const nkv_bank* bank, int32_t layer, nkv_segment_layout* out, uint64_t cap, uint64_t* n);

/* valid_len / capacity / n_segments / total_frames / tokens_per_frame
 * (cache/mod.rs:173-186) and the parked / storage / sampling state. */
int nkv_cache_info(const nkv_bank* bank, int32_t layer, nkv_cache_info_t* out);

/* LifetimeKvCache::metrics (cache/mod.rs:193) of one layer. */
int nkv_cache_metrics(const nkv_bank* bank, int32_t layer, nkv_metrics* out);

/* QvgCodec::with_codebooks (qvg.rs:101-104) — an addition to the reference's
 * cache API, where HistoryCache always fits on its first commit
 * (history.rs:256-262).  `host_cb` is [2 (K,V)][H][stages][2^bits][D] f32.
 * A layer given codebooks never fits; the others still fit on first commit. */
int nkv_cache_set_qvg_codebooks(nkv_bank* bank, int32_t layer, const float* host_cb);

/* Copy a layer's QVG codebooks to the host (same layout); *fitted = 0 when
 * none are fitted/attached yet (QvgCodec::is_fitted, qvg.rs:107-109). */
int nkv_cache_get_qvg_codebooks(const nkv_bank* bank, int32_t layer, float* host_cb, int32_t* fitted);

/* Copy one archived segment's payload (ArchivedPayload, history.rs:25-37) of
 * one layer to the host, components back to back in this order:
 *   FLOAT: k[B,L,H,D], v            (model dtype)
 *   INT8 : kq[B,L,H,D] u8, vq u8, ks[B,L,H] f32, vs f32
 *   QVG  : kcodes[Lv,H,bpt] u8, vcodes, kscales[H,nblocks,stages] f32, vscales,
 *          then (text_tokens > 0) text kq[1,Lt,H,D] u8, vq, ks[1,Lt,H] f32, vs
 * *nbytes = the total size (also when host_buf is NULL or cap is too small,
 * in which case nothing is copied). */
int nkv_cache_export_segment(const nkv_bank* bank, int32_t layer, uint64_t archive_pos, void* host_buf,
                             uint64_t cap, uint64_t* nbytes);

/* --------------------------------------- host policy (no device needed) -- */

/* history_frame_indices (cache/uniform_history.rs:76-125) with its checks;
 * kind selects the raw samplers instead: 0 = uniform_frame_indices (:10-19),
 * 1 = recent_mix_uniform_frame_indices (:23-32), 2 =
 * temporal_context_frame_indices (:40-70), 3 = the validated dispatcher with
 * `sampling` / `gamma`.  *n = count; min(n, cap) written. */
int nkv_frame_indices(int32_t kind, uint64_t total_frames, uint64_t past_frames, int32_t sampling, double gamma,
                      uint64_t* out, uint64_t cap, uint64_t* n);

/* plan_recent_trim + apply_trim (cache/swa.rs:52-130).  records is n x
 * {segment_index, frame_start, frame_count, image_tokens, text_tokens};
 * drop_frames n x {position, frames}; kept n x 5 (the surviving records). */
int nkv_plan_recent_trim(const uint64_t* records, uint64_t n, uint64_t capacity, uint64_t tokens_per_frame,
                         uint64_t* drop_frames, uint64_t* n_drop_frames, uint64_t* drop_records,
                         uint64_t* n_drop_records, uint64_t* evicted_tokens, uint64_t* kept, uint64_t* n_kept);

/* ------------------------------------------------- standalone kernels -- */

/* quantize_kv_pair (cache/int8.rs:85-134) on the device: `rows` rows of D
 * values of k and v (any float dtype; cast to BF16 first like
 * history.rs:249-250), u8 codes (int8 + 128) and f32 scales out.
 * *nonfinite_out (host) gets bit 0 for non-finite k, bit 1 for v; the call
 * synchronizes `stream` and returns NKV_ERR_MSG with the reference message
 * when any bit is set. */
int nkv_int8_quantize(const void* k, const void* v, int32_t in_dtype, uint64_t rows, int64_t head_dim,
                      uint8_t* kq, uint8_t* vq, float* ks, float* vs, uint32_t* nonfinite_out, void* stream);

/* dequantize (cache/int8.rs:139-155): rows x D codes + per-row scales to
 * out_dtype values. */
int nkv_int8_dequantize(const uint8_t* q, const float* scales, uint64_t rows, int64_t head_dim, int32_t out_dtype,
                        void* out, void* stream);

/* QvgCodec::encode (cache/qvg.rs:173-256) of one side of a (1, L, H, D)
 * tensor's first `tokens` tokens, against device codebooks cb_dev
 * [2][H][stages][2^bits][D] f32.  codes: [tokens][H][bpt]; scales:
 * [H][n_blocks][stages]. */
int nkv_qvg_encode(const float* cb_dev, int32_t side, const void* x, int32_t in_dtype, uint64_t L, int64_t heads,
                   int64_t head_dim, uint64_t tokens, int32_t stages, int32_t bits, int32_t block, uint8_t* codes,
                   float* scales, void* stream);

/* QvgCodec::decode (cache/qvg.rs:259-300) to f32 (1, tokens, H, D). */
int nkv_qvg_decode(const float* cb_dev, int32_t side, const uint8_t* codes, const float* scales, uint64_t tokens,
                   int64_t heads, int64_t head_dim, int32_t stages, int32_t bits, int32_t block, float* out,
                   void* stream);

/* The captured K / V of one layer with the commit's quantize in the same
 * kernel (tcgen05 GEMM, TMA, sm_100a), batch 1:
 *   K = apply_rotary(RmsNorm_k(Lin_k(x)))   modules/attention.rs:107-124, 143-144;
 *                                           modules/mod.rs:122-142; norm.rs:55-65;
 *                                           rope.rs:257-306
 *   V = Lin_v(x)
 * with every intermediate rounded to bf16 where the reference rounds it, and
 * for each row of x inside `ranges`, quantize_one (cache/int8.rs:65-81) of
 * that K / V row per head into the INT8 planes (row lo + i of x -> plane row
 * dst + i).  x is (tokens, H*D) bf16; wk / wv the (H*D, H*D) nn.Linear
 * weights ([out][in]) bf16; bk / bv (H*D) bf16 or NULL (no bias);
 * k_norm_gain (D) bf16 or NULL (no gain); qk_norm = 0 skips the norm;
 * rope_cos / rope_sin (tokens, D/2) f32 or NULL (no rotation); k_out / v_out
 * (tokens, H*D) bf16 or NULL; k_codes.. NULL for no codes.  Requirements:
 * D = 128, H*D a multiple of 256, H <= 256, tokens <= 2^26, tensor pointers 16-byte aligned, scales
 * and status 4-byte aligned (else NKV_ERR_ARGUMENT).  *status (device word) gets bit 0 / bit 1 for a
 * non-finite K / V value in a range row, bit 31 if a bounded wait inside the
 * kernel ran out.  Stream-ordered on `stream` on the current device; no
 * synchronisation.  Differences from the reference: the sum of squares is
 * taken as four interleaved f32 partial sums and (var + eps)^-1/2 as
 * 1 / sqrt with IEEE operations (candle: its own reduction order and powf);
 * the GEMM accumulates in f32 on the tensor cores (candle: cuBLAS). */
typedef struct {
  int64_t lo, hi, dst;
} nkv_row_range;
typedef struct {
  int64_t tokens;
  int32_t heads;
  int32_t head_dim;
  const void* x;
  const void* wk;
  const void* bk;
  const void* wv;
  const void* bv;
  int32_t qk_norm;
  float eps;
  const void* k_norm_gain;
  const float* rope_cos;
  const float* rope_sin;
  void* k_out;
  void* v_out;
  uint8_t* k_codes;
  float* k_scales;
  uint8_t* v_codes;
  float* v_scales;
  int32_t n_ranges;
  nkv_row_range ranges[2];
  uint32_t* status;
} nkv_kv_project_args;
int nkv_kv_project(const nkv_kv_project_args* args, void* stream);

/* Deterministic synthetic K/V for tests and benchmarks (no reference
 * counterpart): element (t, h, d) of a (rows = B*L, H, D) tensor is
 *   table[u >> 48] * (chan_scale ? chan_scale[h*D + d] : 1)
 * rounded to `dtype`, with u = mix64(key + (flat_index + 1) * 0x9E3779B97F4A7C15)
 * (mix64 = the SplitMix64 finalizer) and flat_index = (t*H + h)*D + d +
 * index_offset.  table is a 65536-entry f32 device array; chan_scale an H*D
 * f32 device array or NULL. */
int nkv_synth_fill(void* dst, int32_t dtype, uint64_t rows, int64_t heads, int64_t head_dim, uint64_t key,
                   uint64_t index_offset, const float* table, const float* chan_scale, void* stream);

/* ------------------------------------------------ no-allocation variant -- */

/* Most layers one nkv_int8_quantize_layers_noalloc call accepts. */
#define NKV_NOALLOC_MAX_LAYERS 64

/* INT8 quantize (the same kernel and results as nkv_int8_quantize, applied
 * to n_layers K/V pairs in one launch) that allocates no device memory, for
 * callers that cannot call cudaMalloc: a process whose GPU memory is owned
 * by another allocator or capped by a fixed budget, or a caller that must
 * not risk cudaMalloc's device-wide implicit synchronisation (this call
 * waits for `stream` only).  No counterpart in the reference.  k[i], v[i]
 * hold `rows` x head_dim values of in_dtype; kq/vq/ks/vs[i] receive codes
 * and scales; nonfinite_out (host, n_layers words) gets each layer's
 * non-finite bits.  The job table and flags live in one library-wide device
 * array sized for NKV_NOALLOC_MAX_LAYERS layers; larger n_layers is rejected
 * with NKV_ERR_ARGUMENT.  Every call looks up that array's address on the
 * current device.  Calls share the array: within one process the library
 * serialises them per GPU (a mutex held until the call's work finished),
 * whatever host threads and streams they come from.  Synchronizes `stream`
 * before returning. */
int nkv_int8_quantize_layers_noalloc(const void* const* k, const void* const* v, int32_t n_layers, int32_t in_dtype,
                                     uint64_t rows, int64_t head_dim, uint8_t* const* kq, uint8_t* const* vq,
                                     float* const* ks, float* const* vs, uint32_t* nonfinite_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NOMAS_KV_H */
