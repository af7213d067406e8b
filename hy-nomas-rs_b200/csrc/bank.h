// bank.h — host-side lifelong KV cache for a block of DiT layers on one GPU.
//
// `Bank` is the B200 counterpart of the reference's KvBank of HistoryCaches
// (cache/mod.rs:225-320, cache/history.rs:84-569) with the PhaseSwappedCache
// wrapper folded in (cache/phase_swap.rs:27-161).  In a KvBank every layer
// receives the same segment descriptors, so every layer's archive geometry,
// frame timeline, working-set layout and counters are identical; the bank
// keeps that shared state once and one device payload per layer.  Each
// archived segment is one device slab holding every local layer's payload
// at a fixed stride, so one kernel launch commits (or gathers) all layers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "nkv_kernels.h"
#include "nkv_policy.h"
#include "nomas_kv.h"

namespace nkv {

struct Error {
  int code;
  std::string msg;
};
[[noreturn]] void fail(int code, std::string msg);
void check_cuda(cudaError_t e, const char* what);

// Makes `device` current for the lifetime of the scope.
class DeviceScope {
 public:
  explicit DeviceScope(int device);
  ~DeviceScope();

 private:
  int prev_ = -1;
  bool switched_ = false;
};

// LIFO allocator for archive slabs.  The archive only grows at the end
// (commit) and shrinks at the end (rollback), so slabs are carved out of a
// few large chunks in stack order and never fragment.  Chunks are device
// memory up to a device byte limit (none by default); beyond it they are
// pinned host memory mapped into the device's address space, which the
// kernels read and write through the same pointers over the host link: an
// archive larger than HBM (256 segments x 48 layers at the 8B geometry is
// 506 GB) stays usable on one GPU.
class ArchiveArena {
 public:
  ~ArchiveArena();
  unsigned char* push(size_t bytes);
  void pop();
  void reserve(size_t bytes);
  void release();
  void set_device_limit(size_t bytes) { device_limit_ = bytes; }
  size_t device_limit() const { return device_limit_; }
  // bytes of the live slabs in device memory / in host memory
  void usage(size_t* device, size_t* host) const;
  // whether `p` lies in a pinned host chunk
  bool is_host(const void* p) const;

 private:
  struct Chunk {
    unsigned char* base;
    size_t cap;
    bool host;
  };
  unsigned char* alloc_chunk(size_t bytes, bool* host);
  size_t device_limit_ = SIZE_MAX, device_chunk_bytes_ = 0;
  struct Slot {
    size_t chunk, off, size;
  };
  std::vector<Chunk> chunks_;
  std::vector<Slot> stack_;
  size_t free_from_top() const;
};

// Pinned host -> device upload area for per-call metadata (job lists, run
// and tile tables, pointer arrays).  One H2D copy per call, issued on an
// auxiliary stream so that it never sits between two kernels of the cache's
// stream; the cache's stream waits for it with an event.  A ring of slots: a
// call's tables stay untouched on the device until the slot comes round
// again (the upload into a slot waits for the cache-stream work of the
// slot's previous call), and begin() waits only for that slot's host buffer
// to have left, kSlots calls ago.
class Staging {
 public:
  static constexpr int kSlots = 4;
  ~Staging();
  // next slot; `main` is the stream whose work consumes the tables
  void begin(cudaStream_t main);
  size_t add(const void* p, size_t bytes, size_t align = 16);
  // the copy on `aux`, ordered before everything enqueued on `main` afterwards
  void upload(cudaStream_t aux, cudaStream_t main);
  const void* dev(size_t off) const { return slot_[cur_].dev + off; }
  void release();

 private:
  struct Slot {
    unsigned char* host = nullptr;
    unsigned char* dev = nullptr;
    size_t cap = 0;
    cudaEvent_t done = nullptr;      // the upload left the host buffer
    cudaEvent_t consumed = nullptr;  // the cache-stream work of the slot's call
    bool pending = false, used = false;
  };
  Slot slot_[kSlots];
  int cur_ = 0;
  size_t used_ = 0;
};

struct Rec {  // one archived segment (history.rs:40-55), all local layers
  nkv_segment_desc desc;
  unsigned char* slab = nullptr;
  size_t layer_stride = 0;
  // component byte offsets inside a layer block:
  //   FLOAT: 0 k, 1 v | INT8: 0 kq, 1 vq, 2 ks, 3 vs |
  //   QVG  : 0 kcodes, 1 vcodes, 2 kscales, 3 vscales, 4..7 the text INT8 block
  size_t off[8] = {0};
  uint64_t n_blocks = 0;
  uint64_t nbytes = 0;  // payload_bytes (history.rs:70-81) of one layer
};

struct RunSpec {  // a contiguous token range of one archived segment
  size_t rec;
  bool text;  // QVG: the INT8 text block
  int64_t src_tok, dst_tok, ntok;
};

struct Plan {
  std::vector<nkv_segment_layout> layout;
  std::vector<RunSpec> runs;
  uint64_t valid = 0;
};

// Staging offsets of one gather's device tables.
struct GatherTables {
  size_t runs_off = 0, tiles_off = 0, qtiles_off = 0;
  int n_tiles = 0, n_qtiles = 0;
  bool aligned = true;
};

class Bank {
 public:
  Bank(const nkv_cache_config& cfg, int n_layers, int layer_begin, int64_t batch, int64_t heads, int64_t head_dim,
       int dtype, int device, cudaStream_t stream);
  ~Bank();

  void commit(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v);
  // commit, then the new segment decoded in full (decode_segment) into
  // k_out / v_out by the rebuild's gather launch
  void commit_decode(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v,
                     void* const* k_out, void* const* v_out);
  // Two-phase INT8 commit for a producer that writes the archive rows itself
  // (the fused K/V projection): stage validates the segment and reserves its
  // record, commit_staged archives it and rebuilds, discard_staged drops it.
  void stage(const nkv_segment_desc& s, nkv_staged_layer* out);
  void commit_staged();
  void discard_staged();
  bool staged() const { return staged_; }
  void rollback();
  void park();
  void unpark();
  void decode_segment(uint64_t pos, void* const* k_out, void* const* v_out);
  // attention of q (q_len, H, 128) bf16 over `layer`'s history read from
  // the INT8 archive; out (q_len, H, 128) f32, lse (H, q_len) f32
  void attend_history(int layer, const void* q, uint64_t q_len, float scale, float* out, float* lse);
  void synchronize();
  void reserve(uint64_t archive_bytes, uint64_t working_tokens);
  void set_archive_device_limit(uint64_t bytes);
  void archive_usage(uint64_t* device, uint64_t* host) const;
  uint64_t segment_bytes(const nkv_segment_desc& s) const;

  void working_set(int layer, const void** k, const void** v, uint64_t* valid) const;
  const std::vector<nkv_segment_layout>& layout() const { return parked_ ? p_layout_ : layout_; }
  void info(int layer, nkv_cache_info_t* out) const;
  nkv_metrics layer_metrics() const { return m_; }
  nkv_metrics bank_metrics() const;
  void set_codebooks(int layer, const float* host);
  void get_codebooks(int layer, float* host, int32_t* fitted) const;
  uint64_t export_segment(int layer, uint64_t pos, void* host, uint64_t cap);

  void set_timing(bool on);
  void kernel_stats(nkv_kernel_stat* out, bool reset);

  // Archive persistence (no counterpart in the reference, whose archive is
  // in memory only): the timeline, counters, QVG codebooks and every archived
  // payload; load rebuilds the working set.
  void save(const char* path);
  void load(const char* path);

  int n_layers() const { return n_layers_; }

 private:
  Rec make_rec(const nkv_segment_desc& s) const;
  void validate(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v);
  // archive_segment + rebuild of a validated segment whose slab is pushed;
  // `staged`: the codes are already in the slab and the per-layer flags set
  void finish_commit(const nkv_segment_desc& s, Rec r, int kv_dtype, const void* const* k, const void* const* v,
                     bool staged, void* const* dk = nullptr, void* const* dv = nullptr);
  Plan decode_plan(size_t pos) const;
  void no_staged(const char* what) const;
  Plan plan_rebuild();
  // device run/tile tables of `plan` (out_set 0) and, when given, of
  // `plan2` (out_set 1, the second output set of the same launch)
  GatherTables add_runs(const Plan& plan, bool outputs_aligned = true, const Plan* plan2 = nullptr);
  std::vector<int> fit_qvg(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v);
  void launch_gather_into(const GatherTables& t, size_t outk_off, size_t outv_off, uint64_t out_L, bool vector_ok,
                          const uint32_t* abort_flag, int timing_id = NKV_KERNEL_GATHER, size_t out2k_off = 0,
                          size_t out2v_off = 0, uint64_t out2_L = 0);
  void ensure_ws(uint64_t tokens, unsigned char** fresh, uint64_t* fresh_cap);
  unsigned char* ws_plane(unsigned char* base, uint64_t cap, int layer, int side) const;
  size_t ws_plane_bytes(uint64_t cap) const;
  void rebuild_now();  // plan + gather + install (rollback path)
  uint64_t capacity_or_max() const { return cfg_.has_capacity ? cfg_.capacity : UINT64_MAX; }

  void tbegin(int kind);
  void tend(int kind);
  void collect_timing(bool wait);

  nkv_cache_config cfg_;
  int n_layers_, layer_begin_;
  int64_t B_, H_, D_;
  int dtype_, device_;
  cudaStream_t stream_ = nullptr, side_ = nullptr;
  int q_stages_ = 0, q_bits_ = 0, q_block_ = 0, q_E_ = 0, q_bpt_ = 0;

  std::vector<Rec> archive_;
  uint64_t total_frames_ = 0, tpf_ = 0;
  nkv_metrics m_{};
  std::vector<nkv_segment_layout> layout_;
  std::vector<RunSpec> ws_runs_;  // the runs the current working set was gathered from
  std::vector<RunSpec> p_runs_;   // ... of the parked one
  uint32_t* d_attn_status_ = nullptr;
  float* d_attn_part_ = nullptr;  // split units' partial rows: 128 + 2 floats per row
  int64_t attn_part_rows_ = 0;
  int sms_ = 0;
  uint64_t valid_ = 0;

  bool parked_ = false;
  bool staged_ = false;  // a staged segment's slab is the arena's top
  Rec staged_rec_;
  // the working set is the rebuild of the current archive (false after a
  // failed rebuild, or after unpark restored a set older than the archive)
  bool ws_current_ = true;
  bool p_ws_current_ = true, changed_while_parked_ = false;
  std::vector<nkv_segment_layout> p_layout_;
  uint64_t p_valid_ = 0, p_bytes_ = 0;
  std::vector<unsigned char*> p_host_;
  std::vector<size_t> p_host_cap_;

  ArchiveArena arena_;
  unsigned char* ws_ = nullptr;
  uint64_t ws_cap_ = 0;

  float* cb_dev_ = nullptr;
  std::vector<float> cb_host_;
  std::vector<char> fitted_;
  size_t cb_layer_ = 0;

  // Two sets of n_layers + 1 non-finite flags (see the constructor), used
  // by alternate commits: a commit clears its set while the previous commit's
  // gather, which reads the other set, may still run.
  uint32_t* d_flags_[2] = {nullptr, nullptr};
  uint32_t* d_flag_ = nullptr;  // the current commit's set
  int flag_set_ = 0;
  cudaEvent_t flags_free_[2] = {nullptr, nullptr};  // the last gather that read set i is done
  uint32_t* h_flag_ = nullptr;
  cudaEvent_t flag_ev_ = nullptr;  // the flags' read-back has landed
  cudaEvent_t encoded_ = nullptr;  // the commit's archive kernels ran
  cudaStream_t aux_ = nullptr;     // table uploads, flag clears and read-backs
  void next_flags(bool clear_on_aux);
  Staging stg_;

  bool timing_ = false;
  struct Pending {
    int kind;
    cudaEvent_t a, b;
  };
  std::vector<Pending> pending_;
  std::vector<cudaEvent_t> ev_pool_;
  cudaEvent_t cur_a_ = nullptr;
  nkv_kernel_stat stats_[NKV_KERNEL_COUNT] = {};
};

}  // namespace nkv
