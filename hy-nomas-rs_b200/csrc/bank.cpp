// bank.cpp — host logic of the lifelong KV cache (see bank.h).
//
// Reference map (nomas-core):
//   Bank::Bank          HistoryCache::new        cache/history.rs:104-156
//   Bank::validate      validate_segment         cache/history.rs:168-238
//   Bank::commit        commit_segment           cache/history.rs:458-463
//                       archive_segment          cache/history.rs:241-305
//   Bank::plan_rebuild  rebuild                  cache/history.rs:341-446
//   Bank::rollback      rollback_last_segment    cache/history.rs:507-528
//   Bank::park/unpark   PhaseSwappedCache        cache/phase_swap.rs:42-81
//   Bank::bank_metrics  KvBank::metrics          cache/mod.rs:305-319
#include "bank.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>


namespace nkv {

void fail(int code, std::string msg) { throw Error{code, std::move(msg)}; }

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(NKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
#define NKV_CUDA(expr) check_cuda((expr), #expr)

static inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }
static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------ DeviceScope --
DeviceScope::DeviceScope(int device) {
  if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
  if (prev_ != device) {
    NKV_CUDA(cudaSetDevice(device));
    switched_ = true;
  }
}
DeviceScope::~DeviceScope() {
  if (switched_ && prev_ >= 0) cudaSetDevice(prev_);
}

// ----------------------------------------------------------- ArchiveArena --
ArchiveArena::~ArchiveArena() { release(); }

void ArchiveArena::release() {
  for (auto& c : chunks_) {
    if (c.host) cudaFreeHost(c.base);
    else cudaFree(c.base);
  }
  chunks_.clear();
  stack_.clear();
  device_chunk_bytes_ = 0;
}

unsigned char* ArchiveArena::alloc_chunk(size_t bytes, bool* host) {
  unsigned char* p = nullptr;
  if (device_chunk_bytes_ + bytes <= device_limit_) {
    NKV_CUDA(cudaMalloc(&p, bytes));
    device_chunk_bytes_ += bytes;
    *host = false;
    return p;
  }
  NKV_CUDA(cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable));
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, p, 0) != cudaSuccess || d != p) {
    cudaFreeHost(p);
    fail(NKV_ERR_CUDA, "host archive tier: the device does not address mapped host memory by its host pointer");
  }
  *host = true;
  return p;
}

size_t ArchiveArena::free_from_top() const {
  size_t ci = stack_.empty() ? 0 : stack_.back().chunk;
  size_t off = stack_.empty() ? 0 : stack_.back().off + stack_.back().size;
  size_t free = 0;
  for (size_t i = ci; i < chunks_.size(); ++i) free += chunks_[i].cap - (i == ci ? off : 0);
  return free;
}

unsigned char* ArchiveArena::push(size_t bytes) {
  bytes = align_up(std::max<size_t>(bytes, 1));
  size_t ci = stack_.empty() ? 0 : stack_.back().chunk;
  size_t off = stack_.empty() ? 0 : stack_.back().off + stack_.back().size;
  while (ci < chunks_.size() && off + bytes > chunks_[ci].cap) {
    ++ci;
    off = 0;
  }
  if (ci == chunks_.size()) {
    bool host = false;
    unsigned char* p = alloc_chunk(bytes, &host);
    chunks_.push_back({p, bytes, host});
  }
  stack_.push_back({ci, off, bytes});
  return chunks_[ci].base + off;
}

void ArchiveArena::pop() {
  if (!stack_.empty()) stack_.pop_back();
}

void ArchiveArena::reserve(size_t bytes) {
  if (free_from_top() >= bytes) return;
  size_t b = align_up(bytes);
  // what the device limit still allows goes to device memory, the rest to
  // the host tier
  if (device_chunk_bytes_ < device_limit_ && device_chunk_bytes_ + b > device_limit_) {
    const size_t room = (device_limit_ - device_chunk_bytes_) / 256 * 256;
    if (room > 0) {
      bool host = false;
      unsigned char* p = alloc_chunk(room, &host);
      chunks_.push_back({p, room, host});
      b -= std::min(b, room);
    }
  }
  if (b == 0) return;
  bool host = false;
  unsigned char* p = alloc_chunk(b, &host);
  chunks_.push_back({p, b, host});
}

bool ArchiveArena::is_host(const void* p) const {
  const unsigned char* q = static_cast<const unsigned char*>(p);
  for (const auto& c : chunks_)
    if (q >= c.base && q < c.base + c.cap) return c.host;
  return false;
}

void ArchiveArena::usage(size_t* device, size_t* host) const {
  *device = *host = 0;
  for (const auto& sl : stack_) (chunks_[sl.chunk].host ? *host : *device) += sl.size;
}

// ---------------------------------------------------------------- Staging --
Staging::~Staging() { release(); }

void Staging::release() {
  for (auto& sl : slot_) {
    if (sl.done) {
      cudaEventSynchronize(sl.done);
      cudaEventDestroy(sl.done);
    }
    if (sl.consumed) {
      cudaEventSynchronize(sl.consumed);
      cudaEventDestroy(sl.consumed);
    }
    if (sl.host) cudaFreeHost(sl.host);
    if (sl.dev) cudaFree(sl.dev);
    sl = Slot{};
  }
  cur_ = 0;
  used_ = 0;
}

void Staging::begin(cudaStream_t main) {
  // everything the previous call enqueued on `main` has read its slot by the
  // time this event completes
  Slot& prev = slot_[cur_];
  if (prev.used) NKV_CUDA(cudaEventRecord(prev.consumed, main));
  cur_ = (cur_ + 1) % kSlots;
  Slot& sl = slot_[cur_];
  if (!sl.done) {
    NKV_CUDA(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
    NKV_CUDA(cudaEventCreateWithFlags(&sl.consumed, cudaEventDisableTiming));
  }
  if (sl.pending) {
    NKV_CUDA(cudaEventSynchronize(sl.done));
    sl.pending = false;
  }
  sl.used = false;
  used_ = 0;
}

size_t Staging::add(const void* p, size_t bytes, size_t align) {
  Slot& sl = slot_[cur_];
  size_t off = align_up(used_, align);
  if (off + bytes > sl.cap) {
    size_t cap = std::max<size_t>(align_up(off + bytes, 4096) * 2, 64 * 1024);
    unsigned char *h = nullptr, *d = nullptr;
    NKV_CUDA(cudaHostAlloc(&h, cap, cudaHostAllocDefault));
    if (cudaMalloc(&d, cap) != cudaSuccess) {
      cudaFreeHost(h);
      fail(NKV_ERR_CUDA, "staging: cudaMalloc failed");
    }
    if (used_) std::memcpy(h, sl.host, used_);
    // the old device buffer may still be read by kernels in flight
    if (sl.dev) cudaDeviceSynchronize();
    if (sl.host) cudaFreeHost(sl.host);
    if (sl.dev) cudaFree(sl.dev);
    sl.host = h, sl.dev = d, sl.cap = cap;
  }
  if (bytes) std::memcpy(sl.host + off, p, bytes);
  used_ = off + bytes;
  return off;
}

void Staging::upload(cudaStream_t aux, cudaStream_t main) {
  if (used_ == 0) return;
  Slot& sl = slot_[cur_];
  // the slot's previous tables were read by work on `main` (kSlots calls ago)
  NKV_CUDA(cudaStreamWaitEvent(aux, sl.consumed, 0));
  NKV_CUDA(cudaMemcpyAsync(sl.dev, sl.host, used_, cudaMemcpyHostToDevice, aux));
  NKV_CUDA(cudaEventRecord(sl.done, aux));
  NKV_CUDA(cudaStreamWaitEvent(main, sl.done, 0));
  sl.pending = true;
  sl.used = true;
}

// ------------------------------------------------------------------- Bank --
static void validate_config(const nkv_cache_config& c, int n_layers, int64_t batch, int64_t heads, int64_t head_dim,
                            int dtype) {
  // history.rs:112-134, in the reference's order
  if (c.storage < NKV_STORAGE_FLOAT || c.storage > NKV_STORAGE_QVG)
    fail(NKV_ERR_INVALID_CONFIG, "unknown cache storage " + std::to_string(c.storage));
  if (c.sampling < NKV_SAMPLING_RECENT || c.sampling > NKV_SAMPLING_TEMPORAL)
    fail(NKV_ERR_INVALID_CONFIG, "unknown history sampling " + std::to_string(c.sampling));
  if (c.storage == NKV_STORAGE_QVG) {
    if (batch != 1)
      fail(NKV_ERR_INVALID_CONFIG, "QVG storage requires batch=1 (interactive world-model sessions)");
    if (c.qvg.bits_per_stage <= 0 || c.qvg.bits_per_stage > 8 || c.qvg.stages <= 0)
      fail(NKV_ERR_INVALID_CONFIG, "invalid QVG stages/bits");
  }
  if (c.sampling == NKV_SAMPLING_TEMPORAL && (!std::isfinite(c.gamma) || c.gamma <= 0.0))
    fail(NKV_ERR_INVALID_CONFIG, "invalid temporal_context gamma " + rust_f64(c.gamma));
  if (c.has_capacity && c.capacity == 0) fail(NKV_ERR_INVALID_CONFIG, "cache capacity must be > 0");
  if (c.past_frames == 0) fail(NKV_ERR_INVALID_CONFIG, "past_frames must be > 0");
  // Checks with no reference counterpart (the reference would panic or build
  // degenerate tensors): positive geometry, a known dtype, and QVG shapes the
  // device encoder can hold.
  if (n_layers < 1) fail(NKV_ERR_INVALID_CONFIG, "n_layers must be >= 1");
  if (batch < 1 || heads < 1 || head_dim < 1) fail(NKV_ERR_INVALID_CONFIG, "batch, heads and head_dim must be >= 1");
  if (dtype < NKV_F32 || dtype > NKV_F16) fail(NKV_ERR_INVALID_CONFIG, "unknown model dtype");
  if (c.storage == NKV_STORAGE_QVG) {
    if (c.qvg.block_size <= 0) fail(NKV_ERR_INVALID_CONFIG, "QVG block_size must be > 0");
    if (int64_t(c.qvg.stages) * c.qvg.bits_per_stage > 64)
      fail(NKV_ERR_INVALID_CONFIG, "QVG stages * bits_per_stage must be <= 64");
    if (qvg_encode_smem_bytes(int(head_dim), c.qvg.block_size, c.qvg.bits_per_stage) > 200 * 1024)
      fail(NKV_ERR_INVALID_CONFIG, "QVG block_size x head_dim too large for the device encoder");
  }
}

Bank::Bank(const nkv_cache_config& cfg, int n_layers, int layer_begin, int64_t batch, int64_t heads, int64_t head_dim,
           int dtype, int device, cudaStream_t stream)
    : cfg_(cfg),
      n_layers_(n_layers),
      layer_begin_(layer_begin),
      B_(batch),
      H_(heads),
      D_(head_dim),
      dtype_(dtype),
      device_(device),
      stream_(stream) {
  validate_config(cfg, n_layers, batch, heads, head_dim, dtype);
  if (cfg.storage == NKV_STORAGE_QVG) {
    q_stages_ = cfg.qvg.stages, q_bits_ = cfg.qvg.bits_per_stage, q_block_ = cfg.qvg.block_size;
    q_E_ = 1 << q_bits_;
    q_bpt_ = (q_stages_ * q_bits_ + 7) / 8;
  }
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0)
    fail(NKV_ERR_CUDA, "no CUDA device: the cache has no CPU fallback");
  if (device < 0 || device >= n_dev) fail(NKV_ERR_ARGUMENT, "device " + std::to_string(device) + " out of range");
  DeviceScope ds(device_);
  NKV_CUDA(cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking));
  NKV_CUDA(cudaStreamCreateWithFlags(&aux_, cudaStreamNonBlocking));
  // [0]: any layer saw a non-finite value (aborts the gather); [1 + i]: layer i
  for (int b = 0; b < 2; ++b) {
    NKV_CUDA(cudaMalloc(&d_flags_[b], sizeof(uint32_t) * (n_layers_ + 1)));
    NKV_CUDA(cudaMemset(d_flags_[b], 0, sizeof(uint32_t) * (n_layers_ + 1)));
    NKV_CUDA(cudaEventCreateWithFlags(&flags_free_[b], cudaEventDisableTiming));
  }
  d_flag_ = d_flags_[0];
  NKV_CUDA(cudaHostAlloc(&h_flag_, sizeof(uint32_t) * (n_layers_ + 1), cudaHostAllocDefault));
  // the commit's one host wait (its non-finite flags): the thread sleeps
  // instead of spinning, which leaves the host cores to the other ranks'
  // processes; the wake-up is hidden behind the gather queued before the wait
  NKV_CUDA(cudaEventCreateWithFlags(&flag_ev_, cudaEventDisableTiming | cudaEventBlockingSync));
  NKV_CUDA(cudaEventCreateWithFlags(&encoded_, cudaEventDisableTiming));
  std::memset(h_flag_, 0, sizeof(uint32_t) * (n_layers_ + 1));
  if (cfg.storage == NKV_STORAGE_QVG) {
    cb_layer_ = size_t(2) * H_ * q_stages_ * q_E_ * D_;
    NKV_CUDA(cudaMalloc(&cb_dev_, cb_layer_ * n_layers_ * sizeof(float)));
    cb_host_.assign(cb_layer_ * n_layers_, 0.0f);
    fitted_.assign(n_layers_, 0);
  }
  p_host_.assign(n_layers_, nullptr);
  p_host_cap_.assign(n_layers_, 0);
}

Bank::~Bank() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  if (side_) {
    cudaStreamSynchronize(side_);
    cudaStreamDestroy(side_);
  }
  if (aux_) {
    cudaStreamSynchronize(aux_);
    cudaStreamDestroy(aux_);
  }
  for (auto& p : pending_) {
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
  }
  for (auto e : ev_pool_) cudaEventDestroy(e);
  if (cur_a_) cudaEventDestroy(cur_a_);
  if (ws_) cudaFree(ws_);
  if (cb_dev_) cudaFree(cb_dev_);
  for (int b = 0; b < 2; ++b) {
    if (d_flags_[b]) cudaFree(d_flags_[b]);
    if (flags_free_[b]) cudaEventDestroy(flags_free_[b]);
  }
  if (h_flag_) cudaFreeHost(h_flag_);
  if (flag_ev_) cudaEventDestroy(flag_ev_);
  if (encoded_) cudaEventDestroy(encoded_);
  if (d_attn_status_) cudaFree(d_attn_status_);
  if (d_attn_part_) cudaFree(d_attn_part_);
  for (auto p : p_host_)
    if (p) cudaFreeHost(p);
  stg_.release();
  arena_.release();
}

// Archive slab geometry of one segment (ArchivedPayload, history.rs:25-37).
Rec Bank::make_rec(const nkv_segment_desc& s) const {
  Rec r;
  r.desc = s;
  const size_t L = s.image_tokens + s.text_tokens, HD = size_t(H_) * D_, B = size_t(B_);
  size_t o = 0;
  auto put = [&](size_t bytes) {
    size_t at = o;
    o += align_up(bytes);
    return at;
  };
  if (cfg_.storage == NKV_STORAGE_FLOAT) {
    const size_t n = B * L * HD * dtype_size(dtype_);
    r.off[0] = put(n), r.off[1] = put(n);
    r.nbytes = 2 * n;
  } else if (cfg_.storage == NKV_STORAGE_INT8) {
    r.off[0] = put(B * L * HD), r.off[1] = put(B * L * HD);
    r.off[2] = put(B * L * H_ * 4), r.off[3] = put(B * L * H_ * 4);
    r.nbytes = 2 * B * L * HD + 2 * B * L * H_ * 4;  // Int8KvBlock::nbytes (int8.rs:56-61)
  } else {
    const size_t Lv = s.image_tokens, Lt = s.text_tokens;
    r.n_blocks = (Lv + q_block_ - 1) / q_block_;
    r.off[0] = put(Lv * H_ * q_bpt_), r.off[1] = put(Lv * H_ * q_bpt_);
    r.off[2] = put(size_t(H_) * r.n_blocks * q_stages_ * 4), r.off[3] = put(size_t(H_) * r.n_blocks * q_stages_ * 4);
    // QvgPayload::nbytes (qvg.rs:81-83) for k and v
    r.nbytes = 2 * (Lv * H_ * q_bpt_ + size_t(H_) * r.n_blocks * q_stages_ * 4);
    if (Lt > 0) {
      r.off[4] = put(Lt * HD), r.off[5] = put(Lt * HD);
      r.off[6] = put(Lt * H_ * 4), r.off[7] = put(Lt * H_ * 4);
      r.nbytes += 2 * Lt * HD + 2 * Lt * H_ * 4;
    }
  }
  r.layer_stride = std::max<size_t>(align_up(o), 256);
  return r;
}

uint64_t Bank::segment_bytes(const nkv_segment_desc& s) const { return make_rec(s).layer_stride; }

// validate_segment (history.rs:168-238).  Like the reference it records
// tokens_per_frame from the first segment before the later checks run.
void Bank::validate(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v) {
  if (s.frame_count == 0 || s.image_tokens == 0) fail(NKV_ERR_GEOMETRY, "segment must contain at least one frame");
  const uint64_t tpf = s.image_tokens / s.frame_count;
  if (s.image_tokens % s.frame_count != 0 || tpf == 0)
    fail(NKV_ERR_GEOMETRY, "image_tokens " + std::to_string(s.image_tokens) + " not divisible by frame_count " +
                               std::to_string(s.frame_count));
  if (tpf_ == 0)
    tpf_ = tpf;
  else if (tpf_ != tpf)
    fail(NKV_ERR_GEOMETRY,
         "tokens_per_frame changed mid-session: " + std::to_string(tpf_) + " -> " + std::to_string(tpf));
  if (!archive_.empty()) {
    if (s.segment_index <= archive_.back().desc.segment_index)
      fail(NKV_ERR_CACHE_STATE, "history requires one chronological write per segment");
    if (s.frame_start != total_frames_)
      fail(NKV_ERR_GEOMETRY, "segment frame_start " + std::to_string(s.frame_start) +
                                 " does not continue the timeline at " + std::to_string(total_frames_));
  } else if (s.frame_start != 0 && total_frames_ == 0) {
    fail(NKV_ERR_GEOMETRY, "first segment must start at frame 0, got " + std::to_string(s.frame_start));
  }
  if (s.action_start < -1 || s.action_start > int64_t(s.text_tokens))
    fail(NKV_ERR_GEOMETRY, "action_start " + std::to_string(s.action_start) + " outside text block of " +
                               std::to_string(s.text_tokens));
  if (kv_dtype < NKV_F32 || kv_dtype > NKV_F16) fail(NKV_ERR_GEOMETRY, "segment k must be float");
  // "segment KV must live on the cache device" (history.rs:232-236); a
  // staged segment has no input tensors
  if (k && v)
  for (int i = 0; i < n_layers_; ++i)
    for (int side = 0; side < 2; ++side) {
      const void* p = side ? v[i] : k[i];
      cudaPointerAttributes at{};
      if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        fail(NKV_ERR_GEOMETRY, "segment KV must live on the cache device");
      }
      const bool on_dev = (at.type == cudaMemoryTypeDevice && at.device == device_) || at.type == cudaMemoryTypeManaged;
      if (!on_dev) fail(NKV_ERR_GEOMETRY, "segment KV must live on the cache device");
    }
}

// rebuild (history.rs:341-446), host half: which frames of which archived
// segments the working set holds, as contiguous token runs, plus the layout.
// Recent mode adds its evicted tokens to the counters before the capacity
// check, exactly like the reference.
Plan Bank::plan_rebuild() {
  const uint64_t tpf = std::max<uint64_t>(tpf_, 1);
  std::vector<std::pair<size_t, std::vector<uint64_t>>> selection;
  if (cfg_.sampling == NKV_SAMPLING_RECENT) {
    std::vector<DenseRecord> recs;
    recs.reserve(archive_.size());
    for (const auto& a : archive_)
      recs.push_back({a.desc.segment_index, a.desc.frame_start, a.desc.frame_count, a.desc.image_tokens,
                      a.desc.text_tokens});
    TrimPlan plan = plan_recent_trim(recs, capacity_or_max(), tpf);
    m_.evicted_tokens += plan.evicted_tokens;
    for (const auto& r : apply_trim(recs, plan, tpf)) {
      size_t idx = 0;
      for (size_t i = 0; i < archive_.size(); ++i)
        if (archive_[i].desc.segment_index == r.segment_index) {
          idx = i;
          break;
        }
      // The reference keeps frames 0..kept of the segment (its oldest
      // frames) after a partial trim (history.rs:350-358).
      std::vector<uint64_t> frames(r.frame_count);
      for (uint64_t f = 0; f < r.frame_count; ++f) frames[f] = f;
      selection.push_back({idx, std::move(frames)});
    }
  } else {
    std::vector<uint64_t> ids;
    try {
      ids = history_frame_indices(total_frames_, cfg_.past_frames, cfg_.sampling, cfg_.gamma);
    } catch (const PolicyError& e) {
      fail(e.code, e.msg);
    }
    size_t j = 0;  // ids are strictly increasing and archives are chronological
    for (size_t idx = 0; idx < archive_.size(); ++idx) {
      const auto& a = archive_[idx].desc;
      std::vector<uint64_t> sel;
      while (j < ids.size() && ids[j] < a.frame_start) ++j;
      for (size_t t = j; t < ids.size() && ids[t] < a.frame_start + a.frame_count; ++t)
        sel.push_back(ids[t] - a.frame_start);
      if (!sel.empty()) selection.push_back({idx, std::move(sel)});
    }
  }
  Plan p;
  uint64_t cursor = 0;
  for (const auto& [idx, sel] : selection) {
    const auto& a = archive_[idx].desc;
    const uint64_t video_end = cursor + sel.size() * tpf;
    const uint64_t text_end = video_end + a.text_tokens;
    p.layout.push_back({a.segment_index, cursor, video_end, video_end, text_end, a.action_start});
    // consecutive frames merge into one run
    uint64_t dst = cursor;
    for (size_t i = 0; i < sel.size();) {
      size_t j2 = i + 1;
      while (j2 < sel.size() && sel[j2] == sel[j2 - 1] + 1) ++j2;
      const int64_t n = int64_t((j2 - i) * tpf);
      p.runs.push_back({idx, false, int64_t(sel[i] * tpf), int64_t(dst), n});
      dst += uint64_t(n);
      i = j2;
    }
    if (a.text_tokens > 0)
      p.runs.push_back({idx, cfg_.storage == NKV_STORAGE_QVG, int64_t(a.image_tokens), int64_t(video_end),
                        int64_t(a.text_tokens)});
    cursor = text_end;
  }
  if (cursor > capacity_or_max())
    fail(NKV_ERR_GEOMETRY,
         "history needs " + std::to_string(cursor) + " tokens; capacity is " + std::to_string(capacity_or_max()));
  p.valid = cursor;
  return p;
}

// Device run/tile tables for a plan, appended to the staging area.
GatherTables Bank::add_runs(const Plan& plan, bool outputs_aligned, const Plan* plan2) {
  constexpr int64_t kTile = 32;
  std::vector<GatherRun> runs;
  std::vector<GatherTile> tiles;
  std::vector<GatherQvgTile> qtiles;
  // video runs of the default codec go to the table-driven decoder: tiles of
  // <= 64 tokens inside one payload block (one alpha per head and stage)
  const bool qvg_fast = cfg_.storage == NKV_STORAGE_QVG && qvg_gather_fast_ok(int(H_), int(D_), q_stages_, q_bits_) &&
                        B_ == 1 && outputs_aligned;
  runs.reserve(plan.runs.size() + (plan2 ? plan2->runs.size() : 0));
  std::vector<std::pair<const RunSpec*, int32_t>> all;
  for (const auto& rs : plan.runs) all.push_back({&rs, 0});
  if (plan2)
    for (const auto& rs : plan2->runs) all.push_back({&rs, 1});
  for (const auto& [rsp, out_set] : all) {
    const RunSpec& rs = *rsp;
    const Rec& r = archive_[rs.rec];
    GatherRun g{};
    g.out_set = out_set;
    g.src = r.slab;
    g.layer_stride = int64_t(r.layer_stride);
    g.src_tok = rs.src_tok;
    g.dst_tok = rs.dst_tok;
    g.ntok = rs.ntok;
    g.n_blocks = int32_t(r.n_blocks);
    const int64_t L = int64_t(r.desc.image_tokens + r.desc.text_tokens);
    if (cfg_.storage == NKV_STORAGE_FLOAT) {
      g.kind = RUN_FLOAT, g.src_L = L;
      g.off[0] = int64_t(r.off[0]), g.off[1] = int64_t(r.off[1]);
    } else if (cfg_.storage == NKV_STORAGE_INT8) {
      g.kind = RUN_INT8, g.src_L = L;
      for (int i = 0; i < 4; ++i) g.off[i] = int64_t(r.off[i]);
    } else if (!rs.text) {
      g.kind = RUN_QVG_VIDEO, g.src_L = int64_t(r.desc.image_tokens);
      for (int i = 0; i < 4; ++i) g.off[i] = int64_t(r.off[i]);
    } else {
      g.kind = RUN_INT8, g.src_L = int64_t(r.desc.text_tokens);
      g.src_tok = rs.src_tok - int64_t(r.desc.image_tokens);
      for (int i = 0; i < 4; ++i) g.off[i] = int64_t(r.off[4 + i]);
    }
    const int32_t run_id = int32_t(runs.size());
    runs.push_back(g);
    if (g.kind == RUN_QVG_VIDEO && qvg_fast) {
      const int64_t blk_tokens = q_block_;
      for (int64_t t0 = 0; t0 < rs.ntok;) {
        const int64_t tok = rs.src_tok + t0;
        const int64_t blk = tok / blk_tokens;
        const int64_t end = std::min<int64_t>({rs.ntok, (blk + 1) * blk_tokens - rs.src_tok, t0 + kQvgTileTokens});
        qtiles.push_back({run_id, int32_t(t0), int32_t(end - t0), int32_t(blk)});
        t0 = end;
      }
      continue;
    }
    for (int64_t b = 0; b < B_; ++b)
      for (int64_t t0 = 0; t0 < rs.ntok; t0 += kTile)
        tiles.push_back({run_id, int32_t(b), int32_t(t0), int32_t(std::min<int64_t>(kTile, rs.ntok - t0))});
  }
  GatherTables t;
  t.aligned = true;  // slabs, components and working-set planes are 256-byte aligned
  t.runs_off = stg_.add(runs.data(), runs.size() * sizeof(GatherRun));
  t.tiles_off = stg_.add(tiles.data(), tiles.size() * sizeof(GatherTile));
  t.n_tiles = int(tiles.size());
  t.qtiles_off = stg_.add(qtiles.data(), qtiles.size() * sizeof(GatherQvgTile));
  t.n_qtiles = int(qtiles.size());
  return t;
}

void Bank::launch_gather_into(const GatherTables& t, size_t outk_off, size_t outv_off, uint64_t out_L,
                              bool vector_ok, const uint32_t* abort_flag, int timing_id, size_t out2k_off,
                              size_t out2v_off, uint64_t out2_L) {
  if (t.n_tiles + t.n_qtiles == 0) return;
  GatherArgs a{};
  a.runs = static_cast<const GatherRun*>(stg_.dev(t.runs_off));
  a.tiles = static_cast<const GatherTile*>(stg_.dev(t.tiles_off));
  a.n_tiles = t.n_tiles;
  a.qtiles = static_cast<const GatherQvgTile*>(stg_.dev(t.qtiles_off));
  a.n_qtiles = t.n_qtiles;
  a.n_layers = n_layers_;
  a.out_k = static_cast<void* const*>(stg_.dev(outk_off));
  a.out_v = static_cast<void* const*>(stg_.dev(outv_off));
  a.out_L = int64_t(out_L);
  if (out2_L > 0) {
    a.out2_k = static_cast<void* const*>(stg_.dev(out2k_off));
    a.out2_v = static_cast<void* const*>(stg_.dev(out2v_off));
    a.out2_L = int64_t(out2_L);
  }
  a.H = int32_t(H_), a.D = int32_t(D_);
  a.out_dtype = dtype_;
  a.cb = cb_dev_;
  a.cb_layer_stride = int64_t(cb_layer_);
  a.stages = q_stages_, a.bits = q_bits_, a.block = q_block_;
  a.abort_flag = abort_flag;
  const bool hd_ok = ((H_ * D_) % 16) == 0;
  tbegin(timing_id);
  NKV_CUDA(launch_gather(a, vector_ok && hd_ok, stream_));
  tend(timing_id);
}

size_t Bank::ws_plane_bytes(uint64_t cap) const { return align_up(size_t(B_) * cap * H_ * D_ * dtype_size(dtype_)); }

unsigned char* Bank::ws_plane(unsigned char* base, uint64_t cap, int layer, int side) const {
  return base + (size_t(2) * layer + side) * ws_plane_bytes(cap);
}

// Working-set storage for `tokens` tokens per layer: *fresh is a new buffer
// (installed by the caller once the commit is known good) or null when the
// current one is big enough.
void Bank::ensure_ws(uint64_t tokens, unsigned char** fresh, uint64_t* fresh_cap) {
  *fresh = nullptr;
  *fresh_cap = 0;
  if (ws_ && tokens <= ws_cap_) return;
  if (tokens == 0) return;
  uint64_t cap = std::max<uint64_t>(tokens, ws_cap_ + ws_cap_ / 4);
  unsigned char* p = nullptr;
  NKV_CUDA(cudaMalloc(&p, size_t(2) * n_layers_ * ws_plane_bytes(cap)));
  *fresh = p;
  *fresh_cap = cap;
}

std::vector<int> Bank::fit_qvg(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v) {
  std::vector<int> fitted_now;
  for (int i = 0; i < n_layers_; ++i)
    if (!fitted_[i]) fitted_now.push_back(i);
  if (fitted_now.empty()) return fitted_now;  // the usual case
  // history.rs:256-262: fit on the whole first segment, every unfitted layer,
  // on the device (kernels_qvg_fit.cu), in chunks of ~4 GB of scratch
  const uint64_t L = s.image_tokens + s.text_tokens;
  const size_t per = qvg_fit_scratch_bytes(L, int(D_), q_E_);
  const size_t cb_head = size_t(q_stages_) * q_E_ * D_;
  std::vector<QvgFitTask> tasks;
  for (int i : fitted_now)
    for (int side = 0; side < 2; ++side)
      for (int64_t h = 0; h < H_; ++h)
        tasks.push_back({side ? v[i] : k[i], cb_dev_ + cb_layer_ * i + (cb_layer_ / 2) * side + cb_head * h,
                         nullptr, nullptr, nullptr, nullptr, cfg_.qvg.codebook_seed + uint64_t(h), int32_t(h)});
  const size_t chunk = std::max<size_t>(1, std::min(tasks.size(), (size_t(4) << 30) / per));
  unsigned char* scratch = nullptr;
  QvgFitTask* d_tasks = nullptr;
  NKV_CUDA(cudaMalloc(&scratch, chunk * per));
  auto release = [&]() {
    cudaStreamSynchronize(stream_);
    cudaFree(scratch);
    if (d_tasks) cudaFree(d_tasks);
  };
  try {
    NKV_CUDA(cudaMalloc(reinterpret_cast<void**>(&d_tasks), chunk * sizeof(QvgFitTask)));
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
    for (size_t c0 = 0; c0 < tasks.size(); c0 += chunk) {
      const size_t m = std::min(chunk, tasks.size() - c0);
      for (size_t j = 0; j < m; ++j) {
        unsigned char* p = scratch + j * per;
        QvgFitTask& t = tasks[c0 + j];
        t.res = reinterpret_cast<float*>(p);
        p += up(L * D_ * 4);
        t.dmin = reinterpret_cast<double*>(p);
        p += up(L * 8);
        t.sums = reinterpret_cast<double*>(p);
        p += up(size_t(q_E_) * D_ * 8);
        t.codes = p;
      }
      NKV_CUDA(cudaMemcpyAsync(d_tasks, tasks.data() + c0, m * sizeof(QvgFitTask), cudaMemcpyHostToDevice, stream_));
      tbegin(NKV_KERNEL_QVG_FIT);
      NKV_CUDA(launch_qvg_fit(d_tasks, int(m), kv_dtype, L, int(H_), int(D_), q_stages_, q_E_, stream_));
      tend(NKV_KERNEL_QVG_FIT);
      NKV_CUDA(cudaStreamSynchronize(stream_));  // the host task array is reused by the next chunk
    }
    for (int i : fitted_now)
      NKV_CUDA(cudaMemcpyAsync(cb_host_.data() + cb_layer_ * i, cb_dev_ + cb_layer_ * i, cb_layer_ * sizeof(float),
                               cudaMemcpyDeviceToHost, stream_));
  } catch (...) {
    release();
    throw;
  }
  release();
  for (int i : fitted_now) fitted_[i] = 1;
  return fitted_now;
}

// commit_segment (history.rs:458-463).
void Bank::no_staged(const char* what) const {
  if (staged_)
    fail(NKV_ERR_CACHE_STATE, std::string(what) + " with a staged segment pending: commit or discard it first");
}

void Bank::commit(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v) {
  if (!k || !v) fail(NKV_ERR_ARGUMENT, "null K/V pointer array");
  for (int i = 0; i < n_layers_; ++i)
    if (!k[i] || !v[i]) fail(NKV_ERR_ARGUMENT, "null K/V pointer for layer " + std::to_string(i));
  no_staged("commit");
  DeviceScope ds(device_);
  validate(s, kv_dtype, k, v);

  // ---- archive_segment: slab + device encode into it
  Rec r = make_rec(s);
  r.slab = arena_.push(r.layer_stride * n_layers_);
  finish_commit(s, r, kv_dtype, k, v, false);
}

void Bank::commit_decode(const nkv_segment_desc& s, int kv_dtype, const void* const* k, const void* const* v,
                         void* const* k_out, void* const* v_out) {
  if (!k || !v) fail(NKV_ERR_ARGUMENT, "null K/V pointer array");
  if (!k_out || !v_out) fail(NKV_ERR_ARGUMENT, "null output pointer array");
  for (int i = 0; i < n_layers_; ++i) {
    if (!k[i] || !v[i]) fail(NKV_ERR_ARGUMENT, "null K/V pointer for layer " + std::to_string(i));
    if (!k_out[i] || !v_out[i]) fail(NKV_ERR_ARGUMENT, "null output pointer for layer " + std::to_string(i));
  }
  no_staged("commit");
  DeviceScope ds(device_);
  validate(s, kv_dtype, k, v);
  Rec r = make_rec(s);
  r.slab = arena_.push(r.layer_stride * n_layers_);
  finish_commit(s, r, kv_dtype, k, v, false, k_out, v_out);
}

// Picks the next set of non-finite flags and clears it: on the auxiliary
// stream after the last gather that read the set, or (a staged commit,
// whose producer writes the flags on the cache's stream) on the cache's
// stream.
void Bank::next_flags(bool clear_on_aux) {
  flag_set_ ^= 1;
  d_flag_ = d_flags_[flag_set_];
  if (clear_on_aux) {
    NKV_CUDA(cudaStreamWaitEvent(aux_, flags_free_[flag_set_], 0));
    NKV_CUDA(cudaMemsetAsync(d_flag_, 0, sizeof(uint32_t) * (n_layers_ + 1), aux_));
  } else {
    NKV_CUDA(cudaMemsetAsync(d_flag_, 0, sizeof(uint32_t) * (n_layers_ + 1), stream_));
  }
}

// validate_segment (history.rs:168-238) and the record's slab; the
// producer then writes the INT8 rows (int8.rs:65-81 layout: codes (B, L, H, D)
// u8, scales (B, L, H) f32) and ORs its non-finite bits into the layer's
// status word, in work ordered before the bank's stream reaches commit_staged.
void Bank::stage(const nkv_segment_desc& s, nkv_staged_layer* out) {
  if (!out) fail(NKV_ERR_ARGUMENT, "null staged-layer array");
  if (cfg_.storage != NKV_STORAGE_INT8) fail(NKV_ERR_INVALID_CONFIG, "staged commits need INT8 storage");
  if (arena_.device_limit() != SIZE_MAX)
    fail(NKV_ERR_INVALID_CONFIG, "staged commits need the whole archive in device memory (no archive device limit)");
  if (staged_) fail(NKV_ERR_CACHE_STATE, "a staged segment is already pending");
  DeviceScope ds(device_);
  validate(s, NKV_BF16, nullptr, nullptr);
  Rec r = make_rec(s);
  r.slab = arena_.push(r.layer_stride * n_layers_);
  try {
    next_flags(false);
  } catch (...) {
    arena_.pop();
    throw;
  }
  for (int i = 0; i < n_layers_; ++i) {
    unsigned char* lb = r.slab + size_t(i) * r.layer_stride;
    out[i].k_codes = lb + r.off[0];
    out[i].v_codes = lb + r.off[1];
    out[i].k_scales = reinterpret_cast<float*>(lb + r.off[2]);
    out[i].v_scales = reinterpret_cast<float*>(lb + r.off[3]);
    out[i].status = d_flag_ + 1 + i;
  }
  staged_rec_ = r;
  staged_ = true;
}

void Bank::commit_staged() {
  if (!staged_) fail(NKV_ERR_CACHE_STATE, "no staged segment");
  DeviceScope ds(device_);
  Rec r = staged_rec_;
  staged_ = false;
  finish_commit(r.desc, r, NKV_BF16, nullptr, nullptr, true);
}

void Bank::discard_staged() {
  if (!staged_) fail(NKV_ERR_CACHE_STATE, "no staged segment");
  DeviceScope ds(device_);
  NKV_CUDA(cudaStreamSynchronize(stream_));  // a producer may still write into the slab
  arena_.pop();
  staged_ = false;
}

void Bank::finish_commit(const nkv_segment_desc& s, Rec r, int kv_dtype, const void* const* k, const void* const* v,
                         bool staged, void* const* dk, void* const* dv) {
  const nkv_metrics saved = m_;
  const uint64_t L = s.image_tokens + s.text_tokens;
  bool pushed = false, popped = false;
  unsigned char* fresh = nullptr;
  uint64_t fresh_cap = 0;
  try {
    std::vector<int> fitted_now;
    if (cfg_.storage == NKV_STORAGE_QVG) fitted_now = fit_qvg(s, kv_dtype, k, v);  // history.rs:256-262

    archive_.push_back(r);
    pushed = true;
    total_frames_ += s.frame_count;
    m_.encode_calls += cfg_.storage == NKV_STORAGE_FLOAT ? 0 : 1;
    m_.archived_segments += 1;
    m_.archived_bytes += r.nbytes;
    m_.d2h_bytes += r.nbytes;

    // ---- rebuild plan on the new archive
    Plan plan;
    bool plan_ok = true;
    Error plan_err{0, ""};
    try {
      plan = plan_rebuild();
    } catch (const Error& e) {
      plan_ok = false;
      plan_err = e;
    }

    stg_.begin(stream_);
    // a plain commit clears its flag set on the auxiliary stream, ahead of
    // the table upload the cache's stream waits for
    if (!staged) next_flags(true);
    bool in_aligned = true;
    if (!staged)
      for (int i = 0; i < n_layers_; ++i) in_aligned &= aligned16(k[i]) && aligned16(v[i]);
    size_t jobs_off = 0, text_jobs_off = 0;
    if (staged) {
      // the producer wrote the codes and the per-layer flags
    } else if (cfg_.storage == NKV_STORAGE_FLOAT) {
      std::vector<ConvertJob> jobs;
      for (int i = 0; i < n_layers_; ++i) {
        unsigned char* lb = r.slab + size_t(i) * r.layer_stride;
        jobs.push_back({k[i], lb + r.off[0]});
        jobs.push_back({v[i], lb + r.off[1]});
      }
      jobs_off = stg_.add(jobs.data(), jobs.size() * sizeof(ConvertJob));
    } else if (cfg_.storage == NKV_STORAGE_INT8) {
      std::vector<QuantJob> jobs;
      for (int i = 0; i < n_layers_; ++i) {
        unsigned char* lb = r.slab + size_t(i) * r.layer_stride;
        jobs.push_back({k[i], v[i], lb + r.off[0], lb + r.off[1], reinterpret_cast<float*>(lb + r.off[2]),
                        reinterpret_cast<float*>(lb + r.off[3]), d_flag_ + 1 + i});
      }
      jobs_off = stg_.add(jobs.data(), jobs.size() * sizeof(QuantJob));
    } else {
      std::vector<QvgEncodeJob> jobs;
      std::vector<QuantJob> tj;
      for (int i = 0; i < n_layers_; ++i) {
        unsigned char* lb = r.slab + size_t(i) * r.layer_stride;
        const float* cb = cb_dev_ + cb_layer_ * i;
        jobs.push_back({k[i], lb + r.off[0], reinterpret_cast<float*>(lb + r.off[2]), cb});
        jobs.push_back({v[i], lb + r.off[1], reinterpret_cast<float*>(lb + r.off[3]), cb + cb_layer_ / 2});
        tj.push_back({k[i], v[i], lb + r.off[4], lb + r.off[5], reinterpret_cast<float*>(lb + r.off[6]),
                      reinterpret_cast<float*>(lb + r.off[7]), d_flag_ + 1 + i});
      }
      jobs_off = stg_.add(jobs.data(), jobs.size() * sizeof(QvgEncodeJob));
      text_jobs_off = stg_.add(tj.data(), tj.size() * sizeof(QuantJob));
    }

    size_t outk_off = 0, outv_off = 0, out2k_off = 0, out2v_off = 0;
    GatherTables gt;
    // the new segment decoded in full into the caller's buffers, in the same
    // launch as the rebuild (decode_segment, history.rs:308-338)
    Plan dplan;
    const bool decode = dk != nullptr && plan_ok;
    bool dec_aligned = true;
    if (decode) {
      dplan = decode_plan(archive_.size() - 1);
      for (int i = 0; i < n_layers_; ++i) dec_aligned &= aligned16(dk[i]) && aligned16(dv[i]);
      out2k_off = stg_.add(dk, n_layers_ * sizeof(void*));
      out2v_off = stg_.add(dv, n_layers_ * sizeof(void*));
    }
    if (plan_ok && (plan.valid > 0 || decode)) {
      unsigned char* base = ws_;
      uint64_t cap = ws_cap_;
      if (plan.valid > 0) {
        ensure_ws(plan.valid, &fresh, &fresh_cap);
        base = fresh ? fresh : ws_;
        cap = fresh ? fresh_cap : ws_cap_;
      }
      gt = add_runs(plan, dec_aligned, decode ? &dplan : nullptr);
      gt.aligned = dec_aligned;
      std::vector<void*> ok(n_layers_, nullptr), ov(n_layers_, nullptr);
      if (plan.valid > 0)
        for (int i = 0; i < n_layers_; ++i) ok[i] = ws_plane(base, cap, i, 0), ov[i] = ws_plane(base, cap, i, 1);
      outk_off = stg_.add(ok.data(), ok.size() * sizeof(void*));
      outv_off = stg_.add(ov.data(), ov.size() * sizeof(void*));
    }
    stg_.upload(aux_, stream_);

    if (staged) NKV_CUDA(launch_flag_reduce(d_flag_, n_layers_, stream_));  // the gather aborts on word 0
    if (staged) {
    } else if (cfg_.storage == NKV_STORAGE_FLOAT) {
      tbegin(NKV_KERNEL_FLOAT_ARCHIVE);
      NKV_CUDA(launch_convert(static_cast<const ConvertJob*>(stg_.dev(jobs_off)), 2 * n_layers_,
                              uint64_t(B_) * L * H_ * D_, kv_dtype, dtype_, stream_));
      tend(NKV_KERNEL_FLOAT_ARCHIVE);
    } else if (cfg_.storage == NKV_STORAGE_INT8) {
      tbegin(NKV_KERNEL_QUANTIZE);
      NKV_CUDA(launch_int8_quantize(static_cast<const QuantJob*>(stg_.dev(jobs_off)), n_layers_,
                                    uint64_t(B_) * L * H_, 0, D_, kv_dtype, in_aligned, d_flag_, stream_));
      tend(NKV_KERNEL_QUANTIZE);
    } else {
      tbegin(NKV_KERNEL_QVG_ENCODE);
      NKV_CUDA(launch_qvg_encode(static_cast<const QvgEncodeJob*>(stg_.dev(jobs_off)), 2 * n_layers_, kv_dtype, L,
                                 int(H_), int(D_), s.image_tokens, q_stages_, q_bits_, q_block_, in_aligned, stream_));
      tend(NKV_KERNEL_QVG_ENCODE);
      if (s.text_tokens > 0) {
        tbegin(NKV_KERNEL_QUANTIZE);
        NKV_CUDA(launch_int8_quantize(static_cast<const QuantJob*>(stg_.dev(text_jobs_off)), n_layers_,
                                      s.text_tokens * H_, s.image_tokens * H_, D_, kv_dtype, in_aligned, d_flag_,
                                      stream_));
        tend(NKV_KERNEL_QUANTIZE);
      }
    }
    // The non-finite flags are final once the archive kernels ran: they are
    // read back on the auxiliary stream while the rebuild gather (which
    // aborts on them by itself) follows the archive kernels directly on the
    // cache's stream, so the host waits only for the kernels that read the
    // caller's K/V and the gather overlaps the caller's next calls.
    NKV_CUDA(cudaEventRecord(encoded_, stream_));
    NKV_CUDA(cudaStreamWaitEvent(aux_, encoded_, 0));
    NKV_CUDA(cudaMemcpyAsync(h_flag_, d_flag_, sizeof(uint32_t) * (n_layers_ + 1), cudaMemcpyDeviceToHost, aux_));
    NKV_CUDA(cudaEventRecord(flag_ev_, aux_));
    if (gt.n_tiles + gt.n_qtiles > 0)
      launch_gather_into(gt, outk_off, outv_off, plan.valid, gt.aligned, d_flag_, NKV_KERNEL_GATHER, out2k_off,
                         out2v_off, decode ? dplan.valid : 0);
    NKV_CUDA(cudaEventRecord(flags_free_[flag_set_], stream_));
    NKV_CUDA(cudaEventSynchronize(flag_ev_));
    collect_timing(false);

    if (h_flag_[0] != 0) {
      // quantize_kv_pair rejected the segment (int8.rs:99-117): nothing was
      // archived and the working set was left untouched by the gather.  The
      // error is the first failing layer's, as in KvBank::commit's loop
      // (cache/mod.rs:264-266); layers after it never reach their first-commit
      // QVG fit there, so their fit from this segment is dropped.
      int first = 0;
      while (first < n_layers_ && h_flag_[1 + first] == 0) ++first;
      const bool k_bad = first < n_layers_ && (h_flag_[1 + first] & 1u) != 0;
      for (int i : fitted_now)
        if (i > first) fitted_[i] = 0;
      archive_.pop_back();
      pushed = false;
      total_frames_ -= s.frame_count;
      m_ = saved;
      arena_.pop();
      popped = true;
      if (fresh) cudaFree(fresh);
      fresh = nullptr;
      if (h_flag_[0] & kProjectTimeoutBit) fail(NKV_ERR_CUDA, "the K/V producer kernel timed out");
      fail(NKV_ERR_MSG, std::string("cannot quantize non-finite ") + (k_bad ? "k" : "v") + " values");
    }
    if (parked_) changed_while_parked_ = true;
    if (!plan_ok) {
      // like the reference, the segment stays archived when rebuild fails
      if (fresh) cudaFree(fresh);
      fresh = nullptr;
      ws_current_ = false;
      throw plan_err;
    }
    if (fresh) {
      if (ws_) cudaFree(ws_);
      ws_ = fresh, ws_cap_ = fresh_cap;
      fresh = nullptr;
    }
    ws_runs_ = plan.runs;
    layout_ = std::move(plan.layout);
    valid_ = plan.valid;
    ws_current_ = true;
    m_.h2d_bytes += valid_ * B_ * H_ * D_ * dtype_size(dtype_) * 2;  // history.rs:438-439
    m_.rebuilds += 1;
  } catch (const Error& e) {
    if (fresh) cudaFree(fresh);
    if (pushed && (e.code == NKV_ERR_CUDA || e.code == NKV_ERR_ARGUMENT)) {
      archive_.pop_back();
      total_frames_ -= s.frame_count;
      m_ = saved;
      arena_.pop();
    } else if (!pushed && !popped) {
      arena_.pop();
    }
    throw;
  }
}

// rebuild() for rollback: plan, gather into the working set, counters.
void Bank::rebuild_now() {
  Plan plan = plan_rebuild();
  unsigned char* fresh = nullptr;
  uint64_t fresh_cap = 0;
  if (plan.valid > 0) {
    ensure_ws(plan.valid, &fresh, &fresh_cap);
    stg_.begin(stream_);
    const GatherTables gt = add_runs(plan);
    unsigned char* base = fresh ? fresh : ws_;
    const uint64_t cap = fresh ? fresh_cap : ws_cap_;
    std::vector<void*> ok(n_layers_), ov(n_layers_);
    for (int i = 0; i < n_layers_; ++i) ok[i] = ws_plane(base, cap, i, 0), ov[i] = ws_plane(base, cap, i, 1);
    const size_t outk_off = stg_.add(ok.data(), ok.size() * sizeof(void*));
    const size_t outv_off = stg_.add(ov.data(), ov.size() * sizeof(void*));
    stg_.upload(aux_, stream_);
    try {
      launch_gather_into(gt, outk_off, outv_off, plan.valid, gt.aligned, nullptr);
    } catch (...) {
      if (fresh) cudaFree(fresh);
      throw;
    }
    if (fresh) {
      if (ws_) {
        NKV_CUDA(cudaStreamSynchronize(stream_));
        cudaFree(ws_);
      }
      ws_ = fresh, ws_cap_ = fresh_cap;
    }
  }
  ws_runs_ = plan.runs;
  layout_ = std::move(plan.layout);
  valid_ = plan.valid;
  ws_current_ = true;
  m_.h2d_bytes += valid_ * B_ * H_ * D_ * dtype_size(dtype_) * 2;
  m_.rebuilds += 1;
}

// rollback_last_segment (history.rs:507-528).
void Bank::rollback() {
  no_staged("rollback");  // the staged slab sits above the archive's
  if (cfg_.sampling == NKV_SAMPLING_RECENT)
    fail(NKV_ERR_CACHE_STATE, "recent-mode SWA does not support streaming rollback (use an archived sampling)");
  if (archive_.empty()) fail(NKV_ERR_CACHE_STATE, "nothing to roll back");
  DeviceScope ds(device_);
  const Rec last = archive_.back();
  archive_.pop_back();
  arena_.pop();  // stream order keeps earlier readers of the slab ahead of its reuse
  if (last.desc.frame_start + last.desc.frame_count != total_frames_)
    fail(NKV_ERR_CACHE_STATE, "archive does not match the frame timeline");
  total_frames_ -= last.desc.frame_count;
  m_.archived_segments = m_.archived_segments > 0 ? m_.archived_segments - 1 : 0;
  if (parked_) changed_while_parked_ = true;
  ws_current_ = false;  // until the rebuild below succeeds
  rebuild_now();
  m_.rollbacks += 1;
}

// PhaseSwappedCache::park (phase_swap.rs:42-66): the working set goes to
// pinned host memory and its device memory is released.
void Bank::park() {
  if (!cfg_.phase_swap || parked_) return;
  DeviceScope ds(device_);
  p_ws_current_ = ws_current_;
  changed_while_parked_ = false;
  const size_t plane = size_t(B_) * valid_ * H_ * D_ * dtype_size(dtype_);
  cudaEvent_t ready;
  NKV_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
  NKV_CUDA(cudaEventRecord(ready, stream_));
  NKV_CUDA(cudaStreamWaitEvent(side_, ready, 0));
  cudaEventDestroy(ready);
  for (int i = 0; i < n_layers_; ++i) {
    if (p_host_cap_[i] < 2 * plane) {
      if (p_host_[i]) cudaFreeHost(p_host_[i]);
      p_host_[i] = nullptr;
      p_host_cap_[i] = 0;
      NKV_CUDA(cudaHostAlloc(&p_host_[i], std::max<size_t>(2 * plane, 1), cudaHostAllocDefault));
      p_host_cap_[i] = std::max<size_t>(2 * plane, 1);
    }
    if (plane) {
      NKV_CUDA(cudaMemcpyAsync(p_host_[i], ws_plane(ws_, ws_cap_, i, 0), plane, cudaMemcpyDeviceToHost, side_));
      NKV_CUDA(cudaMemcpyAsync(p_host_[i] + plane, ws_plane(ws_, ws_cap_, i, 1), plane, cudaMemcpyDeviceToHost, side_));
    }
  }
  NKV_CUDA(cudaStreamSynchronize(side_));
  if (ws_) cudaFree(ws_);
  ws_ = nullptr, ws_cap_ = 0;
  p_layout_ = layout_;
  p_runs_ = ws_runs_;
  p_valid_ = valid_;
  p_bytes_ = 2 * plane;
  layout_.clear();  // release_working_set (history.rs:539-544)
  valid_ = 0;
  m_.d2h_bytes += p_bytes_;
  parked_ = true;
}

// PhaseSwappedCache::unpark (phase_swap.rs:69-81).  Like the reference, a
// working set rebuilt while parked is replaced by the parked one.
void Bank::unpark() {
  if (!cfg_.phase_swap || !parked_) return;
  DeviceScope ds(device_);
  const size_t plane = size_t(B_) * p_valid_ * H_ * D_ * dtype_size(dtype_);
  if (p_valid_ > 0) {
    unsigned char* fresh = nullptr;
    uint64_t fresh_cap = 0;
    ensure_ws(p_valid_, &fresh, &fresh_cap);
    if (fresh) {
      if (ws_) {
        NKV_CUDA(cudaStreamSynchronize(stream_));
        cudaFree(ws_);
      }
      ws_ = fresh, ws_cap_ = fresh_cap;
    }
    // order after any work still using the old contents of the buffer
    cudaEvent_t ready, done;
    NKV_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    NKV_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
    NKV_CUDA(cudaEventRecord(ready, stream_));
    NKV_CUDA(cudaStreamWaitEvent(side_, ready, 0));
    for (int i = 0; i < n_layers_; ++i) {
      NKV_CUDA(cudaMemcpyAsync(ws_plane(ws_, ws_cap_, i, 0), p_host_[i], plane, cudaMemcpyHostToDevice, side_));
      NKV_CUDA(cudaMemcpyAsync(ws_plane(ws_, ws_cap_, i, 1), p_host_[i] + plane, plane, cudaMemcpyHostToDevice, side_));
    }
    NKV_CUDA(cudaEventRecord(done, side_));
    NKV_CUDA(cudaStreamWaitEvent(stream_, done, 0));
    NKV_CUDA(cudaStreamSynchronize(side_));
    cudaEventDestroy(ready);
    cudaEventDestroy(done);
  }
  layout_ = p_layout_;
  ws_runs_ = p_runs_;
  valid_ = p_valid_;
  ws_current_ = p_ws_current_ && !changed_while_parked_;
  m_.h2d_bytes += p_bytes_;
  parked_ = false;
}

// Runs of a whole archived segment in its own order (decode_segment,
// history.rs:308-338): QVG video then the INT8 text block, else one run.
Plan Bank::decode_plan(size_t pos) const {
  const Rec& r = archive_[pos];
  Plan p;
  const int64_t Lv = int64_t(r.desc.image_tokens), Lt = int64_t(r.desc.text_tokens);
  if (cfg_.storage == NKV_STORAGE_QVG) {
    p.runs.push_back({pos, false, 0, 0, Lv});
    if (Lt > 0) p.runs.push_back({pos, true, Lv, Lv, Lt});
  } else {
    p.runs.push_back({pos, false, 0, 0, Lv + Lt});
  }
  p.valid = uint64_t(Lv + Lt);
  return p;
}

// decode_segment (history.rs:308-338) of every local layer into caller buffers.
void Bank::decode_segment(uint64_t pos, void* const* k_out, void* const* v_out) {
  if (pos >= archive_.size()) fail(NKV_ERR_ARGUMENT, "archive position out of range");
  if (!k_out || !v_out) fail(NKV_ERR_ARGUMENT, "null output pointer array");
  for (int i = 0; i < n_layers_; ++i)
    if (!k_out[i] || !v_out[i]) fail(NKV_ERR_ARGUMENT, "null output pointer for layer " + std::to_string(i));
  DeviceScope ds(device_);
  const Plan p = decode_plan(pos);
  stg_.begin(stream_);
  bool aligned = true;
  for (int i = 0; i < n_layers_; ++i) aligned &= aligned16(k_out[i]) && aligned16(v_out[i]);
  const GatherTables gt = add_runs(p, aligned);
  aligned &= gt.aligned;
  const size_t outk_off = stg_.add(k_out, n_layers_ * sizeof(void*));
  const size_t outv_off = stg_.add(v_out, n_layers_ * sizeof(void*));
  stg_.upload(aux_, stream_);
  launch_gather_into(gt, outk_off, outv_off, p.valid, aligned, nullptr, NKV_KERNEL_SEGMENT_DECODE);
}

// Attention of q over this layer's history, straight from the INT8 archive
// (kernels_attn.cu): key tiles of <= 128 tokens along the runs of the current
// working set, so the keys are the working set's, in its order.
void Bank::attend_history(int layer, const void* q, uint64_t q_len, float scale, float* out, float* lse) {
  if (layer < 0 || layer >= n_layers_) fail(NKV_ERR_ARGUMENT, "layer out of range");
  if (!q || !out || !lse) fail(NKV_ERR_ARGUMENT, "null q / out / lse pointer");
  if (!(scale > 0.0f) || !std::isfinite(scale)) fail(NKV_ERR_ARGUMENT, "scale must be finite and positive");
  if (cfg_.storage != NKV_STORAGE_INT8) fail(NKV_ERR_INVALID_CONFIG, "history attention reads INT8 archives");
  if (D_ != 128 || B_ != 1 || dtype_ != NKV_BF16)
    fail(NKV_ERR_GEOMETRY, "history attention needs head_dim 128, batch 1 and a bf16 model");
  if (parked_) fail(NKV_ERR_CACHE_STATE, "working set is parked; call unpark() before attention");
  if (!ws_current_) fail(NKV_ERR_CACHE_STATE, "the working set is not the rebuild of the archive");
  if (valid_ == 0) fail(NKV_ERR_CACHE_STATE, "no history to attend to");
  if (q_len == 0) return;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15u)
    fail(NKV_ERR_ARGUMENT, "q and out must be 16-byte aligned");
  DeviceScope ds(device_);
  // Codes come by TMA through one tensor map per (record, side) of this
  // layer when every record of the working set is in device memory; a
  // working set that reaches the pinned host tier is read with plain loads.
  bool tma = true;
  std::vector<size_t> recs;                // distinct records, in run order
  std::vector<int> map_of(archive_.size(), -1);
  for (const auto& rs : ws_runs_) {
    if (map_of[rs.rec] >= 0) continue;
    map_of[rs.rec] = int(recs.size());
    recs.push_back(rs.rec);
    if (arena_.is_host(archive_[rs.rec].slab)) tma = false;
  }
  std::vector<TmaDesc> maps;
  if (tma) {
    maps.resize(2 * recs.size());
    for (size_t i = 0; i < recs.size() && tma; ++i) {
      const Rec& r = archive_[recs[i]];
      const unsigned char* lb = r.slab + size_t(layer) * r.layer_stride;
      const uint64_t L = r.desc.image_tokens + r.desc.text_tokens;
      tma = make_codes_map(&maps[2 * i], lb + r.off[0], L, int(H_)) &&
            make_codes_map(&maps[2 * i + 1], lb + r.off[1], L, int(H_));
    }
  }
  if (!d_attn_status_) NKV_CUDA(cudaMalloc(&d_attn_status_, sizeof(uint32_t)));
  stg_.begin(stream_);
  const size_t moff = tma ? stg_.add(maps.data(), maps.size() * sizeof(TmaDesc), 64) : 0;
  std::vector<AttnKeyTile> tiles;
  for (const auto& rs : ws_runs_) {
    const Rec& r = archive_[rs.rec];
    const unsigned char* lb = r.slab + size_t(layer) * r.layer_stride;
    for (int64_t t0 = 0; t0 < rs.ntok; t0 += 128) {
      const int64_t tok = rs.src_tok + t0;
      AttnKeyTile t{};
      t.k_codes = lb + r.off[0] + tok * H_ * D_;
      t.v_codes = lb + r.off[1] + tok * H_ * D_;
      t.k_scales = reinterpret_cast<const float*>(lb + r.off[2]) + tok * H_;
      t.v_scales = reinterpret_cast<const float*>(lb + r.off[3]) + tok * H_;
      t.map = map_of[rs.rec];
      t.tok0 = int32_t(tok);
      t.ntok = int32_t(std::min<int64_t>(128, rs.ntok - t0));
      tiles.push_back(t);
    }
  }
  const size_t toff = stg_.add(tiles.data(), tiles.size() * sizeof(AttnKeyTile));
  stg_.upload(aux_, stream_);
  NKV_CUDA(cudaMemsetAsync(d_attn_status_, 0, sizeof(uint32_t), stream_));
  AttnArgs a{};
  a.tiles = static_cast<const AttnKeyTile*>(stg_.dev(toff));
  a.n_tiles = int32_t(tiles.size());
  a.H = int32_t(H_);
  a.q = static_cast<const uint16_t*>(q);
  a.Lq = int64_t(q_len);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out;
  a.lse = lse;
  a.status = d_attn_status_;
  if (!sms_) NKV_CUDA(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, device_));
  const int64_t part_rows = attend_plan(int64_t(q_len), int(H_), int(tiles.size()), sms_, &a);
  if (part_rows > attn_part_rows_) {
    if (d_attn_part_) NKV_CUDA(cudaFree(d_attn_part_));
    d_attn_part_ = nullptr;
    attn_part_rows_ = 0;
    NKV_CUDA(cudaMalloc(&d_attn_part_, size_t(part_rows) * (128 + 2) * sizeof(float)));
    attn_part_rows_ = part_rows;
  }
  a.part_o = d_attn_part_;
  a.part_ml = d_attn_part_ ? d_attn_part_ + size_t(attn_part_rows_) * 128 : nullptr;
  a.maps = tma ? static_cast<const TmaDesc*>(stg_.dev(moff)) : nullptr;
  tbegin(NKV_KERNEL_ATTEND);
  NKV_CUDA(launch_attend_int8(a, stream_));
  tend(NKV_KERNEL_ATTEND);
  uint32_t st = 0;
  NKV_CUDA(cudaMemcpyAsync(&st, d_attn_status_, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_));
  NKV_CUDA(cudaStreamSynchronize(stream_));
  collect_timing(false);
  if (st) fail(NKV_ERR_CUDA, "history attention: a bounded wait ran out");
}

void Bank::synchronize() {
  DeviceScope ds(device_);
  NKV_CUDA(cudaStreamSynchronize(stream_));
  collect_timing(false);
}

void Bank::set_archive_device_limit(uint64_t bytes) {
  if (staged_) fail(NKV_ERR_CACHE_STATE, "a staged segment is pending");
  arena_.set_device_limit(bytes == 0 ? SIZE_MAX : size_t(bytes));
}

void Bank::archive_usage(uint64_t* device, uint64_t* host) const {
  size_t d = 0, h = 0;
  arena_.usage(&d, &h);
  *device = d, *host = h;
}

void Bank::reserve(uint64_t archive_bytes, uint64_t working_tokens) {
  DeviceScope ds(device_);
  if (archive_bytes) arena_.reserve(archive_bytes);
  if (working_tokens && !parked_) {
    unsigned char* fresh = nullptr;
    uint64_t cap = 0;
    ensure_ws(working_tokens, &fresh, &cap);
    if (fresh) {
      // keep the current contents: the working set may be in use
      if (ws_ && valid_ > 0) {
        for (int i = 0; i < n_layers_; ++i)
          for (int side = 0; side < 2; ++side)
            NKV_CUDA(cudaMemcpyAsync(ws_plane(fresh, cap, i, side), ws_plane(ws_, ws_cap_, i, side),
                                     size_t(B_) * valid_ * H_ * D_ * dtype_size(dtype_), cudaMemcpyDeviceToDevice,
                                     stream_));
      }
      NKV_CUDA(cudaStreamSynchronize(stream_));
      if (ws_) cudaFree(ws_);
      ws_ = fresh, ws_cap_ = cap;
    }
  }
}

void Bank::working_set(int layer, const void** k, const void** v, uint64_t* valid) const {
  if (layer < 0 || layer >= n_layers_) fail(NKV_ERR_ARGUMENT, "layer out of range");
  if (parked_) fail(NKV_ERR_CACHE_STATE, "working set is parked; call unpark() before attention");
  if (valid_ == 0 || !ws_) {
    *k = *v = nullptr;
    *valid = 0;
    return;
  }
  *k = ws_plane(ws_, ws_cap_, layer, 0);
  *v = ws_plane(ws_, ws_cap_, layer, 1);
  *valid = valid_;
}

void Bank::info(int layer, nkv_cache_info_t* o) const {
  if (layer < 0 || layer >= n_layers_) fail(NKV_ERR_ARGUMENT, "layer out of range");
  o->valid_len = parked_ ? p_valid_ : valid_;
  o->capacity = capacity_or_max();
  o->n_segments = archive_.size();
  o->total_frames = total_frames_;
  o->tokens_per_frame = tpf_;
  o->parked = parked_ ? 1 : 0;
  o->storage = cfg_.storage;
  o->sampling = cfg_.sampling;
  o->qvg_fitted = cfg_.storage == NKV_STORAGE_QVG ? fitted_[layer] : 0;
}

// KvBank::metrics (cache/mod.rs:305-319).  Every layer holds the same
// counters, so max-aggregates equal one layer's and sums are n_layers times.
nkv_metrics Bank::bank_metrics() const {
  nkv_metrics o = m_;
  const uint64_t n = uint64_t(n_layers_);
  o.archived_bytes *= n;
  o.encode_calls *= n;
  o.d2h_bytes *= n;
  o.h2d_bytes *= n;
  return o;
}

void Bank::set_codebooks(int layer, const float* host) {
  if (cfg_.storage != NKV_STORAGE_QVG) fail(NKV_ERR_CACHE_STATE, "cache does not use QVG storage");
  if (layer < 0 || layer >= n_layers_) fail(NKV_ERR_ARGUMENT, "layer out of range");
  if (!host) fail(NKV_ERR_ARGUMENT, "null codebook pointer");
  DeviceScope ds(device_);
  float* dst = cb_host_.data() + cb_layer_ * layer;
  std::memcpy(dst, host, cb_layer_ * sizeof(float));
  NKV_CUDA(cudaMemcpyAsync(cb_dev_ + cb_layer_ * layer, dst, cb_layer_ * sizeof(float), cudaMemcpyHostToDevice,
                           stream_));
  NKV_CUDA(cudaStreamSynchronize(stream_));
  fitted_[layer] = 1;
}

void Bank::get_codebooks(int layer, float* host, int32_t* fitted) const {
  if (cfg_.storage != NKV_STORAGE_QVG) fail(NKV_ERR_CACHE_STATE, "cache does not use QVG storage");
  if (layer < 0 || layer >= n_layers_) fail(NKV_ERR_ARGUMENT, "layer out of range");
  *fitted = fitted_[layer];
  if (fitted_[layer] && host) std::memcpy(host, cb_host_.data() + cb_layer_ * layer, cb_layer_ * sizeof(float));
}

uint64_t Bank::export_segment(int layer, uint64_t pos, void* host, uint64_t cap) {
  if (layer < 0 || layer >= n_layers_) fail(NKV_ERR_ARGUMENT, "layer out of range");
  if (pos >= archive_.size()) fail(NKV_ERR_ARGUMENT, "archive position out of range");
  const Rec& r = archive_[pos];
  const size_t L = r.desc.image_tokens + r.desc.text_tokens, HD = size_t(H_) * D_, B = size_t(B_);
  std::vector<std::pair<size_t, size_t>> parts;  // (offset, bytes)
  if (cfg_.storage == NKV_STORAGE_FLOAT) {
    const size_t n = B * L * HD * dtype_size(dtype_);
    parts = {{r.off[0], n}, {r.off[1], n}};
  } else if (cfg_.storage == NKV_STORAGE_INT8) {
    parts = {{r.off[0], B * L * HD}, {r.off[1], B * L * HD}, {r.off[2], B * L * H_ * 4}, {r.off[3], B * L * H_ * 4}};
  } else {
    const size_t Lv = r.desc.image_tokens, Lt = r.desc.text_tokens;
    const size_t cb = Lv * H_ * q_bpt_, sb = size_t(H_) * r.n_blocks * q_stages_ * 4;
    parts = {{r.off[0], cb}, {r.off[1], cb}, {r.off[2], sb}, {r.off[3], sb}};
    if (Lt > 0) {
      parts.push_back({r.off[4], Lt * HD});
      parts.push_back({r.off[5], Lt * HD});
      parts.push_back({r.off[6], Lt * H_ * 4});
      parts.push_back({r.off[7], Lt * H_ * 4});
    }
  }
  uint64_t total = 0;
  for (auto& p : parts) total += p.second;
  if (!host || cap < total) return total;
  DeviceScope ds(device_);
  NKV_CUDA(cudaStreamSynchronize(stream_));
  unsigned char* out = static_cast<unsigned char*>(host);
  const unsigned char* lb = r.slab + size_t(layer) * r.layer_stride;
  for (auto& p : parts) {
    NKV_CUDA(cudaMemcpy(out, lb + p.first, p.second, cudaMemcpyDefault));  // the slab may be in either tier
    out += p.second;
  }
  return total;
}

// ------------------------------------------------------------------ timing --
void Bank::set_timing(bool on) { timing_ = on; }

void Bank::tbegin(int) {
  if (!timing_) return;
  if (ev_pool_.empty()) {
    cudaEvent_t e;
    NKV_CUDA(cudaEventCreate(&e));
    ev_pool_.push_back(e);
  }
  cur_a_ = ev_pool_.back();
  ev_pool_.pop_back();
  NKV_CUDA(cudaEventRecord(cur_a_, stream_));
}

void Bank::tend(int kind) {
  if (!timing_ || !cur_a_) return;
  cudaEvent_t b;
  if (ev_pool_.empty()) {
    NKV_CUDA(cudaEventCreate(&b));
  } else {
    b = ev_pool_.back();
    ev_pool_.pop_back();
  }
  NKV_CUDA(cudaEventRecord(b, stream_));
  pending_.push_back({kind, cur_a_, b});
  cur_a_ = nullptr;
}

void Bank::collect_timing(bool wait) {
  std::vector<Pending> keep;
  for (auto& p : pending_) {
    if (!wait && cudaEventQuery(p.b) != cudaSuccess) {
      keep.push_back(p);
      continue;
    }
    cudaEventSynchronize(p.b);
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
      stats_[p.kind].launches += 1;
      stats_[p.kind].total_ms += ms;
    }
    ev_pool_.push_back(p.a);
    ev_pool_.push_back(p.b);
  }
  pending_.swap(keep);
}

void Bank::kernel_stats(nkv_kernel_stat* out, bool reset) {
  DeviceScope ds(device_);
  collect_timing(true);
  for (int i = 0; i < NKV_KERNEL_COUNT; ++i) out[i] = stats_[i];
  if (reset)
    for (auto& s : stats_) s = nkv_kernel_stat{0, 0.0};
}

// ---------------------------------------------------------------------------
// Archive persistence.  File layout (host byte order):
//   "NKVBANK1"  u32 version (1)
//   config: storage, qvg{stages, bits, block, text_as_int8, seed}, sampling,
//           gamma (f64 bits), has_capacity, capacity, past_frames, phase_swap
//   geometry: n_layers, layer_begin, batch, heads, head_dim, dtype
//   u64 total_frames, u64 tokens_per_frame, the 8 counters
//   u64 n_segments; per segment: the 6 descriptor fields, u64 bytes, the
//       segment's device slab (every local layer's payload, as laid out here)
//   QVG only: n_layers fitted flags (u8), then the codebooks (f32)
//   "NKVEND01"
// ---------------------------------------------------------------------------
namespace {

constexpr char kMagic[8] = {'N', 'K', 'V', 'B', 'A', 'N', 'K', '1'};
constexpr char kEnd[8] = {'N', 'K', 'V', 'E', 'N', 'D', '0', '1'};
constexpr size_t kIoChunk = size_t(64) << 20;

struct File {
  FILE* f = nullptr;
  std::string path;
  ~File() {
    if (f) fclose(f);
  }
  void put(const void* p, size_t n) {
    if (n && fwrite(p, 1, n, f) != n) fail(NKV_ERR_MSG, "write to " + path + " failed");
  }
  void get(void* p, size_t n) {
    if (n && fread(p, 1, n, f) != n) fail(NKV_ERR_MSG, path + " is truncated or unreadable");
  }
  template <class T>
  void put_v(T v) { put(&v, sizeof(T)); }
  template <class T>
  T get_v() {
    T v;
    get(&v, sizeof(T));
    return v;
  }
};

void put_config(File& f, const nkv_cache_config& c) {
  f.put_v<int32_t>(c.storage);
  f.put_v<int32_t>(c.qvg.stages), f.put_v<int32_t>(c.qvg.bits_per_stage), f.put_v<int32_t>(c.qvg.block_size);
  f.put_v<int32_t>(c.qvg.text_as_int8), f.put_v<uint64_t>(c.qvg.codebook_seed);
  f.put_v<int32_t>(c.sampling), f.put_v<double>(c.gamma);
  f.put_v<int32_t>(c.has_capacity), f.put_v<uint64_t>(c.capacity), f.put_v<uint64_t>(c.past_frames);
  f.put_v<int32_t>(c.phase_swap);
}

bool same_config(File& f, const nkv_cache_config& c) {
  bool same = f.get_v<int32_t>() == c.storage;
  same &= f.get_v<int32_t>() == c.qvg.stages;
  same &= f.get_v<int32_t>() == c.qvg.bits_per_stage;
  same &= f.get_v<int32_t>() == c.qvg.block_size;
  same &= f.get_v<int32_t>() == c.qvg.text_as_int8;
  same &= f.get_v<uint64_t>() == c.qvg.codebook_seed;
  same &= f.get_v<int32_t>() == c.sampling;
  const double g = f.get_v<double>();
  same &= std::memcmp(&g, &c.gamma, sizeof(double)) == 0;
  same &= f.get_v<int32_t>() == c.has_capacity;
  same &= f.get_v<uint64_t>() == c.capacity;
  same &= f.get_v<uint64_t>() == c.past_frames;
  same &= f.get_v<int32_t>() == c.phase_swap;
  return same;
}

}  // namespace

void Bank::save(const char* path) {
  if (!path) fail(NKV_ERR_ARGUMENT, "null path");
  no_staged("save");
  if (parked_) fail(NKV_ERR_CACHE_STATE, "cannot save a parked cache; unpark it first");
  if (!ws_current_)
    fail(NKV_ERR_CACHE_STATE,
         "cannot save: the working set is not the rebuild of the archive (a rebuild failed, or a commit or "
         "rollback happened while parked)");
  DeviceScope ds(device_);
  NKV_CUDA(cudaStreamSynchronize(stream_));
  File f;
  f.path = path;
  f.f = std::fopen(path, "wb");
  if (!f.f) fail(NKV_ERR_MSG, std::string("cannot open ") + path + " for writing");
  f.put(kMagic, sizeof(kMagic));
  f.put_v<uint32_t>(1);
  put_config(f, cfg_);
  f.put_v<int32_t>(n_layers_), f.put_v<int32_t>(layer_begin_);
  f.put_v<int64_t>(B_), f.put_v<int64_t>(H_), f.put_v<int64_t>(D_), f.put_v<int32_t>(dtype_);
  f.put_v<uint64_t>(total_frames_), f.put_v<uint64_t>(tpf_);
  f.put(&m_, sizeof(m_));
  f.put_v<uint64_t>(archive_.size());
  std::vector<unsigned char> buf;
  for (const Rec& r : archive_) {
    f.put(&r.desc, sizeof(r.desc));
    const uint64_t bytes = uint64_t(r.layer_stride) * n_layers_;
    f.put_v<uint64_t>(bytes);
    for (uint64_t o = 0; o < bytes; o += kIoChunk) {
      const size_t n = size_t(std::min<uint64_t>(kIoChunk, bytes - o));
      buf.resize(n);
      NKV_CUDA(cudaMemcpy(buf.data(), r.slab + o, n, cudaMemcpyDefault));  // either tier
      f.put(buf.data(), n);
    }
  }
  if (cfg_.storage == NKV_STORAGE_QVG) {
    f.put(fitted_.data(), fitted_.size());
    f.put(cb_host_.data(), cb_host_.size() * sizeof(float));
  }
  f.put(kEnd, sizeof(kEnd));
  if (std::fflush(f.f) != 0) fail(NKV_ERR_MSG, std::string("write to ") + path + " failed");
}

void Bank::load(const char* path) {
  if (!path) fail(NKV_ERR_ARGUMENT, "null path");
  no_staged("load");
  if (!archive_.empty() || total_frames_ != 0 || parked_)
    fail(NKV_ERR_CACHE_STATE, "load needs a fresh cache (nothing committed yet)");
  DeviceScope ds(device_);
  File f;
  f.path = path;
  f.f = std::fopen(path, "rb");
  if (!f.f) fail(NKV_ERR_MSG, std::string("cannot open ") + path);
  char magic[8];
  f.get(magic, sizeof(magic));
  if (std::memcmp(magic, kMagic, sizeof(magic)) != 0 || f.get_v<uint32_t>() != 1)
    fail(NKV_ERR_MSG, std::string(path) + " is not a saved cache archive");
  bool same = same_config(f, cfg_);
  same &= f.get_v<int32_t>() == n_layers_;
  same &= f.get_v<int32_t>() == layer_begin_;
  same &= f.get_v<int64_t>() == B_;
  same &= f.get_v<int64_t>() == H_;
  same &= f.get_v<int64_t>() == D_;
  same &= f.get_v<int32_t>() == dtype_;
  if (!same)
    fail(NKV_ERR_INVALID_CONFIG, std::string(path) + " was saved by a cache with a different configuration or geometry");
  const uint64_t total_frames = f.get_v<uint64_t>(), tpf = f.get_v<uint64_t>();
  nkv_metrics m;
  f.get(&m, sizeof(m));
  const uint64_t n = f.get_v<uint64_t>();
  std::vector<Rec> recs;
  std::vector<unsigned char> buf;
  try {
    uint64_t frames = 0;
    for (uint64_t i = 0; i < n; ++i) {
      nkv_segment_desc d;
      f.get(&d, sizeof(d));
      if (d.frame_start != frames || d.frame_count == 0 || d.image_tokens == 0 ||
          (tpf && d.image_tokens != d.frame_count * tpf) || (i > 0 && d.segment_index <= recs.back().desc.segment_index))
        fail(NKV_ERR_MSG, std::string(path) + ": segment " + std::to_string(i) + " breaks the frame timeline");
      frames += d.frame_count;
      Rec r = make_rec(d);
      const uint64_t bytes = f.get_v<uint64_t>();
      if (bytes != uint64_t(r.layer_stride) * n_layers_)
        fail(NKV_ERR_MSG, std::string(path) + ": segment " + std::to_string(i) + " has the wrong payload size");
      r.slab = arena_.push(size_t(bytes));
      recs.push_back(r);
      for (uint64_t o = 0; o < bytes; o += kIoChunk) {
        const size_t c = size_t(std::min<uint64_t>(kIoChunk, bytes - o));
        buf.resize(c);
        f.get(buf.data(), c);
        NKV_CUDA(cudaMemcpy(r.slab + o, buf.data(), c, cudaMemcpyDefault));  // either tier
      }
    }
    if (frames != total_frames) fail(NKV_ERR_MSG, std::string(path) + ": the segments do not cover the timeline");
    std::vector<char> fitted(fitted_.size());
    std::vector<float> cb(cb_host_.size());
    if (cfg_.storage == NKV_STORAGE_QVG) {
      f.get(fitted.data(), fitted.size());
      f.get(cb.data(), cb.size() * sizeof(float));
    }
    char end[8];
    f.get(end, sizeof(end));
    if (std::memcmp(end, kEnd, sizeof(end)) != 0) fail(NKV_ERR_MSG, std::string(path) + " is corrupt (no end marker)");
    // install
    if (cfg_.storage == NKV_STORAGE_QVG) {
      fitted_ = fitted;
      cb_host_ = cb;
      NKV_CUDA(cudaMemcpy(cb_dev_, cb_host_.data(), cb_host_.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    archive_ = recs;
    total_frames_ = total_frames;
    tpf_ = tpf;
    if (!archive_.empty()) rebuild_now();
    m_ = m;  // the counters as saved (the rebuild above is not a reference rebuild)
    ws_current_ = true;
  } catch (...) {
    // back to a fresh cache
    archive_.clear();
    for (size_t i = 0; i < recs.size(); ++i) arena_.pop();
    total_frames_ = 0, tpf_ = 0;
    m_ = nkv_metrics{};
    layout_.clear();
    valid_ = 0;
    if (cfg_.storage == NKV_STORAGE_QVG) {
      std::fill(fitted_.begin(), fitted_.end(), 0);
      std::fill(cb_host_.begin(), cb_host_.end(), 0.0f);
    }
    throw;
  }
}

}  // namespace nkv
