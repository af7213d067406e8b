// abi.cpp — the extern "C" boundary declared in include/nomas_kv.h.  Each
// entry point validates its arguments, forwards to the Bank / kernels, and
// turns exceptions into an nkv_status plus a thread-local message.
#include <cuda_runtime.h>

#include <cstring>
#include <functional>
#include <string>

#include "bank.h"
#include "nkv_kernels.h"
#include "nkv_policy.h"
#include "nomas_kv.h"

using nkv::Bank;
using nkv::Error;

struct nkv_bank {
  Bank* impl;
};

namespace {
thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return NKV_OK;
  } catch (const Error& e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const nkv::PolicyError& e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return NKV_ERR_CUDA;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return NKV_ERR_MSG;
  }
}

Bank& bank_of(const nkv_bank* b) {
  if (!b || !b->impl) nkv::fail(NKV_ERR_ARGUMENT, "null bank");
  return *b->impl;
}

void need(const void* p, const char* what) {
  if (!p) nkv::fail(NKV_ERR_ARGUMENT, std::string("null ") + what);
}

void check_dtype(int32_t dt) {
  if (dt < NKV_F32 || dt > NKV_F16) nkv::fail(NKV_ERR_ARGUMENT, "unknown dtype " + std::to_string(dt));
}
}  // namespace

namespace nkv {
// Lets entry points outside this file report through nkv_last_error().
void set_abi_error(const std::string& msg) { g_last_error = msg; }
// The exception-to-status guard for entry points outside this file.
int guarded_call(const std::function<void()>& f) { return guarded(f); }
}  // namespace nkv

extern "C" {

const char* nkv_last_error(void) { return g_last_error.c_str(); }

int32_t nkv_abi_version(void) { return NKV_ABI_VERSION; }

int nkv_bank_create(const nkv_cache_config* cfg, int32_t n_layers, int32_t layer_begin, int64_t batch,
                    int64_t heads, int64_t head_dim, int32_t dtype, int32_t device, void* stream, nkv_bank** out) {
  return guarded([&] {
    need(cfg, "config");
    need(out, "output handle");
    *out = nullptr;
    Bank* b = new Bank(*cfg, n_layers, layer_begin, batch, heads, head_dim, dtype, device,
                       static_cast<cudaStream_t>(stream));
    *out = new nkv_bank{b};
  });
}

int nkv_bank_destroy(nkv_bank* bank) {
  return guarded([&] {
    if (!bank) return;
    delete bank->impl;
    bank->impl = nullptr;
    delete bank;
  });
}

int nkv_bank_commit(nkv_bank* bank, const nkv_segment_desc* seg, int32_t kv_dtype, const void* const* k_dev,
                    const void* const* v_dev) {
  return guarded([&] {
    need(seg, "segment descriptor");
    bank_of(bank).commit(*seg, kv_dtype, k_dev, v_dev);
  });
}

int nkv_bank_attend_history(nkv_bank* bank, int32_t layer, const void* q, uint64_t q_len, float scale, float* out,
                            float* lse) {
  return guarded([&] { bank_of(bank).attend_history(layer, q, q_len, scale, out, lse); });
}

int nkv_bank_set_archive_device_limit(nkv_bank* bank, uint64_t device_bytes) {
  return guarded([&] { bank_of(bank).set_archive_device_limit(device_bytes); });
}

int nkv_bank_archive_usage(nkv_bank* bank, uint64_t* device_bytes, uint64_t* host_bytes) {
  return guarded([&] {
    need(device_bytes, "device_bytes");
    need(host_bytes, "host_bytes");
    bank_of(bank).archive_usage(device_bytes, host_bytes);
  });
}

int nkv_bank_commit_decode(nkv_bank* bank, const nkv_segment_desc* seg, int32_t kv_dtype, const void* const* k_dev,
                           const void* const* v_dev, void* const* k_out, void* const* v_out) {
  return guarded([&] {
    need(seg, "segment descriptor");
    bank_of(bank).commit_decode(*seg, kv_dtype, k_dev, v_dev, k_out, v_out);
  });
}

int nkv_bank_rollback(nkv_bank* bank) {
  return guarded([&] { bank_of(bank).rollback(); });
}

int nkv_bank_park(nkv_bank* bank) {
  return guarded([&] { bank_of(bank).park(); });
}

int nkv_bank_unpark(nkv_bank* bank) {
  return guarded([&] { bank_of(bank).unpark(); });
}

int nkv_bank_metrics(const nkv_bank* bank, nkv_metrics* out) {
  return guarded([&] {
    need(out, "output");
    *out = bank_of(bank).bank_metrics();
  });
}

int nkv_bank_synchronize(nkv_bank* bank) {
  return guarded([&] { bank_of(bank).synchronize(); });
}

int nkv_bank_reserve(nkv_bank* bank, uint64_t archive_bytes, uint64_t working_tokens) {
  return guarded([&] { bank_of(bank).reserve(archive_bytes, working_tokens); });
}

int nkv_bank_segment_bytes(const nkv_bank* bank, const nkv_segment_desc* seg, uint64_t* bytes_per_layer) {
  return guarded([&] {
    need(seg, "segment descriptor");
    need(bytes_per_layer, "output");
    *bytes_per_layer = bank_of(bank).segment_bytes(*seg);
  });
}

int nkv_bank_decode_segment(nkv_bank* bank, uint64_t archive_pos, void* const* k_out, void* const* v_out) {
  return guarded([&] { bank_of(bank).decode_segment(archive_pos, k_out, v_out); });
}

int nkv_bank_set_timing(nkv_bank* bank, int32_t enable) {
  return guarded([&] { bank_of(bank).set_timing(enable != 0); });
}

int nkv_bank_kernel_stats(nkv_bank* bank, nkv_kernel_stat* out, int32_t reset) {
  return guarded([&] {
    need(out, "output");
    bank_of(bank).kernel_stats(out, reset != 0);
  });
}

int nkv_bank_save(nkv_bank* bank, const char* path) {
  return guarded([&] { bank_of(bank).save(path); });
}

int nkv_bank_load(nkv_bank* bank, const char* path) {
  return guarded([&] { bank_of(bank).load(path); });
}

int nkv_bank_stage_segment(nkv_bank* bank, const nkv_segment_desc* seg, nkv_staged_layer* out) {
  return guarded([&] {
    need(seg, "seg");
    bank_of(bank).stage(*seg, out);
  });
}

int nkv_bank_commit_staged(nkv_bank* bank) {
  return guarded([&] { bank_of(bank).commit_staged(); });
}

int nkv_bank_discard_staged(nkv_bank* bank) {
  return guarded([&] { bank_of(bank).discard_staged(); });
}

int nkv_cache_working_set(const nkv_bank* bank, int32_t layer, const void** k_dev, const void** v_dev,
                          uint64_t* valid_len) {
  return guarded([&] {
    need(k_dev, "k output");
    need(v_dev, "v output");
    need(valid_len, "valid_len output");
    bank_of(bank).working_set(layer, k_dev, v_dev, valid_len);
  });
}

int nkv_cache_layout(const nkv_bank* bank, int32_t layer, nkv_segment_layout* out, uint64_t cap, uint64_t* n) {
  return guarded([&] {
    need(n, "count output");
    const Bank& b = bank_of(bank);
    if (layer < 0 || layer >= b.n_layers()) nkv::fail(NKV_ERR_ARGUMENT, "layer out of range");
    const auto& lay = b.layout();
    *n = lay.size();
    if (out)
      for (size_t i = 0; i < lay.size() && i < cap; ++i) out[i] = lay[i];
  });
}

int nkv_cache_info(const nkv_bank* bank, int32_t layer, nkv_cache_info_t* out) {
  return guarded([&] {
    need(out, "output");
    bank_of(bank).info(layer, out);
  });
}

int nkv_cache_metrics(const nkv_bank* bank, int32_t layer, nkv_metrics* out) {
  return guarded([&] {
    need(out, "output");
    const Bank& b = bank_of(bank);
    if (layer < 0 || layer >= b.n_layers()) nkv::fail(NKV_ERR_ARGUMENT, "layer out of range");
    *out = b.layer_metrics();
  });
}

int nkv_cache_set_qvg_codebooks(nkv_bank* bank, int32_t layer, const float* host_cb) {
  return guarded([&] { bank_of(bank).set_codebooks(layer, host_cb); });
}

int nkv_cache_get_qvg_codebooks(const nkv_bank* bank, int32_t layer, float* host_cb, int32_t* fitted) {
  return guarded([&] {
    need(fitted, "fitted output");
    bank_of(bank).get_codebooks(layer, host_cb, fitted);
  });
}

int nkv_cache_export_segment(const nkv_bank* bank, int32_t layer, uint64_t archive_pos, void* host_buf,
                             uint64_t cap, uint64_t* nbytes) {
  return guarded([&] {
    need(nbytes, "size output");
    *nbytes = const_cast<Bank&>(bank_of(bank)).export_segment(layer, archive_pos, host_buf, cap);
  });
}

int nkv_frame_indices(int32_t kind, uint64_t total_frames, uint64_t past_frames, int32_t sampling, double gamma,
                      uint64_t* out, uint64_t cap, uint64_t* n) {
  return guarded([&] {
    need(n, "count output");
    std::vector<uint64_t> ids;
    switch (kind) {
      case 0: ids = nkv::uniform_frame_indices(total_frames, past_frames); break;
      case 1: ids = nkv::recent_mix_uniform_frame_indices(total_frames, past_frames); break;
      case 2: ids = nkv::temporal_context_frame_indices(total_frames, past_frames, gamma); break;
      case 3: ids = nkv::history_frame_indices(total_frames, past_frames, sampling, gamma); break;
      default: nkv::fail(NKV_ERR_ARGUMENT, "unknown sampler kind " + std::to_string(kind));
    }
    *n = ids.size();
    if (out)
      for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  });
}

int nkv_plan_recent_trim(const uint64_t* records, uint64_t n, uint64_t capacity, uint64_t tokens_per_frame,
                         uint64_t* drop_frames, uint64_t* n_drop_frames, uint64_t* drop_records,
                         uint64_t* n_drop_records, uint64_t* evicted_tokens, uint64_t* kept, uint64_t* n_kept) {
  return guarded([&] {
    if (n) need(records, "records");
    need(n_drop_frames, "output");
    need(n_drop_records, "output");
    need(evicted_tokens, "output");
    need(n_kept, "output");
    if (tokens_per_frame == 0) nkv::fail(NKV_ERR_ARGUMENT, "tokens_per_frame must be > 0");
    std::vector<nkv::DenseRecord> recs(n);
    for (uint64_t i = 0; i < n; ++i)
      recs[i] = {records[5 * i], records[5 * i + 1], records[5 * i + 2], records[5 * i + 3], records[5 * i + 4]};
    nkv::TrimPlan p = nkv::plan_recent_trim(recs, capacity, tokens_per_frame);
    *n_drop_frames = p.drop_frames.size();
    if (drop_frames)
      for (size_t i = 0; i < p.drop_frames.size(); ++i)
        drop_frames[2 * i] = p.drop_frames[i].first, drop_frames[2 * i + 1] = p.drop_frames[i].second;
    *n_drop_records = p.drop_records.size();
    if (drop_records)
      for (size_t i = 0; i < p.drop_records.size(); ++i) drop_records[i] = p.drop_records[i];
    *evicted_tokens = p.evicted_tokens;
    auto k = nkv::apply_trim(recs, p, tokens_per_frame);
    *n_kept = k.size();
    if (kept)
      for (size_t i = 0; i < k.size(); ++i) {
        kept[5 * i] = k[i].segment_index, kept[5 * i + 1] = k[i].frame_start, kept[5 * i + 2] = k[i].frame_count;
        kept[5 * i + 3] = k[i].image_tokens, kept[5 * i + 4] = k[i].text_tokens;
      }
  });
}

int nkv_kv_project(const nkv_kv_project_args* a, void* stream) {
  return guarded([&] {
    need(a, "args");
    if (a->head_dim != 128 || !nkv::kv_project_shape_ok(a->tokens, a->heads, a->head_dim))
      nkv::fail(NKV_ERR_ARGUMENT, "nkv_kv_project needs head_dim 128, heads * 128 a multiple of 256 (heads <= 256) and 0 < tokens <= 2^26");
    need(a->x, "x"), need(a->wk, "wk"), need(a->wv, "wv"), need(a->status, "status");
    const bool codes = a->k_codes || a->v_codes || a->k_scales || a->v_scales;
    if (codes && !(a->k_codes && a->v_codes && a->k_scales && a->v_scales))
      nkv::fail(NKV_ERR_ARGUMENT, "k_codes, v_codes, k_scales and v_scales go together");
    if (a->rope_cos ? !a->rope_sin : a->rope_sin != nullptr)
      nkv::fail(NKV_ERR_ARGUMENT, "rope_cos and rope_sin go together");
    if (a->n_ranges < 0 || a->n_ranges > 2) nkv::fail(NKV_ERR_ARGUMENT, "n_ranges must be 0, 1 or 2");
    for (int i = 0; i < a->n_ranges; ++i) {
      const nkv_row_range& r = a->ranges[i];
      if (r.lo < 0 || r.hi < r.lo || r.hi > a->tokens || r.dst < 0)
        nkv::fail(NKV_ERR_ARGUMENT, "row range " + std::to_string(i) + " outside [0, tokens)");
    }
    // vector loads / stores and TMA need 16 bytes; scales and the status
    // word are single 4-byte stores / atomics
    const void* vec[] = {a->x, a->wk, a->wv, a->bk, a->bv, a->k_norm_gain, a->rope_cos, a->rope_sin, a->k_out,
                         a->v_out, a->k_codes, a->v_codes};
    for (const void* p : vec)
      if (reinterpret_cast<uintptr_t>(p) & 15u)
        nkv::fail(NKV_ERR_ARGUMENT, "nkv_kv_project tensor pointers must be 16-byte aligned");
    for (const void* p : {static_cast<const void*>(a->k_scales), static_cast<const void*>(a->v_scales),
                          static_cast<const void*>(a->status)})
      if (reinterpret_cast<uintptr_t>(p) & 3u)
        nkv::fail(NKV_ERR_ARGUMENT, "nkv_kv_project scales and status must be 4-byte aligned");
    nkv::KvProjectParams p{};
    p.M = a->tokens;
    p.H = a->heads;
    p.qk_norm = a->qk_norm;
    p.eps = a->eps;
    p.bias_k = static_cast<const uint16_t*>(a->bk);
    p.bias_v = static_cast<const uint16_t*>(a->bv);
    p.k_gain = static_cast<const uint16_t*>(a->k_norm_gain);
    p.rope_cos = a->rope_cos;
    p.rope_sin = a->rope_sin;
    p.k_out = static_cast<uint16_t*>(a->k_out);
    p.v_out = static_cast<uint16_t*>(a->v_out);
    p.k_codes = a->k_codes, p.k_scales = a->k_scales, p.v_codes = a->v_codes, p.v_scales = a->v_scales;
    p.n_ranges = codes ? a->n_ranges : 0;
    for (int i = 0; i < p.n_ranges; ++i)
      p.range_lo[i] = a->ranges[i].lo, p.range_hi[i] = a->ranges[i].hi, p.range_dst[i] = a->ranges[i].dst;
    p.flag = a->status;
    p.err = a->status;
    nkv::check_cuda(nkv::launch_kv_project(a->x, a->wk, a->wv, p, static_cast<cudaStream_t>(stream)),
                    "kv projection launch");
  });
}

int nkv_int8_quantize(const void* k, const void* v, int32_t in_dtype, uint64_t rows, int64_t head_dim,
                      uint8_t* kq, uint8_t* vq, float* ks, float* vs, uint32_t* nonfinite_out, void* stream) {
  return guarded([&] {
    check_dtype(in_dtype);
    if (head_dim < 1) nkv::fail(NKV_ERR_ARGUMENT, "head_dim must be >= 1");
    if (rows == 0) {
      if (nonfinite_out) *nonfinite_out = 0;
      return;
    }
    need(k, "k"), need(v, "v"), need(kq, "kq"), need(vq, "vq"), need(ks, "ks"), need(vs, "vs");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    nkv::QuantJob job{k, v, kq, vq, ks, vs, nullptr};
    nkv::QuantJob* d_job = nullptr;
    uint32_t* d_flag = nullptr;
    nkv::check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&d_job), sizeof(job), s), "cudaMallocAsync");
    nkv::check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&d_flag), sizeof(uint32_t), s), "cudaMallocAsync");
    nkv::check_cuda(cudaMemcpyAsync(d_job, &job, sizeof(job), cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
    nkv::check_cuda(cudaMemsetAsync(d_flag, 0, sizeof(uint32_t), s), "cudaMemsetAsync");
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const bool aligned = a16(k) && a16(v) && a16(kq) && a16(vq);
    nkv::check_cuda(nkv::launch_int8_quantize(d_job, 1, rows, 0, head_dim, in_dtype, aligned, d_flag, s),
                    "int8 quantize launch");
    uint32_t flag = 0;
    nkv::check_cuda(cudaMemcpyAsync(&flag, d_flag, sizeof(uint32_t), cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
    nkv::check_cuda(cudaFreeAsync(d_job, s), "cudaFreeAsync");
    nkv::check_cuda(cudaFreeAsync(d_flag, s), "cudaFreeAsync");
    nkv::check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (nonfinite_out) *nonfinite_out = flag;
    if (flag) nkv::fail(NKV_ERR_MSG, std::string("cannot quantize non-finite ") + ((flag & 1u) ? "k" : "v") + " values");
  });
}

int nkv_int8_dequantize(const uint8_t* q, const float* scales, uint64_t rows, int64_t head_dim, int32_t out_dtype,
                        void* out, void* stream) {
  return guarded([&] {
    check_dtype(out_dtype);
    if (head_dim < 1) nkv::fail(NKV_ERR_ARGUMENT, "head_dim must be >= 1");
    if (rows == 0) return;
    need(q, "codes"), need(scales, "scales"), need(out, "output");
    nkv::check_cuda(nkv::launch_int8_dequantize(q, scales, rows, head_dim, out_dtype, out,
                                                static_cast<cudaStream_t>(stream)),
                    "int8 dequantize launch");
  });
}

int nkv_qvg_encode(const float* cb_dev, int32_t side, const void* x, int32_t in_dtype, uint64_t L, int64_t heads,
                   int64_t head_dim, uint64_t tokens, int32_t stages, int32_t bits, int32_t block, uint8_t* codes,
                   float* scales, void* stream) {
  return guarded([&] {
    check_dtype(in_dtype);
    if (side != 0 && side != 1) nkv::fail(NKV_ERR_ARGUMENT, "side must be 0 (k) or 1 (v)");
    if (stages < 1 || bits < 1 || bits > 8 || stages * bits > 64 || block < 1 || heads < 1 || head_dim < 1)
      nkv::fail(NKV_ERR_INVALID_CONFIG, "invalid QVG stages/bits");
    if (tokens > L)
      nkv::fail(NKV_ERR_GEOMETRY, "qvg encode token range " + std::to_string(tokens) + " > len " + std::to_string(L));
    if (nkv::qvg_encode_smem_bytes(int(head_dim), block, bits) > 200 * 1024)
      nkv::fail(NKV_ERR_INVALID_CONFIG, "QVG block_size x head_dim too large for the device encoder");
    if (tokens == 0) return;
    need(cb_dev, "codebooks"), need(x, "input"), need(codes, "codes"), need(scales, "scales");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t side_floats = size_t(heads) * stages * (size_t(1) << bits) * head_dim;
    nkv::QvgEncodeJob job{x, codes, scales, cb_dev + side_floats * side};
    nkv::QvgEncodeJob* d_job = nullptr;
    nkv::check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&d_job), sizeof(job), s), "cudaMallocAsync");
    nkv::check_cuda(cudaMemcpyAsync(d_job, &job, sizeof(job), cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    nkv::check_cuda(nkv::launch_qvg_encode(d_job, 1, in_dtype, L, int(heads), int(head_dim), tokens, stages, bits,
                                           block, aligned, s),
                    "qvg encode launch");
    nkv::check_cuda(cudaFreeAsync(d_job, s), "cudaFreeAsync");
    nkv::check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  });
}

int nkv_qvg_decode(const float* cb_dev, int32_t side, const uint8_t* codes, const float* scales, uint64_t tokens,
                   int64_t heads, int64_t head_dim, int32_t stages, int32_t bits, int32_t block, float* out,
                   void* stream) {
  return guarded([&] {
    if (side != 0 && side != 1) nkv::fail(NKV_ERR_ARGUMENT, "side must be 0 (k) or 1 (v)");
    if (stages < 1 || bits < 1 || bits > 8 || stages * bits > 64 || block < 1 || heads < 1 || head_dim < 1)
      nkv::fail(NKV_ERR_INVALID_CONFIG, "invalid QVG stages/bits");
    if (tokens == 0) return;
    need(cb_dev, "codebooks"), need(codes, "codes"), need(scales, "scales"), need(out, "output");
    const size_t side_floats = size_t(heads) * stages * (size_t(1) << bits) * head_dim;
    nkv::check_cuda(nkv::launch_qvg_decode(cb_dev + side_floats * side, codes, scales, tokens, int(heads),
                                           int(head_dim), stages, bits, block, out,
                                           static_cast<cudaStream_t>(stream)),
                    "qvg decode launch");
  });
}

int nkv_synth_fill(void* dst, int32_t dtype, uint64_t rows, int64_t heads, int64_t head_dim, uint64_t key,
                   uint64_t index_offset, const float* table, const float* chan_scale, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    if (rows == 0) return;
    need(dst, "destination"), need(table, "table");
    nkv::check_cuda(nkv::launch_synth_fill(dst, dtype, rows, int(heads), int(head_dim), key, index_offset, table,
                                           chan_scale, static_cast<cudaStream_t>(stream)),
                    "synth fill launch");
  });
}

}  // extern "C"
