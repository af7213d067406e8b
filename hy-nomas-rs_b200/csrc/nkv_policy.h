// nkv_policy.h — frame sampling and SWA eviction planning of the lifelong
// KV cache: the integer policy that decides which archived frames the
// working set holds.
//
// Restates cache/uniform_history.rs and cache/swa.rs of nomas-core.  The
// per-index formulas are `__host__ __device__` so a device planner and the
// host planner evaluate identical integer expressions; the list-building
// helpers below are host code used by the bank's rebuild planner.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

#ifdef __CUDACC__
#define NKV_HD __host__ __device__ __forceinline__
#else
#define NKV_HD inline
#endif

namespace nkv {

enum Sampling : int { RECENT = 0, UNIFORM = 1, RECENT_MIX = 2, TEMPORAL = 3 };

// i-th entry of uniform_frame_indices(total, past)
// (cache/uniform_history.rs:10-19): count = min(total, past); count == 1 ->
// [total - 1]; else i * (total - 1) / (count - 1), integer division.
NKV_HD uint64_t uniform_index(uint64_t total, uint64_t count, uint64_t i) {
  return count == 1 ? total - 1 : i * (total - 1) / (count - 1);
}

// i-th entry of recent_mix_uniform_frame_indices (uniform_history.rs:23-32).
NKV_HD uint64_t recent_mix_index(uint64_t total, uint64_t past, uint64_t i) {
  if (total <= past) return i;
  uint64_t recent = past / 2, older_end = total - recent, older = past - recent;
  uint64_t older_count = older_end < older ? older_end : older;
  if (i < older_count) return uniform_index(older_end, older_count, i);
  return older_end + (i - older_count);
}

struct PolicyError {
  int code;  // nkv_status value
  std::string msg;
};

// uniform_frame_indices (uniform_history.rs:10-19)
inline std::vector<uint64_t> uniform_frame_indices(uint64_t total, uint64_t past) {
  uint64_t count = total < past ? total : past;
  std::vector<uint64_t> ids(count);
  for (uint64_t i = 0; i < count; ++i) ids[i] = uniform_index(total, count, i);
  return ids;
}

// recent_mix_uniform_frame_indices (uniform_history.rs:23-32)
inline std::vector<uint64_t> recent_mix_uniform_frame_indices(uint64_t total, uint64_t past) {
  std::vector<uint64_t> ids;
  if (total <= past) {
    for (uint64_t f = 0; f < total; ++f) ids.push_back(f);
    return ids;
  }
  uint64_t recent = past / 2, older_end = total - recent;
  ids = uniform_frame_indices(older_end, past - recent);
  for (uint64_t f = older_end; f < total; ++f) ids.push_back(f);
  return ids;
}

// temporal_context_frame_indices (uniform_history.rs:40-70).  The offsets use
// glibc pow and round-half-away-from-zero in f64, as Rust's f64::powf /
// f64::round do on Linux; they stay on the host for that reason.
inline std::vector<uint64_t> temporal_context_frame_indices(uint64_t total, uint64_t past, double gamma) {
  std::vector<uint64_t> ids;
  if (!std::isfinite(gamma) || gamma <= 0.0) return ids;
  uint64_t count = total < past ? total : past;
  if (count == 0) return ids;
  if (count == 1) return {total - 1};
  if (count == total) {
    for (uint64_t f = 0; f < total; ++f) ids.push_back(f);
    return ids;
  }
  uint64_t slack = total - count;
  ids.resize(count);
  for (uint64_t i = 0; i < count; ++i) {
    double u = double(i) / double(count - 1);
    double off = std::round(double(slack) * std::pow(u, gamma));
    if (off < 0.0) off = 0.0;             // f64::clamp(0, slack)
    if (off > double(slack)) off = double(slack);
    uint64_t o = (off == off) ? uint64_t(off) : 0;  // `as usize`: NaN -> 0
    // distances are reversed and mapped to total - 1 - d: entry i of the
    // result comes from distance index count - 1 - i.
    ids[count - 1 - i] = total - 1 - (i + o);
  }
  return ids;
}

// Rust's `{}` Display of an f64, used in the reference's messages: the
// shortest digits that round-trip, written without an exponent ("0.9",
// "2", "0.0000001", "NaN", "inf").
inline std::string rust_f64(double x) {
  if (x != x) return "NaN";
  if (std::isinf(x)) return x > 0 ? "inf" : "-inf";
  if (x == 0.0) return std::signbit(x) ? "-0" : "0";
  char buf[64];
  int prec = 1;
  for (; prec <= 17; ++prec) {
    snprintf(buf, sizeof buf, "%.*e", prec - 1, x);
    if (std::strtod(buf, nullptr) == x) break;
  }
  std::string s(buf);
  const bool neg = s[0] == '-';
  if (neg) s.erase(0, 1);
  const size_t epos = s.find('e');
  const int exp10 = std::atoi(s.c_str() + epos + 1);
  std::string digits;
  for (size_t i = 0; i < epos; ++i)
    if (s[i] != '.') digits += s[i];
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string out;
  if (exp10 >= 0) {
    if (int(digits.size()) <= exp10 + 1) {
      out = digits + std::string(size_t(exp10 + 1 - int(digits.size())), '0');
    } else {
      out = digits.substr(0, size_t(exp10 + 1)) + "." + digits.substr(size_t(exp10 + 1));
    }
  } else {
    out = "0." + std::string(size_t(-exp10 - 1), '0') + digits;
  }
  return neg ? "-" + out : out;
}

inline std::string sampling_name(int s, double gamma) {
  switch (s) {
    case RECENT: return "recent";
    case UNIFORM: return "uniform";
    case RECENT_MIX: return "recent_mix_uniform";
    default: return "temporal_context(gamma=" + rust_f64(gamma) + ")";  // config.rs:69-78
  }
}

// history_frame_indices (uniform_history.rs:76-125): dispatch + the count,
// range and chronology checks.  Throws PolicyError{ERR_MSG / ERR_INVALID_CONFIG}.
inline std::vector<uint64_t> history_frame_indices(uint64_t total, uint64_t past, int sampling, double gamma_cfg) {
  const int kInvalidConfig = 3, kMsg = 4;
  double gamma = sampling == TEMPORAL ? gamma_cfg : 2.0;
  if (sampling == TEMPORAL && (!std::isfinite(gamma) || gamma <= 0.0))
    throw PolicyError{kInvalidConfig, "temporal_context gamma must be finite and positive, got " + rust_f64(gamma)};
  std::vector<uint64_t> ids;
  if (sampling == UNIFORM) ids = uniform_frame_indices(total, past);
  else if (sampling == RECENT_MIX) ids = recent_mix_uniform_frame_indices(total, past);
  else if (sampling == TEMPORAL) ids = temporal_context_frame_indices(total, past, gamma);
  else {
    uint64_t m = total < past ? total : past;
    for (uint64_t i = 0; i < m; ++i) ids.push_back(total - m + i);
  }
  uint64_t expected = total < past ? total : past;
  std::string name = sampling_name(sampling, gamma);
  if (ids.size() != expected)
    throw PolicyError{kMsg, "history sampling " + name + " selected " + std::to_string(ids.size()) +
                                " frames; expected " + std::to_string(expected)};
  for (uint64_t f : ids)
    if (f >= total)
      throw PolicyError{kMsg, "history sampling " + name + " produced out-of-range frame " + std::to_string(f) +
                                  " (total " + std::to_string(total) + ")"};
  for (size_t i = 1; i < ids.size(); ++i)
    if (ids[i - 1] >= ids[i])
      throw PolicyError{kMsg, "history sampling " + name + " must return chronological, unique frame indices"};
  return ids;
}

// DenseRecord (cache/swa.rs:11-29)
struct DenseRecord {
  uint64_t segment_index, frame_start, frame_count, image_tokens, text_tokens;
  uint64_t total_tokens() const { return image_tokens + text_tokens; }
};

// TrimPlan (cache/swa.rs:33-41)
struct TrimPlan {
  std::vector<std::pair<uint64_t, uint64_t>> drop_frames;  // (archive position, frames dropped from its head)
  std::vector<uint64_t> drop_records;
  uint64_t evicted_tokens = 0;
};

// plan_recent_trim (cache/swa.rs:52-95): oldest record first — drop whole
// records while the deficit needs video and text; else drop only the video
// when that suffices; else drop ceil(deficit / tpf) head frames.
inline TrimPlan plan_recent_trim(const std::vector<DenseRecord>& recs, uint64_t capacity, uint64_t tpf) {
  uint64_t total = 0;
  for (const auto& r : recs) total += r.total_tokens();
  TrimPlan plan;
  for (uint64_t idx = 0; total > capacity && idx < recs.size(); ++idx) {
    const DenseRecord& r = recs[idx];
    uint64_t deficit = total - capacity;
    if (deficit < r.image_tokens) {
      uint64_t frames = (deficit + tpf - 1) / tpf;
      if (frames > r.frame_count) frames = r.frame_count;
      plan.drop_frames.push_back({idx, frames});
      plan.evicted_tokens += frames * tpf;
      break;
    }
    if (total - r.image_tokens <= capacity) {
      plan.drop_frames.push_back({idx, r.frame_count});
      plan.evicted_tokens += r.image_tokens;
      break;
    }
    plan.drop_records.push_back(idx);
    total -= r.total_tokens();
    plan.evicted_tokens += r.total_tokens();
  }
  return plan;
}

// apply_trim (cache/swa.rs:100-130)
inline std::vector<DenseRecord> apply_trim(const std::vector<DenseRecord>& recs, const TrimPlan& plan, uint64_t tpf) {
  std::vector<DenseRecord> out;
  for (uint64_t idx = 0; idx < recs.size(); ++idx) {
    bool dropped = false;
    for (uint64_t d : plan.drop_records) dropped |= (d == idx);
    if (dropped) continue;
    const DenseRecord& r = recs[idx];
    const std::pair<uint64_t, uint64_t>* cut = nullptr;
    for (const auto& p : plan.drop_frames)
      if (p.first == idx) {
        cut = &p;
        break;
      }
    if (!cut) {
      out.push_back(r);
      continue;
    }
    uint64_t kept = r.frame_count - cut->second;
    uint64_t rtpf = r.frame_count > 0 ? r.image_tokens / r.frame_count : tpf;
    out.push_back({r.segment_index, r.frame_start + cut->second, kept, kept * rtpf, r.text_tokens});
  }
  return out;
}

}  // namespace nkv
