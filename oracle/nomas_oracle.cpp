// nomas_oracle.cpp — CPU restatement of the hy-nomas-rs lifelong KV-cache path.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
// calls this file.  It is used by tests/ (as the parity checker), by
// __graft_entry__.smoke() (as the checker of one small GPU call) and by
// bench.py's cpu_baseline / `--impl reference` arm (as the timed CPU
// restatement of the reference algorithm, including its full-segment decode
// before index_select on rebuild).
//
// Every function restates the Rust reference (idrees2516/hy-nomas-rs,
// crate nomas-core) op by op; citations are `path:line` inside that project.
// The reference does its arithmetic through candle-core 0.11.1 and half 2.7.1
// (nomas-core/Cargo.toml:8-9, Cargo.lock:165-167, 754-756), which are not
// available here.  The op semantics assumed for them are:
//   * Tensor::affine(m, a) on f32  : x * (f32)m + (f32)a, two roundings;
//   * round                         : half away from zero (f32::round);
//   * clamp(lo, hi)                 : maximum(lo) then minimum(hi) with
//                                     maximum(a,b) = a < b ? b : a,
//                                     minimum(a,b) = a > b ? b : a;
//   * to_dtype(U8) from f32         : Rust `as u8` (saturating, NaN -> 0);
//   * to_dtype(BF16/F16)            : half's round-to-nearest-even, NaN keeps
//                                     its top payload bits with the quiet bit;
//   * broadcast_div / broadcast_mul : IEEE f32;
//   * Iterator::sum::<f64>          : sequential left fold;
//   * f64::powf / round             : glibc pow, half-away-from-zero round.
//
// Parity status.  The frame samplers and the SWA trim plans are pinned
// exactly by the reference's own known-answer tests
// (cache/uniform_history.rs:131-196, cache/swa.rs:146-230), which
// tests/test_oracle_kats.py replays.  INT8 and QVG byte-level numerics are
// pinned only through the reference's invariant tests (cache/int8.rs:162-244,
// cache/qvg.rs:450-527: error bounds, code ranges, non-finite rejection,
// error decreasing with stages); no reference-generated golden bytes exist
// (the reference is Rust and cannot be built here), so byte-level parity with
// candle itself is "parity unpinned" beyond the semantics listed above.
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off, no -ffast-math, no
// -march: contraction or reassociation would change the f32/f64 roundings).

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <limits>
#include <memory>
#include <string>
#include <thread>
#include <vector>

// Worker threads the checker may use for work the reference does in an
// independent loop (per head of a QVG encode/decode, per represented segment
// of a rebuild).  Every iteration computes the same values in the same order
// as the sequential loop, so results do not depend on it.  1 (the default,
// used by the timed CPU baseline) keeps every loop sequential; tests raise it
// to check the 8B geometry in seconds.
static std::atomic<int> g_threads{1};
static thread_local bool t_in_parallel = false;  // nested loops stay sequential

template <typename F>
static void parallel_for(size_t n, F&& fn) {
  const size_t nt = t_in_parallel ? 1 : std::min<size_t>(size_t(std::max(1, g_threads.load())), n);
  if (nt <= 1) {
    for (size_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<size_t> next{0};
  std::vector<std::thread> th;
  std::vector<std::exception_ptr> err(nt);
  for (size_t t = 0; t < nt; ++t)
    th.emplace_back([&, t]() {
      t_in_parallel = true;
      try {
        for (size_t i = next++; i < n; i = next++) fn(i);
      } catch (...) {
        err[t] = std::current_exception();
      }
    });
  for (auto& x : th) x.join();
  for (auto& e : err)
    if (e) std::rethrow_exception(e);
}

namespace orc {

// ---------------------------------------------------------------- status ---
enum Status : int {
  OK = 0,
  ERR_GEOMETRY = 1,
  ERR_CACHE_STATE = 2,
  ERR_INVALID_CONFIG = 3,
  ERR_MSG = 4,
  ERR_ARGUMENT = 6,
};

struct Error {
  int code;
  std::string msg;
};

static thread_local std::string g_last_error;

[[noreturn]] static void fail(int code, const std::string& msg) { throw Error{code, msg}; }

// ---------------------------------------------------------------- numerics --
enum DType : int { F32 = 0, BF16 = 1, F16 = 2 };

static inline uint32_t f2u(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// half 2.7.1 f32 -> bf16: round to nearest even; NaN keeps its high payload
// and gets the quiet bit.
static inline uint16_t bf16_bits(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return uint16_t((u >> 16) | 0x0040u);
  const uint32_t rb = 0x00008000u;
  if ((u & rb) != 0 && (u & (3 * rb - 1)) != 0) return uint16_t((u >> 16) + 1);
  return uint16_t(u >> 16);
}
static inline float bf16_value(uint16_t b) {
  if ((b & 0x7FFFu) > 0x7F80u) return u2f((uint32_t(b) | 0x0040u) << 16);
  return u2f(uint32_t(b) << 16);
}

// IEEE binary16 from f32, round to nearest even (half's software path and
// x86 F16C agree on this, NaN included).
static inline uint16_t f16_bits(float value) {
  uint32_t x = f2u(value);
  uint32_t sign = x & 0x80000000u, exp = x & 0x7F800000u, man = x & 0x007FFFFFu;
  uint32_t hs = sign >> 16;
  if (exp == 0x7F800000u) {
    if (man == 0) return uint16_t(hs | 0x7C00u);
    return uint16_t(hs | 0x7C00u | 0x0200u | (man >> 13));
  }
  int32_t he = int32_t(exp >> 23) - 127 + 15;
  if (he >= 0x1F) return uint16_t(hs | 0x7C00u);
  if (he <= 0) {
    if (14 - he > 24) return uint16_t(hs);
    uint32_t m = man | 0x00800000u;
    uint32_t hm = m >> (14 - he);
    uint32_t rb = 1u << (13 - he);
    if ((m & rb) != 0 && (m & (3 * rb - 1)) != 0) hm += 1;
    return uint16_t(hs | hm);
  }
  uint32_t hm = man >> 13;
  uint32_t out = hs | (uint32_t(he) << 10) | hm;
  const uint32_t rb = 0x00001000u;
  if ((man & rb) != 0 && (man & (3 * rb - 1)) != 0) out += 1;
  return uint16_t(out);
}
static inline float f16_value(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  if (exp == 0x1F) {
    if (man == 0) return u2f(sign | 0x7F800000u);
    return u2f(sign | 0x7FC00000u | (man << 13));
  }
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    // subnormal: value = man * 2^-24
    float v = float(man) * u2f(0x33800000u);  // 2^-24, exact
    return sign ? -v : v;
  }
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

// Round an f32 value to the value set of `dt` (candle to_dtype, values kept
// as f32 here: every bf16/f16 value is exactly representable in f32).
static inline float round_to(int dt, float x) {
  switch (dt) {
    case BF16: return bf16_value(bf16_bits(x));
    case F16: return f16_value(f16_bits(x));
    default: return x;
  }
}
static inline size_t dtype_size(int dt) { return dt == F32 ? 4 : 2; }

// Raw buffer of dtype `dt` -> f32 values.
static void load_raw(const void* src, int dt, size_t n, float* dst) {
  if (dt == F32) {
    std::memcpy(dst, src, n * 4);
  } else if (dt == BF16) {
    const uint16_t* s = static_cast<const uint16_t*>(src);
    for (size_t i = 0; i < n; ++i) dst[i] = bf16_value(s[i]);
  } else {
    const uint16_t* s = static_cast<const uint16_t*>(src);
    for (size_t i = 0; i < n; ++i) dst[i] = f16_value(s[i]);
  }
}
// f32 values already in the value set of `dt` -> raw buffer.
static void store_raw(const float* src, int dt, size_t n, void* dst) {
  if (dt == F32) {
    std::memcpy(dst, src, n * 4);
  } else if (dt == BF16) {
    uint16_t* d = static_cast<uint16_t*>(dst);
    for (size_t i = 0; i < n; ++i) d[i] = bf16_bits(src[i]);
  } else {
    uint16_t* d = static_cast<uint16_t*>(dst);
    for (size_t i = 0; i < n; ++i) d[i] = f16_bits(src[i]);
  }
}

static inline float cmax(float a, float b) { return a < b ? b : a; }  // candle maximum
static inline float cmin(float a, float b) { return a > b ? b : a; }  // candle minimum
static inline uint8_t as_u8(float v) {                                // Rust `as u8`
  if (!(v == v)) return 0;
  if (v <= 0.0f) return 0;
  if (v >= 255.0f) return 255;
  return uint8_t(v);
}

// ------------------------------------------------------------ SplitMix64 ---
// tensor_utils.rs:65-107
struct SplitMix64 {
  uint64_t state;
  explicit SplitMix64(uint64_t s) : state(s) {}
  uint64_t next_u64() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double next_f64() { return double(next_u64() >> 11) * (1.0 / double(1ull << 53)); }
  double next_normal(bool& has_spare, double& spare) {
    if (has_spare) {
      has_spare = false;
      return spare;
    }
    double u1 = next_f64();
    if (u1 < std::numeric_limits<double>::min()) u1 = std::numeric_limits<double>::min();
    double u2 = next_f64();
    double r = std::sqrt(-2.0 * std::log(u1));
    double theta = 2.0 * 3.141592653589793 * u2;
    spare = r * std::sin(theta);
    has_spare = true;
    return r * std::cos(theta);
  }
};

// tensor_utils.rs:114-138 (deterministic_randn_affine)
static void randn(size_t n, uint64_t seed, double mean, double stdv, float* out) {
  SplitMix64 rng(seed);
  bool has = false;
  double spare = 0.0;
  for (size_t i = 0; i < n; ++i) out[i] = float(rng.next_normal(has, spare) * stdv + mean);
}

// ------------------------------------------------------------------ INT8 ---
// cache/int8.rs:65-81 (quantize_one) over `rows` rows of D values.
static void quantize_rows(const float* x, size_t rows, size_t D, uint8_t* q, float* s) {
  const float inv127 = float(1.0 / 127.0);
  constexpr size_t kChunk = 4096;  // rows are independent (one scale each)
  parallel_for((rows + kChunk - 1) / kChunk, [&](size_t c) {
  for (size_t r = c * kChunk; r < std::min(rows, (c + 1) * kChunk); ++r) {
    const float* xr = x + r * D;
    float peak = std::fabs(xr[0]);
    for (size_t d = 1; d < D; ++d) {
      float a = std::fabs(xr[d]);
      if (a > peak) peak = a;
    }
    float sc = (peak > 0.0f) ? (peak * inv127 + 0.0f) : 1.0f;
    s[r] = sc;
    for (size_t d = 0; d < D; ++d) {
      float t = xr[d] / sc;
      t = std::round(t);
      t = cmin(cmax(t, -127.0f), 127.0f);
      t = t * 1.0f + 128.0f;
      t = cmin(cmax(t, 0.0f), 255.0f);
      q[r * D + d] = as_u8(t);
    }
  }
  });
}

// cache/int8.rs:85-134 (quantize_kv_pair): non-finite scan of k, then v,
// then quantize both.  Inputs are f32 values (already cast to BF16 by the
// caller where the reference casts, history.rs:249-250 / 268-275).
static void check_finite(const float* x, size_t n, const char* name) {
  const float big = float(double(std::numeric_limits<float>::max())) * 1.0f + 0.0f;
  size_t n_nan = 0, n_inf = 0;
  for (size_t i = 0; i < n; ++i) {
    if (x[i] != x[i]) ++n_nan;
    if (std::fabs(x[i]) >= big) ++n_inf;
  }
  if (n_nan + n_inf != 0) fail(ERR_MSG, std::string("cannot quantize non-finite ") + name + " values");
}

struct Int8Block {
  size_t B = 0, L = 0, H = 0, D = 0;
  std::vector<uint8_t> k, v;
  std::vector<float> ks, vs;
  size_t nbytes() const { return k.size() + v.size() + 4 * (ks.size() + vs.size()); }  // int8.rs:56-61
};

static Int8Block quantize_kv_pair(const float* k, const float* v, size_t B, size_t L, size_t H, size_t D) {
  size_t n = B * L * H * D;
  check_finite(k, n, "k");
  check_finite(v, n, "v");
  Int8Block blk;
  blk.B = B, blk.L = L, blk.H = H, blk.D = D;
  blk.k.resize(n), blk.v.resize(n), blk.ks.resize(B * L * H), blk.vs.resize(B * L * H);
  quantize_rows(k, B * L * H, D, blk.k.data(), blk.ks.data());
  quantize_rows(v, B * L * H, D, blk.v.data(), blk.vs.data());
  return blk;
}

// cache/int8.rs:139-155 (dequantize): prefix valid_len of (B, L, H, D).
static void dequantize(const uint8_t* q, const float* s, size_t B, size_t L, size_t H, size_t D, size_t valid,
                       int dt, float* out) {
  if (valid > L) fail(ERR_GEOMETRY, "invalid valid_len " + std::to_string(valid) + " > " + std::to_string(L));
  for (size_t b = 0; b < B; ++b)
    for (size_t l = 0; l < valid; ++l)
      for (size_t h = 0; h < H; ++h) {
        size_t src = ((b * L + l) * H + h);
        size_t dst = ((b * valid + l) * H + h);
        float sc = s[src];
        for (size_t d = 0; d < D; ++d) {
          float sg = float(q[src * D + d]) * 1.0f + (-128.0f);
          out[dst * D + d] = round_to(dt, sg * sc);
        }
      }
}

// ------------------------------------------------------------------- QVG ---
struct QvgConfig {
  size_t stages = 4, bits = 2, block = 64;
  bool text_as_int8 = true;
  uint64_t seed = 0x5EED0002ull;
  size_t entries() const { return size_t(1) << bits; }            // qvg.rs:57-59
  size_t bpt() const { return (stages * bits + 7) / 8; }           // qvg.rs:62-64
  size_t payload_bytes(size_t tokens, size_t heads) const {        // qvg.rs:67-70
    size_t nb = (tokens + block - 1) / block;
    return tokens * heads * bpt() + nb * heads * stages * 4;
  }
};

struct QvgPayload {  // qvg.rs:44-53
  size_t heads = 0, head_dim = 0, tokens = 0, n_blocks = 0;
  std::vector<uint8_t> codes;
  std::vector<float> scales;
  size_t nbytes() const { return codes.size() + scales.size() * 4; }  // qvg.rs:81-83
};

// qvg.rs:303-321 — argmin of the sequential f64 squared distance with the
// early exit `d >= best_d`; ties go to the lower index.
static size_t nearest(const float* cb, size_t entries, size_t D, const float* x) {
  size_t best = 0;
  double best_d = std::numeric_limits<double>::infinity();
  for (size_t i = 0; i < entries; ++i) {
    const float* e = cb + i * D;
    double d = 0.0;
    for (size_t j = 0; j < D; ++j) {
      double diff = double(x[j]) - double(e[j]);
      d += diff * diff;
      if (d >= best_d) break;
    }
    if (d < best_d) {
      best_d = d;
      best = i;
    }
  }
  return best;
}

// qvg.rs:323-347
static void pack_bits(uint8_t* buf, size_t bit_off, size_t bits, size_t value) {
  uint32_t v = uint32_t(value);
  for (size_t i = 0; i < bits; ++i) {
    size_t idx = bit_off + i;
    if (v & 1u) buf[idx / 8] |= uint8_t(1u << (idx % 8));
    v >>= 1;
  }
}
static size_t unpack_bits(const uint8_t* buf, size_t bit_off, size_t bits) {
  size_t v = 0;
  for (size_t i = 0; i < bits; ++i) {
    size_t idx = bit_off + i;
    if (buf[idx / 8] & (1u << (idx % 8))) v |= size_t(1) << i;
  }
  return v;
}

// qvg.rs:396-442 (farthest_point_init) over n rows of d values.
static std::vector<float> farthest_point_init(const std::vector<float>& data, size_t n, size_t entries, size_t d,
                                              SplitMix64& rng) {
  std::vector<float> cents;
  if (n == 0 || d == 0) return std::vector<float>(entries * d, 0.0f);
  size_t first = size_t(rng.next_f64() * double(n)) % n;
  cents.insert(cents.end(), data.begin() + first * d, data.begin() + (first + 1) * d);
  std::vector<double> dists(n, std::numeric_limits<double>::infinity());
  while (cents.size() / d < entries) {
    const float* last = cents.data() + cents.size() - d;
    double total = 0.0;
    for (size_t i = 0; i < n; ++i) {
      const float* r = data.data() + i * d;
      double dd = 0.0;
      for (size_t j = 0; j < d; ++j) {
        double diff = double(r[j]) - double(last[j]);
        dd += diff * diff;
      }
      if (dd < dists[i]) dists[i] = dd;
      total += dists[i];
    }
    if (total <= 1e-12) {
      std::vector<float> j(cents.begin(), cents.begin() + d);
      j[0] += float(cents.size() / d) * 1e-3f;
      cents.insert(cents.end(), j.begin(), j.end());
      continue;
    }
    double pick = rng.next_f64() * total;
    size_t idx = n - 1;
    for (size_t i = 0; i < n; ++i) {
      pick -= dists[i];
      if (pick <= 0.0) {
        idx = i;
        break;
      }
    }
    cents.insert(cents.end(), data.begin() + idx * d, data.begin() + (idx + 1) * d);
  }
  return cents;
}

// qvg.rs:351-394 (fit_head_codebooks): returns stages x entries x d.
static std::vector<float> fit_head_codebooks(const std::vector<float>& mat, size_t n, size_t d, size_t stages,
                                             size_t entries, uint64_t seed) {
  std::vector<float> residual = mat;
  std::vector<float> out;
  SplitMix64 rng(seed);
  for (size_t s = 0; s < stages; ++s) {
    std::vector<float> cb = farthest_point_init(residual, n, entries, d, rng);
    for (int it = 0; it < 2; ++it) {
      std::vector<double> sums(entries * d, 0.0);
      std::vector<size_t> counts(entries, 0);
      for (size_t i = 0; i < n; ++i) {
        const float* r = residual.data() + i * d;
        size_t c = nearest(cb.data(), entries, d, r);
        counts[c] += 1;
        for (size_t j = 0; j < d; ++j) sums[c * d + j] += double(r[j]);
      }
      for (size_t c = 0; c < entries; ++c)
        if (counts[c] > 0)
          for (size_t j = 0; j < d; ++j) cb[c * d + j] = float(sums[c * d + j] / double(counts[c]));
    }
    for (size_t i = 0; i < n; ++i) {
      float* r = residual.data() + i * d;
      size_t c = nearest(cb.data(), entries, d, r);
      for (size_t j = 0; j < d; ++j) r[j] -= cb[c * d + j];
    }
    out.insert(out.end(), cb.begin(), cb.end());
  }
  return out;
}

// Codebooks layout: [side(2)][head][stage][entry][D] f32 (qvg.rs:38-40).
struct QvgCodec {
  QvgConfig cfg;
  size_t H = 0, D = 0;
  bool fitted = false;
  std::vector<float> cb;

  const float* stage_cb(size_t side, size_t h, size_t s) const {
    return cb.data() + (((side * H + h) * cfg.stages + s) * cfg.entries()) * D;
  }

  // qvg.rs:130-167 — per side (k, v), per head, seed = codebook_seed + h.
  void fit(const float* k, const float* v, size_t L) {
    if (fitted) return;
    size_t E = cfg.entries();
    cb.assign(2 * H * cfg.stages * E * D, 0.0f);
    const float* sides[2] = {k, v};
    for (size_t side = 0; side < 2; ++side)
      for (size_t h = 0; h < H; ++h) {
        std::vector<float> mat(L * D);
        for (size_t l = 0; l < L; ++l)
          for (size_t d = 0; d < D; ++d) mat[l * D + d] = sides[side][(l * H + h) * D + d];
        std::vector<float> hc = fit_head_codebooks(mat, L, D, cfg.stages, E, cfg.seed + uint64_t(h));
        std::memcpy(cb.data() + ((side * H + h) * cfg.stages) * E * D, hc.data(), hc.size() * 4);
      }
    fitted = true;
  }

  // qvg.rs:173-256 — encode video tokens [0, tokens) of a (1, L, H, D) tensor.
  QvgPayload encode(size_t side, const float* t, size_t L, size_t tokens) const {
    if (!fitted) fail(ERR_CACHE_STATE, "qvg codebooks not fitted");
    if (tokens > L) fail(ERR_GEOMETRY, "qvg encode token range " + std::to_string(tokens) + " > len " + std::to_string(L));
    QvgPayload p;
    p.heads = H, p.head_dim = D, p.tokens = tokens;
    p.n_blocks = (tokens + cfg.block - 1) / cfg.block;
    size_t bpt = cfg.bpt(), E = cfg.entries();
    p.codes.assign(tokens * H * bpt, 0);
    p.scales.assign(H * p.n_blocks * cfg.stages, 0.0f);
    parallel_for(H, [&](size_t h) {
      std::vector<float> residual;
      std::vector<size_t> codes;
      for (size_t b = 0; b < p.n_blocks; ++b) {
        size_t start = b * cfg.block, end = std::min((b + 1) * cfg.block, tokens);
        size_t n = end - start;
        residual.resize(n * D);
        for (size_t i = 0; i < n; ++i)
          for (size_t d = 0; d < D; ++d) residual[i * D + d] = t[((start + i) * H + h) * D + d];
        for (size_t s = 0; s < cfg.stages; ++s) {
          const float* cbs = stage_cb(side, h, s);
          codes.resize(n);
          for (size_t i = 0; i < n; ++i) codes[i] = nearest(cbs, E, D, residual.data() + i * D);
          double num = 0.0, den = 0.0;
          for (size_t i = 0; i < n; ++i) {
            const float* r = residual.data() + i * D;
            const float* e = cbs + codes[i] * D;
            double in_num = 0.0, in_den = 0.0;
            for (size_t d = 0; d < D; ++d) in_num += double(r[d]) * double(e[d]);
            num += in_num;
            for (size_t d = 0; d < D; ++d) in_den += double(e[d]) * double(e[d]);
            den += in_den;
          }
          float alpha = den > 1e-12 ? float(num / den) : 1.0f;
          p.scales[(h * p.n_blocks + b) * cfg.stages + s] = alpha;
          for (size_t i = 0; i < n; ++i) {
            float* r = residual.data() + i * D;
            const float* e = cbs + codes[i] * D;
            for (size_t d = 0; d < D; ++d) r[d] -= alpha * e[d];
          }
          for (size_t i = 0; i < n; ++i) {
            size_t token = start + i;
            pack_bits(p.codes.data() + (token * H + h) * bpt, s * cfg.bits, cfg.bits, codes[i]);
          }
        }
      }
    });
    return p;
  }

  // qvg.rs:259-300 — decode to (1, tokens, H, D) f32.
  void decode(size_t side, const QvgPayload& p, float* out) const {
    if (!fitted) fail(ERR_CACHE_STATE, "qvg codebooks not fitted");
    size_t bpt = cfg.bpt();
    std::fill(out, out + p.tokens * p.heads * p.head_dim, 0.0f);
    parallel_for(p.heads, [&](size_t h) {
      for (size_t token = 0; token < p.tokens; ++token) {
        const uint8_t* base = p.codes.data() + (token * p.heads + h) * bpt;
        size_t b = token / cfg.block;
        float* o = out + (token * p.heads + h) * p.head_dim;
        for (size_t s = 0; s < cfg.stages; ++s) {
          size_t code = unpack_bits(base, s * cfg.bits, cfg.bits);
          float alpha = p.scales[(h * p.n_blocks + b) * cfg.stages + s];
          const float* e = stage_cb(side, h, s) + code * p.head_dim;
          for (size_t d = 0; d < p.head_dim; ++d) o[d] += alpha * e[d];
        }
      }
    });
  }
};

// -------------------------------------------------------------- samplers ---
enum Sampling : int { RECENT = 0, UNIFORM = 1, RECENT_MIX = 2, TEMPORAL = 3 };

// cache/uniform_history.rs:10-19
static std::vector<size_t> uniform_frame_indices(size_t total, size_t past) {
  size_t count = std::min(total, past);
  std::vector<size_t> ids;
  if (count == 0) return ids;
  if (count == 1) return {total - 1};
  for (size_t i = 0; i < count; ++i) ids.push_back(i * (total - 1) / (count - 1));
  return ids;
}
// cache/uniform_history.rs:23-32
static std::vector<size_t> recent_mix_uniform_frame_indices(size_t total, size_t past) {
  std::vector<size_t> ids;
  if (total <= past) {
    for (size_t i = 0; i < total; ++i) ids.push_back(i);
    return ids;
  }
  size_t recent = past / 2;
  size_t older_end = total - recent;
  ids = uniform_frame_indices(older_end, past - recent);
  for (size_t f = older_end; f < total; ++f) ids.push_back(f);
  return ids;
}
// cache/uniform_history.rs:40-70
static std::vector<size_t> temporal_context_frame_indices(size_t total, size_t past, double gamma) {
  std::vector<size_t> ids;
  if (!std::isfinite(gamma) || gamma <= 0.0) return ids;
  size_t count = std::min(total, past);
  if (count == 0) return ids;
  if (count == 1) return {total - 1};
  if (count == total) {
    for (size_t i = 0; i < total; ++i) ids.push_back(i);
    return ids;
  }
  size_t slack = total - count;
  std::vector<size_t> dist;
  for (size_t i = 0; i < count; ++i) {
    double u = double(i) / double(count - 1);
    double off = std::round(double(slack) * std::pow(u, gamma));
    // f64::clamp then `as usize` (NaN -> 0)
    if (off < 0.0) off = 0.0;
    if (off > double(slack)) off = double(slack);
    size_t o = (off == off) ? size_t(off) : 0;
    dist.push_back(i + o);
  }
  std::reverse(dist.begin(), dist.end());
  for (size_t d : dist) ids.push_back(total - 1 - d);
  return ids;
}
// Rust `{}` for f64: shortest round-trip digits, positional notation.
static std::string rust_display(double x) {
  if (std::isnan(x)) return "NaN";
  if (std::isinf(x)) return x < 0 ? "-inf" : "inf";
  if (x == 0.0) return std::signbit(x) ? "-0" : "0";
  char e[64];
  for (int p = 0; p < 17; ++p) {
    snprintf(e, sizeof e, "%.*e", p, x);
    if (strtod(e, nullptr) == x) break;
  }
  std::string m(e);
  std::string sign = m[0] == '-' ? "-" : "";
  if (!sign.empty()) m = m.substr(1);
  size_t ep = m.find('e');
  int ex = atoi(m.c_str() + ep + 1);
  std::string dig;
  for (size_t i = 0; i < ep; ++i)
    if (isdigit((unsigned char)m[i])) dig.push_back(m[i]);
  while (dig.size() > 1 && dig.back() == '0') dig.pop_back();
  int point = ex + 1;  // digits before the decimal point
  std::string out;
  if (point <= 0) out = "0." + std::string(-point, '0') + dig;
  else if ((size_t)point >= dig.size()) out = dig + std::string(point - dig.size(), '0');
  else out = dig.substr(0, point) + "." + dig.substr(point);
  return sign + out;
}

static std::string sampling_name(int s, double gamma) {
  switch (s) {
    case RECENT: return "recent";
    case UNIFORM: return "uniform";
    case RECENT_MIX: return "recent_mix_uniform";
    default: return "temporal_context(gamma=" + rust_display(gamma) + ")";
  }
}
// cache/uniform_history.rs:76-125
static std::vector<size_t> history_frame_indices(size_t total, size_t past, int sampling, double gamma_in) {
  double gamma = sampling == TEMPORAL ? gamma_in : 2.0;
  if (sampling == TEMPORAL && (!std::isfinite(gamma) || gamma <= 0.0))
    fail(ERR_INVALID_CONFIG, "temporal_context gamma must be finite and positive, got " + rust_display(gamma));
  std::vector<size_t> ids;
  switch (sampling) {
    case UNIFORM: ids = uniform_frame_indices(total, past); break;
    case RECENT_MIX: ids = recent_mix_uniform_frame_indices(total, past); break;
    case TEMPORAL: ids = temporal_context_frame_indices(total, past, gamma); break;
    default: {
      size_t m = std::min(total, past);
      for (size_t i = 0; i < m; ++i) ids.push_back(total - m + i);
    }
  }
  size_t expected = std::min(total, past);
  const std::string name = sampling_name(sampling, gamma);
  if (ids.size() != expected)
    fail(ERR_MSG, std::string("history sampling ") + name + " selected " + std::to_string(ids.size()) +
                      " frames; expected " + std::to_string(expected));
  for (size_t f : ids)
    if (f >= total)
      fail(ERR_MSG, std::string("history sampling ") + name + " produced out-of-range frame " + std::to_string(f) +
                        " (total " + std::to_string(total) + ")");
  for (size_t i = 1; i < ids.size(); ++i)
    if (ids[i - 1] >= ids[i])
      fail(ERR_MSG, std::string("history sampling ") + name + " must return chronological, unique frame indices");
  return ids;
}

// -------------------------------------------------------------- SWA trim ---
struct DenseRecord {  // cache/swa.rs:11-29
  size_t segment_index, frame_start, frame_count, image_tokens, text_tokens;
  size_t total_tokens() const { return image_tokens + text_tokens; }
};
struct TrimPlan {  // cache/swa.rs:33-41
  std::vector<std::pair<size_t, size_t>> drop_frames;
  std::vector<size_t> drop_records;
  size_t evicted_tokens = 0;
};
// cache/swa.rs:52-95
static TrimPlan plan_recent_trim(const std::vector<DenseRecord>& recs, size_t capacity, size_t tpf) {
  size_t total = 0;
  for (auto& r : recs) total += r.total_tokens();
  TrimPlan p;
  size_t idx = 0;
  while (total > capacity && idx < recs.size()) {
    const DenseRecord& rec = recs[idx];
    size_t deficit = total - capacity;
    if (deficit < rec.image_tokens) {
      size_t frames = std::min((deficit + tpf - 1) / tpf, rec.frame_count);
      p.drop_frames.push_back({idx, frames});
      p.evicted_tokens += frames * tpf;
      break;
    } else if (total - rec.image_tokens <= capacity) {
      p.drop_frames.push_back({idx, rec.frame_count});
      p.evicted_tokens += rec.image_tokens;
      break;
    } else {
      p.drop_records.push_back(idx);
      total -= rec.total_tokens();
      p.evicted_tokens += rec.total_tokens();
      idx += 1;
    }
  }
  return p;
}
// cache/swa.rs:100-130
static std::vector<DenseRecord> apply_trim(const std::vector<DenseRecord>& recs, const TrimPlan& p, size_t tpf) {
  std::vector<DenseRecord> out;
  for (size_t idx = 0; idx < recs.size(); ++idx) {
    const DenseRecord& rec = recs[idx];
    if (std::find(p.drop_records.begin(), p.drop_records.end(), idx) != p.drop_records.end()) continue;
    auto it = std::find_if(p.drop_frames.begin(), p.drop_frames.end(), [&](auto& pr) { return pr.first == idx; });
    if (it != p.drop_frames.end()) {
      size_t frames = it->second;
      size_t kept = rec.frame_count - frames;
      size_t rtpf = rec.frame_count > 0 ? rec.image_tokens / rec.frame_count : tpf;
      out.push_back({rec.segment_index, rec.frame_start + frames, kept, kept * rtpf, rec.text_tokens});
    } else {
      out.push_back(rec);
    }
  }
  return out;
}

// ----------------------------------------------------------------- cache ---
enum Storage : int { FLOATING = 0, INT8 = 1, QVG = 2 };

struct CacheConfig {  // config.rs:142-174
  int storage = FLOATING;
  QvgConfig qvg;
  int sampling = RECENT;
  double gamma = 2.0;
  bool has_capacity = false;
  size_t capacity = 0;
  size_t past_frames = 64;
  bool phase_swap = false;
};

struct SegmentDesc {  // cache/mod.rs:100-118
  size_t segment_index, frame_start, frame_count, image_tokens, text_tokens;
  long long action_start;
  size_t len() const { return image_tokens + text_tokens; }
};

struct Layout {  // cache/mod.rs:61-75
  size_t segment_index, video_start, video_end, text_start, text_end;
  long long action_start;
};

struct Metrics {  // cache/mod.rs:133-151
  size_t archived_segments = 0, archived_bytes = 0, encode_calls = 0, d2h_bytes = 0, h2d_bytes = 0, rebuilds = 0,
         evicted_tokens = 0, rollbacks = 0;
};

struct Archived {  // history.rs:25-55
  size_t segment_index, frame_start, frame_count, image_tokens, text_tokens;
  long long action_start;
  std::vector<float> fk, fv;  // FLOATING: model-dtype values
  Int8Block i8;               // INT8
  QvgPayload qk, qv;          // QVG video
  bool has_text = false;
  Int8Block text;             // QVG text
  DenseRecord dense() const { return {segment_index, frame_start, frame_count, image_tokens, text_tokens}; }
};

struct HistoryCache {  // history.rs:84-100 plus the phase_swap.rs:27-40 wrapper
  CacheConfig cfg;
  size_t B, H, D;
  int dtype;
  std::vector<Archived> archive;
  bool has_ws = false;
  std::vector<float> ws_k, ws_v;
  std::vector<Layout> ws_layout;
  size_t valid_len = 0, total_frames = 0, tokens_per_frame = 0;
  Metrics metrics;
  QvgCodec qvg;
  // phase swap state (phase_swap.rs:19-25)
  bool parked = false;
  std::vector<float> pk, pv;
  std::vector<Layout> p_layout;
  size_t p_valid = 0, p_bytes = 0;

  // history.rs:104-156
  HistoryCache(const CacheConfig& c, size_t b, size_t h, size_t d, int dt) : cfg(c), B(b), H(h), D(d), dtype(dt) {
    if (cfg.storage == QVG) {
      if (B != 1) fail(ERR_INVALID_CONFIG, "QVG storage requires batch=1 (interactive world-model sessions)");
      if (cfg.qvg.bits == 0 || cfg.qvg.bits > 8 || cfg.qvg.stages == 0)
        fail(ERR_INVALID_CONFIG, "invalid QVG stages/bits");
    }
    if (cfg.sampling == TEMPORAL && (!std::isfinite(cfg.gamma) || cfg.gamma <= 0.0))
      fail(ERR_INVALID_CONFIG, "invalid temporal_context gamma " + rust_display(cfg.gamma));
    if (cfg.has_capacity && cfg.capacity == 0) fail(ERR_INVALID_CONFIG, "cache capacity must be > 0");
    if (cfg.past_frames == 0) fail(ERR_INVALID_CONFIG, "past_frames must be > 0");
    qvg.cfg = cfg.qvg, qvg.H = H, qvg.D = D;
  }

  size_t capacity_or_max() const { return cfg.has_capacity ? cfg.capacity : SIZE_MAX; }

  // history.rs:168-238 (k/v shapes and dtypes are implied by the desc here)
  void validate_segment(const SegmentDesc& s) {
    if (s.frame_count == 0 || s.image_tokens == 0) fail(ERR_GEOMETRY, "segment must contain at least one frame");
    size_t tpf = s.image_tokens / s.frame_count;
    if (s.image_tokens % s.frame_count != 0 || tpf == 0)
      fail(ERR_GEOMETRY, "image_tokens " + std::to_string(s.image_tokens) + " not divisible by frame_count " +
                             std::to_string(s.frame_count));
    if (tokens_per_frame == 0)
      tokens_per_frame = tpf;
    else if (tokens_per_frame != tpf)
      fail(ERR_GEOMETRY, "tokens_per_frame changed mid-session: " + std::to_string(tokens_per_frame) + " -> " +
                             std::to_string(tpf));
    if (!archive.empty()) {
      if (s.segment_index <= archive.back().segment_index)
        fail(ERR_CACHE_STATE, "history requires one chronological write per segment");
      if (s.frame_start != total_frames)
        fail(ERR_GEOMETRY, "segment frame_start " + std::to_string(s.frame_start) +
                               " does not continue the timeline at " + std::to_string(total_frames));
    } else if (s.frame_start != 0 && total_frames == 0) {
      fail(ERR_GEOMETRY, "first segment must start at frame 0, got " + std::to_string(s.frame_start));
    }
    if (s.action_start < -1 || s.action_start > (long long)s.text_tokens)
      fail(ERR_GEOMETRY, "action_start " + std::to_string(s.action_start) + " outside text block of " +
                             std::to_string(s.text_tokens));
  }

  // history.rs:241-305; k/v are f32 values of the input dtype `in_dt`.
  void archive_segment(const SegmentDesc& s, const float* k, const float* v, int in_dt) {
    size_t L = s.len(), n = B * L * H * D;
    Archived a{s.segment_index, s.frame_start, s.frame_count, s.image_tokens, s.text_tokens, s.action_start};
    size_t nbytes = 0;
    if (cfg.storage == FLOATING) {
      a.fk.resize(n), a.fv.resize(n);
      for (size_t i = 0; i < n; ++i) a.fk[i] = (dtype == F32) ? k[i] : round_to(dtype, k[i]);
      for (size_t i = 0; i < n; ++i) a.fv[i] = (dtype == F32) ? v[i] : round_to(dtype, v[i]);
      nbytes = 2 * n * dtype_size(dtype);
    } else if (cfg.storage == INT8) {
      std::vector<float> kb(n), vb(n);
      for (size_t i = 0; i < n; ++i) kb[i] = (in_dt == BF16) ? k[i] : round_to(BF16, k[i]);
      for (size_t i = 0; i < n; ++i) vb[i] = (in_dt == BF16) ? v[i] : round_to(BF16, v[i]);
      a.i8 = quantize_kv_pair(kb.data(), vb.data(), B, L, H, D);
      nbytes = a.i8.nbytes();
    } else {
      if (!qvg.fitted) qvg.fit(k, v, L);  // first segment, video + text (history.rs:257-262)
      a.qk = qvg.encode(0, k, L, s.image_tokens);
      a.qv = qvg.encode(1, v, L, s.image_tokens);
      if (s.text_tokens > 0) {
        size_t tn = s.text_tokens * H * D, off = s.image_tokens * H * D;
        std::vector<float> kt(tn), vt(tn);
        for (size_t i = 0; i < tn; ++i) kt[i] = round_to(BF16, k[off + i]);
        for (size_t i = 0; i < tn; ++i) vt[i] = round_to(BF16, v[off + i]);
        a.text = quantize_kv_pair(kt.data(), vt.data(), 1, s.text_tokens, H, D);
        a.has_text = true;
      }
      nbytes = a.qk.nbytes() + a.qv.nbytes() + (a.has_text ? a.text.nbytes() : 0);
    }
    metrics.encode_calls += (cfg.storage == FLOATING) ? 0 : 1;
    archive.push_back(std::move(a));
    metrics.archived_segments += 1;
    metrics.archived_bytes += nbytes;
    metrics.d2h_bytes += nbytes;
  }

  // history.rs:308-338 — whole segment back to model dtype, (B, L, H, D).
  void decode_segment(const Archived& a, std::vector<float>& k, std::vector<float>& v) const {
    size_t L = a.image_tokens + a.text_tokens;
    k.resize(B * L * H * D), v.resize(B * L * H * D);
    if (cfg.storage == FLOATING) {
      k = a.fk, v = a.fv;
    } else if (cfg.storage == INT8) {
      dequantize(a.i8.k.data(), a.i8.ks.data(), B, L, H, D, L, dtype, k.data());
      dequantize(a.i8.v.data(), a.i8.vs.data(), B, L, H, D, L, dtype, v.data());
    } else {
      qvg.decode(0, a.qk, k.data());
      qvg.decode(1, a.qv, v.data());
      size_t off = a.image_tokens * H * D;
      if (a.has_text) {
        dequantize(a.text.k.data(), a.text.ks.data(), 1, a.text_tokens, H, D, a.text_tokens, F32, k.data() + off);
        dequantize(a.text.v.data(), a.text.vs.data(), 1, a.text_tokens, H, D, a.text_tokens, F32, v.data() + off);
      }
      // Tensor::cat then to_dtype(model)
      size_t total = (a.image_tokens + (a.has_text ? a.text_tokens : 0)) * H * D;
      k.resize(total), v.resize(total);
      for (auto& x : k) x = round_to(dtype, x);
      for (auto& x : v) x = round_to(dtype, x);
    }
  }

  // history.rs:341-446
  void rebuild() {
    size_t tpf = std::max<size_t>(tokens_per_frame, 1);
    std::vector<std::pair<size_t, std::vector<size_t>>> selection;
    if (cfg.sampling == RECENT) {
      std::vector<DenseRecord> recs;
      for (auto& a : archive) recs.push_back(a.dense());
      TrimPlan plan = plan_recent_trim(recs, capacity_or_max(), tpf);
      metrics.evicted_tokens += plan.evicted_tokens;
      for (auto& r : apply_trim(recs, plan, tpf)) {
        size_t idx = 0;
        for (size_t i = 0; i < archive.size(); ++i)
          if (archive[i].segment_index == r.segment_index) {
            idx = i;
            break;
          }
        std::vector<size_t> frames;
        for (size_t f = 0; f < r.frame_count; ++f) frames.push_back(f);
        selection.push_back({idx, frames});
      }
    } else {
      std::vector<size_t> ids = history_frame_indices(total_frames, cfg.past_frames, cfg.sampling, cfg.gamma);
      for (size_t idx = 0; idx < archive.size(); ++idx) {
        const Archived& a = archive[idx];
        std::vector<size_t> sel;
        for (size_t f : ids)
          if (a.frame_start <= f && f < a.frame_start + a.frame_count) sel.push_back(f - a.frame_start);
        if (!sel.empty()) selection.push_back({idx, sel});
      }
    }
    std::vector<Layout> layout;
    const size_t ns = selection.size();
    std::vector<std::vector<float>> kp(ns), vp(ns);
    std::vector<size_t> part_len(ns);
    // per represented segment: decode the whole segment (the reference,
    // history.rs:398), then index_select its selected frames and text
    parallel_for(ns, [&](size_t p) {
      const auto& [idx, sel] = selection[p];
      const Archived& a = archive[idx];
      std::vector<size_t> indices;
      for (size_t f : sel)
        for (size_t t = f * tpf; t < f * tpf + tpf; ++t) indices.push_back(t);
      for (size_t t = a.image_tokens; t < a.image_tokens + a.text_tokens; ++t) indices.push_back(t);
      std::vector<float> dk, dv;
      decode_segment(a, dk, dv);
      size_t HD = H * D, n = indices.size();
      std::vector<float> k(B * n * HD), v(B * n * HD);
      size_t Ld = dk.size() / (B * HD);
      for (size_t b = 0; b < B; ++b)
        for (size_t j = 0; j < n; ++j) {
          std::memcpy(&k[(b * n + j) * HD], &dk[(b * Ld + indices[j]) * HD], HD * 4);
          std::memcpy(&v[(b * n + j) * HD], &dv[(b * Ld + indices[j]) * HD], HD * 4);
        }
      kp[p] = std::move(k), vp[p] = std::move(v), part_len[p] = n;
    });
    size_t cursor = 0;
    for (const auto& [idx, sel] : selection) {
      const Archived& a = archive[idx];
      size_t video_end = cursor + sel.size() * tpf;
      size_t text_end = video_end + a.text_tokens;
      layout.push_back({a.segment_index, cursor, video_end, video_end, text_end, a.action_start});
      cursor = text_end;
    }
    if (cursor > capacity_or_max())
      fail(ERR_GEOMETRY, "history needs " + std::to_string(cursor) + " tokens; capacity is " +
                             std::to_string(capacity_or_max()));
    // Tensor::cat along dim 1 -> (B, cursor, H, D)
    size_t HD = H * D;
    std::vector<float> K(B * cursor * HD), V(B * cursor * HD);
    for (size_t b = 0; b < B; ++b) {
      size_t off = 0;
      for (size_t p = 0; p < kp.size(); ++p) {
        size_t n = part_len[p];
        std::memcpy(&K[(b * cursor + off) * HD], &kp[p][b * n * HD], n * HD * 4);
        std::memcpy(&V[(b * cursor + off) * HD], &vp[p][b * n * HD], n * HD * 4);
        off += n;
      }
    }
    metrics.h2d_bytes += cursor * B * H * D * dtype_size(dtype) * 2;
    ws_k = std::move(K), ws_v = std::move(V), has_ws = true;
    ws_layout = layout;
    valid_len = cursor;
    metrics.rebuilds += 1;
  }

  // history.rs:458-463 (through phase_swap.rs:103-105)
  void commit(const SegmentDesc& s, const float* k, const float* v, int in_dt) {
    validate_segment(s);
    archive_segment(s, k, v, in_dt);
    total_frames += s.frame_count;
    rebuild();
  }

  // history.rs:507-528
  void rollback() {
    if (cfg.sampling == RECENT)
      fail(ERR_CACHE_STATE, "recent-mode SWA does not support streaming rollback (use an archived sampling)");
    if (archive.empty()) fail(ERR_CACHE_STATE, "nothing to roll back");
    Archived last = std::move(archive.back());
    archive.pop_back();
    if (last.frame_start + last.frame_count != total_frames)
      fail(ERR_CACHE_STATE, "archive does not match the frame timeline");
    total_frames -= last.frame_count;
    metrics.archived_segments = metrics.archived_segments > 0 ? metrics.archived_segments - 1 : 0;
    rebuild();
    metrics.rollbacks += 1;
  }

  // history.rs:465-481 / phase_swap.rs:107-114
  void working_set(std::vector<float>& k, std::vector<float>& v) const {
    if (parked) fail(ERR_CACHE_STATE, "working set is parked; call unpark() before attention");
    if (has_ws) {
      k = ws_k, v = ws_v;
    } else {
      k.clear(), v.clear();
    }
  }
  const std::vector<Layout>& layout() const { return parked ? p_layout : ws_layout; }
  size_t valid() const { return parked ? p_valid : valid_len; }

  // phase_swap.rs:42-66 (only when cfg.phase_swap; otherwise the trait default no-op)
  void park() {
    if (!cfg.phase_swap || parked) return;
    std::vector<float> k, v;
    working_set(k, v);
    p_layout = ws_layout;
    p_valid = valid_len;
    p_bytes = 2 * B * valid_len * H * D * dtype_size(dtype);
    pk = std::move(k), pv = std::move(v);
    has_ws = false, ws_k.clear(), ws_v.clear(), ws_layout.clear(), valid_len = 0;  // release_working_set
    metrics.d2h_bytes += p_bytes;
    parked = true;
  }
  // phase_swap.rs:69-81
  void unpark() {
    if (!cfg.phase_swap || !parked) return;
    ws_k = std::move(pk), ws_v = std::move(pv), has_ws = true;  // restore_working_set
    ws_layout = p_layout;
    valid_len = p_valid;
    metrics.h2d_bytes += p_bytes;
    parked = false;
  }
};

// cache/mod.rs:225-320
struct KvBank {
  std::vector<std::unique_ptr<HistoryCache>> layers;
  size_t B, H, D;
  int dtype;
};

}  // namespace orc

// ================================================================ C API =====
using namespace orc;

extern "C" {

typedef struct {
  int32_t storage;
  int32_t qvg_stages, qvg_bits, qvg_block, qvg_text_as_int8;
  uint64_t qvg_seed;
  int32_t sampling;
  double gamma;
  int32_t has_capacity;
  uint64_t capacity;
  uint64_t past_frames;
  int32_t phase_swap;
} orc_config;

typedef struct {
  uint64_t segment_index, frame_start, frame_count, image_tokens, text_tokens;
  int64_t action_start;
} orc_segment;

typedef struct {
  uint64_t segment_index, video_start, video_end, text_start, text_end;
  int64_t action_start;
} orc_layout;

typedef struct {
  uint64_t archived_segments, archived_bytes, encode_calls, d2h_bytes, h2d_bytes, rebuilds, evicted_tokens,
      rollbacks;
} orc_metrics;

const char* orc_last_error(void) { return g_last_error.c_str(); }
// Worker threads for the checker's independent loops (1 = sequential).
void orc_set_threads(int32_t n) { g_threads = n < 1 ? 1 : n; }

#define ORC_TRY(...)                          \
  try {                                       \
    __VA_ARGS__;                              \
    return OK;                                \
  } catch (const Error& e) {                  \
    g_last_error = e.msg;                     \
    return e.code;                            \
  } catch (const std::exception& e) {         \
    g_last_error = e.what();                  \
    return ERR_MSG;                           \
  }

static CacheConfig to_cfg(const orc_config* c) {
  CacheConfig cfg;
  cfg.storage = c->storage;
  cfg.qvg.stages = size_t(c->qvg_stages), cfg.qvg.bits = size_t(c->qvg_bits), cfg.qvg.block = size_t(c->qvg_block);
  cfg.qvg.text_as_int8 = c->qvg_text_as_int8 != 0, cfg.qvg.seed = c->qvg_seed;
  cfg.sampling = c->sampling, cfg.gamma = c->gamma;
  cfg.has_capacity = c->has_capacity != 0, cfg.capacity = size_t(c->capacity);
  cfg.past_frames = size_t(c->past_frames), cfg.phase_swap = c->phase_swap != 0;
  return cfg;
}
static SegmentDesc to_seg(const orc_segment* s) {
  return {size_t(s->segment_index), size_t(s->frame_start), size_t(s->frame_count), size_t(s->image_tokens),
          size_t(s->text_tokens), (long long)s->action_start};
}
static void fill_metrics(const Metrics& m, orc_metrics* o) {
  o->archived_segments = m.archived_segments, o->archived_bytes = m.archived_bytes;
  o->encode_calls = m.encode_calls, o->d2h_bytes = m.d2h_bytes, o->h2d_bytes = m.h2d_bytes;
  o->rebuilds = m.rebuilds, o->evicted_tokens = m.evicted_tokens, o->rollbacks = m.rollbacks;
}
static HistoryCache& layer_of(void* bank, uint64_t layer) {
  KvBank* b = static_cast<KvBank*>(bank);
  if (layer >= b->layers.size()) fail(ERR_ARGUMENT, "layer out of range");
  return *b->layers[layer];
}

// cache/mod.rs:231-244 + build_cache (mod.rs:208-222)
int orc_bank_create(const orc_config* c, uint64_t n_layers, uint64_t batch, uint64_t heads, uint64_t head_dim,
                    int32_t dtype, void** out) {
  ORC_TRY({
    auto* b = new KvBank();
    b->B = batch, b->H = heads, b->D = head_dim, b->dtype = dtype;
    try {
      for (uint64_t i = 0; i < n_layers; ++i)
        b->layers.emplace_back(new HistoryCache(to_cfg(c), batch, heads, head_dim, dtype));
    } catch (...) {
      delete b;
      throw;
    }
    *out = b;
  })
}
void orc_bank_destroy(void* bank) { delete static_cast<KvBank*>(bank); }

// cache/mod.rs:257-268.  k[i], v[i] are raw (B, L, H, D) buffers of in_dtype
// for layer i.  With nthreads > 1 the layers run concurrently (they are
// independent caches); the first failing layer's error is returned.
int orc_bank_commit(void* bank, const orc_segment* seg, int32_t in_dtype, const void* const* k, const void* const* v,
                    int32_t nthreads) {
  ORC_TRY({
    KvBank* b = static_cast<KvBank*>(bank);
    SegmentDesc s = to_seg(seg);
    size_t n = b->B * s.len() * b->H * b->D;
    size_t nl = b->layers.size();
    auto run = [&](size_t i) {
      std::vector<float> kf(n), vf(n);
      load_raw(k[i], in_dtype, n, kf.data());
      load_raw(v[i], in_dtype, n, vf.data());
      b->layers[i]->commit(s, kf.data(), vf.data(), in_dtype);
    };
    if (nthreads <= 1 || nl <= 1) {
      for (size_t i = 0; i < nl; ++i) run(i);
    } else {
      std::vector<int> codes(nl, OK);
      std::vector<std::string> msgs(nl);
      std::atomic<size_t> next{0};
      std::vector<std::thread> th;
      for (int t = 0; t < nthreads; ++t)
        th.emplace_back([&]() {
          for (size_t i = next++; i < nl; i = next++) {
            try {
              run(i);
            } catch (const Error& e) {
              codes[i] = e.code, msgs[i] = e.msg;
            }
          }
        });
      for (auto& t : th) t.join();
      for (size_t i = 0; i < nl; ++i)
        if (codes[i] != OK) fail(codes[i], msgs[i]);
    }
  })
}

int orc_bank_rollback(void* bank) {
  ORC_TRY({
    for (auto& l : static_cast<KvBank*>(bank)->layers) l->rollback();
  })
}
int orc_bank_park(void* bank) {
  ORC_TRY({
    for (auto& l : static_cast<KvBank*>(bank)->layers) l->park();
  })
}
int orc_bank_unpark(void* bank) {
  ORC_TRY({
    for (auto& l : static_cast<KvBank*>(bank)->layers) l->unpark();
  })
}
// cache/mod.rs:305-319
int orc_bank_metrics(void* bank, orc_metrics* out) {
  ORC_TRY({
    Metrics m;
    for (auto& l : static_cast<KvBank*>(bank)->layers) {
      const Metrics& c = l->metrics;
      m.archived_segments = std::max(m.archived_segments, c.archived_segments);
      m.archived_bytes += c.archived_bytes;
      m.encode_calls += c.encode_calls;
      m.d2h_bytes += c.d2h_bytes;
      m.h2d_bytes += c.h2d_bytes;
      m.rebuilds = std::max(m.rebuilds, c.rebuilds);
      m.evicted_tokens = std::max(m.evicted_tokens, c.evicted_tokens);
      m.rollbacks = std::max(m.rollbacks, c.rollbacks);
    }
    fill_metrics(m, out);
  })
}
int orc_cache_metrics(void* bank, uint64_t layer, orc_metrics* out) {
  ORC_TRY({ fill_metrics(layer_of(bank, layer).metrics, out); })
}
// out = {valid_len, capacity, n_segments, total_frames, tokens_per_frame, parked}
int orc_cache_info(void* bank, uint64_t layer, uint64_t* out) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    out[0] = c.valid(), out[1] = c.capacity_or_max(), out[2] = c.archive.size();
    out[3] = c.total_frames, out[4] = c.tokens_per_frame, out[5] = c.parked ? 1 : 0;
  })
}
int orc_cache_layout(void* bank, uint64_t layer, orc_layout* out, uint64_t cap, uint64_t* n) {
  ORC_TRY({
    const auto& lay = layer_of(bank, layer).layout();
    *n = lay.size();
    for (size_t i = 0; i < lay.size() && i < cap; ++i)
      out[i] = {lay[i].segment_index, lay[i].video_start, lay[i].video_end, lay[i].text_start, lay[i].text_end,
                (int64_t)lay[i].action_start};
  })
}
// Raw model-dtype (B, valid_len, H, D) copies of the working set.
int orc_cache_working_set(void* bank, uint64_t layer, void* k_out, void* v_out) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    std::vector<float> k, v;
    c.working_set(k, v);
    store_raw(k.data(), c.dtype, k.size(), k_out);
    store_raw(v.data(), c.dtype, v.size(), v_out);
  })
}
// history.rs:308-338 for archive position `pos`: raw model dtype, whole segment.
int orc_cache_decode_segment(void* bank, uint64_t layer, uint64_t pos, void* k_out, void* v_out, uint64_t* tokens) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    if (pos >= c.archive.size()) fail(ERR_ARGUMENT, "archive position out of range");
    std::vector<float> k, v;
    c.decode_segment(c.archive[pos], k, v);
    *tokens = k.size() / (c.B * c.H * c.D);
    if (k_out) store_raw(k.data(), c.dtype, k.size(), k_out);
    if (v_out) store_raw(v.data(), c.dtype, v.size(), v_out);
  })
}
// Archived INT8 payload (INT8 storage: the whole segment; QVG: the text block).
int orc_cache_archive_int8(void* bank, uint64_t layer, uint64_t pos, uint8_t* kq, uint8_t* vq, float* ks,
                           float* vs) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    if (pos >= c.archive.size()) fail(ERR_ARGUMENT, "archive position out of range");
    const Archived& a = c.archive[pos];
    const Int8Block* blk = c.cfg.storage == INT8 ? &a.i8 : (c.cfg.storage == QVG && a.has_text ? &a.text : nullptr);
    if (!blk) fail(ERR_ARGUMENT, "segment has no int8 payload");
    std::memcpy(kq, blk->k.data(), blk->k.size());
    std::memcpy(vq, blk->v.data(), blk->v.size());
    std::memcpy(ks, blk->ks.data(), blk->ks.size() * 4);
    std::memcpy(vs, blk->vs.data(), blk->vs.size() * 4);
  })
}
int orc_cache_archive_qvg(void* bank, uint64_t layer, uint64_t pos, uint8_t* kc, uint8_t* vc, float* ksc,
                          float* vsc) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    if (pos >= c.archive.size() || c.cfg.storage != QVG) fail(ERR_ARGUMENT, "no qvg payload");
    const Archived& a = c.archive[pos];
    std::memcpy(kc, a.qk.codes.data(), a.qk.codes.size());
    std::memcpy(vc, a.qv.codes.data(), a.qv.codes.size());
    std::memcpy(ksc, a.qk.scales.data(), a.qk.scales.size() * 4);
    std::memcpy(vsc, a.qv.scales.data(), a.qv.scales.size() * 4);
  })
}
int orc_cache_codebooks(void* bank, uint64_t layer, float* out, int32_t* fitted) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    *fitted = c.qvg.fitted ? 1 : 0;
    if (c.qvg.fitted && out) std::memcpy(out, c.qvg.cb.data(), c.qvg.cb.size() * 4);
  })
}
// QvgCodec::with_codebooks (qvg.rs:101-104) on one layer.
int orc_cache_set_codebooks(void* bank, uint64_t layer, const float* cb) {
  ORC_TRY({
    HistoryCache& c = layer_of(bank, layer);
    if (c.cfg.storage != QVG) fail(ERR_CACHE_STATE, "cache does not use QVG storage");
    size_t n = 2 * c.H * c.cfg.qvg.stages * c.cfg.qvg.entries() * c.D;
    c.qvg.cb.assign(cb, cb + n);
    c.qvg.fitted = true;
  })
}
// Benchmark setup shortcut: append `count` copies of the newest archived
// segment (consecutive segment indices and frames) to every layer, with the
// metrics a real commit would add, without quantizing or rebuilding.
int orc_bank_prefill_clone(void* bank, uint64_t count) {
  ORC_TRY({
    for (auto& lp : static_cast<KvBank*>(bank)->layers) {
      HistoryCache& c = *lp;
      if (c.archive.empty()) fail(ERR_CACHE_STATE, "nothing to clone");
      for (uint64_t i = 0; i < count; ++i) {
        Archived a = c.archive.back();
        a.segment_index += 1;
        a.frame_start = c.total_frames;
        size_t nb = c.cfg.storage == FLOATING ? 2 * a.fk.size() * dtype_size(c.dtype)
                    : c.cfg.storage == INT8   ? a.i8.nbytes()
                                              : a.qk.nbytes() + a.qv.nbytes() + (a.has_text ? a.text.nbytes() : 0);
        c.total_frames += a.frame_count;
        c.archive.push_back(std::move(a));
        c.metrics.encode_calls += c.cfg.storage == FLOATING ? 0 : 1;
        c.metrics.archived_segments += 1, c.metrics.archived_bytes += nb, c.metrics.d2h_bytes += nb;
      }
    }
  })
}

// ------------------------------------------------------- free functions ---
int orc_quantize_kv_pair(const void* k, const void* v, int32_t dtype, uint64_t B, uint64_t L, uint64_t H,
                         uint64_t D, uint8_t* kq, uint8_t* vq, float* ks, float* vs) {
  ORC_TRY({
    size_t n = B * L * H * D;
    std::vector<float> kf(n), vf(n);
    load_raw(k, dtype, n, kf.data());
    load_raw(v, dtype, n, vf.data());
    Int8Block blk = quantize_kv_pair(kf.data(), vf.data(), B, L, H, D);
    std::memcpy(kq, blk.k.data(), n), std::memcpy(vq, blk.v.data(), n);
    std::memcpy(ks, blk.ks.data(), blk.ks.size() * 4), std::memcpy(vs, blk.vs.data(), blk.vs.size() * 4);
  })
}
int orc_dequantize(const uint8_t* q, const float* s, uint64_t B, uint64_t L, uint64_t H, uint64_t D, uint64_t valid,
                   int32_t dtype, void* out) {
  ORC_TRY({
    std::vector<float> o(B * valid * H * D);
    dequantize(q, s, B, L, H, D, valid, dtype, o.data());
    store_raw(o.data(), dtype, o.size(), out);
  })
}
static QvgCodec make_codec(uint64_t H, uint64_t D, uint64_t stages, uint64_t bits, uint64_t block, uint64_t seed) {
  QvgCodec c;
  c.cfg.stages = stages, c.cfg.bits = bits, c.cfg.block = block, c.cfg.seed = seed;
  c.H = H, c.D = D;
  return c;
}
// QvgCodec::fit over (1, L, H, D) f32 k and v; cb_out = [2][H][stages][entries][D].
int orc_qvg_fit(const float* k, const float* v, uint64_t L, uint64_t H, uint64_t D, uint64_t stages, uint64_t bits,
                uint64_t seed, float* cb_out) {
  ORC_TRY({
    QvgCodec c = make_codec(H, D, stages, bits, 64, seed);
    c.fit(k, v, L);
    std::memcpy(cb_out, c.cb.data(), c.cb.size() * 4);
  })
}
int orc_qvg_encode(const float* cb, int32_t side, const float* t, uint64_t L, uint64_t H, uint64_t D,
                   uint64_t tokens, uint64_t stages, uint64_t bits, uint64_t block, uint8_t* codes, float* scales) {
  ORC_TRY({
    QvgCodec c = make_codec(H, D, stages, bits, block, 0);
    c.cb.assign(cb, cb + 2 * H * stages * (size_t(1) << bits) * D);
    c.fitted = true;
    QvgPayload p = c.encode(size_t(side), t, L, tokens);
    std::memcpy(codes, p.codes.data(), p.codes.size());
    std::memcpy(scales, p.scales.data(), p.scales.size() * 4);
  })
}
int orc_qvg_decode(const float* cb, int32_t side, const uint8_t* codes, const float* scales, uint64_t tokens,
                   uint64_t H, uint64_t D, uint64_t stages, uint64_t bits, uint64_t block, float* out) {
  ORC_TRY({
    QvgCodec c = make_codec(H, D, stages, bits, block, 0);
    c.cb.assign(cb, cb + 2 * H * stages * (size_t(1) << bits) * D);
    c.fitted = true;
    QvgPayload p;
    p.heads = H, p.head_dim = D, p.tokens = tokens, p.n_blocks = (tokens + block - 1) / block;
    p.codes.assign(codes, codes + tokens * H * c.cfg.bpt());
    p.scales.assign(scales, scales + H * p.n_blocks * stages);
    c.decode(size_t(side), p, out);
  })
}
int orc_pack_bits(uint8_t* buf, uint64_t bit_off, uint64_t bits, uint64_t value) {
  pack_bits(buf, bit_off, bits, value);
  return OK;
}
uint64_t orc_unpack_bits(const uint8_t* buf, uint64_t bit_off, uint64_t bits) {
  return unpack_bits(buf, bit_off, bits);
}
uint64_t orc_qvg_payload_bytes(uint64_t tokens, uint64_t heads, uint64_t stages, uint64_t bits, uint64_t block) {
  QvgConfig q;
  q.stages = stages, q.bits = bits, q.block = block;
  return q.payload_bytes(tokens, heads);
}

// Samplers: kind 0 = uniform, 1 = recent_mix, 2 = temporal (raw functions),
// 3 = history_frame_indices(sampling) with validation.
int orc_frame_indices(int32_t kind, uint64_t total, uint64_t past, int32_t sampling, double gamma, uint64_t* out,
                      uint64_t cap, uint64_t* n) {
  ORC_TRY({
    std::vector<size_t> ids;
    if (kind == 0) ids = uniform_frame_indices(total, past);
    else if (kind == 1) ids = recent_mix_uniform_frame_indices(total, past);
    else if (kind == 2) ids = temporal_context_frame_indices(total, past, gamma);
    else ids = history_frame_indices(total, past, sampling, gamma);
    *n = ids.size();
    for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  })
}
// recs: n x {segment_index, frame_start, frame_count, image_tokens, text_tokens}.
// Outputs the plan, then the records surviving apply_trim (kept: n x 5).
int orc_plan_recent_trim(const uint64_t* recs, uint64_t n, uint64_t capacity, uint64_t tpf, uint64_t* drop_frames,
                         uint64_t* n_df, uint64_t* drop_records, uint64_t* n_dr, uint64_t* evicted, uint64_t* kept,
                         uint64_t* n_kept) {
  ORC_TRY({
    std::vector<DenseRecord> rs;
    for (uint64_t i = 0; i < n; ++i)
      rs.push_back({recs[i * 5], recs[i * 5 + 1], recs[i * 5 + 2], recs[i * 5 + 3], recs[i * 5 + 4]});
    TrimPlan p = plan_recent_trim(rs, capacity, tpf);
    *n_df = p.drop_frames.size();
    for (size_t i = 0; i < p.drop_frames.size(); ++i)
      drop_frames[2 * i] = p.drop_frames[i].first, drop_frames[2 * i + 1] = p.drop_frames[i].second;
    *n_dr = p.drop_records.size();
    for (size_t i = 0; i < p.drop_records.size(); ++i) drop_records[i] = p.drop_records[i];
    *evicted = p.evicted_tokens;
    auto k = apply_trim(rs, p, tpf);
    *n_kept = k.size();
    for (size_t i = 0; i < k.size(); ++i) {
      kept[i * 5] = k[i].segment_index, kept[i * 5 + 1] = k[i].frame_start, kept[i * 5 + 2] = k[i].frame_count;
      kept[i * 5 + 3] = k[i].image_tokens, kept[i * 5 + 4] = k[i].text_tokens;
    }
  })
}

// tensor_utils.rs:114-138
void orc_randn(uint64_t n, uint64_t seed, double mean, double stdv, float* out) { randn(n, seed, mean, stdv, out); }
uint64_t orc_splitmix_next(uint64_t* state) {
  SplitMix64 r(*state);
  uint64_t v = r.next_u64();
  *state = r.state;
  return v;
}
uint16_t orc_bf16_bits(float x) { return bf16_bits(x); }
uint16_t orc_f16_bits(float x) { return f16_bits(x); }

// The captured K / V of one layer (batch 1), the producer side of a commit:
//   Lin (modules/mod.rs:122-142): bf16 result of x W^T, then + bias in bf16;
//   RmsNorm on K (modules/attention.rs:117-122, modules/norm.rs:55-65) when
//     qk_norm: f32 mean of squares over the head dim, (var + eps)^-1/2, times
//     the optional gain, to bf16;
//   apply_rotary on K (attention.rs:144, rope.rs:257-306) when cos/sin are
//     given: interleaved pairs, r*c - i*s and i*c + r*s in f32, to bf16.
// The matrix product is accumulated in f64 and rounded to f32 before the
// bf16 rounding (exact whenever every partial sum is, which the bit-exact
// tests arrange); squares are summed as four interleaved partial sums
// (d mod 4) added as (s0 + s1) + (s2 + s3), and (var + eps)^-1/2 is
// 1 / sqrt(var + eps) with IEEE square root and division — the order and the
// operations the device epilogue uses (the reference leaves the reduction
// order to candle and uses powf).
int orc_kv_project(const uint16_t* x, const uint16_t* wk, const uint16_t* bk, const uint16_t* wv,
                   const uint16_t* bv, const uint16_t* k_gain, int32_t qk_norm, float eps, const float* cos_t,
                   const float* sin_t, uint64_t M, uint64_t H, uint64_t D, uint16_t* k_out, uint16_t* v_out) {
  const uint64_t dim = H * D;
  std::vector<float> xf(M * dim), wf(dim * dim), row(dim);
  for (uint64_t i = 0; i < M * dim; ++i) xf[i] = bf16_value(x[i]);
  for (int side = 0; side < 2; ++side) {
    const uint16_t* w = side ? wv : wk;
    const uint16_t* b = side ? bv : bk;
    uint16_t* out = side ? v_out : k_out;
    for (uint64_t i = 0; i < dim * dim; ++i) wf[i] = bf16_value(w[i]);
    for (uint64_t t = 0; t < M; ++t) {
      for (uint64_t n = 0; n < dim; ++n) {
        double acc = 0.0;
        const float* xr = &xf[t * dim];
        const float* wr = &wf[n * dim];
        for (uint64_t k = 0; k < dim; ++k) acc += double(xr[k]) * double(wr[k]);
        float y = bf16_value(bf16_bits(float(acc)));
        if (b) y = bf16_value(bf16_bits(y + bf16_value(b[n])));
        row[n] = y;
      }
      for (uint64_t h = 0; h < H; ++h) {
        float* y = &row[h * D];
        if (side == 0 && qk_norm) {
          float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (uint64_t d = 0; d < D; ++d) {
            const float sq = y[d] * y[d];
            s[d & 3] = s[d & 3] + sq;
          }
          const float ss = (s[0] + s[1]) + (s[2] + s[3]);
          const float var = ss * (1.0f / float(D));
          const float root = std::sqrt(var + eps);
          const float inv = 1.0f / root;
          for (uint64_t d = 0; d < D; ++d) {
            float o = y[d] * inv;
            if (k_gain) o = o * bf16_value(k_gain[d]);
            y[d] = bf16_value(bf16_bits(o));
          }
        }
        if (side == 0 && cos_t) {
          for (uint64_t j = 0; j < D / 2; ++j) {
            const float c = cos_t[t * (D / 2) + j], sn = sin_t[t * (D / 2) + j];
            const float xr = y[2 * j], xi = y[2 * j + 1];
            const float a = xr * c, bb = xi * sn, e = xi * c, f = xr * sn;
            y[2 * j] = bf16_value(bf16_bits(a - bb));
            y[2 * j + 1] = bf16_value(bf16_bits(e + f));
          }
        }
      }
      for (uint64_t n = 0; n < dim; ++n) out[t * dim + n] = bf16_bits(row[n]);
    }
  }
  return OK;
}

}  // extern "C"
