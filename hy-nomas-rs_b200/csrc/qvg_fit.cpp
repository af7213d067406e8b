// qvg_fit.cpp — one-time QVG codebook fit on the host (cache/qvg.rs:130-167,
// 351-442): per (side, head), `stages` rounds of seeded farthest-point
// initialisation, two Lloyd iterations with f64 sums in token order, and
// subtraction of each token's nearest entry.  Runs once per cache, on the
// first committed segment (history.rs:256-262), across all host threads.
//
// Compiled with -ffp-contract=off: every f64 / f32 operation rounds where
// the reference's does.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

#include "nkv_qvg_fit.h"

namespace nkv {
namespace {

// SplitMix64 stream (tensor_utils.rs:65-95).
struct Rng {
  uint64_t state;
  uint64_t next() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double uniform() { return double(next() >> 11) * (1.0 / 9007199254740992.0); }
};

// Index of the entry of `cb` (E x D) nearest to x: sequential f64 squared
// distance, strict less-than so ties keep the lower index (qvg.rs:303-321).
// The reference's early exit (stop once the partial sum reaches the best)
// cannot change the answer because partial sums never decrease.
size_t nearest_entry(const float* cb, size_t E, size_t D, const float* x) {
  size_t best = 0;
  double best_d = std::numeric_limits<double>::infinity();
  for (size_t e = 0; e < E; ++e) {
    const float* c = cb + e * D;
    double acc = 0.0;
    for (size_t d = 0; d < D; ++d) {
      const double diff = double(x[d]) - double(c[d]);
      acc += diff * diff;
      if (acc >= best_d) break;
    }
    if (acc < best_d) {
      best_d = acc;
      best = e;
    }
  }
  return best;
}

// farthest_point_init (qvg.rs:396-442): E rows chosen from `rows` (n x D).
void seed_entries(const std::vector<float>& rows, size_t n, size_t D, size_t E, Rng& rng, float* out) {
  if (n == 0 || D == 0) {
    std::fill(out, out + E * D, 0.0f);
    return;
  }
  size_t have = 0;
  const size_t first = size_t(rng.uniform() * double(n)) % n;
  std::memcpy(out, rows.data() + first * D, D * sizeof(float));
  have = 1;
  std::vector<double> dmin(n, std::numeric_limits<double>::infinity());
  while (have < E) {
    const float* last = out + (have - 1) * D;
    double total = 0.0;
    for (size_t i = 0; i < n; ++i) {
      const float* r = rows.data() + i * D;
      double dd = 0.0;
      for (size_t d = 0; d < D; ++d) {
        const double diff = double(r[d]) - double(last[d]);
        dd += diff * diff;
      }
      if (dd < dmin[i]) dmin[i] = dd;
      total += dmin[i];
    }
    if (total <= 1e-12) {
      // every point already coincides with an entry: jitter a copy of the first
      std::memcpy(out + have * D, out, D * sizeof(float));
      out[have * D] += float(have) * 1e-3f;
      ++have;
      continue;
    }
    double pick = rng.uniform() * total;
    size_t idx = n - 1;
    for (size_t i = 0; i < n; ++i) {
      pick -= dmin[i];
      if (pick <= 0.0) {
        idx = i;
        break;
      }
    }
    std::memcpy(out + have * D, rows.data() + idx * D, D * sizeof(float));
    ++have;
  }
}

}  // namespace

// fit_head_codebooks (qvg.rs:351-394).  mat: n x D f32; out: stages x E x D.
void qvg_fit_head(const float* mat, size_t n, size_t D, int stages, int E, uint64_t seed, float* out) {
  std::vector<float> res(mat, mat + n * D);
  Rng rng{seed};
  std::vector<double> sums;
  std::vector<size_t> counts;
  for (int s = 0; s < stages; ++s) {
    float* cb = out + size_t(s) * E * D;
    seed_entries(res, n, D, size_t(E), rng, cb);
    for (int it = 0; it < 2; ++it) {
      sums.assign(size_t(E) * D, 0.0);
      counts.assign(size_t(E), 0);
      for (size_t i = 0; i < n; ++i) {
        const float* r = res.data() + i * D;
        const size_t c = nearest_entry(cb, size_t(E), D, r);
        counts[c] += 1;
        double* sc = sums.data() + c * D;
        for (size_t d = 0; d < D; ++d) sc[d] += double(r[d]);
      }
      for (size_t c = 0; c < size_t(E); ++c)
        if (counts[c] > 0)
          for (size_t d = 0; d < D; ++d) cb[c * D + d] = float(sums[c * D + d] / double(counts[c]));
    }
    for (size_t i = 0; i < n; ++i) {
      float* r = res.data() + i * D;
      const float* c = cb + nearest_entry(cb, size_t(E), D, r) * D;
      for (size_t d = 0; d < D; ++d) r[d] -= c[d];
    }
  }
}

// QvgCodec::fit for one layer: k and v are (L, H, D) f32; out is
// [2][H][stages][E][D].  Head h of both sides uses seed + h (qvg.rs:159).
void qvg_fit_layer(const float* k, const float* v, size_t L, size_t H, size_t D, int stages, int E, uint64_t seed,
                   float* out, int threads) {
  const size_t tasks = 2 * H;
  std::atomic<size_t> next{0};
  auto work = [&]() {
    std::vector<float> mat(L * D);
    for (size_t t = next++; t < tasks; t = next++) {
      const size_t side = t / H, h = t % H;
      const float* src = side == 0 ? k : v;
      for (size_t l = 0; l < L; ++l) std::memcpy(mat.data() + l * D, src + (l * H + h) * D, D * sizeof(float));
      qvg_fit_head(mat.data(), L, D, stages, E, seed + uint64_t(h), out + (side * H + h) * size_t(stages) * E * D);
    }
  };
  int nt = std::max(1, std::min<int>(threads, int(tasks)));
  std::vector<std::thread> pool;
  for (int i = 1; i < nt; ++i) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
}

}  // namespace nkv
