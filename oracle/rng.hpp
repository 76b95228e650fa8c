// ORACLE (test infrastructure only): counter RNG and procedural topology hashes,
// restated from the reference for the CPU checker.  Nothing in the product may
// include this file.
//
//   counter RNG ............ brian2-rust/src/executor.rs:190-336
//   topology hashes ........ brian2-rust/src/large_topology.rs:55-142, 189-260
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <unordered_set>
#include <vector>

namespace oracle {

// executor.rs:190-194
inline uint64_t mix64(uint64_t v) {
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

// executor.rs:196-203
inline double counter_uniform_draw(uint64_t seed, uint64_t stream, uint64_t tick, uint64_t index,
                                   uint64_t draw) {
  uint64_t counter = seed ^ (stream * 0x9e3779b97f4a7c15ull) ^ (tick * 0xd1b54a32d192ed03ull) ^
                     (index * 0x94d049bb133111ebull) ^ (draw * 0x369dea0f31a53f85ull);
  return double(mix64(counter) >> 11) * (1.0 / 9007199254740992.0);
}

inline double counter_uniform(uint64_t seed, uint64_t stream, uint64_t tick, uint64_t index) {
  return counter_uniform_draw(seed, stream, tick, index, 0);
}

// executor.rs:209-222, Marsaglia polar method on pair index/2.
inline double counter_normal(uint64_t seed, uint64_t stream, uint64_t tick, uint64_t index) {
  uint64_t pair = index / 2;
  uint64_t draw = 0;
  while (true) {
    double x1 = 2.0 * counter_uniform_draw(seed, stream, tick, pair, draw) - 1.0;
    double x2 = 2.0 * counter_uniform_draw(seed, stream, tick, pair, draw + 1) - 1.0;
    double radius = x1 * x1 + x2 * x2;
    if (radius < 1.0 && radius != 0.0) {
      double factor = std::sqrt(-2.0 * std::log(radius) / radius);
      return factor * ((index & 1) == 0 ? x1 : x2);
    }
    draw += 2;
  }
}

// executor.rs:224-268, inversion with restart past `bound`.
inline double counter_binomial(uint64_t seed, uint64_t stream, uint64_t tick, uint64_t index,
                               uint64_t n, double p, bool approximate) {
  if (p <= 0.0) return 0.0;
  if (p >= 1.0) return double(n);
  double nf = double(n);
  double loc = nf * p;
  double complement = nf * (1.0 - p);
  if (approximate && loc > 5.0 && complement > 5.0)
    return counter_normal(seed, stream, tick, index) * std::sqrt(loc * (1.0 - p)) + loc;
  bool reverse = p > 0.5;
  double probability = reverse ? 1.0 - p : p;
  double q = 1.0 - probability;
  double qn = std::exp(nf * std::log(q));
  double bound = std::fmin(nf, nf * probability + 10.0 * std::sqrt(nf * probability * q + 1.0));
  uint64_t draw = 0;
  while (true) {
    uint64_t x = 0;
    double px = qn;
    double u = counter_uniform_draw(seed, stream, tick, index, draw);
    bool restart = false;
    while (true) {
      if (u <= px) return double(reverse ? n - x : x);
      x += 1;
      if (double(x) > bound) {
        draw += 1;
        restart = true;
        break;
      }
      u -= px;
      px = (double(n - x + 1) * probability * px) / (double(x) * q);
    }
    if (!restart) break;
  }
  return 0.0;
}

// executor.rs:270-288, Lanczos approximation (g = 7, 8 terms).
inline double log_gamma_positive(double value) {
  // Decimal literals exactly as written in the reference source.
  static const double c[8] = {676.5203681218851,    -1259.1392167224028,
                              771.3234287776531,    -176.6150291621406,
                              12.507343278686905,   -0.13857109526572012,
                              9.984369578019572e-6, 1.5056327351493116e-7};
  double z = value - 1.0;
  double x = 0.9999999999998099;
  for (int i = 0; i < 8; ++i) x += c[i] / (z + double(i) + 1.0);
  double t = z + 7.5;
  return 0.9189385332046727 + (z + 0.5) * std::log(t) - t + std::log(x);
}

// executor.rs:290-336: Knuth product for lambda < 10, Hoermann PTRS above.
inline double counter_poisson(uint64_t seed, uint64_t stream, uint64_t tick, uint64_t index,
                              double lambda) {
  if (lambda == 0.0) return 0.0;
  if (!std::isfinite(lambda) || !(lambda >= 0.0 && lambda <= 1.0e12)) return NAN;
  if (lambda < 10.0) {
    double limit = std::exp(-lambda);
    double product = 1.0;
    uint64_t sample = 0;
    while (true) {
      product *= counter_uniform_draw(seed, stream, tick, index, sample);
      if (product <= limit) return double(sample);
      sample += 1;
    }
  }
  double root = std::sqrt(lambda);
  double b = 0.931 + 2.53 * root;
  double a = -0.059 + 0.02483 * b;
  double inverse_alpha = 1.1239 + 1.1328 / (b - 3.4);
  double squeeze = 0.9277 - 3.6224 / (b - 2.0);
  uint64_t draw = 0;
  while (true) {
    double u = counter_uniform_draw(seed, stream, tick, index, draw) - 0.5;
    double v = counter_uniform_draw(seed, stream, tick, index, draw + 1);
    draw += 2;
    double us = 0.5 - std::fabs(u);
    double candidate = std::floor((2.0 * a / us + b) * u + lambda + 0.43);
    if (us >= 0.07 && v <= squeeze) return candidate;
    if (candidate < 0.0 || (us < 0.013 && v > us)) continue;
    double left = std::log(v * inverse_alpha / (a / (us * us) + b));
    double right = -lambda + candidate * std::log(lambda) - log_gamma_positive(candidate + 1.0);
    if (left <= right) return candidate;
  }
}

// ---- procedural topology (large_topology.rs) ----

inline uint64_t topo_mix64(uint64_t v) {
  v += 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

inline uint64_t topo_draw(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  return topo_mix64(seed ^ (stream * 0xd2b74407b1ce6e93ull) ^ (edge * 0x9e3779b97f4a7c15ull) ^
                    (attempt * 0xca5a826395121157ull));
}

inline uint64_t topo_bounded(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t upper) {
  return uint64_t((unsigned __int128)topo_draw(seed, stream, edge, 0) * upper >> 64);
}

inline double topo_uniform_open(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  uint64_t mantissa = topo_draw(seed, stream, edge, attempt) >> 11;
  return (double(mantissa) + 0.5) * (1.0 / 9007199254740992.0);
}

inline double topo_normal(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  double u1 = topo_uniform_open(seed, stream, edge, attempt * 2);
  double u2 = topo_uniform_open(seed, stream + 1, edge, attempt * 2 + 1);
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// Floyd subset sampling for one target (large_topology.rs:189-208).  `selected`
// is any set of u64 with clear/count/insert (the reference uses a HashSet; the
// set's kind changes nothing but speed).
template <class Set, class Visit>
inline void fixed_indegree_sources(uint64_t source_count, uint64_t indegree, uint64_t target,
                                   uint64_t seed, Set& selected, Visit visit) {
  selected.clear();
  for (uint64_t candidate = source_count - indegree; candidate < source_count; ++candidate) {
    uint64_t logical = target * source_count + candidate;
    uint64_t draw = topo_bounded(seed, 0, logical, candidate + 1);
    uint64_t source = selected.count(draw) ? candidate : draw;
    selected.insert(source);
    visit(source);
  }
}

// Open-addressing set of at most `capacity` u64 keys for the Floyd sampler:
// cleared in O(1) by bumping a generation stamp (a target's selection never
// outlives the target).
class FloydSet {
 public:
  explicit FloydSet(uint64_t capacity) {
    uint64_t n = 16;
    while (n < 2 * capacity) n <<= 1;
    keys_.assign(n, 0);
    stamp_.assign(n, 0);
    mask_ = n - 1;
  }
  void clear() {
    if (++gen_ == 0) {
      std::fill(stamp_.begin(), stamp_.end(), 0u);
      gen_ = 1;
    }
  }
  size_t count(uint64_t k) const {
    for (uint64_t h = slot(k);; h = (h + 1) & mask_) {
      if (stamp_[h] != gen_) return 0;
      if (keys_[h] == k) return 1;
    }
  }
  void insert(uint64_t k) {
    for (uint64_t h = slot(k);; h = (h + 1) & mask_) {
      if (stamp_[h] != gen_) {
        stamp_[h] = gen_;
        keys_[h] = k;
        return;
      }
      if (keys_[h] == k) return;
    }
  }

 private:
  uint64_t slot(uint64_t k) const { return (k * 0x9e3779b97f4a7c15ull >> 17) & mask_; }
  std::vector<uint64_t> keys_;
  std::vector<uint32_t> stamp_;
  uint64_t mask_ = 0;
  uint32_t gen_ = 1;
};

}  // namespace oracle
