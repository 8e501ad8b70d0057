// seeded.cpp -- seeded synthetic weights and token ids for the runtime.
//
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11) keyed by the seed, counter = (element block,
// tensor stream, tag), and the Box-Muller transform in double precision.
// Every element depends only on (seed, stream, index), so generation is split
// across host threads without changing a bit.
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "runtime.h"

namespace gpt2 {

namespace {
constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u, kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
constexpr uint32_t kTag = 0x67707432u;  // "gpt2"

inline void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(kM0) * c[0];
    const uint64_t p1 = static_cast<uint64_t>(kM1) * c[2];
    const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c[3] ^ k1;
    c[1] = static_cast<uint32_t>(p1);
    c[3] = static_cast<uint32_t>(p0);
    c[0] = n0;
    c[2] = n2;
    k0 += kW0;
    k1 += kW1;
  }
}

inline void block_words(uint64_t seed, uint32_t stream, uint64_t block, uint32_t w[4]) {
  w[0] = static_cast<uint32_t>(block);
  w[1] = static_cast<uint32_t>(block >> 32);
  w[2] = stream;
  w[3] = kTag;
  philox(w, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
}

void normal_range(float *out, int64_t n, uint64_t seed, uint32_t stream, double mean, double stdv, int64_t b0,
                  int64_t b1) {
  const double two_pi = 6.283185307179586;
  const double inv32 = 1.0 / 4294967296.0;
  for (int64_t b = b0; b < b1; ++b) {
    uint32_t w[4];
    block_words(seed, stream, static_cast<uint64_t>(b), w);
    double z[4];
    for (int p = 0; p < 2; ++p) {
      const double u1 = (static_cast<double>(w[2 * p]) + 1.0) * inv32;
      const double u2 = static_cast<double>(w[2 * p + 1]) * inv32;
      const double r = sqrt(-2.0 * log(u1));
      const double t = two_pi * u2;
      z[2 * p] = r * cos(t);
      z[2 * p + 1] = r * sin(t);
    }
    for (int j = 0; j < 4 && b * 4 + j < n; ++j) out[b * 4 + j] = static_cast<float>(mean + stdv * z[j]);
  }
}
}  // namespace

void seeded_normal(float *out, int64_t n, uint64_t seed, uint32_t stream, double mean, double stdv) {
  const int64_t blocks = (n + 3) / 4;
  unsigned hw = std::thread::hardware_concurrency();
  int nt = static_cast<int>(std::min<int64_t>(std::max(1u, std::min(hw, 64u)), std::max<int64_t>(1, blocks / 4096)));
  if (nt <= 1) {
    normal_range(out, n, seed, stream, mean, stdv, 0, blocks);
    return;
  }
  std::vector<std::thread> th;
  const int64_t chunk = (blocks + nt - 1) / nt;
  for (int t = 0; t < nt; ++t) {
    const int64_t b0 = t * chunk, b1 = std::min(blocks, b0 + chunk);
    if (b0 >= b1) break;
    th.emplace_back(normal_range, out, n, seed, stream, mean, stdv, b0, b1);
  }
  for (auto &x : th) x.join();
}

void seeded_ids(int64_t *ids, int64_t n, uint64_t seed, uint32_t stream, int64_t vocab) {
  for (int64_t b = 0; b * 4 < n; ++b) {
    uint32_t w[4];
    block_words(seed, stream, static_cast<uint64_t>(b), w);
    for (int j = 0; j < 4 && b * 4 + j < n; ++j)
      ids[b * 4 + j] = static_cast<int64_t>((static_cast<uint64_t>(w[j]) * static_cast<uint64_t>(vocab)) >> 32);
  }
}

void seeded_blob(const ModelDims &m, uint64_t seed, int init_mode, float *blob) {
  const std::vector<TensorSpec> specs = blob_specs(m);
  for (size_t t = 0; t < specs.size(); ++t) {
    const TensorSpec &s = specs[t];
    float *p = blob + s.offset;
    if (s.kind == TensorSpec::kMatrix) {
      seeded_normal(p, s.numel, seed, static_cast<uint32_t>(t), 0.0, 0.02);
    } else if (init_mode == 0) {
      std::fill(p, p + s.numel, s.kind == TensorSpec::kGain ? 1.0f : 0.0f);
    } else {
      const bool gain = s.kind == TensorSpec::kGain;
      seeded_normal(p, s.numel, seed, static_cast<uint32_t>(t), gain ? 1.0 : 0.0, gain ? 0.1 : 0.02);
    }
  }
}

}  // namespace gpt2
