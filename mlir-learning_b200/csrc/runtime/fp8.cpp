// fp8.cpp -- weight-only FP8 (E4M3) quantization of the Conv1D weights.
//
// Per output channel n of a Conv1D weight w [K in, N out]:
//   scale[n] = max_k |w[k, n]| / 448   (448 = largest finite E4M3)
//   q[n, k]  = E4M3(w[k, n] / scale[n]), round to nearest even, saturating
// packed [N, K] (the K-major B operand of the GEMM).  Every E4M3 value is
// exactly a BF16 value, so the GEMM runs on the codes expanded to BF16 and
// applies scale[n] in its epilogue.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "runtime.h"

namespace gpt2 {

uint8_t e4m3_encode(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint8_t sign = static_cast<uint8_t>((b >> 24) & 0x80);
  const uint32_t ab = b & 0x7FFFFFFFu;
  float a;
  memcpy(&a, &ab, 4);
  if (!(a == a) || a >= 448.0f) return static_cast<uint8_t>(sign | 0x7E);
  int e = static_cast<int>((ab >> 23) & 0xFF) - 127;
  if (e >= -6) {  // normal: keep 3 of the 23 mantissa bits, ties to even
    uint32_t m = (ab & 0x7FFFFFu) >> 20;
    const uint32_t rest = ab & 0xFFFFFu;
    if (rest > 0x80000u || (rest == 0x80000u && (m & 1u))) ++m;
    if (m == 8) {
      m = 0;
      ++e;
    }
    if (e > 8 || (e == 8 && m == 7)) {
      e = 8;
      m = 6;
    }
    return static_cast<uint8_t>(sign | (static_cast<uint32_t>(e + 7) << 3) | m);
  }
  // subnormal: multiples of 2^-9 (8 of them is the smallest normal, code 0x08)
  return static_cast<uint8_t>(sign | static_cast<uint8_t>(nearbyintf(a * 512.0f)));
}

void fp8_quantize(const float *w, int K, int N, uint8_t *q, float *scale) {
  auto cols = [&](int n0, int n1) {
    for (int n = n0; n < n1; ++n) {
      float mx = 0.f;
      for (int k = 0; k < K; ++k) mx = std::max(mx, fabsf(w[static_cast<int64_t>(k) * N + n]));
      const float sc = mx > 0.f ? mx / 448.0f : 1.0f;
      scale[n] = sc;
      for (int k = 0; k < K; ++k)
        q[static_cast<int64_t>(n) * K + k] = e4m3_encode(w[static_cast<int64_t>(k) * N + n] / sc);
    }
  };
  const int nt = static_cast<int>(std::max(1u, std::min(32u, std::thread::hardware_concurrency())));
  if (nt == 1 || static_cast<int64_t>(K) * N < (1 << 20)) {
    cols(0, N);
    return;
  }
  std::vector<std::thread> th;
  const int chunk = (N + nt - 1) / nt;
  for (int t = 0; t < nt; ++t) {
    const int n0 = t * chunk, n1 = std::min(N, n0 + chunk);
    if (n0 < n1) th.emplace_back(cols, n0, n1);
  }
  for (auto &x : th) x.join();
}

}  // namespace gpt2
