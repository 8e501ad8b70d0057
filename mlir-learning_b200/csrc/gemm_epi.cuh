// gemm_epi.cuh -- pieces of the tcgen05 GEMM epilogues shared by gemm_tc.cu
// and gemm_tc2sm.cu: the folded LayerNorm (EPI_LN_*) and the row statistics
// of a residual GEMM's output (EPI_BIAS_RESID_STATS).  In both kernels one
// epilogue thread owns one output row of the tile and walks it in chunks of
// columns, so every quantity here is per thread, with no shuffles.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace gpt2 {

template <int EPI>
struct EpiKind {
  static constexpr bool ln = EPI == EPI_LN_BIAS || EPI == EPI_LN_BIAS_GELU || EPI == EPI_LN_BIAS_GELU_ERF;
  static constexpr bool lnres = EPI == EPI_LNRES_BIAS_RESID_STATS;
  static constexpr bool resid = EPI == EPI_BIAS_RESID || EPI == EPI_BIAS_RESID_STATS || lnres;
  static constexpr bool stats = EPI == EPI_BIAS_RESID_STATS || lnres;
  static constexpr bool bias = EPI != EPI_NONE && !ln;
  static constexpr bool gelu_new = EPI == EPI_BIAS_GELU || EPI == EPI_LN_BIAS_GELU;
  static constexpr bool gelu_erf = EPI == EPI_BIAS_GELU_ERF || EPI == EPI_LN_BIAS_GELU_ERF;
  static constexpr int ln_act = gelu_new ? 1 : gelu_erf ? 2 : 0;  // activation after the folded LayerNorm
};

// Mean and 1/sqrt(var + eps) of a row of width k from its nseg segment
// statistics, returned as rstd and -rstd * mean.
__device__ __forceinline__ void seg_row_stats(const float2 *s, int nseg, int k, float eps, float &rstd,
                                              float &neg_mean_rstd) {
  float sum = 0.f, sq = 0.f;
  for (int i = 0; i < nseg; ++i) {
    const float2 v = s[i];
    sum += v.x;
    sq += v.y;
  }
  const float inv_k = 1.f / static_cast<float>(k);
  const float mean = sum * inv_k;
  const float var = fmaxf(fmaf(sq, inv_k, -mean * mean), 0.f);
  rstd = rsqrtf(var + eps);
  neg_mean_rstd = -mean * rstd;
}

// The statistics of a residual row for EPI_LNRES_BIAS_RESID_STATS (width n).
__device__ __forceinline__ void ln_res_row_stats(const LnFold &ln, int row, int n, float &rstd, float &nmr) {
  seg_row_stats(ln.res_stats + (int64_t)row * ln.nseg_out, ln.nseg_out, n, ln.eps, rstd, nmr);
}

// r[0..8) (a 16-byte piece of the bf16 residual at column col) with its
// LayerNorm applied: (r * rstd - mean * rstd) * gain + shift.
__device__ __forceinline__ void ln_res_piece(const uint4 &raw, const LnFold &ln, int col, float rstd, float nmr,
                                             float (&r)[8]) {
  const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&raw);
  const float4 g0 = __ldg(reinterpret_cast<const float4 *>(ln.res_gain + col));
  const float4 g1 = __ldg(reinterpret_cast<const float4 *>(ln.res_gain + col + 4));
  const float4 b0 = __ldg(reinterpret_cast<const float4 *>(ln.res_shift + col));
  const float4 b1 = __ldg(reinterpret_cast<const float4 *>(ln.res_shift + col + 4));
  const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    r[2 * j] = fmaf(fmaf(f.x, rstd, nmr), g[2 * j], b[2 * j]);
    r[2 * j + 1] = fmaf(fmaf(f.y, rstd, nmr), g[2 * j + 1], b[2 * j + 1]);
  }
}

// Mean and 1/sqrt(var + eps) of A's row from its segment statistics; the
// epilogue then computes rstd * acc + (c2 - rstd * mean * c1) per column
// (returned as rstd and -rstd * mean).
__device__ __forceinline__ void ln_row_stats(const LnFold &ln, int row, float &rstd, float &neg_mean_rstd) {
  seg_row_stats(ln.stats_in + (int64_t)row * ln.nseg_in, ln.nseg_in, ln.k, ln.eps, rstd, neg_mean_rstd);
}

// v[0..CH) = rstd * acc + (c2 - rstd * mean * c1) for columns col0.. (the
// vectors are padded, so no column check), then ACT: 0 none, 1 gelu_new,
// 2 the erf GELU.  The vectors are read with 16-byte loads that every lane of
// the warp issues for the same address (one broadcast transaction each).
template <int CH, int ACT>
__device__ __forceinline__ void ln_affine(float *v, const LnFold &ln, int col0, float rstd, float nmr) {
  const float4 *c1 = reinterpret_cast<const float4 *>(ln.c1 + col0);
  const float4 *c2 = reinterpret_cast<const float4 *>(ln.c2 + col0);
#pragma unroll
  for (int g = 0; g < CH / 4; ++g) {
    const float4 a = __ldg(c1 + g), b = __ldg(c2 + g);
    v[4 * g + 0] = fmaf(rstd, v[4 * g + 0], fmaf(nmr, a.x, b.x));
    v[4 * g + 1] = fmaf(rstd, v[4 * g + 1], fmaf(nmr, a.y, b.y));
    v[4 * g + 2] = fmaf(rstd, v[4 * g + 2], fmaf(nmr, a.z, b.z));
    v[4 * g + 3] = fmaf(rstd, v[4 * g + 3], fmaf(nmr, a.w, b.w));
    if (ACT == 1) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * g + i] = gelu_new_fast(v[4 * g + i]);
    }
    if (ACT == 2) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * g + i] = gelu_erf_fast(v[4 * g + i]);
    }
  }
}

// Running (sum, sum of squares) of the bf16-rounded values a thread stores,
// as packed f32 pairs; flushed once per LN_SEG columns.
struct RowStats {
  uint64_t s = 0, q = 0;  // bit patterns of (+0.0f, +0.0f)
  template <int CH>
  __device__ __forceinline__ void add_bf16(const float *v) {
#pragma unroll
    for (int j = 0; j < CH; j += 2) {
      const uint32_t w = pack_bf16x2(v[j], v[j + 1]);
      const uint64_t x2 = pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
      s = add2(s, x2);
      q = fma2(x2, x2, q);
    }
  }
  __device__ __forceinline__ void flush(const LnFold &ln, int row, int seg, bool row_ok) {
    float s0, s1, q0, q1;
    up2(s, s0, s1);
    up2(q, q0, q1);
    if (row_ok && seg < ln.nseg_out)
      ln.stats_out[(int64_t)row * ln.nseg_out + seg] = make_float2(s0 + s1, q0 + q1);
    s = 0;
    q = 0;
  }
};

}  // namespace gpt2
