// gemv_tc.cu -- products of at most 16 activation rows with a bf16 weight
// matrix on the 5th-generation tensor cores: the few-token forward and the
// KV-cache decode steps of the BF16 model.
//
// Replaces, for M <= 16 rows, the reference's linalg.matmul / cblas_sgemm
// calls of its decode loop (src/gpt/lower_gpt_model.py:190-198 re-runs the
// whole forward per token; lib/ConvertMatMulToBlas.cpp:156-160) with the
// weight matrix streamed once per step.
//
// y[M, N] = epi(LN?(x[M, K]) @ W[N, K]^T): the weights are the MMA's A
// operand (M = 128 weight rows per CTA) and the activation rows its B
// operand (N = 16, rows past M zero), D = W x^T in 16 TMEM columns.
//   * A CTA's weight slice (at most 6 k-steps of 128 x 64) streams through a
//     4-stage TMA ring whose first fill goes out before the programmatic-
//     dependency wait: weights depend on no earlier kernel, so they stream
//     while the previous kernel finishes.  About 97 KB of shared memory, so a
//     kernel's CTAs fit beside the previous kernel's (measured: a 6-stage,
//     129 KB version ran a B = 16 decode step at 0.758 ms, this one 0.67).
//   * After the wait all 128 threads compute the rows' LayerNorm statistics
//     (when asked; two passes over K in FP32) and write the CTA's K slice of
//     the rows into the 128-byte-swizzled K-major layout the MMA reads.  A
//     normalised row is FP32: it goes in as two bf16 operands, hi = bf16(v)
//     and lo = bf16(v - hi), and the product is taken with both (about 16
//     significant bits, as the SIMT kernel's FP32 rows times bf16 weights;
//     one bf16 operand measured a flipped top-1 on a tiny model).
//   * One thread issues tcgen05.mma (kind::f16, M=128, N=16, K=16).
//   * K is split over the CTAs of a thread-block cluster (grid x, at most 8)
//     when there are few weight tiles; the partial sums meet in the rank-0
//     CTA through distributed shared memory and are added in rank order, so
//     the result does not depend on timing.
//   * Epilogue: thread = weight row (TMEM lane), 16 values = the 16 rows:
//     per-column scale, bias, gelu_new / erf GELU, residual; bf16 or FP32.
// Every barrier wait is bounded; a timeout records status 2.
#include <atomic>
#include <mutex>
#include <unordered_map>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int TN = 128;                     // weight rows per CTA (the MMA's M)
constexpr int KSTEP = 64;                   // bf16 elements per 128-byte row
constexpr int MAXSTEPS = 6;                 // k-steps per CTA (its activation tiles)
constexpr int WST = 4;                      // weight ring stages (about 97 KB a CTA: two fit on an SM)
constexpr int XROWS = 16;                   // activation rows (the MMA's N)
constexpr int WBYTES = TN * KSTEP * 2;      // 16 KB weight tile
constexpr int XBYTES = XROWS * KSTEP * 2;   // 2 KB activation tile
constexpr int MAXCLUSTER = 8;

struct SmemG {
  static constexpr int W = 0;                        // [WST] weight ring
  static constexpr int X = W + WST * WBYTES;         // [MAXSTEPS] activation tiles
  static constexpr int XLO = X + MAXSTEPS * XBYTES;  // [MAXSTEPS] their low parts (LayerNorm'd rows)
  static constexpr int RED = XLO + MAXSTEPS * XBYTES;  // [16][128] FP32 partial sums (split K)
  static constexpr int BARS = RED + XROWS * TN * 4;  // w_full[WST], w_empty[WST], acc_full
  static constexpr int MISC = BARS + 8 * (2 * WST + 1);
  static constexpr int TOTAL = MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

template <int EPI, bool OUTF32, bool LNP>
__global__ void __launch_bounds__(128, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap map_w, const bf16 *__restrict__ x, void *y, int M, int N,
                   int K, int ldy, int kslice, const float *__restrict__ bias, const bf16 *resid,
                   const float *__restrict__ scale, const float *__restrict__ lng, const float *__restrict__ lnb,
                   float eps, int *status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *w_full = reinterpret_cast<uint64_t *>(sm + SmemG::BARS);
  uint64_t *w_empty = w_full + WST;
  uint64_t *acc_full = w_empty + WST;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + SmemG::MISC);
  __shared__ float s_mean[XROWS], s_rstd[XROWS];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = blockIdx.x, nks = gridDim.x;  // this CTA's K slice; the cluster spans grid x
  const int n0 = blockIdx.y * TN;
  const int k0 = ks * kslice, nsteps = kslice / KSTEP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < WST; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 32);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The weights depend on no earlier kernel: the ring's first fill goes out
  // before the wait.
  if (threadIdx.x == 0) {
    prefetch_tmap(&map_w);
    for (int s = 0; s < nsteps && s < WST; ++s) {
      mbar_arrive_expect_tx(&w_full[s], WBYTES);
      tma_load_2d(sm + SmemG::W + s * WBYTES, &map_w, &w_full[s], k0 + s * KSTEP, n0);
    }
  }
  pdl_wait();     // x and resid belong to earlier kernels
  pdl_trigger();  // the next kernel may start its own weight loads

  if (LNP) {
    // Warp per row: the row's 16-byte chunks stay in registers between the
    // mean and the centred variance (K <= 3072: at most 12 chunks per lane).
    for (int m = warp; m < M; m += 4) {
      const uint4 *xr = reinterpret_cast<const uint4 *>(x + (int64_t)m * K);
      const int nch = K / 8;
      uint4 ch[12];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 12; ++i) {
        const int c = lane + 32 * i;
        ch[i] = c < nch ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {ch[i].x, ch[i].y, ch[i].z, ch[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) sum += bf16_lo(w[e]) + bf16_hi(w[e]);
      }
      const float mu = warp_sum(sum) / K;
      float sq = 0.f;
#pragma unroll
      for (int i = 0; i < 12; ++i) {
        if (lane + 32 * i >= nch) break;
        const uint32_t w[4] = {ch[i].x, ch[i].y, ch[i].z, ch[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float t0 = bf16_lo(w[e]) - mu, t1 = bf16_hi(w[e]) - mu;
          sq = fmaf(t0, t0, fmaf(t1, t1, sq));
        }
      }
      const float r = rsqrtf(warp_sum(sq) / K + eps);
      if (lane == 0) {
        s_mean[m] = mu;
        s_rstd[m] = r;
      }
    }
    __syncthreads();
  }
  // This CTA's K slice of the rows, bf16, 128-byte swizzle: row r of k-step
  // s at s * 2 KB + r * 128, its 16-byte chunk c at (c ^ (r & 7)) * 16.
  for (int idx = threadIdx.x; idx < nsteps * XROWS * 8; idx += 128) {
    const int s = idx >> 7, r = (idx >> 3) & 15, c = idx & 7;
    uint4 v = make_uint4(0u, 0u, 0u, 0u), vlo = make_uint4(0u, 0u, 0u, 0u);
    if (r < M) {
      const int kk = k0 + s * KSTEP + c * 8;
      v = *reinterpret_cast<const uint4 *>(x + (int64_t)r * K + kk);
      if (LNP) {
        const float mu = s_mean[r], rs = s_rstd[r];
        const float4 g0 = *reinterpret_cast<const float4 *>(lng + kk), g1 = *reinterpret_cast<const float4 *>(lng + kk + 4);
        const float4 b0 = *reinterpret_cast<const float4 *>(lnb + kk), b1 = *reinterpret_cast<const float4 *>(lnb + kk + 4);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        uint32_t w4[4] = {v.x, v.y, v.z, v.w}, l4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a0 = fmaf((bf16_lo(w4[e]) - mu) * rs, g[2 * e], bb[2 * e]);
          const float a1 = fmaf((bf16_hi(w4[e]) - mu) * rs, g[2 * e + 1], bb[2 * e + 1]);
          w4[e] = pack_bf16x2(a0, a1);
          l4[e] = pack_bf16x2(a0 - bf16_lo(w4[e]), a1 - bf16_hi(w4[e]));
        }
        v = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        vlo = make_uint4(l4[0], l4[1], l4[2], l4[3]);
      }
    }
    const int off = s * XBYTES + r * 128 + ((c ^ (r & 7)) << 4);
    *reinterpret_cast<uint4 *>(sm + SmemG::X + off) = v;
    if (LNP) *reinterpret_cast<uint4 *>(sm + SmemG::XLO + off) = vlo;
  }
  fence_proxy_async_smem();  // the MMA reads these rows through the async proxy
  __syncthreads();

  // The epilogue's inputs from memory (rank 0 only): residual, bias and scale
  // are loaded now, so their latency overlaps the weight stream and the MMAs.
  const int n_ep = n0 + threadIdx.x;
  const bool ep = ks == 0 && n_ep < N;
  float res[XROWS];
  float sc = 1.f, bn = 0.f;
  if (ep) {
    if (scale) sc = scale[n_ep];
    if (EPI != EPI_NONE) bn = bias[n_ep];
#pragma unroll
    for (int t = 0; t < XROWS; ++t)
      res[t] = (EPI == EPI_BIAS_RESID && t < M) ? __bfloat162float(resid[(int64_t)t * ldy + n_ep]) : 0.f;
  }

  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(TN, XROWS, 0);  // both operands K-major
    bool ok = true;
    for (int s = 0; s < nsteps; ++s) {
      const int st = s % WST;
      const uint32_t ph = (s / WST) & 1;
      if (!mbar_wait(&w_full[st], ph, nullptr, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t a = sdesc_kmajor_sw128(smem_u32(sm + SmemG::W + st * WBYTES));
      const uint64_t b = sdesc_kmajor_sw128(smem_u32(sm + SmemG::X + s * XBYTES));
#pragma unroll
      for (int kk = 0; kk < KSTEP / 16; ++kk) tc_mma_f16(tmem, a + 2 * kk, b + 2 * kk, idesc, (s | kk) != 0);
      if (LNP) {
        const uint64_t bl = sdesc_kmajor_sw128(smem_u32(sm + SmemG::XLO + s * XBYTES));
#pragma unroll
        for (int kk = 0; kk < KSTEP / 16; ++kk) tc_mma_f16(tmem, a + 2 * kk, bl + 2 * kk, idesc, 1);
      }
      if (s + WST < nsteps) {
        // Refill the stage once these products have read it.
        tc_commit(&w_empty[st]);
        if (!mbar_wait(&w_empty[st], ph, nullptr, status)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&w_full[st], WBYTES);
        tma_load_2d(sm + SmemG::W + st * WBYTES, &map_w, &w_full[st], k0 + (s + WST) * KSTEP, n0);
      }
    }
    if (!ok) set_status(status, GPT2_ERR_WAIT_TIMEOUT);
    tc_commit(acc_full);  // arrives once every product issued so far is done
  }
  float v[XROWS];
  {
    if (!mbar_wait(acc_full, 0, nullptr, status)) set_status(status, GPT2_ERR_WAIT_TIMEOUT);
    tc_fence_after();
    uint32_t d[16];
    tmem_ld_32x32b_x16(tmem + (static_cast<uint32_t>(warp * 32) << 16), d);
    tc_wait_ld();
#pragma unroll
    for (int t = 0; t < XROWS; ++t) v[t] = __uint_as_float(d[t]);
  }
  if (nks > 1) {
    // Split K: ranks 1.. leave their partial sums in shared memory, rank 0
    // adds them in rank order; the second barrier keeps every CTA's shared
    // memory alive until rank 0 has read it.
    float *red = reinterpret_cast<float *>(sm + SmemG::RED);
    if (ks != 0) {
#pragma unroll
      for (int t = 0; t < XROWS; ++t) red[t * TN + threadIdx.x] = v[t];
    }
    cluster_sync_all();
    if (ks == 0) {
      const uint32_t base = smem_u32(red + threadIdx.x);
      for (int rk = 1; rk < nks; ++rk) {
        const uint32_t peer = cluster_map_shared(base, static_cast<uint32_t>(rk));
#pragma unroll
        for (int t = 0; t < XROWS; ++t) v[t] += ld_shared_cluster_f32(peer + t * TN * 4);
      }
    }
    cluster_sync_all();
  }
  if (ep) {
#pragma unroll
    for (int t = 0; t < XROWS; ++t) {
      if (t >= M) break;
      float o = fmaf(v[t], sc, bn);
      if (EPI == EPI_BIAS_GELU) o = gelu_new_fast(o);
      if (EPI == EPI_BIAS_GELU_ERF) o = gelu_erf_fast(o);
      if (EPI == EPI_BIAS_RESID) o += res[t];
      const int64_t idx = (int64_t)t * ldy + n_ep;
      if (OUTF32) static_cast<float *>(y)[idx] = o;
      else static_cast<bf16 *>(y)[idx] = __float2bfloat16_rn(o);
    }
  }
  // Every weight copy has landed (the products waited for them, or gave up
  // and wait here once more, bounded) before the CTA's shared memory goes.
  if (threadIdx.x == 0)
    for (int i = 0; i < WST && i < nsteps; ++i) {
      const int cnt = (nsteps - 1 - i) / WST + 1;  // copies that went into stage i
      mbar_wait(&w_full[i], (cnt - 1) & 1, nullptr);
    }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

typedef CUresult (*EncodeTiledFnG)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnG encode_fn_gemv() {
  static std::atomic<EncodeTiledFnG> fn{nullptr};
  EncodeTiledFnG f = fn.load();
  if (f) return f;
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !p)
    return nullptr;
  f = reinterpret_cast<EncodeTiledFnG>(p);
  fn.store(f);
  return f;
}

// Tensor maps of the weight matrices, made once per (pointer, N, K): a
// decode step launches the same few dozen products every time.
struct MapKey {
  const void *w;
  int n, k;
  bool operator==(const MapKey &o) const { return w == o.w && n == o.n && k == o.k; }
};
struct MapKeyHash {
  size_t operator()(const MapKey &k) const {
    return std::hash<const void *>()(k.w) ^ (static_cast<size_t>(k.n) * 0x9E3779B97F4A7C15ull) ^
           (static_cast<size_t>(k.k) << 20);
  }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

bool weight_map(const bf16 *W, int N, int K, CUtensorMap *out) {
  std::lock_guard<std::mutex> lk(g_map_mu);
  const MapKey key{W, N, K};
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return true;
  }
  EncodeTiledFnG f = encode_fn_gemv();
  if (!f) return false;
  CUtensorMap m;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {KSTEP, TN};
  const cuuint32_t estr[2] = {1, 1};
  if (f(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16 *>(W), dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  g_maps.emplace(key, m);
  *out = m;
  return true;
}

// K split: the fewest CTAs per weight tile that keep a CTA's slice within
// MAXSTEPS k-steps, raised while the grid is under one CTA per SM (a
// divisor of the k-steps, at most a portable cluster of 8).
int pick_ksplit(int nsteps, int ntiles, int sms) {
  int best = 0;
  for (int d = 1; d <= MAXCLUSTER; ++d) {
    if (nsteps % d || nsteps / d > MAXSTEPS) continue;
    best = d;
    if ((int64_t)ntiles * d >= sms) break;
  }
  return best;
}

template <int EPI, bool OUTF32>
cudaError_t launch_typed(const CUtensorMap &map, const bf16 *x, void *y, int M, int N, int K, int ldy, int ksplit,
                         const float *bias, const bf16 *resid, const float *scale, const GemvLn *ln, int *status,
                         cudaStream_t st, bool pdl) {
  auto kern = ln ? gemv_tc_kernel<EPI, OUTF32, true> : gemv_tc_kernel<EPI, OUTF32, false>;
  static std::atomic<uint64_t> done_ln{0}, done_plain{0};
  cudaError_t e = set_smem_once(kern, SmemG::ALLOC, ln ? done_ln : done_plain);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ksplit, (N + TN - 1) / TN);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = SmemG::ALLOC;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = ksplit;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl && pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const float *g = ln ? ln->gain : nullptr, *b = ln ? ln->shift : nullptr;
  const float eps = ln ? ln->eps : 0.f;
  e = cudaLaunchKernelEx(&cfg, kern, map, x, y, M, N, K, ldy, K / ksplit, bias, resid, scale, g, b, eps, status);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t gemv_tc_launch(const bf16 *x, const bf16 *W, void *y, bool out_f32, int M, int N, int K, int ldy,
                           const float *bias, const bf16 *resid, const float *scale, int epi, const GemvLn *ln,
                           int *status, cudaStream_t st, bool pdl) {
  if (!gemv_tc_supported(M, N, K, ldy) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(W) & 15))
    return cudaErrorInvalidValue;
  if (ln && (epi == EPI_BIAS_RESID || (reinterpret_cast<uintptr_t>(ln->gain) & 15) ||
             (reinterpret_cast<uintptr_t>(ln->shift) & 15)))
    return cudaErrorInvalidValue;
  if (epi != EPI_NONE && !bias) return cudaErrorInvalidValue;
  if (epi == EPI_BIAS_RESID && !resid) return cudaErrorInvalidValue;
  CUtensorMap map;
  if (!weight_map(W, N, K, &map)) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ksplit = pick_ksplit(K / KSTEP, (N + TN - 1) / TN, sms);
  if (ksplit < 1) return cudaErrorInvalidValue;
  if (out_f32) {
    if (epi != EPI_NONE) return cudaErrorInvalidValue;
    return launch_typed<EPI_NONE, true>(map, x, y, M, N, K, ldy, ksplit, bias, resid, scale, ln, status, st, pdl);
  }
  switch (epi) {
    case EPI_NONE:
      return launch_typed<EPI_NONE, false>(map, x, y, M, N, K, ldy, ksplit, bias, resid, scale, ln, status, st, pdl);
    case EPI_BIAS:
      return launch_typed<EPI_BIAS, false>(map, x, y, M, N, K, ldy, ksplit, bias, resid, scale, ln, status, st, pdl);
    case EPI_BIAS_GELU:
      return launch_typed<EPI_BIAS_GELU, false>(map, x, y, M, N, K, ldy, ksplit, bias, resid, scale, ln, status, st,
                                                pdl);
    case EPI_BIAS_GELU_ERF:
      return launch_typed<EPI_BIAS_GELU_ERF, false>(map, x, y, M, N, K, ldy, ksplit, bias, resid, scale, ln, status,
                                                    st, pdl);
    case EPI_BIAS_RESID:
      return launch_typed<EPI_BIAS_RESID, false>(map, x, y, M, N, K, ldy, ksplit, bias, resid, scale, nullptr, status,
                                                 st, pdl);
    default:
      return cudaErrorInvalidValue;
  }
}
}  // namespace

bool gemv_tc_supported(int M, int N, int K, int ldy) {
  if (M < 1 || M > XROWS || N < 1 || K < KSTEP || K % KSTEP || K > 12 * 256 || ldy < N) return false;
  const int nsteps = K / KSTEP;
  for (int d = 1; d <= MAXCLUSTER; ++d)
    if (nsteps % d == 0 && nsteps / d <= MAXSTEPS) return true;
  return false;
}

cudaError_t launch_gemv_tc_bf16(const bf16 *x, const bf16 *W, bf16 *y, int M, int N, int K, int ldy,
                                const float *bias, const bf16 *resid, const float *scale, int epi, int *status,
                                cudaStream_t st, const GemvLn *ln, bool pdl) {
  return gemv_tc_launch(x, W, y, false, M, N, K, ldy, bias, resid, scale, epi, ln, status, st, pdl);
}

cudaError_t launch_gemv_tc_bf16_f32out(const bf16 *x, const bf16 *W, float *y, int M, int N, int K, int ldy,
                                       int *status, cudaStream_t st, const GemvLn *ln, bool pdl) {
  return gemv_tc_launch(x, W, y, true, M, N, K, ldy, nullptr, nullptr, nullptr, EPI_NONE, ln, status, st, pdl);
}

}  // namespace gpt2

namespace gpt2 {

bool gemv_tc_enabled() {
  static const bool on = [] {
    const char *e = getenv("GPT2_GEMV_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

namespace {
// Every precondition of the tensor-core kernel, and at least 8 rows: with
// fewer the SIMT kernel's shorter chain wins (B = 1 / 4 / 16 decode steps:
// 0.34 / 0.42 / 0.90 ms SIMT, 0.44 / 0.47 / 0.67 ms tensor cores, measured).
constexpr int kTcMinRows = 8;
bool tc_fits(const bf16 *x, const bf16 *W, int M, int N, int K, int ldy, int epi, const GemvLn *ln) {
  auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!gemv_tc_enabled() || M < kTcMinRows || !gemv_tc_supported(M, N, K, ldy) || !a16(x) || !a16(W)) return false;
  if (ln && (epi == EPI_BIAS_RESID || !a16(ln->gain) || !a16(ln->shift))) return false;
  return true;
}
}  // namespace

cudaError_t launch_gemv_bf16_auto(const bf16 *x, const bf16 *W, bf16 *y, int M, int N, int K, int ldy,
                                  const float *bias, const bf16 *resid, const float *scale, int epi, int *status,
                                  cudaStream_t st, const GemvLn *ln, bool pdl) {
  if (tc_fits(x, W, M, N, K, ldy, epi, ln))
    return launch_gemv_tc_bf16(x, W, y, M, N, K, ldy, bias, resid, scale, epi, status, st, ln, pdl);
  return launch_gemv_bf16(x, W, y, M, N, K, ldy, bias, resid, scale, epi, st, ln, pdl);
}

cudaError_t launch_gemv_bf16_f32out_auto(const bf16 *x, const bf16 *W, float *y, int M, int N, int K, int ldy,
                                         int *status, cudaStream_t st, const GemvLn *ln, bool pdl) {
  if (tc_fits(x, W, M, N, K, ldy, EPI_NONE, ln))
    return launch_gemv_tc_bf16_f32out(x, W, y, M, N, K, ldy, status, st, ln, pdl);
  return launch_gemv_bf16_f32out(x, W, y, M, N, K, ldy, st, ln, pdl);
}

}  // namespace gpt2
