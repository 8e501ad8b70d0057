// decode.cu -- the kernels of incremental (KV-cache) decoding: one new token
// per sequence per step, so every matrix product has M = B <= 16 rows and is
// bound by streaming the weights once.
//
// Replaces the reference's generation pattern -- re-running the whole
// forward on the grown sequence each step and taking logits[:, -1]
// (src/gpt/lower_gpt_model.py:190-198; HF generate's greedy search in
// src/gpt/run_gpt.py:20-24) -- with per-token work against cached keys and
// values.  Results equal the last position of the full forward on the same
// sequence (up to accumulation order).
#include <math.h>
#include <stdlib.h>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

// Programmatic dependent launch of the few-token chain (GEMV, short and
// decode attention): on unless the environment sets GPT2_PDL=0.
bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("GPT2_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

namespace {
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) {
  return __float2bfloat16_rn(v);
}


// kern<<<grid, block, smem, st>>>(args...), as a programmatic dependent of
// the previous kernel on st when pdl is set (the kernel calls pdl_wait()
// before it reads anything an earlier kernel wrote).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// 16-byte chunk of a row as floats: 4 (f32) or 8 (bf16) values.
template <typename T>
struct Chunk {
  static constexpr int N = 16 / sizeof(T);
};
template <typename T>
__device__ __forceinline__ void load_chunk(const T *p, float (&v)[Chunk<T>::N]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(p);
  if constexpr (sizeof(T) == 4) {
    v[0] = __uint_as_float(u.x), v[1] = __uint_as_float(u.y), v[2] = __uint_as_float(u.z), v[3] = __uint_as_float(u.w);
  } else {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// x[b] = wte[tok[b]] + wpe[*d_pos]: one warp per sequence.  The position is
// read from device memory so that one captured step serves every position.
template <typename T>
__global__ void decode_embed_kernel(const int64_t *__restrict__ tok, const T *__restrict__ wte,
                                    const T *__restrict__ wpe, T *__restrict__ x, int B, int d, int V,
                                    const int *__restrict__ d_pos, int P, int *status) {
  pdl_trigger();  // the first GEMV may start streaming its weights
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (b >= B) return;
  const int64_t id = tok[b];
  const int pos0 = *d_pos;
  const bool pos_ok = pos0 >= 0 && pos0 < P;
  const int pos = pos_ok ? pos0 : 0;
  if (!pos_ok && lane == 0) set_status(status, GPT2_ERR_TOKEN_RANGE);
  const bool ok = id >= 0 && id < V;
  if (!ok && lane == 0) set_status(status, GPT2_ERR_TOKEN_RANGE);
  const T *e = wte + (ok ? id : 0) * (int64_t)d;
  const T *p = wpe + (int64_t)pos * d;
  for (int i = lane; i < d; i += 32) x[(int64_t)b * d + i] = from_f<T>((ok ? to_f(e[i]) : 0.f) + to_f(p[i]));
}

// Butterfly reduce-scatter of 32 per-lane values over the warp: afterwards
// lane j holds the warp's sum of value j (31 shuffles in all, where a full
// reduction of each value would take 32 x 5).
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// y[m, n] = epi(sum_k x[m, k] W[n, k]) for m < M <= MMAX: each warp streams
// NC = 32 / MMAX rows of W (16-byte loads along k; the NC loads of a step are
// issued together, each warp takes a 1/KS slice of k) for all M rows of x at
// once, x coming from L1 (it is tiny and shared by every warp).  FP32
// accumulation.  A lane's NC x MMAX partial sums are reduce-scattered over
// the warp, leaving output (m, column) = (j % MMAX, j / MMAX) on lane j; the
// KS slices are added through shared memory; the epilogue runs on that lane.
// With LNP, x is first put through a LayerNorm (gain lng, shift lnb, biased
// variance over K, FP32): each block computes its rows' mean and 1/std (two
// passes per row, one warp per row) and normalises the x chunks as it reads
// them, so the LayerNorm needs no launch and no output buffer of its own.
// FP32 weights with 8-row accumulators (forwards of 5-8 tokens, the
// reference host program's B1 x S5 call among them): at most 80 registers,
// so three blocks fit an SM (the LayerNorm variants spill about 140 bytes of
// the row kept for the statistics).  A whole wave of the fc product then
// fits the GPU and the next kernel's blocks become resident sooner: that
// forward went from 0.390 to 0.359 ms.  Other instances keep the compiler's
// choice (the same bound measured slower for 4 and 16 rows, and spills
// heavily for bf16 weights).
template <typename WT, int MMAX>
constexpr int gemv_min_blocks() {
  return sizeof(WT) == 4 && MMAX == 8 ? 3 : 0;
}

template <typename WT, typename AT, typename OT, int EPI, bool EXACT, int MMAX, int KS, bool LNP>
__global__ void __launch_bounds__(256, (gemv_min_blocks<WT, MMAX>())) gemv_nk_kernel(const AT *__restrict__ x, const WT *__restrict__ W,
                                                      OT *__restrict__ y, int M, int N, int K, int ldy,
                                                      const float *__restrict__ bias, const OT *resid,
                                                      const float *__restrict__ scale, const float *__restrict__ lng,
                                                      const float *__restrict__ lnb, float eps) {
  constexpr int NC = 32 / MMAX;
  constexpr int WC = Chunk<WT>::N;  // weights per 16-byte chunk
  __shared__ float part[8][32];
  __shared__ float s_mean[16], s_rstd[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * (8 / KS) + warp / KS) * NC, ks = warp % KS;
  {
    // The block's weight rows (contiguous: 8 / KS column groups of NC rows)
    // depend on no earlier kernel: they go to L2 while the previous kernel
    // of a programmatic launch finishes, in 4 KB pieces spread over the
    // threads.  K * sizeof(WT) is a multiple of 16, so every piece is too.
    constexpr int ROWS = (8 / KS) * NC;
    const int nb0 = blockIdx.x * ROWS;
    if (nb0 < N) {
      const char *base = reinterpret_cast<const char *>(W + (int64_t)nb0 * K);
      const uint32_t bytes = static_cast<uint32_t>(min(ROWS, N - nb0)) * static_cast<uint32_t>(K) * sizeof(WT);
      for (uint32_t off = threadIdx.x * 4096u; off < bytes; off += 256u * 4096u)
        prefetch_l2_bulk(base + off, min(4096u, bytes - off));
    }
  }
  // The first k step's weights and LayerNorm gain / shift, and the
  // epilogue's scale and bias, are parameters no kernel of the chain writes
  // (a programmatic dependent overlaps only its predecessors in the chain,
  // which write activations): with PRE they are loaded before the wait, so
  // that their latency overlaps it and the LayerNorm statistics instead of
  // following them.  Same values and order of operations either way.  Not
  // for 16-row accumulators, where it measured slower (0.86 -> 0.91 ms for
  // a 16-token FP32 forward; 2-6 % faster at 1-5 rows).
  constexpr bool PRE = MMAX <= 8;
  const int kfirst = (ks * 32 + lane) * WC;
  const WT *wr[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) wr[c] = W + (int64_t)(n0 + c < N ? n0 + c : n0) * K;  // past N: a valid row, unused
  auto load_step = [&](int k0, float (&w)[NC][WC], float *g, float *b) {
#pragma unroll
    for (int c = 0; c < NC; ++c) load_chunk<WT>(wr[c] + k0, w[c]);
    if (LNP) {
#pragma unroll
      for (int j = 0; j < WC; j += 4) {
        const float4 g4 = *reinterpret_cast<const float4 *>(lng + k0 + j);
        const float4 b4 = *reinterpret_cast<const float4 *>(lnb + k0 + j);
        g[j] = g4.x, g[j + 1] = g4.y, g[j + 2] = g4.z, g[j + 3] = g4.w;
        b[j] = b4.x, b[j + 1] = b4.y, b[j + 2] = b4.z, b[j + 3] = b4.w;
      }
    }
  };
  float w0[NC][WC], g0[LNP ? WC : 1], b0[LNP ? WC : 1];
  if (PRE && n0 < N && kfirst < K) load_step(kfirst, w0, g0, b0);
  const int m_out = lane % MMAX, n_out = n0 + lane / MMAX;
  const bool out_ok = n_out < N && m_out < M && (KS == 1 || ks == 0);
  float pre_scale = 1.f, pre_bias = 0.f, pre_res = 0.f;
  if (out_ok) {
    if (scale) pre_scale = scale[n_out];
    if (EPI != EPI_NONE) pre_bias = bias[n_out];
  }
  pdl_wait();     // x, resid and y belong to earlier kernels
  pdl_trigger();  // the next kernel may start its own weight prefetch
  // The residual, loaded now so that its latency overlaps the product.
  if (out_ok && EPI == EPI_BIAS_RESID) pre_res = to_f(resid[(int64_t)m_out * ldy + n_out]);
  float mean[MMAX], rstd[MMAX];
  if (LNP) {
    constexpr int LNR = 32;  // row values a lane keeps in registers (K <= 1024)
    for (int m = warp; m < M; m += 8) {
      const AT *xr = x + (int64_t)m * K;
      float mu, sq = 0.f;
      if (K <= 32 * LNR) {
        // One pass over memory: the row stays in registers between the mean
        // and the centred variance (same order of additions as two passes).
        float xv[LNR];
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < LNR; ++i) {
          const int k = lane + 32 * i;
          xv[i] = k < K ? to_f(xr[k]) : 0.f;
          if (k < K) sum += xv[i];
        }
        mu = warp_sum(sum) / K;
#pragma unroll
        for (int i = 0; i < LNR; ++i) {
          if (lane + 32 * i < K) {
            const float t = xv[i] - mu;
            sq = fmaf(t, t, sq);
          }
        }
      } else {
        float sum = 0.f;
        for (int k = lane; k < K; k += 32) sum += to_f(xr[k]);
        mu = warp_sum(sum) / K;
        for (int k = lane; k < K; k += 32) {
          const float t = to_f(xr[k]) - mu;
          sq = fmaf(t, t, sq);
        }
      }
      const float r = rsqrtf(warp_sum(sq) / K + eps);
      if (lane == 0) {
        s_mean[m] = mu;
        s_rstd[m] = r;
      }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MMAX; ++m) {
      mean[m] = m < M ? s_mean[m] : 0.f;
      rstd[m] = m < M ? s_rstd[m] : 0.f;
    }
  }
  float acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0.f;
  // One k step: acc += x[:, k0 .. k0 + WC) (LayerNorm applied) . w rows.
  auto fma_step = [&](int k0, const float (&w)[NC][WC], const float *g, const float *b) {
#pragma unroll
    for (int m = 0; m < MMAX; ++m) {
      if (m < M) {
        const AT *xr = x + (int64_t)m * K + k0;
#pragma unroll
        for (int j = 0; j < WC; j += Chunk<AT>::N) {
          float xv[Chunk<AT>::N];
          load_chunk<AT>(xr + j, xv);
          if (LNP) {
#pragma unroll
            for (int e = 0; e < Chunk<AT>::N; ++e) xv[e] = fmaf((xv[e] - mean[m]) * rstd[m], g[j + e], b[j + e]);
          }
#pragma unroll
          for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int e = 0; e < Chunk<AT>::N; ++e) acc[c * MMAX + m] = fmaf(xv[e], w[c][j + e], acc[c * MMAX + m]);
        }
      }
    }
  };
  if (n0 < N) {
    // With PRE the first step runs from the values loaded before the wait
    // (peeled, so they are dead before the loop).
    int k0 = kfirst;
    if (PRE && k0 < K) {
      fma_step(k0, w0, g0, b0);
      k0 += 32 * KS * WC;
    }
#pragma unroll 1
    for (; k0 < K; k0 += 32 * KS * WC) {
      float w[NC][WC];
      float g[LNP ? WC : 1], b[LNP ? WC : 1];
      load_step(k0, w, g, b);
      fma_step(k0, w, g, b);
    }
  }
  float v = warp_reduce_scatter32(acc);
  if (KS > 1) {
    part[warp][lane] = v;
    __syncthreads();
    if (ks != 0) return;
#pragma unroll
    for (int i = 1; i < KS; ++i) v += part[warp + i][lane];
  }
  if (n_out < N && m_out < M) {
    if (scale) v *= pre_scale;
    if (EPI != EPI_NONE) v += pre_bias;
    if (EPI == EPI_BIAS_GELU) v = EXACT ? gelu_new_exact(v) : gelu_new_fast(v);
    if (EPI == EPI_BIAS_GELU_ERF) v = EXACT ? gelu_erf(v) : gelu_erf_fast(v);
    if (EPI == EPI_BIAS_RESID) v += pre_res;
    y[(int64_t)m_out * ldy + n_out] = from_f<OT>(v);
  }
}

// Attention of a short sequence (S <= 16, the few-token forward): one warp
// per (sequence, head, query row), lane l holding dimensions l and l + 32 of
// the head.  Scores q.k / 8 by warp reduction, softmax with max subtraction
// (expf), O = P V.  Masked keys (causal future, key_valid 0) contribute
// exactly 0; a row with no attendable key is left to the masked-rows kernel.
template <typename T>
__global__ void __launch_bounds__(128) attn_short_kernel(const T *__restrict__ qkv, const uint8_t *__restrict__ key_valid,
                                                         T *__restrict__ o, int B, int S, int H, int causal) {
  constexpr int DH = 64, SMAX = 16;
  pdl_wait();
  pdl_trigger();
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= B * H * S) return;
  const int i = wid % S, h = (wid / S) % H, b = wid / (S * H);
  const int D = H * DH;
  const int64_t row = (int64_t)b * S;
  const T *q = qkv + (row + i) * 3 * D + h * DH;
  // Every load of the row is issued before any is used (the query, the
  // sequence's keys and values, the key mask), so the kernel waits for one
  // L2 round trip instead of one per dependent step.
  const float q0 = to_f(q[lane]) * 0.125f, q1 = to_f(q[lane + 32]) * 0.125f;
  float k0[SMAX], k1[SMAX], v0[SMAX], v1[SMAX];
  bool use[SMAX];
#pragma unroll
  for (int j = 0; j < SMAX; ++j) {
    use[j] = false;
    k0[j] = k1[j] = v0[j] = v1[j] = 0.f;
    if (j < S) {
      const T *k = qkv + (row + j) * 3 * D + D + h * DH;
      k0[j] = to_f(k[lane]), k1[j] = to_f(k[lane + 32]);
      v0[j] = to_f(k[D + lane]), v1[j] = to_f(k[D + lane + 32]);
      use[j] = (!causal || j <= i) && (!key_valid || key_valid[row + j]);
    }
  }
  float sc[SMAX];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < SMAX; ++j) {
    sc[j] = -INFINITY;
    if (use[j]) {
      const float s = warp_sum(fmaf(q0, k0[j], q1 * k1[j]));
      sc[j] = s;
      mx = fmaxf(mx, s);
    }
  }
  if (mx == -INFINITY) return;
  float l = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
  for (int j = 0; j < SMAX; ++j) {
    if (sc[j] != -INFINITY) {
      const float p = expf(sc[j] - mx);
      l += p;
      o0 = fmaf(p, v0[j], o0);
      o1 = fmaf(p, v1[j], o1);
    }
  }
  T *out = o + (row + i) * D + h * DH;
  out[lane] = from_f<T>(o0 / l);
  out[lane + 32] = from_f<T>(o1 / l);
}

// Copies the keys and values of S tokens per sequence (positions pos0 ..
// pos0 + S - 1) from qkv [B*S, 3D] into the cache [B][max_len][2D].
template <typename T>
__global__ void kv_store_kernel(const T *__restrict__ qkv, T *__restrict__ cache, int B, int S, int D, int max_len,
                                int pos0) {
  const int64_t total = (int64_t)B * S * 2 * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / (2 * D);
    const int c = static_cast<int>(i % (2 * D));
    const int b = static_cast<int>(t / S), s = static_cast<int>(t % S);
    cache[((int64_t)b * max_len + pos0 + s) * 2 * D + c] = qkv[t * 3 * D + D + c];
  }
}

// Attention of one new query per sequence at position pos against cached
// keys / values 0 .. pos - 1 and its own (taken from qkv, and appended to the
// cache).  One 128-thread block per (sequence, head): scores in shared memory,
// block max and sum, then O = P V with two key groups of 64 threads.
template <typename T, bool EXACT>
__global__ void __launch_bounds__(128) attn_decode_kernel(const T *__restrict__ qkv, T *__restrict__ cache,
                                                          T *__restrict__ out, int H, const int *__restrict__ d_pos,
                                                          int max_len, int *status) {
  constexpr int DH = 64;
  extern __shared__ float sc[];  // max(max_len, 1024) floats: the scores, then partial output rows
  pdl_trigger();  // the next GEMV may start its own early loads
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int D = H * DH;
  T *cb = cache + (int64_t)b * max_len * 2 * D;
  // The position and the cached keys and values of positions 0 .. pos - 1
  // were written before this step's chain began (a programmatic dependent
  // overlaps only its predecessors in the chain, which write qkv): the
  // cached rows are prefetched into L1 before the wait, so that the scores
  // and P V after it read them without an L2 round trip.
  const int pos = *d_pos;
  if (pos >= 0 && pos < max_len) {
    for (int j = tid; j < pos; j += blockDim.x) {
      const char *kr = reinterpret_cast<const char *>(cb + (int64_t)j * 2 * D + h * DH);
      const char *vr = kr + sizeof(T) * D;
#pragma unroll
      for (int o = 0; o < DH * (int)sizeof(T); o += 128) {
        asm volatile("prefetch.global.L1 [%0];" ::"l"(kr + o));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(vr + o));
      }
    }
  }
  pdl_wait();
  if (pos < 0 || pos >= max_len) {  // the cache is full: report, touch nothing
    if (tid == 0) set_status(status, GPT2_ERR_BAD_LAUNCH);
    return;
  }
  const int n = pos + 1;
  const T *q = qkv + (int64_t)b * 3 * D + h * DH;
  const T *knew = q + D, *vnew = q + 2 * D;
  __shared__ float qs[DH], red[2 * DH];
  __shared__ float stat[4];
  if (tid < DH) qs[tid] = to_f(q[tid]);
  // append this token's key and value
  if (tid < DH) {
    cb[(int64_t)pos * 2 * D + h * DH + tid] = knew[tid];
    cb[(int64_t)pos * 2 * D + D + h * DH + tid] = vnew[tid];
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = tid; j < n; j += blockDim.x) {
    const T *kr = j == pos ? knew : cb + (int64_t)j * 2 * D + h * DH;
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < DH; c += Chunk<T>::N) {
      float kv[Chunk<T>::N];
      load_chunk<T>(kr + c, kv);
#pragma unroll
      for (int e = 0; e < Chunk<T>::N; ++e) s = fmaf(qs[c + e], kv[e], s);
    }
    s *= 0.125f;
    sc[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) stat[0] = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  const float m = stat[0];
  float sum = 0.f;
  for (int j = tid; j < n; j += blockDim.x) {
    const float p = EXACT ? expf(sc[j] - m) : __expf(sc[j] - m);
    sc[j] = p;
    sum += p;
  }
  sum = warp_sum(sum);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = sum;
  __syncthreads();
  if (tid == 0) stat[1] = (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();
  const float inv = 1.0f / stat[1];
  // O = P V: thread = (key group kg of 128 / CPR, 16-byte column chunk cc);
  // each key row is read with one 16-byte load per chunk, the key groups'
  // partial rows are added through shared memory.
  constexpr int CW = Chunk<T>::N, CPR = DH / CW;  // values per chunk, chunks per row
  constexpr int KG = 128 / CPR;                     // key groups
  const int cc = tid % CPR, kg = tid / CPR;
  float acc[CW];
#pragma unroll
  for (int e = 0; e < CW; ++e) acc[e] = 0.f;
#pragma unroll 4
  for (int j = kg; j < n; j += KG) {
    const T *vr = j == pos ? vnew : cb + (int64_t)j * 2 * D + D + h * DH;
    float v[CW];
    load_chunk<T>(vr + cc * CW, v);
    const float p = sc[j];
#pragma unroll
    for (int e = 0; e < CW; ++e) acc[e] = fmaf(p, v[e], acc[e]);
  }
  __syncthreads();  // every thread is done with sc before it is reused
#pragma unroll
  for (int e = 0; e < CW; ++e) sc[kg * DH + cc * CW + e] = acc[e];
  __syncthreads();
  if (tid < DH) {
    float o = 0.f;
    for (int g = 0; g < KG; ++g) o += sc[g * DH + tid];
    out[(int64_t)b * D + h * DH + tid] = from_f<T>(o * inv);
  }
}

// tokens[b] = argmax_n logits[b, n] (the first maximum, as torch.argmax).
__global__ void argmax_rows_kernel(const float *__restrict__ logits, int64_t ld, int V, int64_t *__restrict__ tokens) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const float *r = logits + (int64_t)b * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += blockDim.x) {
    const float v = r[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  if ((tid & 31) == 0) {
    sv[tid >> 5] = best;
    si[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    tokens[b] = bi == 0x7fffffff ? 0 : bi;
  }
}

__global__ void transpose_f32_kernel(const float *__restrict__ src, float *__restrict__ dst, int rows, int cols) {
  __shared__ float tile[32][33];
  const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = by + i, c = bx + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? src[(int64_t)r * cols + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = bx + i, r = by + threadIdx.x;
    if (c < cols && r < rows) dst[(int64_t)c * rows + r] = tile[threadIdx.x][i];
  }
}

template <typename WT, typename AT, typename OT, bool EXACT, int MMAX, int KS>
cudaError_t gemv_launch(const AT *x, const WT *W, OT *y, int M, int N, int K, int ldy, const float *bias,
                        const OT *resid, const float *scale, int epi, const GemvLn *ln, cudaStream_t st, bool pdl) {
  constexpr int NC = 32 / MMAX, GROUPS_PER_BLOCK = 8 / KS;
  const int groups = (N + NC - 1) / NC;
  const int blocks = (groups + GROUPS_PER_BLOCK - 1) / GROUPS_PER_BLOCK;
#define GEMV_CASE(E)                                                                                          \
  case E:                                                                                                     \
    return launch_k(gemv_nk_kernel<WT, AT, OT, E, EXACT, MMAX, KS, false>, dim3(blocks), dim3(256), 0, st, pdl, \
                    x, W, y, M, N, K, ldy, bias, resid, scale, nullptr, nullptr, 0.f);
#define GEMV_LN_CASE(E)                                                                                       \
  case E:                                                                                                     \
    return launch_k(gemv_nk_kernel<WT, AT, OT, E, EXACT, MMAX, KS, true>, dim3(blocks), dim3(256), 0, st, pdl,  \
                    x, W, y, M, N, K, ldy, bias, resid, scale, ln->gain, ln->shift, ln->eps);
  if (ln) {
    // A LayerNorm ahead of the product: the QKV, fc and lm_head inputs.
    switch (epi) {
      GEMV_LN_CASE(EPI_NONE)
      GEMV_LN_CASE(EPI_BIAS)
      GEMV_LN_CASE(EPI_BIAS_GELU)
      default:
        return cudaErrorInvalidValue;
    }
  }
  switch (epi) {
    GEMV_CASE(EPI_NONE)
    GEMV_CASE(EPI_BIAS)
    GEMV_CASE(EPI_BIAS_GELU)
    GEMV_CASE(EPI_BIAS_RESID)
    GEMV_CASE(EPI_BIAS_GELU_ERF)
    default:
      return cudaErrorInvalidValue;
  }
#undef GEMV_CASE
#undef GEMV_LN_CASE
}

template <typename WT, typename AT, typename OT, bool EXACT, int MMAX>
cudaError_t gemv_ks(const AT *x, const WT *W, OT *y, int M, int N, int K, int ldy, const float *bias,
                    const OT *resid, const float *scale, int epi, const GemvLn *ln, cudaStream_t st, bool pdl) {
  // Split k over KS warps until about 4096 warps stream the matrix (a few
  // dozen per SM keep enough loads in flight), with at least one 16-byte step
  // of k per lane for every warp.
  constexpr int NC = 32 / MMAX;
  const int groups = (N + NC - 1) / NC;
  const int steps = (K + 32 * Chunk<WT>::N - 1) / (32 * Chunk<WT>::N);
  int ks = 1;
  while (ks < 8 && groups * ks < 4096 && 2 * ks <= steps) ks *= 2;
  switch (ks) {
    case 1:
      return gemv_launch<WT, AT, OT, EXACT, MMAX, 1>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
    case 2:
      return gemv_launch<WT, AT, OT, EXACT, MMAX, 2>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
    case 4:
      return gemv_launch<WT, AT, OT, EXACT, MMAX, 4>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
    default:
      return gemv_launch<WT, AT, OT, EXACT, MMAX, 8>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
  }
}

// Accumulators sized to the rows: 4, 8 or 16 (8, 4 or 2 columns per warp).
template <typename WT, typename AT, typename OT, bool EXACT>
cudaError_t gemv_dispatch(const AT *x, const WT *W, OT *y, int M, int N, int K, int ldy, const float *bias,
                          const OT *resid, const float *scale, int epi, const GemvLn *ln, cudaStream_t st,
                          bool pdl) {
  if (ln && (!ln->gain || !ln->shift || K % 4 || !(ln->eps > 0.f) || (reinterpret_cast<uintptr_t>(ln->gain) & 15) ||
             (reinterpret_cast<uintptr_t>(ln->shift) & 15)))
    return cudaErrorInvalidValue;  // the gain and shift are read as 16-byte vectors
  if (M <= 4) return gemv_ks<WT, AT, OT, EXACT, 4>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
  if (M <= 8) return gemv_ks<WT, AT, OT, EXACT, 8>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
  return gemv_ks<WT, AT, OT, EXACT, 16>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
}
}  // namespace

cudaError_t launch_decode_embed_f32(const int64_t *tok, const float *wte, const float *wpe, float *x, int B, int d,
                                    int V, const int *d_pos, int P, int *status, cudaStream_t st) {
  decode_embed_kernel<float><<<(B * 32 + 127) / 128, 128, 0, st>>>(tok, wte, wpe, x, B, d, V, d_pos, P, status);
  return cudaGetLastError();
}
cudaError_t launch_decode_embed_bf16(const int64_t *tok, const bf16 *wte, const bf16 *wpe, bf16 *x, int B, int d,
                                     int V, const int *d_pos, int P, int *status, cudaStream_t st) {
  decode_embed_kernel<bf16><<<(B * 32 + 127) / 128, 128, 0, st>>>(tok, wte, wpe, x, B, d, V, d_pos, P, status);
  return cudaGetLastError();
}

cudaError_t launch_gemv_f32(const float *x, const float *W, float *y, int M, int N, int K, int ldy, const float *bias,
                            const float *resid, int epi, cudaStream_t st, const GemvLn *ln, bool pdl) {
  if (M < 1 || M > 16 || K % 4 || ldy < N) return cudaErrorInvalidValue;
  return gemv_dispatch<float, float, float, true>(x, W, y, M, N, K, ldy, bias, resid, nullptr, epi, ln, st, pdl);
}
cudaError_t launch_gemv_bf16(const bf16 *x, const bf16 *W, bf16 *y, int M, int N, int K, int ldy, const float *bias,
                             const bf16 *resid, const float *scale, int epi, cudaStream_t st, const GemvLn *ln,
                             bool pdl) {
  if (M < 1 || M > 16 || K % 8 || ldy < N) return cudaErrorInvalidValue;
  return gemv_dispatch<bf16, bf16, bf16, false>(x, W, y, M, N, K, ldy, bias, resid, scale, epi, ln, st, pdl);
}
cudaError_t launch_gemv_bf16_f32out(const bf16 *x, const bf16 *W, float *y, int M, int N, int K, int ldy,
                                    cudaStream_t st, const GemvLn *ln, bool pdl) {
  if (M < 1 || M > 16 || K % 8 || ldy < N) return cudaErrorInvalidValue;
  return gemv_dispatch<bf16, bf16, float, false>(x, W, y, M, N, K, ldy, nullptr, nullptr, nullptr, EPI_NONE, ln, st,
                                                 pdl);
}

cudaError_t launch_attention_short_f32(const float *qkv, const uint8_t *key_valid, float *o, int B, int S, int H,
                                      int causal, cudaStream_t st, bool pdl) {
  if (S < 1 || S > 16) return cudaErrorInvalidValue;
  const int warps = B * H * S;
  return launch_k(attn_short_kernel<float>, dim3((warps + 3) / 4), dim3(128), 0, st, pdl, qkv, key_valid, o, B, S, H,
                  causal);
}
cudaError_t launch_attention_short_bf16(const bf16 *qkv, const uint8_t *key_valid, bf16 *o, int B, int S, int H,
                                       int causal, cudaStream_t st, bool pdl) {
  if (S < 1 || S > 16) return cudaErrorInvalidValue;
  const int warps = B * H * S;
  return launch_k(attn_short_kernel<bf16>, dim3((warps + 3) / 4), dim3(128), 0, st, pdl, qkv, key_valid, o, B, S, H,
                  causal);
}

cudaError_t launch_kv_store_f32(const float *qkv, float *cache, int B, int S, int D, int max_len, int pos0,
                                cudaStream_t st) {
  kv_store_kernel<float><<<592, 256, 0, st>>>(qkv, cache, B, S, D, max_len, pos0);
  return cudaGetLastError();
}
cudaError_t launch_kv_store_bf16(const bf16 *qkv, bf16 *cache, int B, int S, int D, int max_len, int pos0,
                                 cudaStream_t st) {
  kv_store_kernel<bf16><<<592, 256, 0, st>>>(qkv, cache, B, S, D, max_len, pos0);
  return cudaGetLastError();
}

cudaError_t launch_attn_decode_f32(const float *qkv, float *cache, float *out, int B, int H, const int *d_pos,
                                   int max_len, int *status, cudaStream_t st, bool pdl) {
  if (max_len < 1 || max_len > 8192) return cudaErrorInvalidValue;
  const int sm = max_len > 1024 ? max_len : 1024;  // scores, then the key groups' partial rows
  return launch_k(attn_decode_kernel<float, true>, dim3(H, B), dim3(128), sizeof(float) * sm, st, pdl, qkv, cache,
                  out, H, d_pos, max_len, status);
}
cudaError_t launch_attn_decode_bf16(const bf16 *qkv, bf16 *cache, bf16 *out, int B, int H, const int *d_pos,
                                    int max_len, int *status, cudaStream_t st, bool pdl) {
  if (max_len < 1 || max_len > 8192) return cudaErrorInvalidValue;
  const int sm = max_len > 1024 ? max_len : 1024;  // scores, then the key groups' partial rows
  return launch_k(attn_decode_kernel<bf16, false>, dim3(H, B), dim3(128), sizeof(float) * sm, st, pdl, qkv, cache,
                  out, H, d_pos, max_len, status);
}

namespace {
__global__ void set_int_kernel(int *p, int v) { *p = v; }
__global__ void add_int_kernel(int *p, int v) { *p += v; }
// hist[(*d_pos - base) * B + b] = cur[b] (the generated-token history).
__global__ void append_tokens_kernel(const int64_t *__restrict__ cur, int64_t *__restrict__ hist,
                                     const int *__restrict__ d_pos, int base, int B, int cap) {
  const int b = threadIdx.x;
  const int i = *d_pos - base;
  if (b < B && i >= 0 && (int64_t)i * B + b < cap) hist[(int64_t)i * B + b] = cur[b];
}
}  // namespace

cudaError_t launch_set_int(int *p, int v, cudaStream_t st) {
  set_int_kernel<<<1, 1, 0, st>>>(p, v);
  return cudaGetLastError();
}
cudaError_t launch_add_int(int *p, int v, cudaStream_t st) {
  add_int_kernel<<<1, 1, 0, st>>>(p, v);
  return cudaGetLastError();
}
cudaError_t launch_append_tokens(const int64_t *cur, int64_t *hist, const int *d_pos, int base, int B, int cap,
                                 cudaStream_t st) {
  append_tokens_kernel<<<1, 32, 0, st>>>(cur, hist, d_pos, base, B, cap);
  return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const float *logits, int64_t ld, int B, int V, int64_t *tokens, cudaStream_t st) {
  argmax_rows_kernel<<<B, 1024, 0, st>>>(logits, ld, V, tokens);
  return cudaGetLastError();
}

cudaError_t launch_transpose_f32(const float *src, float *dst, int rows, int cols, cudaStream_t st) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  transpose_f32_kernel<<<grid, block, 0, st>>>(src, dst, rows, cols);
  return cudaGetLastError();
}

}  // namespace gpt2
