// elementwise.cu -- the bandwidth-bound kernels of the GPT-2 forward:
// mask preparation, token + position embedding, LayerNorm, weight packing.
//
// These replace the reference's gather / reduction / elementwise
// linalg.generic launches (README.md:11, :49; LayerNorm mean/var over 768
// columns, the wte[id] + wpe[pos] gathers) with one launch per op, 128-bit
// accesses and warp-shuffle reductions.
#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

// ---------------------------------------------------------------------------
// Mask preparation: one block per sequence.
// ---------------------------------------------------------------------------
__global__ void seq_info_kernel(const int64_t *__restrict__ mask, int S, int *__restrict__ first_valid,
                                uint8_t *__restrict__ key_valid, int *__restrict__ kv_end) {
  const int b = blockIdx.x;
  __shared__ int first, last;
  if (threadIdx.x == 0) {
    first = S;
    last = -1;
  }
  __syncthreads();
  int lo = S, hi = -1;
  for (int k = threadIdx.x; k < S; k += blockDim.x) {
    const bool v = mask[(int64_t)b * S + k] != 0;
    key_valid[(int64_t)b * S + k] = v ? 1 : 0;
    if (v) {
      lo = min(lo, k);
      hi = max(hi, k);
    }
  }
  if (lo < S) atomicMin(&first, lo);
  if (hi >= 0) atomicMax(&last, hi);
  __syncthreads();
  if (threadIdx.x == 0) {
    first_valid[b] = first;
    if (kv_end) kv_end[b] = last + 1;
  }
}

cudaError_t launch_seq_info(const int64_t *mask, int B, int S, int *first_valid, uint8_t *key_valid,
                            cudaStream_t st, int *kv_end) {
  seq_info_kernel<<<B, 256, 0, st>>>(mask, S, first_valid, key_valid, kv_end);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Embedding.  One warp per token row; d % 4 == 0 (f32) / d % 8 == 0 (bf16).
// ---------------------------------------------------------------------------
__global__ void embed_f32_kernel(const int64_t *__restrict__ ids, const float *__restrict__ wte,
                                 const float *__restrict__ wpe, float *__restrict__ x, int T, int S, int d, int V,
                                 int *status) {
  pdl_trigger();  // a programmatic dependent (the first GEMV of a few-token forward) may start
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const int64_t id = ids[warp];
  const bool ok = id >= 0 && id < V;
  if (!ok && lane == 0) set_status(status, GPT2_ERR_TOKEN_RANGE);
  const float4 *e = reinterpret_cast<const float4 *>(wte + (ok ? id : 0) * (int64_t)d);
  const float4 *p = reinterpret_cast<const float4 *>(wpe + (int64_t)(warp % S) * d);
  float4 *o = reinterpret_cast<float4 *>(x + (int64_t)warp * d);
  for (int i = lane; i < d / 4; i += 32) {
    const float4 a = ok ? e[i] : make_float4(0.f, 0.f, 0.f, 0.f), b = p[i];
    o[i] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  }
}

__global__ void embed_bf16_kernel(const int64_t *__restrict__ ids, const bf16 *__restrict__ wte,
                                  const bf16 *__restrict__ wpe, bf16 *__restrict__ x, int T, int S, int d, int V,
                                  int *status, float2 *__restrict__ stats) {
  pdl_trigger();  // a programmatic dependent (the first GEMV of a few-token forward) may start
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const int64_t id = ids[warp];
  const bool ok = id >= 0 && id < V;
  if (!ok && lane == 0) set_status(status, GPT2_ERR_TOKEN_RANGE);
  const uint4 *e = reinterpret_cast<const uint4 *>(wte + (ok ? id : 0) * (int64_t)d);
  const uint4 *p = reinterpret_cast<const uint4 *>(wpe + (int64_t)(warp % S) * d);
  uint4 *o = reinterpret_cast<uint4 *>(x + (int64_t)warp * d);
  const int nv = d / 8, nseg = (d + LN_SEG - 1) / LN_SEG;
  // 32 vectors of 8 per pass = two LN_SEG-column segments: lanes 0-15 hold
  // segment 2 * pass, lanes 16-31 segment 2 * pass + 1.
  for (int i0 = 0; i0 < nv; i0 += 32) {
    const int i = i0 + lane;
    float sum = 0.f, sq = 0.f;
    if (i < nv) {
      uint4 a = ok ? e[i] : make_uint4(0, 0, 0, 0);
      const uint4 b = p[i];
      const __nv_bfloat162 *a2 = reinterpret_cast<const __nv_bfloat162 *>(&a);
      const __nv_bfloat162 *b2 = reinterpret_cast<const __nv_bfloat162 *>(&b);
      uint4 r;
      uint32_t *r2 = reinterpret_cast<uint32_t *>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __bfloat1622float2(a2[j]), fb = __bfloat1622float2(b2[j]);
        r2[j] = pack_bf16x2(fa.x + fb.x, fa.y + fb.y);
        const float lo = __uint_as_float(r2[j] << 16), hi = __uint_as_float(r2[j] & 0xffff0000u);
        sum += lo + hi;
        sq = fmaf(lo, lo, fmaf(hi, hi, sq));
      }
      o[i] = r;
    }
    if (stats) {
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
        sq += __shfl_xor_sync(0xffffffffu, sq, off);
      }
      const int seg = i0 / 16 + (lane >> 4);
      if ((lane & 15) == 0 && seg < nseg) stats[(int64_t)warp * nseg + seg] = make_float2(sum, sq);
    }
  }
}

cudaError_t launch_embed_f32(const int64_t *ids, const float *wte, const float *wpe, float *x, int T, int S, int d,
                             int V, int *status, cudaStream_t st) {
  if (d % 4) return cudaErrorInvalidValue;
  const int threads = 256, rows = threads / 32;
  embed_f32_kernel<<<(T + rows - 1) / rows, threads, 0, st>>>(ids, wte, wpe, x, T, S, d, V, status);
  return cudaGetLastError();
}

cudaError_t launch_embed_bf16(const int64_t *ids, const bf16 *wte, const bf16 *wpe, bf16 *x, int T, int S, int d,
                              int V, int *status, cudaStream_t st, float2 *stats) {
  if (d % 8) return cudaErrorInvalidValue;
  const int threads = 256, rows = threads / 32;
  embed_bf16_kernel<<<(T + rows - 1) / rows, threads, 0, st>>>(ids, wte, wpe, x, T, S, d, V, status, stats);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// LayerNorm: one warp per row, the row held in registers (VPT 128-bit vectors
// per lane), mean then centred variance from the registers, FP32 throughout.
// ---------------------------------------------------------------------------
template <int VPT>
__global__ void layernorm_f32_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                     const float *__restrict__ b, float *__restrict__ y, int T, int d, float eps) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int nv = d / 4;
  const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)row * d);
  float4 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < nv ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = warp_sum(s) / d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      const float a = v[i].x - mean, bb = v[i].y - mean, cc = v[i].z - mean, dd = v[i].w - mean;
      q += (a * a + bb * bb) + (cc * cc + dd * dd);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / d + eps);
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  const float4 *b4 = reinterpret_cast<const float4 *>(b);
  float4 *yr = reinterpret_cast<float4 *>(y + (int64_t)row * d);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      const float4 gg = g4[c], bb = b4[c];
      yr[c] = make_float4((v[i].x - mean) * rstd * gg.x + bb.x, (v[i].y - mean) * rstd * gg.y + bb.y,
                          (v[i].z - mean) * rstd * gg.z + bb.z, (v[i].w - mean) * rstd * gg.w + bb.w);
    }
  }
}

// BF16 rows: a grid-stride loop of warps over rows, the next row's loads
// issued before the current row is reduced (two rows in flight per warp), the
// gain and shift staged once per block in shared memory.
template <int VPT, typename OutT>
__global__ void __launch_bounds__(256) layernorm_bf16_kernel(const bf16 *__restrict__ x, const float *__restrict__ g,
                                                             const float *__restrict__ b, OutT *__restrict__ y, int T,
                                                             int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nv = d / 8;
  extern __shared__ float4 gb_sm[];  // gain then shift, d floats each
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
    gb_sm[i] = reinterpret_cast<const float4 *>(g)[i];
    gb_sm[d / 4 + i] = reinterpret_cast<const float4 *>(b)[i];
  }
  __syncthreads();
  auto load = [&](int row, uint4 (&dst)[VPT]) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + (int64_t)row * d);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      dst[i] = c < nv ? xr[c] : make_uint4(0, 0, 0, 0);
    }
  };
  int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  uint4 cur[VPT], nxt[VPT];
  if (row < T) load(row, cur);
  for (; row < T; row += nwarps) {
    if (row + nwarps < T) load(row + nwarps, nxt);
    float v[VPT][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&cur[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        v[i][2 * j] = f.x;
        v[i][2 * j + 1] = f.y;
        s += f.x + f.y;
      }
    }
    const float mean = warp_sum(s) / d;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float e = v[i][j] - mean;
          q += e * e;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(q) / d + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        const float4 g0 = gb_sm[2 * c], g1 = gb_sm[2 * c + 1];
        const float4 b0 = gb_sm[d / 4 + 2 * c], b1 = gb_sm[d / 4 + 2 * c + 1];
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * rstd * gg[j] + bb[j];
        if constexpr (sizeof(OutT) == 4) {  // FP32 output (the encoder's last LayerNorm)
          float4 *yr = reinterpret_cast<float4 *>(y + (int64_t)row * d);
          yr[2 * c] = make_float4(o[0], o[1], o[2], o[3]);
          yr[2 * c + 1] = make_float4(o[4], o[5], o[6], o[7]);
        } else {
          uint4 *yr = reinterpret_cast<uint4 *>(y + (int64_t)row * d);
          yr[c] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                             pack_bf16x2(o[6], o[7]));
        }
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) cur[i] = nxt[i];
  }
}

#define LN_CASE(V, KERNEL, ...)                                              \
  case V:                                                                    \
    KERNEL<V><<<(T + rows - 1) / rows, threads, 0, st>>>(__VA_ARGS__);       \
    break;

cudaError_t launch_layernorm_f32(const float *x, const float *g, const float *b, float *y, int T, int d, float eps,
                                 cudaStream_t st) {
  if (d % 4 || d > 128 * 16) return cudaErrorInvalidValue;
  const int threads = 256, rows = threads / 32;
  switch ((d + 127) / 128) {
    LN_CASE(1, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(2, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(3, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(4, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(5, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(6, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(7, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(8, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(10, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(13, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    LN_CASE(16, layernorm_f32_kernel, x, g, b, y, T, d, eps)
    default:
      if (d <= 128 * 10) layernorm_f32_kernel<10><<<(T + rows - 1) / rows, threads, 0, st>>>(x, g, b, y, T, d, eps);
      else if (d <= 128 * 13) layernorm_f32_kernel<13><<<(T + rows - 1) / rows, threads, 0, st>>>(x, g, b, y, T, d, eps);
      else layernorm_f32_kernel<16><<<(T + rows - 1) / rows, threads, 0, st>>>(x, g, b, y, T, d, eps);
  }
  return cudaGetLastError();
}

namespace {
template <typename OutT>
cudaError_t layernorm_bf16_any(const bf16 *x, const float *g, const float *b, OutT *y, int T, int d, float eps,
                               cudaStream_t st) {
  if (d % 8 || d > 256 * 8) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Enough warps to keep two rows in flight each on every SM, no more than there are rows.
  const int threads = 256, rows_per_block = threads / 32;
  const size_t smem = 2 * sizeof(float) * d;
  const int want = (T + rows_per_block - 1) / rows_per_block;
  // One resident wave: as many blocks as the SMs hold at once.
  auto grid_for = [&](auto kernel) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    const int cap = sms * per_sm;
    return want < cap ? want : cap;
  };
  switch ((d + 255) / 256) {
    case 1: layernorm_bf16_kernel<1, OutT><<<grid_for(layernorm_bf16_kernel<1, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 2: layernorm_bf16_kernel<2, OutT><<<grid_for(layernorm_bf16_kernel<2, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 3: layernorm_bf16_kernel<3, OutT><<<grid_for(layernorm_bf16_kernel<3, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 4: layernorm_bf16_kernel<4, OutT><<<grid_for(layernorm_bf16_kernel<4, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 5: layernorm_bf16_kernel<5, OutT><<<grid_for(layernorm_bf16_kernel<5, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 6: layernorm_bf16_kernel<6, OutT><<<grid_for(layernorm_bf16_kernel<6, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 7: layernorm_bf16_kernel<7, OutT><<<grid_for(layernorm_bf16_kernel<7, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    case 8: layernorm_bf16_kernel<8, OutT><<<grid_for(layernorm_bf16_kernel<8, OutT>), threads, smem, st>>>(x, g, b, y, T, d, eps); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_layernorm_bf16(const bf16 *x, const float *g, const float *b, bf16 *y, int T, int d, float eps,
                                  cudaStream_t st) {
  return layernorm_bf16_any(x, g, b, y, T, d, eps, st);
}

cudaError_t launch_layernorm_bf16_f32out(const bf16 *x, const float *g, const float *b, float *y, int T, int d,
                                         float eps, cudaStream_t st) {
  return layernorm_bf16_any(x, g, b, y, T, d, eps, st);
}

// ---------------------------------------------------------------------------
// Weight packing (run once per weight load).
// ---------------------------------------------------------------------------
// kgain (optional): a factor per element of the K axis of the packed [N, K]
// result (src columns without transpose, src rows with it), for the
// gain-scaled weights of a folded LayerNorm.
__global__ void pack_bf16_kernel(const float *__restrict__ src, bf16 *__restrict__ dst, int rows, int cols,
                                 int transpose, const float *__restrict__ kgain) {
  __shared__ float tile[32][33];
  const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
  if (!transpose) {
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int r = by + i, c = bx + threadIdx.x;
      if (r < rows && c < cols)
        dst[(int64_t)r * cols + c] = __float2bfloat16_rn(src[(int64_t)r * cols + c] * (kgain ? kgain[c] : 1.f));
    }
    return;
  }
  // dst[cols, rows] = src[rows, cols]^T
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = by + i, c = bx + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? src[(int64_t)r * cols + c] * (kgain ? kgain[r] : 1.f) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = bx + i, r = by + threadIdx.x;
    if (c < cols && r < rows) dst[(int64_t)c * rows + r] = __float2bfloat16_rn(tile[threadIdx.x][i]);
  }
}

__global__ void e4m3_to_bf16_kernel(const uint8_t *__restrict__ src, bf16 *__restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t q = src[i];
    const int e = (q >> 3) & 0xF, m = q & 7;
    // E4M3 value: m * 2^-9 (e == 0) or (1 + m/8) * 2^(e-7); both exact in float and bf16
    const float v = e == 0 ? m * (1.0f / 512.0f) : __int_as_float(((e + 120) << 23) | (m << 20));
    dst[i] = __float2bfloat16_rn((q & 0x80) ? -v : v);
  }
}

cudaError_t launch_e4m3_to_bf16(const uint8_t *src, bf16 *dst, int64_t n, cudaStream_t st) {
  e4m3_to_bf16_kernel<<<1184, 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_pack_bf16(const float *src, bf16 *dst, int rows, int cols, int transpose, cudaStream_t st) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  pack_bf16_kernel<<<grid, block, 0, st>>>(src, dst, rows, cols, transpose, nullptr);
  return cudaGetLastError();
}

// c1[n] = sum_k Wp[n, k] (the bf16 gain-scaled weight the GEMM multiplies),
// c2[n] = sum_k W[n, k] * shift[k] + bias[n] (the FP32 master weight), in
// double; one warp per n, zeros in the padding up to npad.
__global__ void ln_fold_vectors_kernel(const float *__restrict__ W, int w_kn, const float *__restrict__ shift,
                                       const float *__restrict__ bias, const bf16 *__restrict__ Wp,
                                       float *__restrict__ c1, float *__restrict__ c2, int N, int K, int npad) {
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= npad) return;
  double a = 0.0, b = 0.0;
  if (n < N) {
    for (int k = lane; k < K; k += 32) {
      a += (double)__bfloat162float(Wp[(int64_t)n * K + k]);
      const float w = w_kn ? W[(int64_t)k * N + n] : W[(int64_t)n * K + k];
      b += (double)w * (double)shift[k];
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, off);
    b += __shfl_xor_sync(0xffffffffu, b, off);
  }
  if (lane == 0) {
    c1[n] = n < N ? (float)a : 0.f;
    c2[n] = n < N ? (float)(b + (bias ? (double)bias[n] : 0.0)) : 0.f;
  }
}

cudaError_t launch_ln_fold_pack(const float *W, int w_kn, const float *gain, const float *shift, const float *bias,
                                bf16 *Wp, float *c1, float *c2, int N, int K, cudaStream_t st) {
  if (N <= 0 || K <= 0 || !W || !gain || !shift || !Wp || !c1 || !c2) return cudaErrorInvalidValue;
  // Wp [N, K]: from W [K, N] transposed (w_kn) or W [N, K] as stored.
  const int rows = w_kn ? K : N, cols = w_kn ? N : K;
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  pack_bf16_kernel<<<grid, block, 0, st>>>(W, Wp, rows, cols, w_kn, gain);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int npad = (int)ln_vector_len(N);
  ln_fold_vectors_kernel<<<(npad + 7) / 8, 256, 0, st>>>(W, w_kn, shift, bias, Wp, c1, c2, N, K, npad);
  return cudaGetLastError();
}

}  // namespace gpt2
