// attention_f32.cu -- exact-FP32 fused causal attention (flash-style online
// softmax) for head dim 64, the verification path of the GPT-2 forward.
//
// Replaces, per layer, the reference's two linalg.batch_matmul (q k^T and
// p v), the 1/sqrt(64) scale, the causal `where` against the 1024x1024 bool
// buffer, the additive padding mask and the max / sub / exp / sum / div
// softmax chain (src/gpt/README.md:6, lib/DeadArgmaxElimination.cpp:4-6):
// the S x S scores never leave shared memory and no argmax is computed.
//
// With causal = 0 it is the BERT encoder's self-attention
// (src/bert-base-uncased/lower_bert_model.py:12-18: every key of the
// sequence, padding mask only).
//
// Semantics (identical to the reference on every row that has at least one
// attendable key): key k is attendable from query q iff mask[b, k] != 0 and,
// when causal, k <= q; masked keys weigh exactly 0 (exp(finfo.min - max) == 0 in
// FP32).  Rows without an attendable key are finished by
// attn_masked_rows_*_kernel (mean of V over all S keys, which is what the
// reference's uniform finfo.min row produces).
//
// Block: 64 queries x one (batch, head), 256 threads; each thread owns a 4x4
// block of scores and a 4x4 block of the output (rows ty*4.., columns tx*4..).
// The 16 threads of a row sit in one half-warp, so row max / sum reductions
// are 4 xor-shuffles.  expf is CUDA's accurate expf (no fast-math).
#include <math.h>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int DH = 64, BQ = 64, BKV = 64, NT = 256, PLD = 68;

struct AttnSmem {
  float qt[DH][BQ];    // Q transposed
  float kt[DH][BKV];   // K transposed
  float vs[BKV][DH];   // V
  float ps[BQ][PLD];   // probabilities
};

__device__ __forceinline__ float hsum16(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  return v;
}
__device__ __forceinline__ float hmax16(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  return v;
}

__global__ void __launch_bounds__(NT) attention_f32_kernel(const float *__restrict__ qkv,
                                                           const uint8_t *__restrict__ key_valid,
                                                           float *__restrict__ o, int S, int H, int causal) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_raw);
  const int nqb = (S + BQ - 1) / BQ;
  const int qb = nqb - 1 - blockIdx.x;  // heaviest query blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int D = H * DH;
  const int64_t ld = 3 * (int64_t)D;
  const float *base = qkv + (int64_t)b * S * ld;
  const uint8_t *kv_ok = key_valid ? key_valid + (int64_t)b * S : nullptr;
  const int q0 = qb * BQ;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const float scale = 1.0f / sqrtf((float)DH);

  // Q tile, transposed: element (q, d) -> qt[d][q].
  for (int idx = tid; idx < BQ * DH / 4; idx += NT) {
    const int q = idx % BQ, d4 = (idx / BQ) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + q < S) v = *reinterpret_cast<const float4 *>(base + (int64_t)(q0 + q) * ld + h * DH + d4);
    sm.qt[d4 + 0][q] = v.x;
    sm.qt[d4 + 1][q] = v.y;
    sm.qt[d4 + 2][q] = v.z;
    sm.qt[d4 + 3][q] = v.w;
  }

  float acc[4][4], m_run[4], l_run[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m_run[r] = -INFINITY;
    l_run[r] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
  }

  const int kv_end = causal ? min(S, q0 + BQ) : S;  // causal: keys beyond the last query are never needed
  for (int kv0 = 0; kv0 < kv_end; kv0 += BKV) {
    __syncthreads();
    for (int idx = tid; idx < BKV * DH / 4; idx += NT) {
      const int k = idx % BKV, d4 = (idx / BKV) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kv0 + k < S) kv = *reinterpret_cast<const float4 *>(base + (int64_t)(kv0 + k) * ld + D + h * DH + d4);
      sm.kt[d4 + 0][k] = kv.x;
      sm.kt[d4 + 1][k] = kv.y;
      sm.kt[d4 + 2][k] = kv.z;
      sm.kt[d4 + 3][k] = kv.w;
    }
    for (int idx = tid; idx < BKV * DH / 4; idx += NT) {
      const int k = idx / (DH / 4), d4 = (idx % (DH / 4)) * 4;
      float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kv0 + k < S) vv = *reinterpret_cast<const float4 *>(base + (int64_t)(kv0 + k) * ld + 2 * D + h * DH + d4);
      *reinterpret_cast<float4 *>(&sm.vs[k][d4]) = vv;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[r][c] = 0.f;
#pragma unroll 8
    for (int d = 0; d < DH; ++d) {
      const float4 a = *reinterpret_cast<const float4 *>(&sm.qt[d][ty * 4]);
      const float4 k4 = *reinterpret_cast<const float4 *>(&sm.kt[d][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[r][c] = fmaf(av[r], kv[c], s[r][c]);
    }

#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qi = q0 + ty * 4 + r;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int kj = kv0 + tx * 4 + c;
        const bool ok = (!causal || kj <= qi) && kj < S && (!kv_ok || kv_ok[kj]);
        s[r][c] = ok ? s[r][c] * scale : -INFINITY;
        mt = fmaxf(mt, s[r][c]);
      }
      mt = hmax16(mt);
      const float m_new = fmaxf(m_run[r], mt);
      float alpha, rs = 0.f;
      if (m_new == -INFINITY) {
        alpha = 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) s[r][c] = 0.f;
      } else {
        alpha = expf(m_run[r] - m_new);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s[r][c] = expf(s[r][c] - m_new);
          rs += s[r][c];
        }
      }
      rs = hsum16(rs);
      l_run[r] = l_run[r] * alpha + rs;
      m_run[r] = m_new;
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] *= alpha;
      *reinterpret_cast<float4 *>(&sm.ps[ty * 4 + r][tx * 4]) = make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
    }
    __syncthreads();

#pragma unroll 4
    for (int j = 0; j < BKV; ++j) {
      const float4 v4 = *reinterpret_cast<const float4 *>(&sm.vs[j][tx * 4]);
      const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float p = sm.ps[ty * 4 + r][j];
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(p, vv[c], acc[r][c]);
      }
    }
  }

#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int qi = q0 + ty * 4 + r;
    if (qi >= S) continue;
    const float inv = l_run[r] > 0.f ? 1.0f / l_run[r] : 0.f;
    *reinterpret_cast<float4 *>(o + ((int64_t)b * S + qi) * D + h * DH + tx * 4) =
        make_float4(acc[r][0] * inv, acc[r][1] * inv, acc[r][2] * inv, acc[r][3] * inv);
  }
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// One block per (head, batch), one thread per head column.
template <typename T>
__global__ void attn_masked_rows_kernel(const T *__restrict__ qkv, const int *__restrict__ first_valid,
                                        T *__restrict__ o, int S, int H, int causal) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int nrows = causal ? min(first_valid[b], S) : (first_valid[b] >= S ? S : 0);
  if (nrows == 0) return;
  const int D = H * DH;
  const int64_t ld = 3 * (int64_t)D;
  const T *v = qkv + (int64_t)b * S * ld + 2 * D + h * DH + d;
  float sum = 0.f;
  for (int k = 0; k < S; ++k) sum += to_f<T>(v[(int64_t)k * ld]);
  const T mean = from_f<T>(sum / (float)S);
  for (int q = 0; q < nrows; ++q) o[((int64_t)b * S + q) * D + h * DH + d] = mean;
}
}  // namespace

cudaError_t launch_attention_f32(const float *qkv, const uint8_t *key_valid, float *o, int B, int S, int H,
                                 cudaStream_t st, int causal) {
  if (B <= 0 || S <= 0 || H <= 0 || H > 65535 || B > 65535) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  const int smem = (int)sizeof(AttnSmem);
  cudaError_t e = set_smem_once(attention_f32_kernel, smem, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid((S + BQ - 1) / BQ, H, B);
  attention_f32_kernel<<<grid, NT, smem, st>>>(qkv, key_valid, o, S, H, causal);
  return cudaGetLastError();
}

cudaError_t launch_attn_masked_rows_f32(const float *qkv, const int *first_valid, float *o, int B, int S, int H,
                                        cudaStream_t st, int causal) {
  attn_masked_rows_kernel<float><<<dim3(H, B), DH, 0, st>>>(qkv, first_valid, o, S, H, causal);
  return cudaGetLastError();
}

cudaError_t launch_attn_masked_rows_bf16(const bf16 *qkv, const int *first_valid, bf16 *o, int B, int S, int H,
                                         cudaStream_t st, int causal) {
  attn_masked_rows_kernel<bf16><<<dim3(H, B), DH, 0, st>>>(qkv, first_valid, o, S, H, causal);
  return cudaGetLastError();
}

}  // namespace gpt2
