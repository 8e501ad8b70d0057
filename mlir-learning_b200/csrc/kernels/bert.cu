// bert.cu -- the two kernels the BERT encoder needs beyond the GPT-2 set:
// the fused embedding sum + LayerNorm and the pooler.
//
// Replaces the reference BERT export's embedding gathers (word, position,
// token type), their adds and the embeddings LayerNorm generics, and the
// pooler's first-token slice, matmul, bias and tanh
// (src/bert-base-uncased/lower_bert_model.py:12-18, the last_hidden_state /
// pooler_output pair of call_bert.cpp:41-44), one launch each.
#include <math.h>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
// One warp per token: the three FP32 rows are summed in registers
// ((word + position) + type, the order of transformers' BertEmbeddings),
// normalised with FP32 mean and centred variance, and written once.
template <int VPT, typename OutT>
__global__ void bert_embed_ln_kernel(const int64_t *__restrict__ ids, const int64_t *__restrict__ tt,
                                     const int64_t *__restrict__ pos_ids, const float *__restrict__ word,
                                     const float *__restrict__ pos, const float *__restrict__ type,
                                     const float *__restrict__ g, const float *__restrict__ b, OutT *__restrict__ x,
                                     int T, int S, int d, int V, int P, int TV, float eps, int *status) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int64_t id = ids[row];
  const int64_t ty = tt ? tt[row] : 0;
  const int64_t p = pos_ids ? pos_ids[row % S] : row % S;
  const bool ok = id >= 0 && id < V && ty >= 0 && ty < TV && p >= 0 && p < P;
  if (!ok && lane == 0) set_status(status, GPT2_ERR_TOKEN_RANGE);
  const float4 *wr = reinterpret_cast<const float4 *>(word + (ok ? id : 0) * (int64_t)d);
  const float4 *pr = reinterpret_cast<const float4 *>(pos + (ok ? p : 0) * (int64_t)d);
  const float4 *tr = reinterpret_cast<const float4 *>(type + (ok ? ty : 0) * (int64_t)d);
  const int nv = d / 4;
  float4 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      const float4 a = wr[c], e = pr[c], f = tr[c];
      v[i] = make_float4((a.x + e.x) + f.x, (a.y + e.y) + f.y, (a.z + e.z) + f.z, (a.w + e.w) + f.w);
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
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
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      const float4 gg = g4[c], bb = b4[c];
      const float o0 = (v[i].x - mean) * rstd * gg.x + bb.x, o1 = (v[i].y - mean) * rstd * gg.y + bb.y;
      const float o2 = (v[i].z - mean) * rstd * gg.z + bb.z, o3 = (v[i].w - mean) * rstd * gg.w + bb.w;
      if constexpr (sizeof(OutT) == 4) {
        reinterpret_cast<float4 *>(x + (int64_t)row * d)[c] = make_float4(o0, o1, o2, o3);
      } else {
        reinterpret_cast<uint2 *>(x + (int64_t)row * d)[c] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
      }
    }
  }
}

template <typename OutT>
cudaError_t launch_embed_ln(const int64_t *ids, const int64_t *tt, const int64_t *pos_ids, const float *word,
                            const float *pos, const float *type, const float *g, const float *b, OutT *x, int T,
                            int S, int d, int V, int P, int TV, float eps, int *status, cudaStream_t st) {
  if (T <= 0 || S <= 0 || d % 4 || d > 128 * 16) return cudaErrorInvalidValue;
  const int threads = 256, blocks = (T + threads / 32 - 1) / (threads / 32);
#define EMB_CASE(N)                                                                                           \
  case N:                                                                                                     \
    bert_embed_ln_kernel<N, OutT><<<blocks, threads, 0, st>>>(ids, tt, pos_ids, word, pos, type, g, b, x, T, S, \
                                                              d, V, P, TV, eps, status);                      \
    break;
  switch ((d + 127) / 128) {
    EMB_CASE(1)
    EMB_CASE(2)
    EMB_CASE(3)
    EMB_CASE(4)
    EMB_CASE(5)
    EMB_CASE(6)
    EMB_CASE(7)
    EMB_CASE(8)
    EMB_CASE(12)
    EMB_CASE(16)
    default:
      if ((d + 127) / 128 <= 12) {
        bert_embed_ln_kernel<12, OutT><<<blocks, threads, 0, st>>>(ids, tt, pos_ids, word, pos, type, g, b, x, T,
                                                                   S, d, V, P, TV, eps, status);
      } else {
        bert_embed_ln_kernel<16, OutT><<<blocks, threads, 0, st>>>(ids, tt, pos_ids, word, pos, type, g, b, x, T,
                                                                   S, d, V, P, TV, eps, status);
      }
  }
#undef EMB_CASE
  return cudaGetLastError();
}

// One warp per pooled element (b, n): the dot product of the sequence's
// first hidden row with weight row n, lanes striding 16-byte vectors, then
// tanh (CUDA's accurate tanhf).
__global__ void bert_pooler_kernel(const float *__restrict__ hidden, const float *__restrict__ w,
                                   const float *__restrict__ bias, float *__restrict__ pooled, int B, int S, int d) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)B * d) return;
  const int bi = static_cast<int>(gw / d), n = static_cast<int>(gw % d);
  const float4 *h = reinterpret_cast<const float4 *>(hidden + (int64_t)bi * S * d);
  const float4 *wr = reinterpret_cast<const float4 *>(w + (int64_t)n * d);
  float acc = 0.f;
  for (int c = lane; c < d / 4; c += 32) {
    const float4 a = h[c], bb = wr[c];
    acc = fmaf(a.x, bb.x, acc);
    acc = fmaf(a.y, bb.y, acc);
    acc = fmaf(a.z, bb.z, acc);
    acc = fmaf(a.w, bb.w, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) pooled[gw] = tanhf(acc + bias[n]);
}
}  // namespace

cudaError_t launch_bert_embed_ln_f32(const int64_t *ids, const int64_t *tt, const int64_t *pos_ids, const float *word,
                                     const float *pos, const float *type, const float *g, const float *b, float *x,
                                     int T, int S, int d, int V, int P, int TV, float eps, int *status,
                                     cudaStream_t st) {
  return launch_embed_ln(ids, tt, pos_ids, word, pos, type, g, b, x, T, S, d, V, P, TV, eps, status, st);
}

cudaError_t launch_bert_embed_ln_bf16(const int64_t *ids, const int64_t *tt, const int64_t *pos_ids,
                                      const float *word, const float *pos, const float *type, const float *g,
                                      const float *b, bf16 *x, int T, int S, int d, int V, int P, int TV, float eps,
                                      int *status, cudaStream_t st) {
  return launch_embed_ln(ids, tt, pos_ids, word, pos, type, g, b, x, T, S, d, V, P, TV, eps, status, st);
}

cudaError_t launch_bert_pooler(const float *hidden, const float *w, const float *bias, float *pooled, int B, int S,
                               int d, cudaStream_t st) {
  if (B <= 0 || S <= 0 || d % 4) return cudaErrorInvalidValue;
  const int64_t warps = (int64_t)B * d;
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  bert_pooler_kernel<<<static_cast<unsigned>(blocks), threads, 0, st>>>(hidden, w, bias, pooled, B, S, d);
  return cudaGetLastError();
}

}  // namespace gpt2
