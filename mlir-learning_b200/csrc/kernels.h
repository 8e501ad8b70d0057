// kernels.h -- host launchers of the GPT-2 device kernels (internal API of
// libgpt2_b200.so; the public C ABI is include/gpt2_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace gpt2 {

typedef __nv_bfloat16 bf16;

// Raises a kernel's dynamic shared-memory limit once per device (the
// attribute is per device; `done` holds one bit per device ordinal).
template <typename Kernel>
inline cudaError_t set_smem_once(Kernel kernel, int bytes, std::atomic<uint64_t> &done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load() & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

// Epilogue applied to C = A @ B (+ ...), fused into every GEMM:
//   EPI_NONE       C = acc
//   EPI_BIAS       C = acc + bias[col]
//   EPI_BIAS_GELU  C = gelu_new(acc + bias[col])
//   EPI_BIAS_RESID C = resid[row, col] + (acc + bias[col])   (resid may alias C)
//   EPI_BIAS_GELU_ERF C = gelu(acc + bias[col]), the exact (erf) GELU of BERT
//   EPI_LN_BIAS    C = rstd[row] * acc - rstd[row] * mean[row] * c1[col] + c2[col]
//   EPI_LN_BIAS_GELU  gelu_new of the same: a LayerNorm of A folded into the
//                  GEMM (LnFold below)
//   EPI_BIAS_RESID_STATS  EPI_BIAS_RESID, and the row statistics of the bf16
//                  C it stores for the LayerNorm folded into the next GEMM
//   EPI_LN_BIAS_GELU_ERF  the erf GELU of EPI_LN_BIAS (BERT's intermediate
//                  layer after its folded attention-output LayerNorm)
//   EPI_LNRES_BIAS_RESID_STATS  EPI_BIAS_RESID_STATS with a LayerNorm applied
//                  to the residual as it is read: C = LN(resid)[row, col] +
//                  acc + bias[col], LN from the residual rows' statistics and
//                  the gain / shift of LnFold (BERT's post-LN residual
//                  stream, kept un-normalised in memory)
enum Epilogue : int {
  EPI_NONE = 0,
  EPI_BIAS = 1,
  EPI_BIAS_GELU = 2,
  EPI_BIAS_RESID = 3,
  EPI_BIAS_GELU_ERF = 4,
  EPI_LN_BIAS = 5,
  EPI_LN_BIAS_GELU = 6,
  EPI_BIAS_RESID_STATS = 7,
  EPI_LN_BIAS_GELU_ERF = 8,
  EPI_LNRES_BIAS_RESID_STATS = 9,
};

// A pre-LayerNorm folded into the GEMM that consumes it:
//   LN(x) @ W^T + bias = rstd * (x @ W'^T) - rstd * mean * c1 + c2,
//   W'[n, k] = bf16(W[n, k] * gain[k]),  c1[n] = sum_k W'[n, k],
//   c2[n] = sum_k W[n, k] * shift[k] + bias[n],
// so the GEMM reads x itself and the LayerNorm kernel and its output go
// away.  mean and rstd come from row statistics that the producer of x (the
// embedding or a residual GEMM) writes while it stores x: per row and per
// LN_SEG-column segment, the sum and the sum of squares of the bf16 values.
constexpr int LN_SEG = 128;
struct LnFold {
  const float *c1 = nullptr, *c2 = nullptr;  // [N rounded up to 256], 16-byte aligned, zero past N
  const float2 *stats_in = nullptr;          // [M][nseg_in] statistics of A's rows
  int nseg_in = 0, k = 0;                    // ceil(k / LN_SEG); the row width (K)
  float eps = 1e-5f;
  float2 *stats_out = nullptr;               // [M][nseg_out] of C's rows (EPI_BIAS_RESID_STATS)
  int nseg_out = 0;                          // ceil(N / LN_SEG)
  // EPI_LNRES_BIAS_RESID_STATS: the residual's LayerNorm (width N).
  const float2 *res_stats = nullptr;         // [M][nseg_out] statistics of the residual rows
  const float *res_gain = nullptr, *res_shift = nullptr;  // [N], 16-byte aligned
};
inline int ln_segments(int width) { return (width + LN_SEG - 1) / LN_SEG; }
inline int64_t ln_vector_len(int n) { return ((int64_t)n + 255) / 256 * 256; }
// W' (bf16 [N, K], transposed from a [K, N] master when w_kn) and c1 / c2.
cudaError_t launch_ln_fold_pack(const float *W, int w_kn, const float *gain, const float *shift, const float *bias,
                                bf16 *Wp, float *c1, float *c2, int N, int K, cudaStream_t st);

// ---- sequence / mask preparation -------------------------------------------
// first_valid[b] = smallest k with mask[b, k] != 0 (S if none);
// key_valid[b*S + k] = mask[b, k] != 0; kv_end[b] (optional) = 1 + the
// largest such k (0 if none).  mask is contiguous [B, S] int64.
cudaError_t launch_seq_info(const int64_t *mask, int B, int S, int *first_valid, uint8_t *key_valid,
                            cudaStream_t st, int *kv_end = nullptr);

// ---- FP32 SIMT throughput, measured (denominator of the exact-FP32 roofline) ----
cudaError_t measure_ffma_peak(float *tflops, cudaStream_t st);

// ---- embedding: x[t] = wte[ids[t]] + wpe[t % S] -------------------------------
cudaError_t launch_embed_f32(const int64_t *ids, const float *wte, const float *wpe, float *x, int T, int S, int d,
                             int V, int *status, cudaStream_t st);
// stats (optional, [T][ceil(d / LN_SEG)]): the row statistics of the bf16 x
// for a LayerNorm folded into the next GEMM (LnFold).
cudaError_t launch_embed_bf16(const int64_t *ids, const bf16 *wte, const bf16 *wpe, bf16 *x, int T, int S, int d,
                              int V, int *status, cudaStream_t st, float2 *stats = nullptr);

// ---- LayerNorm (biased variance, FP32 statistics) ----------------------------
cudaError_t launch_layernorm_f32(const float *x, const float *g, const float *b, float *y, int T, int d, float eps,
                                 cudaStream_t st);
cudaError_t launch_layernorm_bf16(const bf16 *x, const float *g, const float *b, bf16 *y, int T, int d, float eps,
                                  cudaStream_t st);
cudaError_t launch_layernorm_bf16_f32out(const bf16 *x, const float *g, const float *b, float *y, int T, int d,
                                         float eps, cudaStream_t st);

// ---- BERT encoder ------------------------------------------------------------
// x[t] = LayerNorm(word[ids[t]] + pos[p(t)] + type[tt[t]]) with p(t) =
// pos_ids[t % S] (t % S when pos_ids is null) and tt null meaning type 0;
// FP32 tables, FP32 statistics; ids / types / positions out of range record
// status 1 and read row 0.  d % 4 == 0, d <= 2048.
cudaError_t launch_bert_embed_ln_f32(const int64_t *ids, const int64_t *tt, const int64_t *pos_ids, const float *word,
                                     const float *pos, const float *type, const float *g, const float *b, float *x,
                                     int T, int S, int d, int V, int P, int TV, float eps, int *status,
                                     cudaStream_t st);
cudaError_t launch_bert_embed_ln_bf16(const int64_t *ids, const int64_t *tt, const int64_t *pos_ids,
                                      const float *word, const float *pos, const float *type, const float *g,
                                      const float *b, bf16 *x, int T, int S, int d, int V, int P, int TV, float eps,
                                      int *status, cudaStream_t st);
// pooled[b, n] = tanh(hidden[b, 0, :] . w[n, :] + bias[n]) (nn.Linear [out, in]).
cudaError_t launch_bert_pooler(const float *hidden, const float *w, const float *bias, float *pooled, int B, int S,
                               int d, cudaStream_t st);

// ---- exact-FP32 SIMT GEMM ----------------------------------------------------
// C[M, N] (row stride ldc) = epilogue(A[M, K] @ op(B)), op(B) = B[K, N] when
// b_nk == 0 (Conv1D weight) or B[N, K]^T when b_nk == 1 (tied lm_head).
// resid has row stride ldc.
cudaError_t launch_gemm_f32(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                            const float *bias, const float *resid, int epi, cudaStream_t st);

// ---- tcgen05 BF16 GEMM -------------------------------------------------------
// C[M, N] = epilogue(A[M, K] @ B[N, K]^T), A and B bf16 K-major, f32 accumulate
// in TMEM.  out_f32 selects an FP32 output (lm_head logits) instead of bf16.
struct TcGemmPlan {
  CUtensorMap map_a;
  CUtensorMap map_b;
  CUtensorMap map_c;  // output, when the output can be stored by TMA
  int M, N, K;
  int bn;  // width of the B box: 128 or 256
  int two_sm = 0;  // 256 x 256 tiles on CTA pairs (gemm_tc2sm.cu); B boxes of 128 rows
  const void *c_ptr = nullptr;
  int c_ld = 0, c_f32 = 0, has_c = 0;
};
// Builds the TMA descriptors of A and B; returns 0 or a negative error.
// bn = 128 or 256: one SM per 128 x bn output tile (gemm_tc.cu);
// bn = TC_TILE_PAIR: two SMs per 256 x 256 tile (gemm_tc2sm.cu), used when
// C can be stored by TMA (else the 128 x 128 single-SM kernel runs).
constexpr int TC_TILE_PAIR = 2;
int tc_gemm_plan(TcGemmPlan *plan, const bf16 *A, const bf16 *B, int M, int N, int K, int bn);
// Builds the output descriptor for C (row stride ldc elements, f32 or bf16)
// when C is 16-byte aligned and ldc * element size is a multiple of 16;
// otherwise the kernel falls back to direct stores.  Returns has_c.
int tc_gemm_set_output(TcGemmPlan *plan, const void *C, int ldc, int out_f32);
// scale (optional, [N]): per-output-column factor applied to the accumulator
// before the epilogue (weight-only FP8 dequantization).
// ln: the folded LayerNorm of EPI_LN_* and the statistics output of
// EPI_BIAS_RESID_STATS (checked by ln_fold_valid).
cudaError_t launch_gemm_tc(const TcGemmPlan &plan, void *C, int ldc, int out_f32, const float *bias,
                           const bf16 *resid, int epi, int *status, int num_sms, cudaStream_t st,
                           const float *scale = nullptr, const LnFold *ln = nullptr);
bool ln_fold_valid(const TcGemmPlan &plan, int epi, int out_f32, const LnFold *ln);
// Test hook of the bounded-wait error path: the single-SM kernel (plan.bn =
// 128, C bf16 [M, N] by direct stores, no epilogue) with CTA 0's producer
// withholding its first stage, so that CTA 0's MMA thread waits for data that
// never comes, gives up after GPT2_WAIT_TIMEOUT_NS, records status 2, and
// every role unwinds (drains what it issued, frees TMEM, returns).
cudaError_t launch_gemm_tc_withheld_load(const TcGemmPlan &plan, void *C, int *status, int num_sms,
                                         cudaStream_t st);
// The CTA-pair kernel (called by launch_gemm_tc for TC_TILE_PAIR plans).
bool gemm_tc2sm_usable(const TcGemmPlan &plan, const void *C, int ldc, int out_f32);
cudaError_t launch_gemm_tc2sm(const TcGemmPlan &plan, void *C, int ldc, int out_f32, const float *bias,
                              const bf16 *resid, int epi, int *status, int num_sms, cudaStream_t st,
                              const float *scale, const LnFold &ln);

// ---- attention ----------------------------------------------------------------
// qkv [B*S, 3*H*64] (q | k | v, head h at columns h*64), o [B*S, H*64].
// key_valid may be null (all keys valid); a query row with no attendable key
// is written by launch_attn_masked_rows afterwards.
// causal = 0: every key of the sequence is attendable (the BERT encoder).
cudaError_t launch_attention_f32(const float *qkv, const uint8_t *key_valid, float *o, int B, int S, int H,
                                 cudaStream_t st, int causal = 1);
// tcgen05 attention: TMA descriptor over qkv viewed as [B][S][3*H*64].
struct AttnTcPlan {
  CUtensorMap map_qkv;
  CUtensorMap map_out;  // o viewed as [B][S][H*64], for the TMA-stored epilogue
  const bf16 *qkv = nullptr;
  const bf16 *out = nullptr;
  int B = 0, S = 0, H = 0;
};
// Builds the qkv descriptor and, when o is given, the output descriptor.
int attention_tc_plan(AttnTcPlan *plan, const bf16 *qkv, int B, int S, int H, const bf16 *o = nullptr);
// tcgen05 attention: three independent 128-query-tile slots per SM over
// 64-key blocks, one softmax thread per query row, P kept in tensor memory
// (the P.V MMA reads its A operand from TMEM); o must be the output the plan
// was built with.  kv_end (optional, [B]): keys at or past kv_end[b] are all
// masked, so their blocks are skipped (right padding costs no attention work).
cudaError_t launch_attention_tc3(const AttnTcPlan &plan, const uint8_t *key_valid, bf16 *o, int *status,
                                 cudaStream_t st, int causal = 1, const int *kv_end = nullptr);
// Rows without an attendable key get the mean of V over all S keys: with the
// causal mask the rows q < first_valid[b]; without it, every row of a
// sequence whose mask is all zero.
cudaError_t launch_attn_masked_rows_f32(const float *qkv, const int *first_valid, float *o, int B, int S, int H,
                                        cudaStream_t st, int causal = 1);
cudaError_t launch_attn_masked_rows_bf16(const bf16 *qkv, const int *first_valid, bf16 *o, int B, int S, int H,
                                         cudaStream_t st, int causal = 1);

// ---- incremental decoding (KV cache; M = B <= 16 rows per product) -----------
// The step's position is read from device memory (*d_pos), so one captured
// step serves every position.
cudaError_t launch_decode_embed_f32(const int64_t *tok, const float *wte, const float *wpe, float *x, int B, int d,
                                    int V, const int *d_pos, int P, int *status, cudaStream_t st);
cudaError_t launch_decode_embed_bf16(const int64_t *tok, const bf16 *wte, const bf16 *wpe, bf16 *x, int B, int d,
                                     int V, const int *d_pos, int P, int *status, cudaStream_t st);
// y[M, N] (row stride ldy) = epi(x[M, K] @ W[N, K]^T); resid has stride ldy;
// scale (optional) multiplies the product per column before the epilogue.
// ln (optional): a LayerNorm of x's rows (gain, shift over K, eps) applied
// inside the kernel before the product; with EPI_NONE / EPI_BIAS /
// EPI_BIAS_GELU only.
struct GemvLn {
  const float *gain = nullptr, *shift = nullptr;
  float eps = 1e-5f;
};
//
// pdl (here and in the short / decode attention launchers): launch as a
// programmatic dependent of the previous kernel on st (which must be a
// kernel): the grid may start while that kernel runs, prefetches its weights
// into L2, and waits (griddepcontrol.wait) for the previous grid to complete
// before it reads anything that grid or an earlier one wrote.  Environment
// GPT2_PDL=0 turns it off.
cudaError_t launch_gemv_f32(const float *x, const float *W, float *y, int M, int N, int K, int ldy, const float *bias,
                            const float *resid, int epi, cudaStream_t st, const GemvLn *ln = nullptr,
                            bool pdl = false);
cudaError_t launch_gemv_bf16(const bf16 *x, const bf16 *W, bf16 *y, int M, int N, int K, int ldy, const float *bias,
                             const bf16 *resid, const float *scale, int epi, cudaStream_t st,
                             const GemvLn *ln = nullptr, bool pdl = false);
cudaError_t launch_gemv_bf16_f32out(const bf16 *x, const bf16 *W, float *y, int M, int N, int K, int ldy,
                                    cudaStream_t st, const GemvLn *ln = nullptr, bool pdl = false);
// Programmatic dependent launch of the few-token chain: on unless the
// environment sets GPT2_PDL=0.
bool pdl_enabled();
// The same products on the tensor cores (gemv_tc.cu): bf16 weights W[N, K]
// (16-byte aligned, K a multiple of 64 that splits into at most 8 slices of
// at most 6 k-steps), x 16-byte aligned, M <= 16 rows.  Epilogues EPI_NONE,
// EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_GELU_ERF (ln allowed) and
// EPI_BIAS_RESID (no ln); a wait timeout records status 2 in *status.
bool gemv_tc_supported(int M, int N, int K, int ldy);
cudaError_t launch_gemv_tc_bf16(const bf16 *x, const bf16 *W, bf16 *y, int M, int N, int K, int ldy,
                                const float *bias, const bf16 *resid, const float *scale, int epi, int *status,
                                cudaStream_t st, const GemvLn *ln = nullptr, bool pdl = false);
cudaError_t launch_gemv_tc_bf16_f32out(const bf16 *x, const bf16 *W, float *y, int M, int N, int K, int ldy,
                                       int *status, cudaStream_t st, const GemvLn *ln = nullptr, bool pdl = false);
// The few-token and decode products: the tensor-core kernel where
// gemv_tc_supported, else launch_gemv_bf16 (environment GPT2_GEMV_TC=0: always
// the SIMT kernel).
bool gemv_tc_enabled();
cudaError_t launch_gemv_bf16_auto(const bf16 *x, const bf16 *W, bf16 *y, int M, int N, int K, int ldy,
                                  const float *bias, const bf16 *resid, const float *scale, int epi, int *status,
                                  cudaStream_t st, const GemvLn *ln = nullptr, bool pdl = false);
cudaError_t launch_gemv_bf16_f32out_auto(const bf16 *x, const bf16 *W, float *y, int M, int N, int K, int ldy,
                                         int *status, cudaStream_t st, const GemvLn *ln = nullptr, bool pdl = false);
// Attention of sequences of S <= 16 tokens (one warp per query row); rows
// with no attendable key are left for launch_attn_masked_rows_*.
cudaError_t launch_attention_short_f32(const float *qkv, const uint8_t *key_valid, float *o, int B, int S, int H,
                                      int causal, cudaStream_t st, bool pdl = false);
cudaError_t launch_attention_short_bf16(const bf16 *qkv, const uint8_t *key_valid, bf16 *o, int B, int S, int H,
                                       int causal, cudaStream_t st, bool pdl = false);
// cache [B][max_len][2D] (keys | values of every head) <- qkv rows of positions pos0 ..
cudaError_t launch_kv_store_f32(const float *qkv, float *cache, int B, int S, int D, int max_len, int pos0,
                                cudaStream_t st);
cudaError_t launch_kv_store_bf16(const bf16 *qkv, bf16 *cache, int B, int S, int D, int max_len, int pos0,
                                 cudaStream_t st);
// One query per sequence at position *d_pos (qkv [B, 3D]) against cache
// positions 0 .. pos - 1 plus its own key / value, which it appends; a
// position at or past max_len records status 3 and changes nothing.
cudaError_t launch_attn_decode_f32(const float *qkv, float *cache, float *out, int B, int H, const int *d_pos,
                                   int max_len, int *status, cudaStream_t st, bool pdl = false);
cudaError_t launch_attn_decode_bf16(const bf16 *qkv, bf16 *cache, bf16 *out, int B, int H, const int *d_pos,
                                    int max_len, int *status, cudaStream_t st, bool pdl = false);
cudaError_t launch_set_int(int *p, int v, cudaStream_t st);
cudaError_t launch_add_int(int *p, int v, cudaStream_t st);
// hist[(*d_pos - base) * B + b] = cur[b] for b < B (bounded by cap entries)
cudaError_t launch_append_tokens(const int64_t *cur, int64_t *hist, const int *d_pos, int base, int B, int cap,
                                 cudaStream_t st);
// tokens[b] = first argmax of logits[b, :V]
cudaError_t launch_argmax_rows(const float *logits, int64_t ld, int B, int V, int64_t *tokens, cudaStream_t st);
// dst[cols, rows] = src[rows, cols]^T (FP32)
cudaError_t launch_transpose_f32(const float *src, float *dst, int rows, int cols, cudaStream_t st);

// ---- weight packing --------------------------------------------------------
// dst[i] = bf16(decode_e4m3(src[i])), exact (every E4M3 value is a BF16 value).
cudaError_t launch_e4m3_to_bf16(const uint8_t *src, bf16 *dst, int64_t n, cudaStream_t st);
// dst[N, K] (bf16) = transpose(src[K, N] fp32); dst[r, c] = bf16(src[r, c]) when transpose == 0.
cudaError_t launch_pack_bf16(const float *src, bf16 *dst, int rows, int cols, int transpose, cudaStream_t st);

}  // namespace gpt2
