/*
 * gpt2_b200.h -- C ABI of libgpt2_b200.so, a B200 (sm_100a) implementation of
 * the GPT-2 forward (prefill) pass that drops in for the object file the
 * reference compiles from its linalg MLIR.
 *
 * No function aborts the process.  Functions returning int return 0 on
 * success and a negative GPT2_E* code on failure; gpt2_last_error() then
 * describes the failure.  The decoder entry points return an all-zero
 * descriptor on failure.
 */
#ifndef GPT2_B200_H
#define GPT2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ------------------------------------------------------------------------ */
/* MLIR memref descriptors                                                   */
/* ------------------------------------------------------------------------ */

/* memref<?x?x?xf32>: the result struct of the reference's compiled
 * gpt2_decoder (src/gpt/gpt2_call.cpp:23-29; layout of the MLIR C ABI,
 * docs/Chapter4.md:97-106). */
typedef struct MemRef3D {
  float *allocated;
  float *aligned;
  int64_t offset;
  int64_t sizes[3];
  int64_t strides[3];
} MemRef3D;

/* memref<?x?xi64>: the token-id and attention-mask operands. */
typedef struct MemRef2D_i64 {
  int64_t *allocated;
  int64_t *aligned;
  int64_t offset;
  int64_t sizes[2];
  int64_t strides[2];
} MemRef2D_i64;

/* ------------------------------------------------------------------------ */
/* Drop-in forward entry points                                              */
/* ------------------------------------------------------------------------ */

/* Replaces the compiled `gpt2_decoder` declared at src/gpt/gpt2_call.cpp:31-37
 * (decomposed memref ABI: memref<1x?xi64> ids, memref<1x?xi64> mask ->
 * memref<1x?x50257xf32> logits).
 *
 * ids / mask: int64 [B, S] with the given offset and strides (any strides);
 * mask value != 0 means "attend" (all ones in the reference call,
 * src/gpt/gpt2_call.cpp:55).  B >= 1 and 1 <= S <= n_positions (the
 * reference's export fixes B = 1 and S <= 128).
 *
 * Returns FP32 logits [B, S, vocab] in host memory obtained from malloc(),
 * contiguous, offset 0, strides {S*V, V, 1}; the caller frees `allocated`
 * with free() as src/gpt/gpt2_call.cpp:94 does.  Synchronous.
 *
 * The model is the one loaded by gpt2_init / gpt2_load_weights /
 * gpt2_init_seeded; when none is loaded, the first call creates GPT-2 small
 * on the current CUDA device with seeded weights (env GPT2_SEED, default
 * 1234; env GPT2_DTYPE = "f32" (default) | "bf16"). */
MemRef3D gpt2_decoder(int64_t *in_alloc, int64_t *in_align, int64_t in_offs, int64_t in_s0, int64_t in_s1,
                      int64_t in_str0, int64_t in_str1, int64_t *mask_alloc, int64_t *mask_align,
                      int64_t mask_offs, int64_t mask_s0, int64_t mask_s1, int64_t mask_str0, int64_t mask_str1);

/* The `-llvm-request-c-wrappers` form of the same function
 * (src/gpt/run_mlir_pipeline.sh:7; convention of docs/Chapter4.md:78-112,
 * e.g. src/bert-base-uncased/call_bert.cpp:46-53).  On failure *result is
 * zeroed. */
void _mlir_ciface_gpt2_decoder(MemRef3D *result, MemRef2D_i64 *input_ids, MemRef2D_i64 *attention_mask);

/* ------------------------------------------------------------------------ */
/* Model configuration and weights (companions; the reference bakes its    */
/* weights into the object as constants, README.md:11, :30)                 */
/* ------------------------------------------------------------------------ */

enum {
  GPT2_DTYPE_F32 = 0,  /* exact FP32 (SIMT FFMA); logits within 1e-4 of the CPU lowering */
  GPT2_DTYPE_BF16 = 1, /* BF16 weights and activations, FP32 accumulate and statistics (tcgen05) */
  GPT2_DTYPE_FP8W = 2  /* as BF16, but the Conv1D weights are E4M3 with a per-output-channel FP32
                          scale (weight-only FP8); embeddings and the tied lm_head stay BF16 */
};

typedef struct Gpt2Config {
  int32_t n_layer;       /* 12 */
  int32_t n_embd;        /* 768; multiple of 64 */
  int32_t n_head;        /* 12; n_embd / n_head must be 64 */
  int32_t n_inner;       /* 3072 */
  int32_t vocab_size;    /* 50257 */
  int32_t n_positions;   /* 1024 */
  float layer_norm_eps;  /* 1e-5 */
  int32_t dtype;         /* GPT2_DTYPE_* */
} Gpt2Config;

/* Error codes (negative returns). */
enum {
  GPT2_EINVAL = -1,   /* bad argument or shape */
  GPT2_ECUDA = -2,    /* a CUDA call failed */
  GPT2_ENOMODEL = -3, /* no model loaded */
  GPT2_EDEVICE = -4,  /* a kernel reported an error in the status word */
  GPT2_ENOMEM = -5
};

/* Creates (or replaces) the process-wide model on CUDA device `device`
 * (-1: the current device).  No weights are loaded yet. */
int gpt2_init(const Gpt2Config *cfg, int device);

/* Number of floats of the canonical FP32 weight blob of `cfg`: tensors in
 * the order wte [V,d], wpe [P,d], then per layer ln_1.{weight,bias},
 * attn.c_attn.{weight [d,3d], bias}, attn.c_proj.{weight [d,d], bias},
 * ln_2.{weight,bias}, mlp.c_fc.{weight [d,ff], bias},
 * mlp.c_proj.{weight [ff,d], bias}, then ln_f.{weight,bias}; Conv1D weights
 * are [in, out] as in HF GPT-2, lm_head is tied to wte. */
int64_t gpt2_blob_floats(const Gpt2Config *cfg);

/* Loads a canonical FP32 blob (bytes == 4 * gpt2_blob_floats).  manifest_json
 * may be NULL, or a JSON object whose "layout" is "gpt2-canonical-f32-v1". */
int gpt2_load_weights(const void *packed, size_t bytes, const char *manifest_json);

/* Reads an HF safetensors checkpoint of a GPT-2 model (transformers names,
 * with or without the "transformer." prefix; F32, F16 or BF16 tensors,
 * widened exactly to FP32) whose shapes match cfg, into out[0 ..
 * gpt2_blob_floats(cfg)) in the canonical order.  Needs no GPU.  Extra
 * tensors (attn.bias buffers, a tied lm_head.weight) are ignored; a missing
 * or mis-shaped tensor is an error naming it. */
int gpt2_safetensors_to_blob(const char *path, const Gpt2Config *cfg, float *out);

/* The same checkpoint loaded into the current model (gpt2_init first). */
int gpt2_load_safetensors(const char *path);

/* Generates the seeded synthetic weights (Philox4x32-10 + Box-Muller) and
 * loads them.  init_mode 0: matrices N(0, 0.02), LayerNorm gain 1, every
 * bias 0.  init_mode 1: also gains 1 + N(0, 0.1) and biases N(0, 0.02). */
int gpt2_init_seeded(uint64_t seed, int init_mode);

/* Fills out[0 .. gpt2_blob_floats(cfg)) with the seeded blob on the host. */
int gpt2_seeded_blob(const Gpt2Config *cfg, uint64_t seed, int init_mode, float *out);

/* Weight-only FP8 quantization of one Conv1D weight w [K in, N out]:
 * scale[n] = max_k |w[k,n]| / 448, q[n*K + k] = E4M3(w[k,n] / scale[n])
 * (round to nearest even, saturating), codes packed [N, K].  The model does
 * this itself at load time for GPT2_DTYPE_FP8W; exported for callers that
 * store quantized checkpoints. */
int gpt2_fp8_quantize(const float *w, int K, int N, uint8_t *q, float *scale);

/* Seeded token ids: ids[i] = floor(w_i * vocab / 2^32), w_i a Philox word. */
int gpt2_seeded_ids(int64_t *ids, int64_t n, uint64_t seed, uint32_t stream, int64_t vocab);

/* Copies the loaded model's configuration into *out (GPT2_ENOMODEL if none). */
int gpt2_get_config(Gpt2Config *out);

/* Releases the model and every device buffer. */
void gpt2_shutdown(void);

/* Text of the last failure on this thread ("" if none). */
const char *gpt2_last_error(void);

/* Device status word of the model (0 = OK; 1 = token id out of range,
 * 2 = a barrier wait timed out, 3 = bad launch); reading clears it. */
int gpt2_status(void);

/* ------------------------------------------------------------------------ */
/* Device-resident forward (benchmarks and device callers)                  */
/* ------------------------------------------------------------------------ */

/* logits [B, S, vocab] (row stride ld_logits >= vocab elements) of the
 * loaded model, everything on the model's device.  Columns [vocab, ld_logits)
 * of a row may be overwritten up to the next 16-byte boundary.  d_ids /
 * d_mask: contiguous int64 [B, S] device arrays (d_mask may be NULL = all
 * ones).  Enqueued on `stream` (a cudaStream_t; NULL = the CUDA default
 * stream); returns when enqueued.
 * logits_dtype GPT2_DTYPE_F32: FP32 logits, the reference's output type
 * (memref<1x?x50257xf32>, src/gpt/gpt2_call.cpp:17-21).  GPT2_DTYPE_BF16:
 * the same FP32-accumulated logits rounded once to bf16 in the lm_head
 * epilogue (half the bytes written, moved over PCIe or NVLink); BF16 and
 * FP8-weight models only, ld_logits a multiple of 8. */
int gpt2_forward_device(const int64_t *d_ids, const int64_t *d_mask, int B, int S, void *d_logits,
                        int64_t ld_logits, int logits_dtype, void *stream);

/* Forward with the host-side contract of gpt2_decoder but caller-owned host
 * buffers: ids / mask contiguous int64 [B, S] (mask may be NULL), logits
 * [B, S, vocab] FP32 host memory.  Copies in, runs, copies out, synchronises. */
int gpt2_forward_host(const int64_t *ids, const int64_t *mask, int B, int S, float *logits);

/* Number of kernel launches one forward of (B, S) enqueues. */
int gpt2_forward_launches(int B, int S, int has_mask);

/* ------------------------------------------------------------------------ */
/* Incremental decoding with a key / value cache                            */
/* ------------------------------------------------------------------------ */
/* The reference generates by re-running the whole forward on the grown
 * sequence (src/gpt/lower_gpt_model.py:190-198, HF generate in
 * src/gpt/run_gpt.py:20-24); these entry points keep every layer's keys and
 * values in HBM so that each new token costs one token's work.  Sequences
 * advance together (all-ones mask).  Logits of a step equal those of the
 * full forward at that position, up to accumulation order. */

/* Reserves the cache for B (1..16) sequences of up to max_len tokens and
 * empties it. */
int gpt2_kv_reserve(int B, int max_len);

/* The forward over d_ids [B, S] (device) that also fills cache positions
 * 0 .. S-1; writes only the last position's logits, d_logits [B, ld_logits]. */
int gpt2_prefill(const int64_t *d_ids, int B, int S, float *d_logits, int64_t ld_logits, void *stream);

/* One token per sequence (d_tokens [B], device) at the next position;
 * d_logits [B, ld_logits].  Fails when the cache is full. */
int gpt2_decode_step(const int64_t *d_tokens, int B, float *d_logits, int64_t ld_logits, void *stream);

/* Positions currently cached. */
int gpt2_kv_length(void);

/* Greedy generation (argmax, first maximum on ties): prompt ids [B, S]
 * (host), n_new tokens per sequence into out_tokens [B, n_new] (host).
 * Synchronous. */
int gpt2_generate(const int64_t *ids, int B, int S, int n_new, int64_t *out_tokens);

/* Per-kernel timing: between gpt2_profile_begin() and gpt2_profile_end(),
 * every launch of the forward is bracketed by CUDA events on its stream.
 * gpt2_profile_end waits for them and writes, per kernel kind, the summed
 * milliseconds and the launch count.  Kinds: 0 seq_info, 1 embed,
 * 2 layernorm, 3 qkv GEMM, 4 attention, 5 masked-row fix-up, 6 attention
 * out-proj GEMM, 7 MLP fc GEMM, 8 MLP proj GEMM, 9 lm_head GEMM. */
enum { GPT2_KERNEL_KINDS = 10 };
int gpt2_profile_begin(void);
int gpt2_profile_end(double *ms_per_kind, int64_t *launches_per_kind, int n_kinds);

/* ------------------------------------------------------------------------ */
/* Kernel-level entry points (device pointers, enqueued on `stream`)         */
/* ------------------------------------------------------------------------ */

/* Epilogues fused into the GEMMs. */
enum { GPT2_EPI_NONE = 0, GPT2_EPI_BIAS = 1, GPT2_EPI_BIAS_GELU = 2, GPT2_EPI_BIAS_RESID = 3,
       GPT2_EPI_BIAS_GELU_ERF = 4 /* exact erf GELU of the BERT intermediate layer */,
       GPT2_EPI_LN_BIAS = 5 /* a LayerNorm of A folded in (gpt2k_gemm_bf16_ln) */,
       GPT2_EPI_LN_BIAS_GELU = 6 /* the same, then gelu_new */,
       GPT2_EPI_BIAS_RESID_STATS = 7 /* EPI_BIAS_RESID and the row statistics of C */ };

/* The call a BLAS lowering of linalg.matmul emits, on the GPU: the argument
 * list of cblas_sgemm exactly as lib/ConvertMatMulToBlas.cpp:84-160 builds it
 * (CblasRowMajor = 101, CblasNoTrans = 111, alpha 1, beta 0, lda = K,
 * ldb = N, ldc = N), so a lowering retargets by changing only the callee's
 * name.  A, B, C may be host or device memory (host operands are staged
 * through device buffers); the product runs on the exact-FP32 SIMT GEMM and
 * C is complete when the call returns.  Also accepted: transB = 112
 * (CblasTrans, B given as [N, K] with ldb = K) and any ldc >= N.  Other
 * orders, transposed A, alpha != 1 or beta != 0 return GPT2_EINVAL (the
 * lowering never emits them).  Returns 0 on success; a lowering that
 * declares the callee void may ignore the result. */
int gpt2_blas_sgemm(int order, int transA, int transB, int M, int N, int K, float alpha, const float *A, int lda,
                    const float *B, int ldb, float beta, float *C, int ldc);

/* Exact-FP32 SIMT GEMM: C[M,N] (row stride ldc) = epi(A[M,K] @ op(B)),
 * op(B) = B[K,N] (b_nk = 0) or B[N,K]^T (b_nk = 1); resid row stride ldc. */
int gpt2k_gemm_f32(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                   const float *bias, const float *resid, int epi, void *stream);

/* tcgen05 BF16 GEMM: C[M,N] = epi(A[M,K] @ B[N,K]^T), A and B bf16
 * row-major; C bf16 (out_f32 = 0) or f32 (out_f32 = 1, EPI_NONE / EPI_BIAS);
 * resid bf16 with row stride ldc; bn = 128 or 256: one SM per 128 x bn
 * output tile; bn = 2: two SMs (a CTA pair) per 256 x 256 tile. */
int gpt2k_gemm_bf16(const void *A, const void *B, void *C, int M, int N, int K, int ldc, int out_f32,
                    const float *bias, const void *resid, int epi, int bn, void *stream);

/* The products of the few-token forward and of decode steps: y[M, N] =
 * epi(LN(x)[M, K] @ W[N, K]^T) for M <= 16 rows, x, W and a bf16 y (row
 * stride ldy; resid has the same stride and may alias y), or an FP32 y with
 * out_f32 = 1 (epi GPT2_EPI_NONE).  ln_gain / ln_shift (FP32 [K], both or
 * neither): a LayerNorm of x's rows (FP32 statistics, eps) applied before the
 * product; not with GPT2_EPI_BIAS_RESID.  impl 0: one SIMT kernel (warp per
 * few weight rows); impl 1: the tensor-core kernel (weights as the 128-row
 * MMA operand, K a multiple of 64, 16-byte aligned x and W).  They replace
 * the linalg.matmul calls the reference's decode loop re-runs per token
 * (src/gpt/lower_gpt_model.py:190-198). */
int gpt2k_gemv_bf16(const void *x, const void *W, void *y, int M, int N, int K, int ldy, const float *bias,
                    const void *resid, int epi, const float *ln_gain, const float *ln_shift, float eps, int out_f32,
                    int impl, void *stream);

/* Test hook of the kernels' bounded-wait error path; no counterpart in the
 * reference, which has no error path at all (src/gpt/gpt2_call.cpp:42-46
 * checks cuInit only).  Runs the single-SM tcgen05 GEMM of gpt2k_gemm_bf16
 * (bn = 128, C bf16 [M, N] with row stride N, no epilogue) with CTA 0's TMA
 * producer withholding the copy of its first stage, so that CTA 0's MMA
 * thread waits for data that never comes.  That wait gives up after its
 * limit (2 s); the kernel records status 2 (GPT2 "a barrier wait timed
 * out") in *d_status, stops issuing, waits for the copies it issued, frees
 * its tensor memory and returns, and the CUDA context stays usable.  C is
 * left partly written.  Enqueued on `stream`; nothing faults or hangs. */
int gpt2k_test_gemm_withheld_load(const void *A, const void *B, void *C, int M, int N, int K, int *d_status,
                                  void *stream);

/* The GEMM epilogues of the BF16 forward's folded LayerNorms (C bf16, or f32
 * for GPT2_EPI_LN_BIAS).  A LayerNorm LN(a) = (a - mean) * rstd * gain + shift
 * of A's rows followed by a linear layer with weight W [N, K] and bias is
 * computed as C = rstd * (A @ B^T) - rstd * mean * c1 + c2 with
 * B = bf16(W * gain) (gpt2k_ln_fold_pack), c1[n] = sum_k B[n, k] and
 * c2 = W @ shift + bias ([N rounded up to 256] floats, 16-byte aligned,
 * zero past N).  mean and rstd (1/sqrt(var + eps), biased variance over K)
 * come from stats_in [M][ceil(K / 128)]: per row and 128-column segment the
 * sum and the sum of squares (float pairs) of A's bf16 values.
 * GPT2_EPI_BIAS_RESID_STATS: C = resid + A @ B^T + bias and stats_out
 * [M][ceil(N / 128)] of the bf16 C, in the stats_in format.  Other epi values
 * behave as in gpt2k_gemm_bf16. */
int gpt2k_gemm_bf16_ln(const void *A, const void *B, void *C, int M, int N, int K, int ldc, int out_f32,
                       const float *bias, const void *resid, int epi, int bn, const float *c1, const float *c2,
                       const float *stats_in, float *stats_out, float eps, void *stream);
/* B [N, K] = bf16(W * gain) and the c1 / c2 vectors of a folded LayerNorm,
 * from an FP32 weight W stored [K, N] (w_kn = 1, the GPT-2 Conv1D layout) or
 * [N, K] (w_kn = 0); bias may be null. */
int gpt2k_ln_fold_pack(const float *W, int w_kn, const float *gain, const float *shift, const float *bias, void *B,
                       float *c1, float *c2, int N, int K, void *stream);

/* Measured FP32 FFMA throughput of the current device in TFLOP/s (a
 * microbenchmark of independent fma.rn.f32 chains on every SM, best of
 * three launches): the roofline denominator of the exact-FP32 path. */
int gpt2k_ffma_peak(float *tflops, void *stream);

/* LayerNorm over rows of width d (FP32 statistics): dtype GPT2_DTYPE_F32
 * (x, y float) or GPT2_DTYPE_BF16 (x, y bf16); gain and shift are float. */
int gpt2k_layernorm(const void *x, const float *gain, const float *shift, void *y, int T, int d, float eps,
                    int dtype, void *stream);

/* Causal attention of one layer, head dim 64: qkv [B*S, 3*H*64] (q | k | v),
 * o [B*S, H*64] (16-byte aligned for BF16), in dtype: GPT2_DTYPE_F32 (SIMT)
 * or GPT2_DTYPE_BF16 (tcgen05: one thread per query row, P in tensor
 * memory).  d_mask: contiguous int64 [B, S] or NULL.  workspace: device
 * memory of gpt2k_attention_workspace_bytes(B, S) bytes (unused, may be
 * NULL, when d_mask is NULL). */
size_t gpt2k_attention_workspace_bytes(int B, int S);
int gpt2k_attention(const void *qkv, const int64_t *d_mask, void *o, int B, int S, int H, int dtype,
                    void *workspace, void *stream);

/* Attention with the causal mask selectable: causal = 1 is gpt2k_attention;
 * causal = 0 lets every query attend to every unmasked key of its sequence
 * (the BERT encoder's self-attention), and a sequence whose mask is all
 * zero gets the mean of V in every row.  With a mask, key tiles past a
 * sequence's last unmasked key are skipped.  workspace: device memory of
 * gpt2k_attention_ex_workspace_bytes(B, S) bytes (may be NULL without a
 * mask). */
size_t gpt2k_attention_ex_workspace_bytes(int B, int S);
int gpt2k_attention_ex(const void *qkv, const int64_t *d_mask, void *o, int B, int S, int H, int dtype, int causal,
                       void *workspace, void *stream);

/* Attention without a workspace argument, for callers that cannot allocate
 * device memory at call time: hosts whose device memory is reserved up front
 * by another allocator, generated code with no allocation hook at this call,
 * real-time loops that must not pay for an allocation.  (No counterpart in
 * the reference.)  Same arguments and results as gpt2k_attention; the mask
 * scratch comes from a fixed 4 MiB array in the library's device image,
 * present on every GPU that loads the library until the process exits, so
 * 256 + 4*B + B*S must not exceed 4 MiB (a larger shape returns GPT2_EINVAL
 * with a message).  The first call on a device looks up the array's address
 * (make it before any stream capture).  Calls share the array: calls that
 * overlap on the GPU race; each call rewrites the bytes it reads. */
int gpt2k_attention_noalloc(const void *qkv, const int64_t *d_mask, void *o, int B, int S, int H, int dtype,
                            void *stream);

/* Token + position embedding: x[t] = wte[ids[t]] + wpe[t % S] in dtype;
 * out-of-range ids set the model-independent status word *d_status to 1. */
int gpt2k_embed(const int64_t *d_ids, const void *wte, const void *wpe, void *x, int T, int S, int d, int V,
                int dtype, int *d_status, void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* GPT2_B200_H */
