/*
 * gpt2_oracle.c -- CPU oracle for the GPT-2 forward (prefill) pass.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke()
 * entry and bench.py's cpu_baseline / reference legs may load it; the product
 * library never links or calls it.
 *
 * It restates, in plain FP32 C, the computation that the reference compiles
 * into its `gpt2_decoder` object:
 *   - model semantics: HF GPT-2 wrapped by src/gpt/lower_gpt_model.py:20-50
 *     (full logits, use_cache=False at :86), i.e. transformers' GPT2LMHeadModel
 *     forward with eager attention;
 *   - CPU lowering: src/gpt/run_mlir_pipeline.sh:5-10 runs
 *     -linalg-to-bufferization / -bufferization-to-llvm (tools/tutorial-opt.cpp:35-79),
 *     where every 2-D f32 linalg.matmul becomes cblas_sgemm(RowMajor, NoTrans,
 *     NoTrans, M, N, K, 1.0, A, lda, B, ldb, 0.0, C, ldc)
 *     (lib/ConvertMatMulToBlas.cpp:84-92, :156-160) and everything else
 *     (batch_matmul, LayerNorm, softmax, GELU, adds) stays a single-threaded
 *     loop nest (tools/tutorial-opt.cpp:55-61).  This file mirrors that split:
 *     the five 2-D matmul kinds call an sgemm (OpenBLAS through dlopen when
 *     available, else a blocked fallback), the rest are loops whose thread
 *     count defaults to 1.
 *
 * Parity of this restatement is pinned against transformers' GPT2LMHeadModel
 * run in the build container on the same seeded weights (tests/golden/).
 *
 * Seeded synthetic inputs: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11)
 * counter-based generator plus the Box-Muller transform, so that the weights
 * do not depend on any framework's RNG.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------- */
/* Configuration and packed-weight layout                                    */
/* ------------------------------------------------------------------------- */

/* Same field order as the product's Gpt2Config (first seven fields). */
typedef struct OracleCfg {
  int32_t n_layer;
  int32_t n_embd;
  int32_t n_head;
  int32_t n_inner;
  int32_t vocab_size;
  int32_t n_positions;
  float layer_norm_eps;
  int32_t dtype; /* ignored: the oracle is FP32 */
} OracleCfg;

/* Canonical FP32 blob: tensors in this order, row-major, HF Conv1D weights
 * stored [in, out] (x @ W + b), wte [V, d] used both for the lookup and,
 * transposed, as the tied lm_head.
 *   0 wte [V,d]   1 wpe [P,d]
 *   per layer l, index 2 + 12 l + j:
 *     j=0 ln_1.weight [d]   1 ln_1.bias [d]
 *       2 attn.c_attn.weight [d,3d]   3 attn.c_attn.bias [3d]
 *       4 attn.c_proj.weight [d,d]    5 attn.c_proj.bias [d]
 *       6 ln_2.weight [d]   7 ln_2.bias [d]
 *       8 mlp.c_fc.weight [d,ff]      9 mlp.c_fc.bias [ff]
 *      10 mlp.c_proj.weight [ff,d]   11 mlp.c_proj.bias [d]
 *   2 + 12 L: ln_f.weight [d]    3 + 12 L: ln_f.bias [d]
 */
enum { T_LN1_G, T_LN1_B, T_QKV_W, T_QKV_B, T_PROJ_W, T_PROJ_B, T_LN2_G, T_LN2_B,
       T_FC_W, T_FC_B, T_MPROJ_W, T_MPROJ_B, T_PER_LAYER };

int oracle_num_tensors(const OracleCfg *c) { return 4 + T_PER_LAYER * c->n_layer; }

/* kind: 0 = matrix N(0, 0.02), 1 = LN gain, 2 = LN/linear bias */
static int64_t tensor_numel(const OracleCfg *c, int t, int *kind) {
  const int64_t d = c->n_embd, ff = c->n_inner;
  const int L = c->n_layer;
  if (t == 0) { *kind = 0; return (int64_t)c->vocab_size * d; }
  if (t == 1) { *kind = 0; return (int64_t)c->n_positions * d; }
  if (t == 2 + T_PER_LAYER * L) { *kind = 1; return d; }
  if (t == 3 + T_PER_LAYER * L) { *kind = 2; return d; }
  switch ((t - 2) % T_PER_LAYER) {
    case T_LN1_G: case T_LN2_G: *kind = 1; return d;
    case T_LN1_B: case T_LN2_B: *kind = 2; return d;
    case T_QKV_W: *kind = 0; return d * 3 * d;
    case T_QKV_B: *kind = 2; return 3 * d;
    case T_PROJ_W: *kind = 0; return d * d;
    case T_PROJ_B: *kind = 2; return d;
    case T_FC_W: *kind = 0; return d * ff;
    case T_FC_B: *kind = 2; return ff;
    case T_MPROJ_W: *kind = 0; return ff * d;
    case T_MPROJ_B: *kind = 2; return d;
  }
  return 0;
}

/* Fills offsets[0..num_tensors] (in floats); returns the total float count. */
int64_t oracle_blob_layout(const OracleCfg *c, int64_t *offsets) {
  int64_t off = 0;
  const int n = oracle_num_tensors(c);
  for (int t = 0; t < n; ++t) {
    int kind;
    if (offsets) offsets[t] = off;
    off += tensor_numel(c, t, &kind);
  }
  if (offsets) offsets[n] = off;
  return off;
}

/* ------------------------------------------------------------------------- */
/* A minimal pthread parallel-for for the loop nests.  The thread count      */
/* defaults to 1, which is how the reference's CPU lowering runs them.       */
/* ------------------------------------------------------------------------- */

static int g_loop_threads = 1;

void oracle_set_loop_threads(int n) { g_loop_threads = n < 1 ? 1 : n; }

typedef void (*range_fn)(void *ctx, int64_t begin, int64_t end, int tid);
typedef struct { range_fn fn; void *ctx; int64_t n; int nt; int tid; } range_job;

static void *range_thread(void *arg) {
  range_job *j = (range_job *)arg;
  const int64_t chunk = (j->n + j->nt - 1) / j->nt;
  const int64_t b = (int64_t)j->tid * chunk;
  const int64_t e = b + chunk < j->n ? b + chunk : j->n;
  if (b < e) j->fn(j->ctx, b, e, j->tid);
  return NULL;
}

static void parallel_for(int64_t n, range_fn fn, void *ctx) {
  int nt = g_loop_threads;
  if (nt > n) nt = (int)(n > 0 ? n : 1);
  if (nt <= 1) { if (n > 0) fn(ctx, 0, n, 0); return; }
  pthread_t th[256];
  range_job jobs[256];
  if (nt > 256) nt = 256;
  for (int t = 0; t < nt; ++t) {
    jobs[t] = (range_job){fn, ctx, n, nt, t};
    if (t) pthread_create(&th[t], NULL, range_thread, &jobs[t]);
  }
  range_thread(&jobs[0]);
  for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* Philox4x32-10 + Box-Muller                                                */
/* ------------------------------------------------------------------------- */

#define PHILOX_M0 0xD2511F53u
#define PHILOX_M1 0xCD9E8D57u
#define PHILOX_W0 0x9E3779B9u
#define PHILOX_W1 0xBB67AE85u
#define SEED_TAG 0x67707432u /* "gpt2" */

void oracle_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)PHILOX_M0 * c0;
    const uint64_t p1 = (uint64_t)PHILOX_M1 * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c1 ^ k0;
    const uint32_t n1 = lo1;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    const uint32_t n3 = lo0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += PHILOX_W0;
    k1 += PHILOX_W1;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static void philox_block(uint64_t seed, uint32_t stream, uint64_t block, uint32_t out[4]) {
  const uint32_t ctr[4] = {(uint32_t)block, (uint32_t)(block >> 32), stream, SEED_TAG};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  oracle_philox4x32_10(ctr, key, out);
}

typedef struct { float *out; int64_t n; uint64_t seed; uint32_t stream; double mean, std; } fill_ctx;

static void fill_blocks(void *vctx, int64_t b0, int64_t b1, int tid) {
  const fill_ctx *c = (const fill_ctx *)vctx;
  const double two_pi = 6.283185307179586;
  const double inv32 = 1.0 / 4294967296.0;
  for (int64_t b = b0; b < b1; ++b) {
    uint32_t w[4];
    philox_block(c->seed, c->stream, (uint64_t)b, w);
    double z[4];
    for (int p = 0; p < 2; ++p) {
      const double u1 = ((double)w[2 * p] + 1.0) * inv32;
      const double u2 = (double)w[2 * p + 1] * inv32;
      const double r = sqrt(-2.0 * log(u1));
      const double t = two_pi * u2;
      z[2 * p] = r * cos(t);
      z[2 * p + 1] = r * sin(t);
    }
    for (int j = 0; j < 4 && b * 4 + j < c->n; ++j) c->out[b * 4 + j] = (float)(c->mean + c->std * z[j]);
  }
}

/* out[i] = float(mean + std * z_i), z_i standard normal from Box-Muller on
 * Philox block i/4: words (0,1) give z0 = r cos t, z1 = r sin t and words
 * (2,3) give z2, z3, with u1 = (w + 1) / 2^32 and u2 = w' / 2^32.  The value
 * of every element depends only on (seed, stream, i), so the fill is split
 * over all host threads without changing a bit. */
void oracle_normal_fill(float *out, int64_t n, uint64_t seed, uint32_t stream, double mean, double std) {
  fill_ctx c = {out, n, seed, stream, mean, std};
  const int saved = g_loop_threads;
  const long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
  g_loop_threads = ncpu > 1 ? (int)(ncpu < 64 ? ncpu : 64) : 1;
  parallel_for((n + 3) / 4, fill_blocks, &c);
  g_loop_threads = saved;
}

/* ids[i] = floor(w * vocab / 2^32) with w the (i % 4)-th Philox word of block i/4. */
void oracle_token_ids(int64_t *ids, int64_t n, uint64_t seed, uint32_t stream, int64_t vocab) {
  for (int64_t b = 0; b * 4 < n; ++b) {
    uint32_t w[4];
    philox_block(seed, stream, (uint64_t)b, w);
    for (int j = 0; j < 4 && b * 4 + j < n; ++j)
      ids[b * 4 + j] = (int64_t)(((uint64_t)w[j] * (uint64_t)vocab) >> 32);
  }
}

/* init_mode 0: the benchmark init (matrices N(0,0.02), LN gain 1, LN/linear
 * bias 0).  init_mode 1: every tensor random (matrices N(0,0.02), gains
 * 1 + N(0,0.1), biases N(0,0.02)), so that parity tests exercise the bias,
 * gain and shift paths. */
int oracle_seeded_blob(const OracleCfg *c, uint64_t seed, int init_mode, float *blob) {
  const int n = oracle_num_tensors(c);
  int64_t off = 0;
  for (int t = 0; t < n; ++t) {
    int kind;
    const int64_t numel = tensor_numel(c, t, &kind);
    float *p = blob + off;
    if (kind == 0) {
      oracle_normal_fill(p, numel, seed, (uint32_t)t, 0.0, 0.02);
    } else if (init_mode == 0) {
      const float v = kind == 1 ? 1.0f : 0.0f;
      for (int64_t i = 0; i < numel; ++i) p[i] = v;
    } else {
      oracle_normal_fill(p, numel, seed, (uint32_t)t, kind == 1 ? 1.0 : 0.0, kind == 1 ? 0.1 : 0.02);
    }
    off += numel;
  }
  return 0;
}


/* ------------------------------------------------------------------------- */
/* FP8 E4M3 weight quantization (the weight-only FP8 configuration)           */
/* ------------------------------------------------------------------------- */

/* float -> E4M3 code (1 sign, 4 exponent bits with bias 7, 3 mantissa bits;
 * largest finite 448, no infinities), round to nearest even on the float's
 * bits, saturating at 448.  Subnormals are steps of 2^-9. */
uint8_t oracle_e4m3_encode(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint8_t sign = (uint8_t)((b >> 24) & 0x80);
  const uint32_t ab = b & 0x7FFFFFFF;
  float a;
  memcpy(&a, &ab, 4);
  if (!(a == a)) return (uint8_t)(sign | 0x7E); /* NaN input: saturate (not produced by the quantizer) */
  if (a >= 448.0f) return (uint8_t)(sign | 0x7E);
  int e = (int)((ab >> 23) & 0xFF) - 127;
  if (e >= -6) {
    uint32_t r = (ab & 0x7FFFFF) >> 20, rem = ab & 0xFFFFF;
    if (rem > 0x80000 || (rem == 0x80000 && (r & 1))) ++r;
    if (r == 8) { r = 0; ++e; }
    if (e > 8 || (e == 8 && r == 7)) { e = 8; r = 6; }
    return (uint8_t)(sign | ((uint32_t)(e + 7) << 3) | r);
  }
  /* subnormal range: a / 2^-9 rounded to nearest even (0..8; 8 is the smallest normal) */
  const float u = a * 512.0f;
  float n = rintf(u); /* the default rounding mode is round to nearest even */
  return (uint8_t)(sign | (uint8_t)n);
}

float oracle_e4m3_decode(uint8_t q) {
  const int e = (q >> 3) & 0xF, m = q & 7;
  const float v = e == 0 ? ldexpf((float)m, -9) : ldexpf(1.0f + m / 8.0f, e - 7);
  return (q & 0x80) ? -v : v;
}

/* Conv1D weight w [K in, N out]: per output channel n, scale[n] = max_k |w[k,n]| / 448
 * and q[n*K + k] = e4m3(w[k,n] / scale[n]) (packed [N, K]).  A zero column gets scale 1. */
void oracle_fp8_quantize(const float *w, int K, int N, uint8_t *q, float *scale) {
  for (int n = 0; n < N; ++n) {
    float mx = 0.f;
    for (int k = 0; k < K; ++k) { const float a = fabsf(w[(int64_t)k * N + n]); if (a > mx) mx = a; }
    const float sc = mx > 0.f ? mx / 448.0f : 1.0f;
    scale[n] = sc;
    for (int k = 0; k < K; ++k) q[(int64_t)n * K + k] = oracle_e4m3_encode(w[(int64_t)k * N + n] / sc);
  }
}

/* Replaces the four Conv1D weights of every layer of a canonical blob by their
 * FP8-dequantized values e4m3_decode(q) * scale, in place. */
int oracle_fp8_dequantize_blob(const OracleCfg *c, float *blob) {
  int64_t *off = (int64_t *)malloc(sizeof(int64_t) * (oracle_num_tensors(c) + 1));
  if (!off) return -3;
  oracle_blob_layout(c, off);
  const int d = c->n_embd, ff = c->n_inner;
  const int kinds[4] = {T_QKV_W, T_PROJ_W, T_FC_W, T_MPROJ_W};
  for (int l = 0; l < c->n_layer; ++l)
    for (int i = 0; i < 4; ++i) {
      const int K = kinds[i] == T_MPROJ_W ? ff : d;
      const int N = kinds[i] == T_QKV_W ? 3 * d : kinds[i] == T_FC_W ? ff : d;
      float *w = blob + off[2 + T_PER_LAYER * l + kinds[i]];
      uint8_t *q = (uint8_t *)malloc((size_t)K * N);
      float *sc = (float *)malloc(sizeof(float) * N);
      if (!q || !sc) { free(q); free(sc); free(off); return -3; }
      oracle_fp8_quantize(w, K, N, q, sc);
      for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n) w[(int64_t)k * N + n] = oracle_e4m3_decode(q[(int64_t)n * K + k]) * sc[n];
      free(q);
      free(sc);
    }
  free(off);
  return 0;
}

/* ------------------------------------------------------------------------- */
/* sgemm: OpenBLAS through dlopen (as the reference's -lopenblas link), or a  */
/* blocked fallback.  Row-major C[M,N] = A[M,K] * op(B).                      */
/* ------------------------------------------------------------------------- */

typedef void (*cblas_sgemm_lp64_t)(int, int, int, int, int, int, float, const float *, int,
                                   const float *, int, float, float *, int);
typedef void (*cblas_sgemm_ilp64_t)(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float,
                                    const float *, int64_t, const float *, int64_t, float, float *,
                                    int64_t);
static cblas_sgemm_lp64_t g_sgemm32;
static cblas_sgemm_ilp64_t g_sgemm64;
static char g_blas_name[512] = "builtin-blocked";

/* Loads an OpenBLAS-style library; returns 0 on success. */
int oracle_set_blas(const char *path) {
  g_sgemm32 = NULL;
  g_sgemm64 = NULL;
  snprintf(g_blas_name, sizeof g_blas_name, "builtin-blocked");
  if (!path || !*path) return 0;
  void *h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) return -1;
  static const char *lp64[] = {"scipy_cblas_sgemm", "cblas_sgemm"};
  static const char *ilp64[] = {"scipy_cblas_sgemm64_", "cblas_sgemm64_"};
  for (int i = 0; i < 2 && !g_sgemm32; ++i) g_sgemm32 = (cblas_sgemm_lp64_t)dlsym(h, lp64[i]);
  for (int i = 0; i < 2 && !g_sgemm32 && !g_sgemm64; ++i) g_sgemm64 = (cblas_sgemm_ilp64_t)dlsym(h, ilp64[i]);
  if (!g_sgemm32 && !g_sgemm64) return -2;
  snprintf(g_blas_name, sizeof g_blas_name, "%s", path);
  return 0;
}

const char *oracle_blas_name(void) { return g_blas_name; }

typedef struct { int M, N, K, transB; const float *A, *B; float *C; } gemm_ctx;

static void sgemm_rows(void *vctx, int64_t rb, int64_t re, int tid) {
  const gemm_ctx *g = (const gemm_ctx *)vctx;
  const int N = g->N, K = g->K, KB = 256;
  const int i0 = (int)rb * 64, i1 = (int)(re * 64 < g->M ? re * 64 : g->M);
  for (int i = i0; i < i1; ++i)
    for (int j = 0; j < N; ++j) g->C[(int64_t)i * N + j] = 0.f;
  if (!g->transB) {
    for (int k0 = 0; k0 < K; k0 += KB) {
      const int k1 = k0 + KB < K ? k0 + KB : K;
      for (int i = i0; i < i1; ++i) {
        float *c = g->C + (int64_t)i * N;
        for (int k = k0; k < k1; ++k) {
          const float a = g->A[(int64_t)i * K + k];
          const float *b = g->B + (int64_t)k * N;
          for (int j = 0; j < N; ++j) c[j] += a * b[j];
        }
      }
    }
  } else {
    for (int i = i0; i < i1; ++i)
      for (int j = 0; j < N; ++j) {
        const float *a = g->A + (int64_t)i * K, *b = g->B + (int64_t)j * K;
        float s = 0.f;
        for (int k = 0; k < K; ++k) s += a[k] * b[k];
        g->C[(int64_t)i * N + j] = s;
      }
  }
}

/* Blocked sgemm used when no OpenBLAS can be loaded (rows split in blocks of 64). */
static void sgemm_fallback(int M, int N, int K, const float *A, const float *B, int transB, float *C) {
  gemm_ctx g = {M, N, K, transB, A, B, C};
  parallel_for((M + 63) / 64, sgemm_rows, &g);
}

/* C = A @ B (B [K,N]) or A @ B^T (B [N,K]); the cblas call matches
 * lib/ConvertMatMulToBlas.cpp:156-160 (alpha 1, beta 0, row-major). */
static void sgemm(int M, int N, int K, const float *A, const float *B, int transB, float *C) {
  enum { RowMajor = 101, NoTrans = 111, Trans = 112 };
  const int tb = transB ? Trans : NoTrans;
  const int ldb = transB ? K : N;
  if (g_sgemm32) g_sgemm32(RowMajor, NoTrans, tb, M, N, K, 1.0f, A, K, B, ldb, 0.0f, C, N);
  else if (g_sgemm64) g_sgemm64(RowMajor, NoTrans, tb, M, N, K, 1.0f, A, K, B, ldb, 0.0f, C, N);
  else sgemm_fallback(M, N, K, A, B, transB, C);
}

/* ------------------------------------------------------------------------- */
/* Loop-nest ops                                                              */
/* ------------------------------------------------------------------------- */

typedef struct { const float *x, *g, *b; float *y; int d; float eps; } ln_ctx;

static void ln_rows(void *vctx, int64_t t0, int64_t t1, int tid) {
  const ln_ctx *c = (const ln_ctx *)vctx;
  const int d = c->d;
  for (int64_t t = t0; t < t1; ++t) {
    const float *r = c->x + t * d;
    double s = 0.0;
    for (int i = 0; i < d; ++i) s += r[i];
    const double mean = s / d;
    double v = 0.0;
    for (int i = 0; i < d; ++i) { const double e = r[i] - mean; v += e * e; }
    const float rstd = (float)(1.0 / sqrt(v / d + (double)c->eps));
    const float m = (float)mean;
    float *o = c->y + t * d;
    for (int i = 0; i < d; ++i) o[i] = (r[i] - m) * rstd * c->g[i] + c->b[i];
  }
}

/* torch.nn.LayerNorm: biased variance, eps inside the square root. */
static void layer_norm(const float *x, const float *g, const float *b, float *y, int64_t T, int d, float eps) {
  ln_ctx c = {x, g, b, y, d, eps};
  parallel_for(T, ln_rows, &c);
}

/* transformers' NewGELUActivation ("gelu_new"), the tanh approximation. */
static inline float gelu_new(float x) {
  const float k = 0.7978845608028654f; /* sqrt(2/pi) */
  return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
}

typedef struct { const float *qkv; const int64_t *mask; float *o; int B, S, d, H; float *scratch; int causal; } attn_ctx;

static void attn_heads(void *vctx, int64_t i0, int64_t i1, int tid) {
  const attn_ctx *c = (const attn_ctx *)vctx;
  const int S = c->S, d = c->d, H = c->H, dh = d / H;
  const float scale = (float)(1.0 / sqrt((double)dh));
  const int64_t ld = 3 * (int64_t)d;
  float *p = c->scratch + (int64_t)tid * S;
  for (int64_t bh = i0; bh < i1; ++bh) {
    const int b = (int)(bh / H), h = (int)(bh % H);
    const float *base = c->qkv + (int64_t)b * S * ld;
    const int64_t *m = c->mask ? c->mask + (int64_t)b * S : NULL;
    int first_valid = 0;
    if (m) { first_valid = S; for (int k = 0; k < S; ++k) if (m[k]) { first_valid = k; break; } }
    /* Without the causal mask a row lacks an attendable key only when the whole sequence is masked. */
    if (!c->causal && first_valid < S) first_valid = 0;
    for (int q = 0; q < S; ++q) {
      float *out = c->o + ((int64_t)b * S + q) * d + h * dh;
      const int klast = c->causal ? q : S - 1;
      if (q < first_valid) {
        for (int j = 0; j < dh; ++j) {
          double acc = 0.0;
          for (int k = 0; k < S; ++k) acc += base[(int64_t)k * ld + 2 * d + h * dh + j];
          out[j] = (float)(acc / S);
        }
        continue;
      }
      const float *qv = base + (int64_t)q * ld + h * dh;
      float mx = -INFINITY;
      for (int k = 0; k <= klast; ++k) {
        if (m && !m[k]) { p[k] = -INFINITY; continue; }
        const float *kv = base + (int64_t)k * ld + d + h * dh;
        float s = 0.f;
        for (int j = 0; j < dh; ++j) s += qv[j] * kv[j];
        s *= scale;
        p[k] = s;
        if (s > mx) mx = s;
      }
      float sum = 0.f;
      for (int k = 0; k <= klast; ++k) {
        const float e = p[k] == -INFINITY ? 0.f : expf(p[k] - mx);
        p[k] = e;
        sum += e;
      }
      const float inv = 1.0f / sum;
      for (int j = 0; j < dh; ++j) out[j] = 0.f;
      for (int k = 0; k <= klast; ++k) {
        if (p[k] == 0.f) continue;
        const float w = p[k] * inv;
        const float *vv = base + (int64_t)k * ld + 2 * d + h * dh;
        for (int j = 0; j < dh; ++j) out[j] += w * vv[j];
      }
    }
  }
}

/* Causal self-attention of one layer (the two batch_matmuls, the scale, the
 * mask and the softmax), heads merged back into o [T, d].
 * Key k is attendable from query q when k <= q and mask[b, k] != 0; the
 * reference adds finfo(f32).min for every other key before the softmax, so
 * masked keys weigh exp(min - max) = 0 exactly.  A query row with no
 * attendable key (a left-padded prefix) sees the same additive value on
 * every key and therefore averages V uniformly over all S keys. */
static void attention(const float *qkv, const int64_t *mask, float *o, int B, int S, int d, int H,
                      float *scratch_all) {
  attn_ctx c = {qkv, mask, o, B, S, d, H, scratch_all, 1};
  parallel_for((int64_t)B * H, attn_heads, &c);
}

/* ------------------------------------------------------------------------- */
/* Forward                                                                    */
/* ------------------------------------------------------------------------- */

/* logits [B, S, V] = GPT2LMHeadModel(ids, mask).logits in FP32.
 * ids/mask are contiguous [B, S]; mask may be NULL (all ones).
 * Returns 0, or a negative code: -1 bad shape, -2 id out of range, -3 OOM. */
int oracle_gpt2_forward(const OracleCfg *c, const float *blob, const int64_t *ids, const int64_t *mask,
                        int B, int S, float *logits) {
  const int d = c->n_embd, H = c->n_head, ff = c->n_inner, V = c->vocab_size, L = c->n_layer;
  if (B < 1 || S < 1 || S > c->n_positions || d % H) return -1;
  const int64_t T = (int64_t)B * S;
  for (int64_t i = 0; i < T; ++i)
    if (ids[i] < 0 || ids[i] >= V) return -2;
  int64_t *off = (int64_t *)malloc(sizeof(int64_t) * (oracle_num_tensors(c) + 1));
  oracle_blob_layout(c, off);
  float *x = (float *)malloc(sizeof(float) * T * d);
  float *a = (float *)malloc(sizeof(float) * T * d);
  float *o = (float *)malloc(sizeof(float) * T * d);
  float *tmp = (float *)malloc(sizeof(float) * T * d);
  float *big = (float *)malloc(sizeof(float) * T * (ff > 3 * d ? ff : 3 * d));
  float *scr = (float *)malloc(sizeof(float) * (int64_t)S * 257);
  if (!off || !x || !a || !o || !tmp || !big || !scr) {
    free(off); free(x); free(a); free(o); free(tmp); free(big); free(scr);
    return -3;
  }
  const float *wte = blob + off[0], *wpe = blob + off[1];

  /* x0 = wte[ids] + wpe[arange(S)] */
  for (int64_t t = 0; t < T; ++t) {
    const float *e = wte + ids[t] * d, *p = wpe + (int64_t)(t % S) * d;
    for (int i = 0; i < d; ++i) x[t * d + i] = e[i] + p[i];
  }

  for (int l = 0; l < L; ++l) {
    const int64_t *lo = off + 2 + T_PER_LAYER * l;
    const float *ln1g = blob + lo[T_LN1_G], *ln1b = blob + lo[T_LN1_B];
    const float *wqkv = blob + lo[T_QKV_W], *bqkv = blob + lo[T_QKV_B];
    const float *wpr = blob + lo[T_PROJ_W], *bpr = blob + lo[T_PROJ_B];
    const float *ln2g = blob + lo[T_LN2_G], *ln2b = blob + lo[T_LN2_B];
    const float *wfc = blob + lo[T_FC_W], *bfc = blob + lo[T_FC_B];
    const float *wmp = blob + lo[T_MPROJ_W], *bmp = blob + lo[T_MPROJ_B];

    layer_norm(x, ln1g, ln1b, a, T, d, c->layer_norm_eps);
    sgemm((int)T, 3 * d, d, a, wqkv, 0, big);
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < 3 * d; ++j) big[t * 3 * d + j] += bqkv[j];
    attention(big, mask, o, B, S, d, H, scr);
    sgemm((int)T, d, d, o, wpr, 0, tmp);
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < d; ++j) x[t * d + j] += tmp[t * d + j] + bpr[j];

    layer_norm(x, ln2g, ln2b, a, T, d, c->layer_norm_eps);
    sgemm((int)T, ff, d, a, wfc, 0, big);
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < ff; ++j) big[t * ff + j] = gelu_new(big[t * ff + j] + bfc[j]);
    sgemm((int)T, d, ff, big, wmp, 0, tmp);
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < d; ++j) x[t * d + j] += tmp[t * d + j] + bmp[j];
  }
  const int64_t *fo = off + 2 + T_PER_LAYER * L;
  layer_norm(x, blob + fo[0], blob + fo[1], a, T, d, c->layer_norm_eps);
  /* tied lm_head: logits = ln_f(x) @ wte^T */
  sgemm((int)T, V, d, a, wte, 1, logits);

  free(off); free(x); free(a); free(o); free(tmp); free(big); free(scr);
  return 0;
}

/* ------------------------------------------------------------------------- */
/* BERT encoder (the reference's second exported model)                       */
/* ------------------------------------------------------------------------- */
/*
 * Restates transformers' BertModel as wrapped by
 * src/bert-base-uncased/lower_bert_model.py:7-18 (last_hidden_state and
 * pooler_output) with eager attention: embeddings word + position + token
 * type, LayerNorm; per layer (post-LN) ctx = softmax(q k^T / sqrt(dh) +
 * key mask) v, h = LN(x + ctx Wo^T + bo), x = LN(h + gelu(h Wi^T + bi) Wo2^T
 * + bo2) with the exact (erf) GELU; pooler tanh(x[:, 0] Wp^T + bp).  A
 * sequence with no unmasked key averages V over all keys (the reference adds
 * the same finfo.min to every score).  nn.Linear weights are [out, in].
 *
 * Canonical FP32 blob, HF order:
 *   0 word_embeddings [V,d]  1 position_embeddings [P,d]  2 token_type_embeddings [TV,d]
 *   3 embeddings.LayerNorm.weight [d]  4 .bias [d]
 *   per layer l, index 5 + 16 l + j:
 *     0 query.weight [d,d] 1 query.bias  2 key.weight 3 key.bias  4 value.weight 5 value.bias
 *     6 attention.output.dense.weight [d,d] 7 .bias  8 attention.output.LayerNorm.weight 9 .bias
 *    10 intermediate.dense.weight [ff,d] 11 .bias [ff]  12 output.dense.weight [d,ff] 13 .bias
 *    14 output.LayerNorm.weight 15 .bias
 *   5 + 16 L: pooler.dense.weight [d,d]   6 + 16 L: pooler.dense.bias [d]
 */
typedef struct OracleBertCfg {
  int32_t n_layer, n_embd, n_head, n_inner, vocab_size, n_positions;
  float layer_norm_eps;
  int32_t type_vocab;
} OracleBertCfg;

enum { B_Q_W, B_Q_B, B_K_W, B_K_B, B_V_W, B_V_B, B_AO_W, B_AO_B, B_AOLN_G, B_AOLN_B, B_I_W, B_I_B, B_O_W, B_O_B,
       B_OLN_G, B_OLN_B, B_PER_LAYER };

int oracle_bert_num_tensors(const OracleBertCfg *c) { return 7 + B_PER_LAYER * c->n_layer; }

static int64_t bert_numel(const OracleBertCfg *c, int t, int *kind) {
  const int64_t d = c->n_embd, ff = c->n_inner;
  const int L = c->n_layer;
  if (t == 0) { *kind = 0; return (int64_t)c->vocab_size * d; }
  if (t == 1) { *kind = 0; return (int64_t)c->n_positions * d; }
  if (t == 2) { *kind = 0; return (int64_t)c->type_vocab * d; }
  if (t == 3) { *kind = 1; return d; }
  if (t == 4) { *kind = 2; return d; }
  if (t == 5 + B_PER_LAYER * L) { *kind = 0; return d * d; }
  if (t == 6 + B_PER_LAYER * L) { *kind = 2; return d; }
  switch ((t - 5) % B_PER_LAYER) {
    case B_Q_W: case B_K_W: case B_V_W: case B_AO_W: *kind = 0; return d * d;
    case B_I_W: *kind = 0; return ff * d;
    case B_O_W: *kind = 0; return d * ff;
    case B_AOLN_G: case B_OLN_G: *kind = 1; return d;
    case B_I_B: *kind = 2; return ff;
    default: *kind = 2; return d;
  }
}

int64_t oracle_bert_blob_layout(const OracleBertCfg *c, int64_t *offsets) {
  int64_t off = 0;
  const int n = oracle_bert_num_tensors(c);
  for (int t = 0; t < n; ++t) {
    int kind;
    if (offsets) offsets[t] = off;
    off += bert_numel(c, t, &kind);
  }
  if (offsets) offsets[n] = off;
  return off;
}

/* Same generator and init modes as the GPT-2 blob; Philox streams 0x20000 + tensor index. */
int oracle_bert_seeded_blob(const OracleBertCfg *c, uint64_t seed, int init_mode, float *blob) {
  const int n = oracle_bert_num_tensors(c);
  int64_t off = 0;
  for (int t = 0; t < n; ++t) {
    int kind;
    const int64_t numel = bert_numel(c, t, &kind);
    float *p = blob + off;
    const uint32_t stream = 0x20000u + (uint32_t)t;
    if (kind == 0) oracle_normal_fill(p, numel, seed, stream, 0.0, 0.02);
    else if (init_mode == 0) { const float v = kind == 1 ? 1.0f : 0.0f; for (int64_t i = 0; i < numel; ++i) p[i] = v; }
    else oracle_normal_fill(p, numel, seed, stream, kind == 1 ? 1.0 : 0.0, kind == 1 ? 0.1 : 0.02);
    off += numel;
  }
  return 0;
}

static inline float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }

/* hidden [B,S,d] and pooled [B,d] of BertModel(ids, token_type_ids, mask) with
 * position ids pos[S] (NULL: 0..S-1); tt and mask may be NULL (zeros / ones).
 * Returns 0, -1 bad shape, -2 an id out of range, -3 OOM. */
int oracle_bert_forward(const OracleBertCfg *c, const float *blob, const int64_t *ids, const int64_t *tt,
                        const int64_t *pos, const int64_t *mask, int B, int S, float *hidden, float *pooled) {
  const int d = c->n_embd, H = c->n_head, ff = c->n_inner, L = c->n_layer;
  if (B < 1 || S < 1 || S > c->n_positions || d % H) return -1;
  const int64_t T = (int64_t)B * S;
  for (int64_t i = 0; i < T; ++i) {
    if (ids[i] < 0 || ids[i] >= c->vocab_size) return -2;
    if (tt && (tt[i] < 0 || tt[i] >= c->type_vocab)) return -2;
  }
  for (int s = 0; s < S && pos; ++s)
    if (pos[s] < 0 || pos[s] >= c->n_positions) return -2;
  int64_t *off = (int64_t *)malloc(sizeof(int64_t) * (oracle_bert_num_tensors(c) + 1));
  float *x = (float *)malloc(sizeof(float) * T * d);
  float *h = (float *)malloc(sizeof(float) * T * d);
  float *o = (float *)malloc(sizeof(float) * T * d);
  float *tmp = (float *)malloc(sizeof(float) * T * d);
  float *big = (float *)malloc(sizeof(float) * T * (ff > 3 * d ? ff : 3 * d));
  float *wqkv = (float *)malloc(sizeof(float) * 3 * (int64_t)d * d);
  float *bqkv = (float *)malloc(sizeof(float) * 3 * d);
  float *scr = (float *)malloc(sizeof(float) * (int64_t)S * 257);
  if (!off || !x || !h || !o || !tmp || !big || !wqkv || !bqkv || !scr) {
    free(off); free(x); free(h); free(o); free(tmp); free(big); free(wqkv); free(bqkv); free(scr);
    return -3;
  }
  oracle_bert_blob_layout(c, off);
  const float *we = blob + off[0], *pe = blob + off[1], *te = blob + off[2];
  for (int64_t t = 0; t < T; ++t) {
    const int64_t p = pos ? pos[t % S] : t % S;
    const int64_t ty = tt ? tt[t] : 0;
    for (int i = 0; i < d; ++i) tmp[t * d + i] = (we[ids[t] * d + i] + pe[p * d + i]) + te[ty * d + i];
  }
  layer_norm(tmp, blob + off[3], blob + off[4], x, T, d, c->layer_norm_eps);
  for (int l = 0; l < L; ++l) {
    const int64_t *lo = off + 5 + B_PER_LAYER * l;
    /* q, k, v as one [3d, d] weight: qkv [T, 3d] = x @ [Wq; Wk; Wv]^T + [bq; bk; bv] */
    memcpy(wqkv, blob + lo[B_Q_W], sizeof(float) * d * d);
    memcpy(wqkv + (int64_t)d * d, blob + lo[B_K_W], sizeof(float) * d * d);
    memcpy(wqkv + 2 * (int64_t)d * d, blob + lo[B_V_W], sizeof(float) * d * d);
    memcpy(bqkv, blob + lo[B_Q_B], sizeof(float) * d);
    memcpy(bqkv + d, blob + lo[B_K_B], sizeof(float) * d);
    memcpy(bqkv + 2 * d, blob + lo[B_V_B], sizeof(float) * d);
    sgemm((int)T, 3 * d, d, x, wqkv, 1, big);
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < 3 * d; ++j) big[t * 3 * d + j] += bqkv[j];
    attn_ctx ac = {big, mask, o, B, S, d, H, scr, 0};
    parallel_for((int64_t)B * H, attn_heads, &ac);
    sgemm((int)T, d, d, o, blob + lo[B_AO_W], 1, tmp);
    const float *bao = blob + lo[B_AO_B];
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < d; ++j) tmp[t * d + j] = (tmp[t * d + j] + bao[j]) + x[t * d + j];
    layer_norm(tmp, blob + lo[B_AOLN_G], blob + lo[B_AOLN_B], h, T, d, c->layer_norm_eps);
    sgemm((int)T, ff, d, h, blob + lo[B_I_W], 1, big);
    const float *bi = blob + lo[B_I_B];
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < ff; ++j) big[t * ff + j] = gelu_erf(big[t * ff + j] + bi[j]);
    sgemm((int)T, d, ff, big, blob + lo[B_O_W], 1, tmp);
    const float *bo = blob + lo[B_O_B];
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < d; ++j) tmp[t * d + j] = (tmp[t * d + j] + bo[j]) + h[t * d + j];
    layer_norm(tmp, blob + lo[B_OLN_G], blob + lo[B_OLN_B], x, T, d, c->layer_norm_eps);
  }
  memcpy(hidden, x, sizeof(float) * T * d);
  if (pooled) {
    const float *wp = blob + off[5 + B_PER_LAYER * L], *bp = blob + off[6 + B_PER_LAYER * L];
    for (int b = 0; b < B; ++b)
      for (int n = 0; n < d; ++n) {
        const float *r = x + (int64_t)b * S * d, *w = wp + (int64_t)n * d;
        float acc = 0.f;
        for (int k = 0; k < d; ++k) acc += r[k] * w[k];
        pooled[(int64_t)b * d + n] = tanhf(acc + bp[n]);
      }
  }
  free(off); free(x); free(h); free(o); free(tmp); free(big); free(wqkv); free(bqkv); free(scr);
  return 0;
}
