// context.cu -- model context, weight upload and packing, workspace and the
// forward schedule of the GPT-2 prefill.
//
// The schedule is the layer structure of HF GPT-2 as exported by the
// reference (src/gpt/lower_gpt_model.py:20-50, full logits, use_cache=False):
//   x = wte[ids] + wpe[pos]
//   per layer: a = ln_1(x); qkv = a @ W_attn + b; o = attention(qkv, mask);
//              x = x + (o @ W_proj + b); a = ln_2(x);
//              u = gelu_new(a @ W_fc + b); x = x + (u @ W_mproj + b)
//   logits = ln_f(x) @ wte^T
// as 3 + 7 L launches (+ 1 + L when a mask is given) instead of
// the reference's ~797 (README.md:96).
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "runtime.h"

namespace gpt2 {

namespace {
thread_local std::string g_err;
Context *g_ctx = nullptr;

void free_ws(Workspace &w) {
  void *ptrs[] = {w.x, w.a, w.qkv, w.o, w.u, w.stats, w.first_valid, w.key_valid, w.ids, w.mask};
  for (void *p : ptrs)
    if (p) cudaFree(p);
  if (w.logits) cudaFree(w.logits);
  w = Workspace();
}
}  // namespace

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

const char *last_error_text() { return g_err.c_str(); }
void clear_error() { g_err.clear(); }

std::vector<TensorSpec> blob_specs(const ModelDims &m) {
  std::vector<TensorSpec> s;
  int64_t off = 0;
  auto add = [&](int64_t n, TensorSpec::Kind k) {
    s.push_back({off, n, k});
    off += n;
  };
  const int64_t d = m.n_embd, ff = m.n_inner;
  add((int64_t)m.vocab * d, TensorSpec::kMatrix);
  add((int64_t)m.n_pos * d, TensorSpec::kMatrix);
  for (int l = 0; l < m.n_layer; ++l) {
    add(d, TensorSpec::kGain);
    add(d, TensorSpec::kBias);
    add(d * 3 * d, TensorSpec::kMatrix);
    add(3 * d, TensorSpec::kBias);
    add(d * d, TensorSpec::kMatrix);
    add(d, TensorSpec::kBias);
    add(d, TensorSpec::kGain);
    add(d, TensorSpec::kBias);
    add(d * ff, TensorSpec::kMatrix);
    add(ff, TensorSpec::kBias);
    add(ff * d, TensorSpec::kMatrix);
    add(d, TensorSpec::kBias);
  }
  add(d, TensorSpec::kGain);
  add(d, TensorSpec::kBias);
  return s;
}

int64_t blob_floats(const ModelDims &m) {
  const auto s = blob_specs(m);
  return s.back().offset + s.back().numel;
}

Context *context() { return g_ctx; }

void drop_graph(GraphCache &g) {
  if (g.exec) cudaGraphExecDestroy(g.exec);
  g = GraphCache();
}

void destroy_context() {
  if (!g_ctx) return;
  Context *c = g_ctx;
  g_ctx = nullptr;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  drop_graph(c->graph);
  drop_graph(c->dec_graph);
  free_decode(c->dec);
  for (cudaEvent_t e : c->prof.pool) cudaEventDestroy(e);
  free_ws(c->ws);
  if (c->d_blob) cudaFree(c->d_blob);
  if (c->wte_h) cudaFree(c->wte_h);
  if (c->wpe_h) cudaFree(c->wpe_h);
  if (c->wte_ln) cudaFree(c->wte_ln);
  if (c->head_c1) cudaFree(c->head_c1);
  if (c->head_c2) cudaFree(c->head_c2);
  for (auto &l : c->layers) {
    void *p[] = {l.qkv_wt, l.proj_wt, l.fc_wt, l.mproj_wt, l.qkv_q, l.proj_q, l.fc_q, l.mproj_q,
                 l.qkv_s, l.proj_s, l.fc_s, l.mproj_s, l.qkv_lnw, l.fc_lnw, l.qkv_c1, l.qkv_c2,
                 l.fc_c1, l.fc_c2};
    for (void *q : p)
      if (q) cudaFree(q);
  }
  if (c->d_status) cudaFree(c->d_status);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  cudaSetDevice(prev);
}

int create_context(const ModelDims &m, int dtype, int device) {
  if (m.n_layer < 1 || m.n_embd < 64 || m.n_embd % 64 || m.n_head < 1 || m.n_embd / m.n_head != 64 ||
      m.n_embd % m.n_head || m.n_inner < 64 || m.n_inner % 64 || m.vocab < 1 || m.n_pos < 1 || !(m.eps > 0.f)) {
    set_error("unsupported GPT-2 configuration (need n_embd %% 64 == 0, head dim 64, n_inner %% 64 == 0)");
    return -1;
  }
  if (dtype < 0 || dtype > 2) {
    set_error("unsupported dtype %d", dtype);
    return -1;
  }
  destroy_context();
  if (device < 0) CK(cudaGetDevice(&device));
  CK(cudaSetDevice(device));
  Context *c = new Context();
  c->dims = m;
  c->dtype = dtype;
  c->device = device;
  cudaError_t e = cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, sizeof(int));
  if (e != cudaSuccess) {
    g_ctx = c;
    destroy_context();
    return cuda_fail(e, "context setup");
  }
  c->specs = blob_specs(m);
  if (const char *e = getenv("GPT2_GRAPHS")) c->use_graphs = strcmp(e, "0") != 0;
  g_ctx = c;
  return 0;
}

int load_blob(Context &c, const float *host_blob) {
  CK(cudaSetDevice(c.device));
  const ModelDims &m = c.dims;
  const int64_t n = blob_floats(m);
  if (!c.d_blob) CK(cudaMalloc(&c.d_blob, sizeof(float) * n));
  CK(cudaMemcpy(c.d_blob, host_blob, sizeof(float) * n, cudaMemcpyHostToDevice));
  const auto &s = c.specs;
  auto at = [&](size_t i) -> float * { return c.d_blob + s[i].offset; };
  c.wte = at(0);
  c.wpe = at(1);
  c.lnf_g = at(2 + PER_LAYER * m.n_layer);
  c.lnf_b = at(3 + PER_LAYER * m.n_layer);
  c.layers.resize(m.n_layer);
  const int d = m.n_embd, ff = m.n_inner;
  for (int l = 0; l < m.n_layer; ++l) {
    LayerWeights &w = c.layers[l];
    const size_t b = 2 + PER_LAYER * l;
    w.ln1_g = at(b + LN1_G);
    w.ln1_b = at(b + LN1_B);
    w.qkv_w = at(b + QKV_W);
    w.qkv_b = at(b + QKV_B);
    w.proj_w = at(b + PROJ_W);
    w.proj_b = at(b + PROJ_B);
    w.ln2_g = at(b + LN2_G);
    w.ln2_b = at(b + LN2_B);
    w.fc_w = at(b + FC_W);
    w.fc_b = at(b + FC_B);
    w.mproj_w = at(b + MPROJ_W);
    w.mproj_b = at(b + MPROJ_B);
  }
  if (c.dtype >= 1) {
    // BF16 copies: wte / wpe as stored ([V, d] is already the K-major B of the
    // lm_head), Conv1D weights transposed to [out, in] (K-major B operands).
    if (!c.wte_h) CK(cudaMalloc(&c.wte_h, sizeof(bf16) * (size_t)m.vocab * d));
    if (!c.wpe_h) CK(cudaMalloc(&c.wpe_h, sizeof(bf16) * (size_t)m.n_pos * d));
    CK(launch_pack_bf16(c.wte, c.wte_h, m.vocab, d, 0, c.stream));
    CK(launch_pack_bf16(c.wpe, c.wpe_h, m.n_pos, d, 0, c.stream));
    std::vector<uint8_t> hq;
    std::vector<float> hs;
    for (int l = 0; l < m.n_layer; ++l) {
      LayerWeights &w = c.layers[l];
      if (!w.qkv_wt) CK(cudaMalloc(&w.qkv_wt, sizeof(bf16) * (size_t)d * 3 * d));
      if (!w.proj_wt) CK(cudaMalloc(&w.proj_wt, sizeof(bf16) * (size_t)d * d));
      if (!w.fc_wt) CK(cudaMalloc(&w.fc_wt, sizeof(bf16) * (size_t)d * ff));
      if (!w.mproj_wt) CK(cudaMalloc(&w.mproj_wt, sizeof(bf16) * (size_t)ff * d));
      if (c.dtype == 1) {
        CK(launch_pack_bf16(w.qkv_w, w.qkv_wt, d, 3 * d, 1, c.stream));
        CK(launch_pack_bf16(w.proj_w, w.proj_wt, d, d, 1, c.stream));
        CK(launch_pack_bf16(w.fc_w, w.fc_wt, d, ff, 1, c.stream));
        CK(launch_pack_bf16(w.mproj_w, w.mproj_wt, ff, d, 1, c.stream));
        // ln_1 into QKV and ln_2 into fc: gain-scaled copies and their c1 / c2
        // (the unscaled copies above serve the decode step).
        if (!w.qkv_lnw) CK(cudaMalloc(&w.qkv_lnw, sizeof(bf16) * (size_t)d * 3 * d));
        if (!w.fc_lnw) CK(cudaMalloc(&w.fc_lnw, sizeof(bf16) * (size_t)d * ff));
        float **vec[4] = {&w.qkv_c1, &w.qkv_c2, &w.fc_c1, &w.fc_c2};
        const int vlen[4] = {3 * d, 3 * d, ff, ff};
        for (int i = 0; i < 4; ++i)
          if (!*vec[i]) CK(cudaMalloc(vec[i], sizeof(float) * ln_vector_len(vlen[i])));
        CK(launch_ln_fold_pack(w.qkv_w, 1, w.ln1_g, w.ln1_b, w.qkv_b, w.qkv_lnw, w.qkv_c1, w.qkv_c2, 3 * d, d,
                               c.stream));
        CK(launch_ln_fold_pack(w.fc_w, 1, w.ln2_g, w.ln2_b, w.fc_b, w.fc_lnw, w.fc_c1, w.fc_c2, ff, d, c.stream));
        continue;
      }
      // Weight-only FP8: quantize on the host (per-output-channel scale), keep
      // the E4M3 codes and scales resident, expand the codes exactly to the
      // BF16 operands; the GEMM epilogue applies the scale.
      const size_t b = 2 + PER_LAYER * l;
      struct {
        size_t idx;
        int K, N;
        uint8_t **q;
        float **sc;
        bf16 *wt;
      } mats[4] = {{b + QKV_W, d, 3 * d, &w.qkv_q, &w.qkv_s, w.qkv_wt},
                   {b + PROJ_W, d, d, &w.proj_q, &w.proj_s, w.proj_wt},
                   {b + FC_W, d, ff, &w.fc_q, &w.fc_s, w.fc_wt},
                   {b + MPROJ_W, ff, d, &w.mproj_q, &w.mproj_s, w.mproj_wt}};
      for (auto &mt : mats) {
        const size_t n = (size_t)mt.K * mt.N;
        hq.resize(n);
        hs.resize(mt.N);
        fp8_quantize(host_blob + s[mt.idx].offset, mt.K, mt.N, hq.data(), hs.data());
        if (!*mt.q) CK(cudaMalloc(mt.q, n));
        if (!*mt.sc) CK(cudaMalloc(mt.sc, sizeof(float) * mt.N));
        CK(cudaMemcpy(*mt.q, hq.data(), n, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(*mt.sc, hs.data(), sizeof(float) * mt.N, cudaMemcpyHostToDevice));
        CK(launch_e4m3_to_bf16(*mt.q, mt.wt, (int64_t)n, c.stream));
      }
    }
    // BF16 folds ln_f into the lm_head: wte * ln_f gain, c2 = wte @ ln_f shift.
    // Weight-only FP8 keeps its weights exactly on the E4M3 grid and runs the
    // LayerNorm kernels instead.
    c.ln_fold = c.dtype == 1;
    if (c.ln_fold) {
      if (!c.wte_ln) CK(cudaMalloc(&c.wte_ln, sizeof(bf16) * (size_t)m.vocab * d));
      if (!c.head_c1) CK(cudaMalloc(&c.head_c1, sizeof(float) * ln_vector_len(m.vocab)));
      if (!c.head_c2) CK(cudaMalloc(&c.head_c2, sizeof(float) * ln_vector_len(m.vocab)));
      CK(launch_ln_fold_pack(c.wte, 0, c.lnf_g, c.lnf_b, nullptr, c.wte_ln, c.head_c1, c.head_c2, m.vocab, d,
                             c.stream));
    }
    CK(cudaStreamSynchronize(c.stream));
  }
  c.loaded = true;
  c.plans_T = -1;  // weights moved: rebuild TMA descriptors
  drop_graph(c.graph);
  // A decode cache (and the FP32 transposed weights) belongs to the old weights.
  CK(cudaDeviceSynchronize());
  drop_graph(c.dec_graph);
  free_decode(c.dec);
  return 0;
}

int ensure_workspace(Context &c, int B, int S) {
  const int64_t T = (int64_t)B * S;
  Workspace &w = c.ws;
  if (T <= w.T && B <= w.B) return 0;
  const int64_t Tn = std::max(T, w.T);
  const int Bn = std::max(B, w.B);
  CK(cudaDeviceSynchronize());  // earlier forwards may still read the buffers on any stream
  drop_graph(c.graph);           // it captured the old buffers
  Workspace keep_logits;
  keep_logits.logits = w.logits;
  keep_logits.logits_T = w.logits_T;
  w.logits = nullptr;
  free_ws(w);
  w.logits = keep_logits.logits;
  w.logits_T = keep_logits.logits_T;
  const size_t es = c.dtype >= 1 ? 2 : 4;
  const int64_t d = c.dims.n_embd, ff = c.dims.n_inner;
  CK(cudaMalloc(&w.x, es * Tn * d));
  CK(cudaMalloc(&w.a, es * Tn * d));
  CK(cudaMalloc(&w.qkv, es * Tn * 3 * d));
  CK(cudaMalloc(&w.o, es * Tn * d));
  CK(cudaMalloc(&w.u, es * Tn * ff));
  if (c.dtype >= 1) CK(cudaMalloc(&w.stats, sizeof(float2) * Tn * ln_segments((int)d)));
  CK(cudaMalloc(&w.first_valid, sizeof(int) * Bn));
  CK(cudaMalloc(&w.key_valid, Tn));
  CK(cudaMalloc(&w.ids, sizeof(int64_t) * Tn));
  CK(cudaMalloc(&w.mask, sizeof(int64_t) * Tn));
  w.T = Tn;
  w.B = Bn;
  c.plans_T = -1;
  return 0;
}

namespace {
// TMA descriptors of every BF16 GEMM for M = T tokens over the current
// workspace: per layer qkv, proj, fc, mproj, then the lm_head.
int ensure_plans(Context &c, int64_t T) {
  if (c.plans_T == T) return 0;
  const ModelDims &m = c.dims;
  const int d = m.n_embd, ff = m.n_inner;
  c.plans.resize(4 * m.n_layer + 1);
  const bf16 *o = static_cast<const bf16 *>(c.ws.o), *u = static_cast<const bf16 *>(c.ws.u);
  // With the LayerNorms folded, QKV, fc and the lm_head read the residual
  // stream x itself and the gain-scaled weights.
  const bf16 *a = static_cast<const bf16 *>(c.ln_fold ? c.ws.x : c.ws.a);
  auto pick_bn = [&](int N) {
    // 128 x 256 tiles once they fill the GPU at least once: at 8192 tokens the
    // 768-wide residual GEMMs measured 22.8 vs 24.8 us (K = 768) and 47.1 vs
    // 58.6 us (K = 3072) with 256-wide tiles at 1.3 waves.
    const int64_t tiles256 = ((T + 127) / 128) * ((N + 255) / 256);
    return tiles256 >= c.num_sms ? 256 : 128;
  };
  // 256 x 256 tiles on CTA pairs where there are enough of them to fill the
  // GPU twice over; measured faster for the QKV, fc, MLP-proj and lm_head
  // shapes and slower for the narrow short-K attention out-proj (N = K = d),
  // which keeps the single-SM tiles.
  auto pick_tile = [&](int N) {
    const int64_t pair_tiles = ((T + 255) / 256) * ((N + 255) / 256);
    return pair_tiles >= 2 * (c.num_sms / 2) ? TC_TILE_PAIR : pick_bn(N);
  };
  for (int l = 0; l < m.n_layer; ++l) {
    const LayerWeights &w = c.layers[l];
    TcGemmPlan *p = &c.plans[4 * l];
    int r = tc_gemm_plan(&p[0], a, c.ln_fold ? w.qkv_lnw : w.qkv_wt, (int)T, 3 * d, d, pick_tile(3 * d));
    if (!r) r = tc_gemm_plan(&p[1], o, w.proj_wt, (int)T, d, d, pick_bn(d));
    if (!r) r = tc_gemm_plan(&p[2], a, c.ln_fold ? w.fc_lnw : w.fc_wt, (int)T, ff, d, pick_tile(ff));
    if (!r) r = tc_gemm_plan(&p[3], u, w.mproj_wt, (int)T, d, ff, pick_tile(d));
    if (r) {
      set_error("TMA descriptor creation failed (%d)", r);
      return -2;
    }
    tc_gemm_set_output(&p[0], c.ws.qkv, 3 * d, 0);
    tc_gemm_set_output(&p[1], c.ws.x, d, 0);
    tc_gemm_set_output(&p[2], c.ws.u, ff, 0);
    tc_gemm_set_output(&p[3], c.ws.x, d, 0);
  }
  c.head_tile = pick_tile(m.vocab);
  c.head_bn = pick_bn(m.vocab);
  if (tc_gemm_plan(&c.plans[4 * m.n_layer], a, c.ln_fold ? c.wte_ln : c.wte_h, (int)T, m.vocab, d, c.head_tile)) {
    set_error("TMA descriptor creation failed (lm_head)");
    return -2;
  }
  c.plans_T = T;
  return 0;
}
}  // namespace

int cuda_fail(cudaError_t e, const char *what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return -2;
}

cudaEvent_t prof_event(Profiler &p) {
  if (p.used == p.pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    p.pool.push_back(e);
  }
  return p.pool[p.used++];
}

int profile_begin(Profiler &p) {
  p.on = true;
  p.used = 0;
  p.kinds.clear();
  return 0;
}

int profile_end(Profiler &p, double *ms, int64_t *count, int n) {
  p.on = false;
  for (int k = 0; k < n; ++k) {
    ms[k] = 0.0;
    count[k] = 0;
  }
  for (size_t i = 0; i < p.kinds.size(); ++i) {
    cudaEvent_t a = p.pool[2 * i], b = p.pool[2 * i + 1];
    CK(cudaEventSynchronize(b));
    float t = 0.f;
    CK(cudaEventElapsedTime(&t, a, b));
    const int k = p.kinds[i];
    if (k < n) {
      ms[k] += t;
      count[k] += 1;
    }
  }
  p.kinds.clear();
  p.used = 0;
  return 0;
}

int forward_launch_count(const Context &c, int64_t T, int has_mask) {
  // embed + 7 per layer + ln_f + lm_head; with a mask, seq_info + 1 per layer.
  // With the LayerNorms folded into the GEMMs: embed + 5 per layer + lm_head.
  // A few-token forward: embed + 5 per layer (LayerNorms inside the GEMVs) + lm_head.
  const bool fold = T <= kFewRows || c.ln_fold;
  const int base = fold ? 2 + 5 * c.dims.n_layer : 3 + 7 * c.dims.n_layer;
  return base + (has_mask ? 1 + c.dims.n_layer : 0);
}

// Buffers, TMA descriptors and output descriptor of a forward of (B, S) into
// d_logits: everything that allocates or encodes on the host, done before
// any launch (and outside any graph capture).
int prepare_forward(Context &c, int B, int S, void *d_logits, int64_t ld_logits, int logits_f32) {
  const ModelDims &m = c.dims;
  int r = ensure_workspace(c, B, S);
  if (!r && c.dtype == 0 && (int64_t)B * S <= kFewRows) r = ensure_nk_f32(c);
  if (r || c.dtype == 0) return r;
  Workspace &w = c.ws;
  r = ensure_plans(c, (int64_t)B * S);
  if (r) return r;
  if (c.attn_plan.qkv != w.qkv || c.attn_plan.out != w.o || c.attn_plan.B != B || c.attn_plan.S != S ||
      c.attn_plan.H != m.n_head) {
    if (attention_tc_plan(&c.attn_plan, static_cast<const bf16 *>(w.qkv), B, S, m.n_head,
                          static_cast<const bf16 *>(w.o))) {
      set_error("TMA descriptor creation failed (attention)");
      return -2;
    }
  }
  TcGemmPlan &head = c.plans[4 * m.n_layer];
  if (d_logits && (head.c_ptr != d_logits || head.c_ld != (int)ld_logits || head.c_f32 != logits_f32)) {
    // Logits rows that TMA cannot store (unaligned base or row stride) go
    // through the single-SM kernel's direct stores, with its own tile width.
    const bool storable =
        !(reinterpret_cast<uintptr_t>(d_logits) & 15) && (ld_logits * (logits_f32 ? 4 : 2)) % 16 == 0;
    const int tile = storable ? c.head_tile : c.head_bn;
    if (head.two_sm != (tile == TC_TILE_PAIR) || (!head.two_sm && head.bn != tile)) {
      if (tc_gemm_plan(&head, static_cast<const bf16 *>(c.ln_fold ? w.x : w.a), c.ln_fold ? c.wte_ln : c.wte_h,
                       B * S, m.vocab, m.n_embd, tile)) {
        set_error("TMA descriptor creation failed (lm_head)");
        return -2;
      }
    }
    tc_gemm_set_output(&head, d_logits, (int)ld_logits, logits_f32);
  }
  return 0;
}

namespace {
// The forward of at most kFewRows tokens (the reference host program's own
// B1 x S5 call, short prompts): LayerNorm kernels and the split-K GEMV
// kernels of the decode step, which spread each weight's stream over the
// whole GPU, instead of the tiled GEMMs, which would give a handful of rows
// one M-tile on a few SMs.  Same results contract as the tiled path.
int launch_forward_few(Context &c, const int64_t *d_ids, const uint8_t *kv, const int64_t *d_mask, int B, int S,
                       void *d_logits_v, int64_t ld_logits, cudaStream_t st, bool kv_fill, int logits_f32) {
  float *d_logits = static_cast<float *>(d_logits_v);
  const ModelDims &m = c.dims;
  const int T = B * S;
  const int d = m.n_embd, ff = m.n_inner, H = m.n_head, V = m.vocab;
  Workspace &w = c.ws;
  const GemvLn lnf{c.lnf_g, c.lnf_b, m.eps};
  // ln_1, ln_2 and ln_f run inside the GEMVs that read them (GemvLn); the
  // attention of these short sequences is one warp per query row.
  // Every GEMV and attention launch here follows a kernel, so it can be a
  // programmatic dependent of it (its weight prefetch overlaps the previous
  // kernel); not in a profiled step, whose events bracket each kernel.
  const bool pdl = !c.prof.on;
  if (c.dtype == 0) {
    float *x = static_cast<float *>(w.x), *qkv = static_cast<float *>(w.qkv), *o = static_cast<float *>(w.o),
          *u = static_cast<float *>(w.u);
    CKP(K_EMBED, launch_embed_f32(d_ids, c.wte, c.wpe, x, T, S, d, V, c.d_status, st));
    for (int l = 0; l < m.n_layer; ++l) {
      const LayerWeights &lw = c.layers[l];
      float *const *wt = &c.dec.wt[4 * l];
      const GemvLn ln1{lw.ln1_g, lw.ln1_b, m.eps}, ln2{lw.ln2_g, lw.ln2_b, m.eps};
      CKP(K_GEMM_QKV, launch_gemv_f32(x, wt[0], qkv, T, 3 * d, d, 3 * d, lw.qkv_b, nullptr, EPI_BIAS, st, &ln1, pdl));
      if (kv_fill)
        CK(launch_kv_store_f32(qkv, static_cast<float *>(c.dec.cache[l]), B, S, d, c.dec.max_len, 0, st));
      CKP(K_ATTENTION, launch_attention_short_f32(qkv, kv, o, B, S, H, 1, st, pdl));
      if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_f32(qkv, w.first_valid, o, B, S, H, st));
      CKP(K_GEMM_PROJ, launch_gemv_f32(o, wt[1], x, T, d, d, d, lw.proj_b, x, EPI_BIAS_RESID, st, nullptr, pdl));
      CKP(K_GEMM_FC, launch_gemv_f32(x, wt[2], u, T, ff, d, ff, lw.fc_b, nullptr, EPI_BIAS_GELU, st, &ln2, pdl));
      CKP(K_GEMM_MPROJ, launch_gemv_f32(u, wt[3], x, T, d, ff, d, lw.mproj_b, x, EPI_BIAS_RESID, st, nullptr, pdl));
    }
    if (kv_fill) {
      float *xl = static_cast<float *>(c.dec.a_last);
      CK(cudaMemcpy2DAsync(xl, sizeof(float) * d, x + (int64_t)(S - 1) * d, sizeof(float) * S * d,
                           sizeof(float) * d, B, cudaMemcpyDeviceToDevice, st));
      CKP(K_LM_HEAD,
          launch_gemv_f32(xl, c.wte, d_logits, B, V, d, (int)ld_logits, nullptr, nullptr, EPI_NONE, st, &lnf));
      return 0;
    }
    CKP(K_LM_HEAD,
        launch_gemv_f32(x, c.wte, d_logits, T, V, d, (int)ld_logits, nullptr, nullptr, EPI_NONE, st, &lnf, pdl));
    return 0;
  }
  bf16 *x = static_cast<bf16 *>(w.x), *qkv = static_cast<bf16 *>(w.qkv), *o = static_cast<bf16 *>(w.o),
       *u = static_cast<bf16 *>(w.u);
  CKP(K_EMBED, launch_embed_bf16(d_ids, c.wte_h, c.wpe_h, x, T, S, d, V, c.d_status, st));
  for (int l = 0; l < m.n_layer; ++l) {
    const LayerWeights &lw = c.layers[l];
    const GemvLn ln1{lw.ln1_g, lw.ln1_b, m.eps}, ln2{lw.ln2_g, lw.ln2_b, m.eps};
    CKP(K_GEMM_QKV, launch_gemv_bf16_auto(x, lw.qkv_wt, qkv, T, 3 * d, d, 3 * d, lw.qkv_b, nullptr, lw.qkv_s, EPI_BIAS, c.d_status,
                                     st, &ln1, pdl));
    if (kv_fill) CK(launch_kv_store_bf16(qkv, static_cast<bf16 *>(c.dec.cache[l]), B, S, d, c.dec.max_len, 0, st));
    CKP(K_ATTENTION, launch_attention_short_bf16(qkv, kv, o, B, S, H, 1, st, pdl));
    if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_bf16(qkv, w.first_valid, o, B, S, H, st));
    CKP(K_GEMM_PROJ, launch_gemv_bf16_auto(o, lw.proj_wt, x, T, d, d, d, lw.proj_b, x, lw.proj_s, EPI_BIAS_RESID, c.d_status, st, nullptr, pdl));
    CKP(K_GEMM_FC,
        launch_gemv_bf16_auto(x, lw.fc_wt, u, T, ff, d, ff, lw.fc_b, nullptr, lw.fc_s, EPI_BIAS_GELU, c.d_status, st, &ln2, pdl));
    CKP(K_GEMM_MPROJ,
        launch_gemv_bf16_auto(u, lw.mproj_wt, x, T, d, ff, d, lw.mproj_b, x, lw.mproj_s, EPI_BIAS_RESID, c.d_status, st, nullptr, pdl));
  }
  if (kv_fill) {
    bf16 *xl = static_cast<bf16 *>(c.dec.a_last);
    CK(cudaMemcpy2DAsync(xl, sizeof(bf16) * d, x + (int64_t)(S - 1) * d, sizeof(bf16) * S * d, sizeof(bf16) * d, B,
                         cudaMemcpyDeviceToDevice, st));
    CKP(K_LM_HEAD, launch_gemv_bf16_f32out_auto(xl, c.wte_h, d_logits, B, V, d, (int)ld_logits, c.d_status, st, &lnf));
    return 0;
  }
  if (!logits_f32) {
    CKP(K_LM_HEAD, launch_gemv_bf16_auto(x, c.wte_h, static_cast<bf16 *>(d_logits_v), T, V, d, (int)ld_logits, nullptr,
                                    nullptr, nullptr, EPI_NONE, c.d_status, st, &lnf, pdl));
    return 0;
  }
  CKP(K_LM_HEAD, launch_gemv_bf16_f32out_auto(x, c.wte_h, d_logits, T, V, d, (int)ld_logits, c.d_status, st, &lnf, pdl));
  return 0;
}
}  // namespace

// Enqueues the forward's kernels on st (prepare_forward has run).  With
// kv_fill, every layer's keys and values also go to the decode cache, and
// only the last position's logits are computed, into d_logits [B, ld_logits].
int launch_forward(Context &c, const int64_t *d_ids, const int64_t *d_mask, int B, int S, void *d_logits_v,
                   int64_t ld_logits, cudaStream_t st, bool kv_fill, int logits_f32) {
  float *d_logits = static_cast<float *>(d_logits_v);
  const ModelDims &m = c.dims;
  const int64_t T = (int64_t)B * S;
  const int d = m.n_embd, ff = m.n_inner, H = m.n_head, V = m.vocab;
  Workspace &w = c.ws;
  const uint8_t *kv = nullptr;
  if (d_mask) {
    CKP(K_SEQ_INFO, launch_seq_info(d_mask, B, S, w.first_valid, w.key_valid, st));
    kv = w.key_valid;
  }
  if (T <= kFewRows)
    return launch_forward_few(c, d_ids, kv, d_mask, B, S, d_logits_v, ld_logits, st, kv_fill, logits_f32);
  if (c.dtype == 0) {
    float *x = static_cast<float *>(w.x), *a = static_cast<float *>(w.a), *qkv = static_cast<float *>(w.qkv),
          *o = static_cast<float *>(w.o), *u = static_cast<float *>(w.u);
    CKP(K_EMBED, launch_embed_f32(d_ids, c.wte, c.wpe, x, (int)T, S, d, V, c.d_status, st));
    for (int l = 0; l < m.n_layer; ++l) {
      const LayerWeights &lw = c.layers[l];
      CKP(K_LAYERNORM, launch_layernorm_f32(x, lw.ln1_g, lw.ln1_b, a, (int)T, d, m.eps, st));
      CKP(K_GEMM_QKV, launch_gemm_f32(a, lw.qkv_w, 0, qkv, (int)T, 3 * d, d, 3 * d, lw.qkv_b, nullptr, EPI_BIAS, st));
      if (kv_fill)
        CK(launch_kv_store_f32(qkv, static_cast<float *>(c.dec.cache[l]), B, S, d, c.dec.max_len, 0, st));
      CKP(K_ATTENTION, launch_attention_f32(qkv, kv, o, B, S, H, st));
      if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_f32(qkv, w.first_valid, o, B, S, H, st));
      CKP(K_GEMM_PROJ, launch_gemm_f32(o, lw.proj_w, 0, x, (int)T, d, d, d, lw.proj_b, x, EPI_BIAS_RESID, st));
      CKP(K_LAYERNORM, launch_layernorm_f32(x, lw.ln2_g, lw.ln2_b, a, (int)T, d, m.eps, st));
      CKP(K_GEMM_FC, launch_gemm_f32(a, lw.fc_w, 0, u, (int)T, ff, d, ff, lw.fc_b, nullptr, EPI_BIAS_GELU, st));
      CKP(K_GEMM_MPROJ, launch_gemm_f32(u, lw.mproj_w, 0, x, (int)T, d, ff, d, lw.mproj_b, x, EPI_BIAS_RESID, st));
    }
    CKP(K_LAYERNORM, launch_layernorm_f32(x, c.lnf_g, c.lnf_b, a, (int)T, d, m.eps, st));
    if (kv_fill) {
      float *al = static_cast<float *>(c.dec.a_last);
      CK(cudaMemcpy2DAsync(al, sizeof(float) * d, a + (int64_t)(S - 1) * d, sizeof(float) * S * d,
                           sizeof(float) * d, B, cudaMemcpyDeviceToDevice, st));
      CKP(K_LM_HEAD, launch_gemv_f32(al, c.wte, d_logits, B, V, d, (int)ld_logits, nullptr, nullptr, EPI_NONE, st));
      return 0;
    }
    CKP(K_LM_HEAD, launch_gemm_f32(a, c.wte, 1, d_logits, (int)T, V, d, (int)ld_logits, nullptr, nullptr, EPI_NONE, st));
    return 0;
  }
  bf16 *x = static_cast<bf16 *>(w.x), *a = static_cast<bf16 *>(w.a), *qkv = static_cast<bf16 *>(w.qkv),
       *o = static_cast<bf16 *>(w.o), *u = static_cast<bf16 *>(w.u);
  const int ns = c.num_sms;
  if (c.ln_fold) {
    // Every LayerNorm folded into the GEMM after it: the embedding and the two
    // residual GEMMs of each layer also write the row statistics of x, which
    // the QKV / fc / lm_head epilogues turn into mean and 1/std.
    LnFold stats_out;
    stats_out.stats_out = w.stats;
    stats_out.nseg_out = ln_segments(d);
    auto fold = [&](const float *c1, const float *c2) {
      LnFold f;
      f.c1 = c1;
      f.c2 = c2;
      f.stats_in = w.stats;
      f.nseg_in = ln_segments(d);
      f.k = d;
      f.eps = m.eps;
      return f;
    };
    CKP(K_EMBED, launch_embed_bf16(d_ids, c.wte_h, c.wpe_h, x, (int)T, S, d, V, c.d_status, st, w.stats));
    for (int l = 0; l < m.n_layer; ++l) {
      const LayerWeights &lw = c.layers[l];
      const TcGemmPlan *p = &c.plans[4 * l];
      const LnFold ln1 = fold(lw.qkv_c1, lw.qkv_c2), ln2 = fold(lw.fc_c1, lw.fc_c2);
      CKP(K_GEMM_QKV,
          launch_gemm_tc(p[0], qkv, 3 * d, 0, nullptr, nullptr, EPI_LN_BIAS, c.d_status, ns, st, nullptr, &ln1));
      if (kv_fill) CK(launch_kv_store_bf16(qkv, static_cast<bf16 *>(c.dec.cache[l]), B, S, d, c.dec.max_len, 0, st));
      CKP(K_ATTENTION, launch_attention_tc3(c.attn_plan, kv, o, c.d_status, st));
      if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_bf16(qkv, w.first_valid, o, B, S, H, st));
      CKP(K_GEMM_PROJ, launch_gemm_tc(p[1], x, d, 0, lw.proj_b, x, EPI_BIAS_RESID_STATS, c.d_status, ns, st,
                                      nullptr, &stats_out));
      CKP(K_GEMM_FC,
          launch_gemm_tc(p[2], u, ff, 0, nullptr, nullptr, EPI_LN_BIAS_GELU, c.d_status, ns, st, nullptr, &ln2));
      CKP(K_GEMM_MPROJ, launch_gemm_tc(p[3], x, d, 0, lw.mproj_b, x, EPI_BIAS_RESID_STATS, c.d_status, ns, st,
                                       nullptr, &stats_out));
    }
    if (!kv_fill) {
      const LnFold lnf = fold(c.head_c1, c.head_c2);
      const TcGemmPlan &head = c.plans[4 * m.n_layer];
      CKP(K_LM_HEAD, launch_gemm_tc(head, d_logits_v, (int)ld_logits, logits_f32, nullptr, nullptr, EPI_LN_BIAS,
                                    c.d_status, ns, st, nullptr, &lnf));
      return 0;
    }
  } else {
    CKP(K_EMBED, launch_embed_bf16(d_ids, c.wte_h, c.wpe_h, x, (int)T, S, d, V, c.d_status, st));
    for (int l = 0; l < m.n_layer; ++l) {
      const LayerWeights &lw = c.layers[l];
      const TcGemmPlan *p = &c.plans[4 * l];
      CKP(K_LAYERNORM, launch_layernorm_bf16(x, lw.ln1_g, lw.ln1_b, a, (int)T, d, m.eps, st));
      CKP(K_GEMM_QKV,
          launch_gemm_tc(p[0], qkv, 3 * d, 0, lw.qkv_b, nullptr, EPI_BIAS, c.d_status, ns, st, lw.qkv_s));
      if (kv_fill) CK(launch_kv_store_bf16(qkv, static_cast<bf16 *>(c.dec.cache[l]), B, S, d, c.dec.max_len, 0, st));
      CKP(K_ATTENTION, launch_attention_tc3(c.attn_plan, kv, o, c.d_status, st));
      if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_bf16(qkv, w.first_valid, o, B, S, H, st));
      CKP(K_GEMM_PROJ, launch_gemm_tc(p[1], x, d, 0, lw.proj_b, x, EPI_BIAS_RESID, c.d_status, ns, st, lw.proj_s));
      CKP(K_LAYERNORM, launch_layernorm_bf16(x, lw.ln2_g, lw.ln2_b, a, (int)T, d, m.eps, st));
      CKP(K_GEMM_FC, launch_gemm_tc(p[2], u, ff, 0, lw.fc_b, nullptr, EPI_BIAS_GELU, c.d_status, ns, st, lw.fc_s));
      CKP(K_GEMM_MPROJ,
          launch_gemm_tc(p[3], x, d, 0, lw.mproj_b, x, EPI_BIAS_RESID, c.d_status, ns, st, lw.mproj_s));
    }
  }
  // ln_f over every row: the input of the lm_head, or (kv_fill) of the last
  // position's logits.
  CKP(K_LAYERNORM, launch_layernorm_bf16(x, c.lnf_g, c.lnf_b, a, (int)T, d, m.eps, st));
  if (kv_fill) {
    bf16 *al = static_cast<bf16 *>(c.dec.a_last);
    CK(cudaMemcpy2DAsync(al, sizeof(bf16) * d, a + (int64_t)(S - 1) * d, sizeof(bf16) * S * d, sizeof(bf16) * d, B,
                         cudaMemcpyDeviceToDevice, st));
    CKP(K_LM_HEAD, launch_gemv_bf16_f32out_auto(al, c.wte_h, d_logits, B, V, d, (int)ld_logits, c.d_status, st));
    return 0;
  }
  const TcGemmPlan &head = c.plans[4 * m.n_layer];
  CKP(K_LM_HEAD, launch_gemm_tc(head, d_logits_v, (int)ld_logits, logits_f32, nullptr, nullptr, EPI_NONE,
                                c.d_status, ns, st));
  return 0;
}

int forward_device(Context &c, const int64_t *d_ids, const int64_t *d_mask, int B, int S, void *d_logits,
                   int64_t ld_logits, int logits_f32, cudaStream_t st) {
  const ModelDims &m = c.dims;
  if (!c.loaded) {
    set_error("no weights loaded");
    return -3;
  }
  if (B < 1 || S < 1 || S > m.n_pos || (int64_t)B * S > (int64_t)1 << 30 || ld_logits < m.vocab) {
    set_error("bad forward shape B=%d S=%d (n_positions %d) ld_logits=%lld", B, S, m.n_pos, (long long)ld_logits);
    return -1;
  }
  if (!logits_f32 && (c.dtype == 0 || ld_logits % 8)) {
    set_error("bf16 logits need a BF16 or FP8-weight model and a row stride that is a multiple of 8 (got dtype %d, "
              "ld_logits %lld)", c.dtype, (long long)ld_logits);
    return -1;
  }
  int r = prepare_forward(c, B, S, d_logits, ld_logits, logits_f32);
  if (r) return r;
  auto launch = [&](cudaStream_t s) {
    return launch_forward(c, d_ids, d_mask, B, S, d_logits, ld_logits, s, false, logits_f32);
  };
  if (c.prof.on) return launch(st);  // per-launch events need plain launches
  const uintptr_t key[7] = {reinterpret_cast<uintptr_t>(d_ids), reinterpret_cast<uintptr_t>(d_mask),
                            reinterpret_cast<uintptr_t>(d_logits), static_cast<uintptr_t>(ld_logits),
                            static_cast<uintptr_t>(B), static_cast<uintptr_t>(S),
                            static_cast<uintptr_t>(logits_f32)};
  return run_with_graph(c.graph, &c.use_graphs, key, 7, c.stream, st, launch);
}

}  // namespace gpt2
