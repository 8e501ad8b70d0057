// bert.cu -- the BERT encoder's context, weight upload and forward schedule.
//
// The schedule is transformers' BertModel as exported by the reference
// (src/bert-base-uncased/lower_bert_model.py:7-18: last_hidden_state and
// pooler_output, eager attention, no dropout), post-LayerNorm:
//   x = LN_emb(word[ids] + pos[position_ids] + type[token_type_ids])
//   per layer: qkv = x @ [Wq; Wk; Wv]^T + b; o = attention(qkv, mask), not causal;
//              h = LN_1(x + (o @ Wao^T + b)); u = gelu_erf(h @ Wi^T + b);
//              x = LN_2(h + (u @ Wo^T + b))
//   hidden = x (FP32); pooled = tanh(hidden[:, 0] @ Wp^T + b)
// as 2 + 7 L launches (+ 1 + L with a mask).  Linear weights are [out, in],
// which is already the K-major B operand of the tcgen05 GEMM.
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "bert.h"

namespace gpt2 {

namespace {
BertContext *g_bert = nullptr;

void free_bert_ws(BertWorkspace &w) {
  void *ptrs[] = {w.x, w.qkv, w.o, w.y, w.h, w.u, w.stats_h, w.stats_y, w.first_valid, w.kv_end, w.key_valid,
                  w.ids, w.tt, w.pos, w.mask, w.hidden, w.pooled};
  for (void *p : ptrs)
    if (p) cudaFree(p);
  w = BertWorkspace();
}
}  // namespace

std::vector<TensorSpec> bert_blob_specs(const BertDims &m) {
  std::vector<TensorSpec> s;
  int64_t off = 0;
  auto add = [&](int64_t n, TensorSpec::Kind k) {
    s.push_back({off, n, k});
    off += n;
  };
  const int64_t d = m.n_embd, ff = m.n_inner;
  add((int64_t)m.vocab * d, TensorSpec::kMatrix);
  add((int64_t)m.n_pos * d, TensorSpec::kMatrix);
  add((int64_t)m.type_vocab * d, TensorSpec::kMatrix);
  add(d, TensorSpec::kGain);
  add(d, TensorSpec::kBias);
  for (int l = 0; l < m.n_layer; ++l) {
    for (int j = 0; j < 4; ++j) {  // query, key, value, attention.output.dense
      add(d * d, TensorSpec::kMatrix);
      add(d, TensorSpec::kBias);
    }
    add(d, TensorSpec::kGain);
    add(d, TensorSpec::kBias);
    add(ff * d, TensorSpec::kMatrix);
    add(ff, TensorSpec::kBias);
    add(d * ff, TensorSpec::kMatrix);
    add(d, TensorSpec::kBias);
    add(d, TensorSpec::kGain);
    add(d, TensorSpec::kBias);
  }
  add(d * d, TensorSpec::kMatrix);
  add(d, TensorSpec::kBias);
  return s;
}

int64_t bert_blob_floats(const BertDims &m) {
  const auto s = bert_blob_specs(m);
  return s.back().offset + s.back().numel;
}

void bert_seeded_blob(const BertDims &m, uint64_t seed, int init_mode, float *blob) {
  const std::vector<TensorSpec> specs = bert_blob_specs(m);
  for (size_t t = 0; t < specs.size(); ++t) {
    const TensorSpec &s = specs[t];
    float *p = blob + s.offset;
    const uint32_t stream = 0x20000u + static_cast<uint32_t>(t);
    if (s.kind == TensorSpec::kMatrix) {
      seeded_normal(p, s.numel, seed, stream, 0.0, 0.02);
    } else if (init_mode == 0) {
      std::fill(p, p + s.numel, s.kind == TensorSpec::kGain ? 1.0f : 0.0f);
    } else {
      const bool gain = s.kind == TensorSpec::kGain;
      seeded_normal(p, s.numel, seed, stream, gain ? 1.0 : 0.0, gain ? 0.1 : 0.02);
    }
  }
}

BertContext *bert_context() { return g_bert; }

void bert_destroy_context() {
  if (!g_bert) return;
  BertContext *c = g_bert;
  g_bert = nullptr;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  drop_graph(c->graph);
  free_bert_ws(c->ws);
  if (c->d_blob) cudaFree(c->d_blob);
  for (auto &l : c->layers) {
    void *p[] = {l.qkv_w, l.qkv_b, l.qkv_h, l.ao_h, l.i_h, l.o_h, l.qkv_fold_h, l.i_fold_h, l.qkv_c1, l.qkv_c2,
                 l.i_c1, l.i_c2};
    for (void *q : p)
      if (q) cudaFree(q);
  }
  for (cudaEvent_t e : c->prof.pool) cudaEventDestroy(e);
  if (c->d_status) cudaFree(c->d_status);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  cudaSetDevice(prev);
}

int bert_create_context(const BertDims &m, int dtype, int device) {
  if (m.n_layer < 1 || m.n_embd < 64 || m.n_embd % 64 || m.n_head < 1 || m.n_embd % m.n_head ||
      m.n_embd / m.n_head != 64 || m.n_embd > 2048 || m.n_inner < 64 || m.n_inner % 64 || m.vocab < 1 ||
      m.n_pos < 1 || m.type_vocab < 1 || !(m.eps > 0.f)) {
    set_error("unsupported BERT configuration (need n_embd %% 64 == 0 and <= 2048, head dim 64, n_inner %% 64 == 0)");
    return -1;
  }
  if (dtype != 0 && dtype != 1) {
    set_error("unsupported BERT dtype %d (f32 or bf16)", dtype);
    return -1;
  }
  bert_destroy_context();
  if (device < 0) CK(cudaGetDevice(&device));
  CK(cudaSetDevice(device));
  BertContext *c = new BertContext();
  c->dims = m;
  c->dtype = dtype;
  c->device = device;
  cudaError_t e = cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, sizeof(int));
  if (e != cudaSuccess) {
    g_bert = c;
    bert_destroy_context();
    return cuda_fail(e, "BERT context setup");
  }
  c->specs = bert_blob_specs(m);
  if (const char *e = getenv("GPT2_GRAPHS")) c->use_graphs = strcmp(e, "0") != 0;
  g_bert = c;
  return 0;
}

int bert_load_blob(BertContext &c, const float *host_blob) {
  CK(cudaSetDevice(c.device));
  const BertDims &m = c.dims;
  const int64_t n = bert_blob_floats(m);
  if (!c.d_blob) CK(cudaMalloc(&c.d_blob, sizeof(float) * n));
  CK(cudaMemcpy(c.d_blob, host_blob, sizeof(float) * n, cudaMemcpyHostToDevice));
  const auto &s = c.specs;
  auto at = [&](size_t i) -> float * { return c.d_blob + s[i].offset; };
  c.word = at(0);
  c.pos = at(1);
  c.type = at(2);
  c.emb_g = at(3);
  c.emb_b = at(4);
  c.pool_w = at(5 + BERT_PER_LAYER * m.n_layer);
  c.pool_b = at(6 + BERT_PER_LAYER * m.n_layer);
  c.layers.resize(m.n_layer);
  const int d = m.n_embd, ff = m.n_inner;
  const size_t dd = (size_t)d * d;
  for (int l = 0; l < m.n_layer; ++l) {
    BertLayer &w = c.layers[l];
    const size_t b = 5 + BERT_PER_LAYER * l;
    // q, k and v stacked into one [3d, d] weight and [3d] bias: one GEMM
    // produces the [T, 3d] (q | k | v) rows the attention kernels read.
    if (!w.qkv_w) CK(cudaMalloc(&w.qkv_w, sizeof(float) * 3 * dd));
    if (!w.qkv_b) CK(cudaMalloc(&w.qkv_b, sizeof(float) * 3 * d));
    const size_t wi[3] = {b + BQ_W, b + BK_W, b + BV_W}, bi[3] = {b + BQ_B, b + BK_B, b + BV_B};
    for (int j = 0; j < 3; ++j) {
      CK(cudaMemcpyAsync(w.qkv_w + j * dd, at(wi[j]), sizeof(float) * dd, cudaMemcpyDeviceToDevice, c.stream));
      CK(cudaMemcpyAsync(w.qkv_b + j * d, at(bi[j]), sizeof(float) * d, cudaMemcpyDeviceToDevice, c.stream));
    }
    w.ao_w = at(b + BAO_W);
    w.ao_b = at(b + BAO_B);
    w.aoln_g = at(b + BAOLN_G);
    w.aoln_b = at(b + BAOLN_B);
    w.i_w = at(b + BI_W);
    w.i_b = at(b + BI_B);
    w.o_w = at(b + BO_W);
    w.o_b = at(b + BO_B);
    w.oln_g = at(b + BOLN_G);
    w.oln_b = at(b + BOLN_B);
    if (c.dtype == 1) {
      if (!w.qkv_h) CK(cudaMalloc(&w.qkv_h, sizeof(bf16) * 3 * dd));
      if (!w.ao_h) CK(cudaMalloc(&w.ao_h, sizeof(bf16) * dd));
      if (!w.i_h) CK(cudaMalloc(&w.i_h, sizeof(bf16) * (size_t)ff * d));
      if (!w.o_h) CK(cudaMalloc(&w.o_h, sizeof(bf16) * (size_t)d * ff));
      CK(launch_pack_bf16(w.qkv_w, w.qkv_h, 3 * d, d, 0, c.stream));
      CK(launch_pack_bf16(w.ao_w, w.ao_h, d, d, 0, c.stream));
      CK(launch_pack_bf16(w.i_w, w.i_h, ff, d, 0, c.stream));
      CK(launch_pack_bf16(w.o_w, w.o_h, d, ff, 0, c.stream));
      // Folded LayerNorms: the intermediate layer takes this layer's
      // attention-output LayerNorm; QKV (after the first layer) the previous
      // layer's output LayerNorm.
      if (!w.i_fold_h) CK(cudaMalloc(&w.i_fold_h, sizeof(bf16) * (size_t)ff * d));
      if (!w.i_c1) CK(cudaMalloc(&w.i_c1, sizeof(float) * ln_vector_len(ff)));
      if (!w.i_c2) CK(cudaMalloc(&w.i_c2, sizeof(float) * ln_vector_len(ff)));
      CK(launch_ln_fold_pack(w.i_w, 0, w.aoln_g, w.aoln_b, w.i_b, w.i_fold_h, w.i_c1, w.i_c2, ff, d, c.stream));
      if (l > 0) {
        const BertLayer &prev = c.layers[l - 1];
        if (!w.qkv_fold_h) CK(cudaMalloc(&w.qkv_fold_h, sizeof(bf16) * 3 * dd));
        if (!w.qkv_c1) CK(cudaMalloc(&w.qkv_c1, sizeof(float) * ln_vector_len(3 * d)));
        if (!w.qkv_c2) CK(cudaMalloc(&w.qkv_c2, sizeof(float) * ln_vector_len(3 * d)));
        CK(launch_ln_fold_pack(w.qkv_w, 0, prev.oln_g, prev.oln_b, w.qkv_b, w.qkv_fold_h, w.qkv_c1, w.qkv_c2, 3 * d,
                               d, c.stream));
      }
    }
  }
  CK(cudaStreamSynchronize(c.stream));
  c.loaded = true;
  c.plans_T = -1;
  drop_graph(c.graph);
  return 0;
}

int bert_ensure_workspace(BertContext &c, int B, int S) {
  const int64_t T = (int64_t)B * S;
  BertWorkspace &w = c.ws;
  if (T <= w.T && B <= w.B) return 0;
  const int64_t Tn = std::max(T, w.T);
  const int Bn = std::max(B, w.B);
  CK(cudaDeviceSynchronize());  // earlier forwards may still read the buffers
  drop_graph(c.graph);           // it captured the old buffers
  free_bert_ws(w);
  const size_t es = c.dtype == 1 ? 2 : 4;
  const int64_t d = c.dims.n_embd, ff = c.dims.n_inner;
  CK(cudaMalloc(&w.x, es * Tn * d));
  CK(cudaMalloc(&w.qkv, es * Tn * 3 * d));
  CK(cudaMalloc(&w.o, es * Tn * d));
  CK(cudaMalloc(&w.y, es * Tn * d));
  CK(cudaMalloc(&w.h, es * Tn * d));
  CK(cudaMalloc(&w.u, es * Tn * ff));
  CK(cudaMalloc(&w.stats_h, sizeof(float2) * Tn * ln_segments((int)d)));
  CK(cudaMalloc(&w.stats_y, sizeof(float2) * Tn * ln_segments((int)d)));
  CK(cudaMalloc(&w.first_valid, sizeof(int) * Bn));
  CK(cudaMalloc(&w.kv_end, sizeof(int) * Bn));
  CK(cudaMalloc(&w.key_valid, Tn));
  CK(cudaMalloc(&w.ids, sizeof(int64_t) * Tn));
  CK(cudaMalloc(&w.tt, sizeof(int64_t) * Tn));
  CK(cudaMalloc(&w.pos, sizeof(int64_t) * c.dims.n_pos));
  CK(cudaMalloc(&w.mask, sizeof(int64_t) * Tn));
  CK(cudaMalloc(&w.hidden, sizeof(float) * Tn * d));
  CK(cudaMalloc(&w.pooled, sizeof(float) * Bn * d));
  w.T = Tn;
  w.B = Bn;
  c.plans_T = -1;
  return 0;
}

namespace {
int bert_ensure_plans(BertContext &c, int64_t T) {
  if (c.plans_T == T) return 0;
  const BertDims &m = c.dims;
  const int d = m.n_embd, ff = m.n_inner;
  c.plans.resize(4 * m.n_layer);
  const BertWorkspace &ws = c.ws;
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
    const BertLayer &w = c.layers[l];
    TcGemmPlan *p = &c.plans[4 * l];
    // The residual stream stays un-normalised in memory (h after the
    // attention output, y after the layer; their LayerNorms are folded into
    // the GEMMs that read them): QKV reads the embedding output x in the
    // first layer and the previous layer's y after it.
    const bool first = l == 0;
    int r = tc_gemm_plan(&p[0], static_cast<const bf16 *>(first ? ws.x : ws.y), first ? w.qkv_h : w.qkv_fold_h,
                         (int)T, 3 * d, d, pick_tile(3 * d));
    if (!r) r = tc_gemm_plan(&p[1], static_cast<const bf16 *>(ws.o), w.ao_h, (int)T, d, d, pick_tile(d));
    if (!r) r = tc_gemm_plan(&p[2], static_cast<const bf16 *>(ws.h), w.i_fold_h, (int)T, ff, d, pick_tile(ff));
    if (!r) r = tc_gemm_plan(&p[3], static_cast<const bf16 *>(ws.u), w.o_h, (int)T, d, ff, pick_tile(d));
    if (r) {
      set_error("TMA descriptor creation failed (%d)", r);
      return -2;
    }
    tc_gemm_set_output(&p[0], ws.qkv, 3 * d, 0);
    tc_gemm_set_output(&p[1], ws.h, d, 0);
    tc_gemm_set_output(&p[2], ws.u, ff, 0);
    tc_gemm_set_output(&p[3], ws.y, d, 0);
  }
  c.plans_T = T;
  return 0;
}
}  // namespace

int bert_forward_launch_count(const BertContext &c, int has_mask, int has_pooler) {
  // embedding + per layer 7 (FP32: with two LayerNorm kernels) or 5 (BF16:
  // LayerNorms folded into the GEMMs) + the BF16 path's final LayerNorm
  // (+ pooler); with a mask, seq_info + 1 per layer
  const int L = c.dims.n_layer;
  const int body = c.dtype == 1 ? 5 * L + 1 : 7 * L;
  return 1 + body + (has_pooler ? 1 : 0) + (has_mask ? 1 + L : 0);
}

namespace {
int bert_prepare(BertContext &c, int B, int S);
int bert_launch(BertContext &c, const int64_t *d_ids, const int64_t *d_tt, const int64_t *d_pos,
                const int64_t *d_mask, int B, int S, float *d_hidden, float *d_pooled, cudaStream_t st);
}  // namespace

int bert_forward_device(BertContext &c, const int64_t *d_ids, const int64_t *d_tt, const int64_t *d_pos,
                        const int64_t *d_mask, int B, int S, float *d_hidden, float *d_pooled, cudaStream_t st) {
  const BertDims &m = c.dims;
  if (!c.loaded) {
    set_error("no BERT weights loaded");
    return -3;
  }
  if (B < 1 || S < 1 || S > m.n_pos || (int64_t)B * S > (int64_t)1 << 30 || !d_ids || !d_hidden ||
      (reinterpret_cast<uintptr_t>(d_hidden) & 15) || (reinterpret_cast<uintptr_t>(d_pooled) & 15)) {
    set_error("bad BERT forward: B=%d S=%d (n_positions %d), hidden / pooled must be 16-byte aligned", B, S,
              m.n_pos);
    return -1;
  }
  int r = bert_prepare(c, B, S);
  if (r) return r;
  auto launch = [&](cudaStream_t s) { return bert_launch(c, d_ids, d_tt, d_pos, d_mask, B, S, d_hidden, d_pooled, s); };
  if (c.prof.on) return launch(st);  // per-launch events need plain launches
  const uintptr_t key[8] = {reinterpret_cast<uintptr_t>(d_ids),    reinterpret_cast<uintptr_t>(d_tt),
                            reinterpret_cast<uintptr_t>(d_pos),    reinterpret_cast<uintptr_t>(d_mask),
                            reinterpret_cast<uintptr_t>(d_hidden), reinterpret_cast<uintptr_t>(d_pooled),
                            static_cast<uintptr_t>(B),             static_cast<uintptr_t>(S)};
  return run_with_graph(c.graph, &c.use_graphs, key, 8, c.stream, st, launch);
}

namespace {
// Buffers and descriptors of a forward of (B, S), before any launch (and
// outside any graph capture).
int bert_prepare(BertContext &c, int B, int S) {
  int r = bert_ensure_workspace(c, B, S);
  if (r || c.dtype == 0) return r;
  BertWorkspace &w = c.ws;
  r = bert_ensure_plans(c, (int64_t)B * S);
  if (r) return r;
  if (c.attn_plan.qkv != w.qkv || c.attn_plan.out != w.o || c.attn_plan.B != B || c.attn_plan.S != S ||
      c.attn_plan.H != c.dims.n_head) {
    if (attention_tc_plan(&c.attn_plan, static_cast<const bf16 *>(w.qkv), B, S, c.dims.n_head,
                          static_cast<const bf16 *>(w.o))) {
      set_error("TMA descriptor creation failed (attention)");
      return -2;
    }
  }
  return 0;
}

int bert_launch(BertContext &c, const int64_t *d_ids, const int64_t *d_tt, const int64_t *d_pos,
                const int64_t *d_mask, int B, int S, float *d_hidden, float *d_pooled, cudaStream_t st) {
  const BertDims &m = c.dims;
  const int64_t T = (int64_t)B * S;
  const int d = m.n_embd, ff = m.n_inner, H = m.n_head;
  BertWorkspace &w = c.ws;
  const uint8_t *kv = nullptr;
  const int *kv_end = nullptr;
  if (d_mask) {
    CKP(K_SEQ_INFO, launch_seq_info(d_mask, B, S, w.first_valid, w.key_valid, st, w.kv_end));
    kv = w.key_valid;
    kv_end = w.kv_end;
  }
  const int L = m.n_layer;
  if (c.dtype == 0) {
    float *x = static_cast<float *>(w.x), *qkv = static_cast<float *>(w.qkv), *o = static_cast<float *>(w.o),
          *y = static_cast<float *>(w.y), *h = static_cast<float *>(w.h), *u = static_cast<float *>(w.u);
    CKP(K_EMBED, launch_bert_embed_ln_f32(d_ids, d_tt, d_pos, c.word, c.pos, c.type, c.emb_g, c.emb_b, x, (int)T, S,
                                          d, m.vocab, m.n_pos, m.type_vocab, m.eps, c.d_status, st));
    for (int l = 0; l < L; ++l) {
      const BertLayer &lw = c.layers[l];
      CKP(K_GEMM_QKV, launch_gemm_f32(x, lw.qkv_w, 1, qkv, (int)T, 3 * d, d, 3 * d, lw.qkv_b, nullptr, EPI_BIAS, st));
      CKP(K_ATTENTION, launch_attention_f32(qkv, kv, o, B, S, H, st, 0));
      if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_f32(qkv, w.first_valid, o, B, S, H, st, 0));
      CKP(K_GEMM_PROJ, launch_gemm_f32(o, lw.ao_w, 1, y, (int)T, d, d, d, lw.ao_b, x, EPI_BIAS_RESID, st));
      CKP(K_LAYERNORM, launch_layernorm_f32(y, lw.aoln_g, lw.aoln_b, h, (int)T, d, m.eps, st));
      CKP(K_GEMM_FC, launch_gemm_f32(h, lw.i_w, 1, u, (int)T, ff, d, ff, lw.i_b, nullptr, EPI_BIAS_GELU_ERF, st));
      CKP(K_GEMM_MPROJ, launch_gemm_f32(u, lw.o_w, 1, y, (int)T, d, ff, d, lw.o_b, h, EPI_BIAS_RESID, st));
      CKP(K_LAYERNORM, launch_layernorm_f32(y, lw.oln_g, lw.oln_b, l == L - 1 ? d_hidden : x, (int)T, d, m.eps, st));
    }
  } else {
    bf16 *x = static_cast<bf16 *>(w.x), *qkv = static_cast<bf16 *>(w.qkv), *o = static_cast<bf16 *>(w.o),
         *y = static_cast<bf16 *>(w.y), *h = static_cast<bf16 *>(w.h), *u = static_cast<bf16 *>(w.u);
    const int ns = c.num_sms;
    CKP(K_EMBED, launch_bert_embed_ln_bf16(d_ids, d_tt, d_pos, c.word, c.pos, c.type, c.emb_g, c.emb_b, x, (int)T,
                                           S, d, m.vocab, m.n_pos, m.type_vocab, m.eps, c.d_status, st));
    // Post-LN with the LayerNorms folded: h = LN_out_prev(y) + o Wo + bo (x in
    // the first layer) and y = LN_att(h) + gelu(LN_att(h) Wi + bi) Wo2 + bo2
    // are stored un-normalised with their row statistics; every GEMM that
    // reads one applies its LayerNorm (as A: folded weights, EPI_LN_*; as the
    // residual: EPI_LNRES_*).  Only the last layer's output is normalised by
    // a kernel, into the FP32 hidden state.
    const int nseg = ln_segments(d);
    LnFold base;
    base.eps = m.eps;
    float2 *sh = w.stats_h, *sy = w.stats_y;
    for (int l = 0; l < L; ++l) {
      const BertLayer &lw = c.layers[l];
      const TcGemmPlan *p = &c.plans[4 * l];
      if (l == 0) {
        CKP(K_GEMM_QKV, launch_gemm_tc(p[0], qkv, 3 * d, 0, lw.qkv_b, nullptr, EPI_BIAS, c.d_status, ns, st));
      } else {
        LnFold f = base;
        f.c1 = lw.qkv_c1;
        f.c2 = lw.qkv_c2;
        f.stats_in = sy;
        f.nseg_in = nseg;
        f.k = d;
        CKP(K_GEMM_QKV, launch_gemm_tc(p[0], qkv, 3 * d, 0, nullptr, nullptr, EPI_LN_BIAS, c.d_status, ns, st,
                                       nullptr, &f));
      }
      CKP(K_ATTENTION, launch_attention_tc3(c.attn_plan, kv, o, c.d_status, st, 0, kv_end));
      if (d_mask) CKP(K_MASKED_ROWS, launch_attn_masked_rows_bf16(qkv, w.first_valid, o, B, S, H, st, 0));
      {
        LnFold f = base;
        f.stats_out = sh;
        f.nseg_out = nseg;
        if (l == 0) {
          CKP(K_GEMM_PROJ, launch_gemm_tc(p[1], h, d, 0, lw.ao_b, x, EPI_BIAS_RESID_STATS, c.d_status, ns, st,
                                          nullptr, &f));
        } else {
          const BertLayer &prev = c.layers[l - 1];
          f.res_stats = sy;
          f.res_gain = prev.oln_g;
          f.res_shift = prev.oln_b;
          CKP(K_GEMM_PROJ, launch_gemm_tc(p[1], h, d, 0, lw.ao_b, y, EPI_LNRES_BIAS_RESID_STATS, c.d_status, ns,
                                          st, nullptr, &f));
        }
      }
      {
        LnFold f = base;
        f.c1 = lw.i_c1;
        f.c2 = lw.i_c2;
        f.stats_in = sh;
        f.nseg_in = nseg;
        f.k = d;
        CKP(K_GEMM_FC, launch_gemm_tc(p[2], u, ff, 0, nullptr, nullptr, EPI_LN_BIAS_GELU_ERF, c.d_status, ns, st,
                                      nullptr, &f));
      }
      {
        LnFold f = base;
        f.stats_out = sy;
        f.nseg_out = nseg;
        f.res_stats = sh;
        f.res_gain = lw.aoln_g;
        f.res_shift = lw.aoln_b;
        CKP(K_GEMM_MPROJ, launch_gemm_tc(p[3], y, d, 0, lw.o_b, h, EPI_LNRES_BIAS_RESID_STATS, c.d_status, ns, st,
                                         nullptr, &f));
      }
    }
    const BertLayer &last = c.layers[L - 1];
    CKP(K_LAYERNORM, launch_layernorm_bf16_f32out(y, last.oln_g, last.oln_b, d_hidden, (int)T, d, m.eps, st));
  }
  if (d_pooled) CKP(K_LM_HEAD, launch_bert_pooler(d_hidden, c.pool_w, c.pool_b, d_pooled, B, S, d, st));
  return 0;
}
}  // namespace

}  // namespace gpt2
