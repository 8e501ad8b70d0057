// decode.cu -- incremental decoding of the GPT-2 model with a key / value
// cache: prefill (the forward over the prompt that also fills the cache and
// returns the last position's logits), one-token decode steps, and greedy
// generation.
//
// The reference generates by re-running the whole exported forward on the
// grown sequence and taking logits[:, -1] (src/gpt/lower_gpt_model.py:190-198;
// the loop pattern of src/flan-t5-small/flan_call.cpp:64-180; HF generate's
// greedy search in src/gpt/run_gpt.py:20-24).  Each decode step here costs
// one token: per layer LayerNorm, the QKV / out-proj / fc / proj products on
// B <= 16 rows (GEMV kernels streaming each weight once), and attention of
// the new query against the cache.  Masks are all ones (every sequence has
// the same length), as in the reference's generation calls.
#include <string.h>

#include <algorithm>

#include "runtime.h"

namespace gpt2 {

void free_decode(DecodeState &d) {
  for (void *p : d.cache)
    if (p) cudaFree(p);
  void *ptrs[] = {d.x, d.a, d.qkv, d.o, d.u, d.a_last, d.logits, d.tokens, d.cur, d.d_pos};
  for (void *p : ptrs)
    if (p) cudaFree(p);
  for (float *p : d.wt)
    if (p) cudaFree(p);
  d = DecodeState();
}

int kv_reserve(Context &c, int B, int max_len) {
  const ModelDims &m = c.dims;
  if (!c.loaded) {
    set_error("no weights loaded");
    return -3;
  }
  if (B < 1 || B > 16 || max_len < 1 || max_len > m.n_pos) {
    set_error("KV cache for B=%d (1..16) sequences of max_len=%d (1..%d) tokens", B, max_len, m.n_pos);
    return -1;
  }
  CK(cudaSetDevice(c.device));
  DecodeState &d = c.dec;
  const int64_t D = m.n_embd, ff = m.n_inner;
  const size_t es = c.dtype >= 1 ? 2 : 4;
  if (d.B != B || d.max_len != max_len || d.cache.empty()) {
    CK(cudaDeviceSynchronize());
    drop_graph(c.dec_graph);  // it captured the old buffers
    std::vector<float *> keep_wt;
    keep_wt.swap(d.wt);
    free_decode(d);
    d.wt.swap(keep_wt);
    d.cache.assign(m.n_layer, nullptr);
    for (int l = 0; l < m.n_layer; ++l) CK(cudaMalloc(&d.cache[l], es * B * (size_t)max_len * 2 * D));
    CK(cudaMalloc(&d.x, es * B * D));
    CK(cudaMalloc(&d.a, es * B * D));
    CK(cudaMalloc(&d.qkv, es * B * 3 * D));
    CK(cudaMalloc(&d.o, es * B * D));
    CK(cudaMalloc(&d.u, es * B * ff));
    CK(cudaMalloc(&d.a_last, es * B * D));
    d.ld_logits = (m.vocab + 3) / 4 * 4;
    CK(cudaMalloc(&d.logits, sizeof(float) * B * d.ld_logits));
    CK(cudaMalloc(&d.cur, sizeof(int64_t) * B));
    CK(cudaMalloc(&d.d_pos, sizeof(int)));
    d.B = B;
    d.max_len = max_len;
  }
  d.len = 0;
  CK(launch_set_int(d.d_pos, 0, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  return ensure_nk_f32(c);
}

int ensure_nk_f32(Context &c) {
  DecodeState &d = c.dec;
  if (c.dtype != 0 || !d.wt.empty()) return 0;
  // The GEMV kernels read weights as [out, in]; the FP32 blob holds the
  // Conv1D weights as [in, out].
  const ModelDims &m = c.dims;
  const int D = m.n_embd, ff = m.n_inner;
  d.wt.assign(4 * m.n_layer, nullptr);
  for (int l = 0; l < m.n_layer; ++l) {
    const LayerWeights &w = c.layers[l];
    const float *src[4] = {w.qkv_w, w.proj_w, w.fc_w, w.mproj_w};
    const int rows[4] = {D, D, D, ff}, cols[4] = {3 * D, D, ff, D};
    for (int j = 0; j < 4; ++j) {
      CK(cudaMalloc(&d.wt[4 * l + j], sizeof(float) * rows[j] * cols[j]));
      CK(launch_transpose_f32(src[j], d.wt[4 * l + j], rows[j], cols[j], c.stream));
    }
  }
  CK(cudaStreamSynchronize(c.stream));
  return 0;
}

int prefill(Context &c, const int64_t *d_ids, int B, int S, float *d_logits, int64_t ld, cudaStream_t st) {
  DecodeState &d = c.dec;
  if (d.cache.empty() || B != d.B || S < 1 || S > d.max_len || ld < c.dims.vocab) {
    set_error("prefill of B=%d x S=%d needs a KV cache reserved for B=%d and >= S positions (have %d), ld >= V",
              B, S, d.B, d.max_len);
    return -1;
  }
  int r = prepare_forward(c, B, S, nullptr, 0);
  if (r) return r;
  r = launch_forward(c, d_ids, nullptr, B, S, d_logits, ld, st, true);
  if (r) return r;
  CK(launch_set_int(d.d_pos, S, st));
  d.len = S;
  return 0;
}

namespace {
// The kernels of one decode step at position *d.d_pos, then the position
// advance; everything reads its position from the device.
int launch_step(Context &c, const int64_t *d_tokens, int B, float *d_logits, int64_t ld, cudaStream_t st) {
  const ModelDims &m = c.dims;
  DecodeState &d = c.dec;
  const int D = m.n_embd, ff = m.n_inner, H = m.n_head, V = m.vocab;
  const int *dp = d.d_pos;
  // Each GEMV and attention launch follows a kernel: a programmatic
  // dependent of it (not in a profiled step, whose events bracket each kernel).
  const bool pdl = !c.prof.on;

  if (c.dtype == 0) {
    float *x = static_cast<float *>(d.x), *qkv = static_cast<float *>(d.qkv),
          *o = static_cast<float *>(d.o), *u = static_cast<float *>(d.u);
    CKP(K_EMBED, launch_decode_embed_f32(d_tokens, c.wte, c.wpe, x, B, D, V, dp, m.n_pos, c.d_status, st));
    // ln_1, ln_2 and ln_f run inside the GEMVs that read them (GemvLn).
    for (int l = 0; l < m.n_layer; ++l) {
      const LayerWeights &lw = c.layers[l];
      float *const *wt = &d.wt[4 * l];
      const GemvLn ln1{lw.ln1_g, lw.ln1_b, m.eps}, ln2{lw.ln2_g, lw.ln2_b, m.eps};
      CKP(K_GEMM_QKV, launch_gemv_f32(x, wt[0], qkv, B, 3 * D, D, 3 * D, lw.qkv_b, nullptr, EPI_BIAS, st, &ln1, pdl));
      CKP(K_ATTENTION,
          launch_attn_decode_f32(qkv, static_cast<float *>(d.cache[l]), o, B, H, dp, d.max_len, c.d_status, st, pdl));
      CKP(K_GEMM_PROJ, launch_gemv_f32(o, wt[1], x, B, D, D, D, lw.proj_b, x, EPI_BIAS_RESID, st, nullptr, pdl));
      CKP(K_GEMM_FC, launch_gemv_f32(x, wt[2], u, B, ff, D, ff, lw.fc_b, nullptr, EPI_BIAS_GELU, st, &ln2, pdl));
      CKP(K_GEMM_MPROJ, launch_gemv_f32(u, wt[3], x, B, D, ff, D, lw.mproj_b, x, EPI_BIAS_RESID, st, nullptr, pdl));
    }
    const GemvLn lnf{c.lnf_g, c.lnf_b, m.eps};
    CKP(K_LM_HEAD, launch_gemv_f32(x, c.wte, d_logits, B, V, D, (int)ld, nullptr, nullptr, EPI_NONE, st, &lnf, pdl));
  } else {
    bf16 *x = static_cast<bf16 *>(d.x), *qkv = static_cast<bf16 *>(d.qkv),
         *o = static_cast<bf16 *>(d.o), *u = static_cast<bf16 *>(d.u);
    CKP(K_EMBED, launch_decode_embed_bf16(d_tokens, c.wte_h, c.wpe_h, x, B, D, V, dp, m.n_pos, c.d_status, st));
    for (int l = 0; l < m.n_layer; ++l) {
      const LayerWeights &lw = c.layers[l];
      const GemvLn ln1{lw.ln1_g, lw.ln1_b, m.eps}, ln2{lw.ln2_g, lw.ln2_b, m.eps};
      CKP(K_GEMM_QKV, launch_gemv_bf16_auto(x, lw.qkv_wt, qkv, B, 3 * D, D, 3 * D, lw.qkv_b, nullptr, lw.qkv_s, EPI_BIAS, c.d_status,
                                       st, &ln1, pdl));
      CKP(K_ATTENTION, launch_attn_decode_bf16(qkv, static_cast<bf16 *>(d.cache[l]), o, B, H, dp, d.max_len, c.d_status, st, pdl));
      CKP(K_GEMM_PROJ, launch_gemv_bf16_auto(o, lw.proj_wt, x, B, D, D, D, lw.proj_b, x, lw.proj_s, EPI_BIAS_RESID, c.d_status, st, nullptr, pdl));
      CKP(K_GEMM_FC, launch_gemv_bf16_auto(x, lw.fc_wt, u, B, ff, D, ff, lw.fc_b, nullptr, lw.fc_s, EPI_BIAS_GELU, c.d_status, st,
                                      &ln2, pdl));
      CKP(K_GEMM_MPROJ,
          launch_gemv_bf16_auto(u, lw.mproj_wt, x, B, D, ff, D, lw.mproj_b, x, lw.mproj_s, EPI_BIAS_RESID, c.d_status, st, nullptr, pdl));
    }
    const GemvLn lnf{c.lnf_g, c.lnf_b, m.eps};
    CKP(K_LM_HEAD, launch_gemv_bf16_f32out_auto(x, c.wte_h, d_logits, B, V, D, (int)ld, c.d_status, st, &lnf, pdl));
  }
  CK(launch_add_int(d.d_pos, 1, st));
  return 0;
}
}  // namespace

int decode_step(Context &c, const int64_t *d_tokens, int B, float *d_logits, int64_t ld, cudaStream_t st) {
  const ModelDims &m = c.dims;
  DecodeState &d = c.dec;
  if (d.cache.empty() || B != d.B || d.len < 1 || d.len >= d.max_len || ld < m.vocab) {
    set_error("decode step: cache for B=%d holds %d of %d positions (prefill first; B must match; ld >= V)", d.B,
              d.len, d.max_len);
    return -1;
  }
  auto launch = [&](cudaStream_t s) { return launch_step(c, d_tokens, B, d_logits, ld, s); };
  int r;
  if (c.prof.on) {
    r = launch(st);
  } else {
    const uintptr_t key[5] = {1, reinterpret_cast<uintptr_t>(d_tokens), static_cast<uintptr_t>(B),
                              reinterpret_cast<uintptr_t>(d_logits), static_cast<uintptr_t>(ld)};
    r = run_with_graph(c.dec_graph, &c.use_graphs, key, 5, c.stream, st, launch);
  }
  if (r) return r;
  d.len += 1;
  return 0;
}

int generate(Context &c, const int64_t *ids, int B, int S, int n_new, int64_t *out_tokens) {
  const ModelDims &m = c.dims;
  if (B < 1 || S < 1 || n_new < 1 || S + n_new - 1 > m.n_pos) {
    set_error("generate: B=%d S=%d n_new=%d exceeds n_positions %d", B, S, n_new, m.n_pos);
    return -1;
  }
  for (int64_t i = 0; i < (int64_t)B * S; ++i)
    if (ids[i] < 0 || ids[i] >= m.vocab) {
      set_error("token id %lld at position %lld outside [0, %d)", (long long)ids[i], (long long)i, m.vocab);
      return -1;
    }
  // The last generated token is never fed back, so the cache needs S + n_new - 1 positions.
  int r = kv_reserve(c, B, std::max(S + n_new - 1, 1));
  if (r) return r;
  r = ensure_workspace(c, B, S);
  if (r) return r;
  DecodeState &d = c.dec;
  if (d.tokens_cap < (int64_t)n_new * B) {
    if (d.tokens) cudaFree(d.tokens);
    d.tokens = nullptr;
    d.tokens_cap = 0;
    CK(cudaMalloc(&d.tokens, sizeof(int64_t) * n_new * B));
    d.tokens_cap = (int64_t)n_new * B;
  }
  cudaStream_t st = c.stream;
  CK(cudaMemcpyAsync(c.ws.ids, ids, sizeof(int64_t) * B * S, cudaMemcpyHostToDevice, st));
  r = prefill(c, c.ws.ids, B, S, d.logits, d.ld_logits, st);
  if (r) return r;
  CK(launch_argmax_rows(d.logits, d.ld_logits, B, m.vocab, d.cur, st));
  CK(launch_append_tokens(d.cur, d.tokens, d.d_pos, S, B, (int)d.tokens_cap, st));  // token 0 at *d_pos == S
  // One greedy step: decode the latest tokens, argmax, record them at index
  // (position - S + 1), advance; captured once and replayed per token.
  auto greedy = [&](cudaStream_t s) -> int {
    int rr = launch_step(c, d.cur, B, d.logits, d.ld_logits, s);
    if (rr) return rr;
    CK(launch_argmax_rows(d.logits, d.ld_logits, B, m.vocab, d.cur, s));
    CK(launch_append_tokens(d.cur, d.tokens, d.d_pos, S, B, (int)d.tokens_cap, s));
    return 0;
  };
  const uintptr_t key[4] = {2, static_cast<uintptr_t>(B), static_cast<uintptr_t>(S),
                            reinterpret_cast<uintptr_t>(d.tokens)};
  for (int i = 1; i < n_new; ++i) {
    r = run_with_graph(c.dec_graph, &c.use_graphs, key, 4, c.stream, st, greedy);
    if (r) return r;
    d.len += 1;
  }
  std::vector<int64_t> t((size_t)n_new * B);
  CK(cudaMemcpyAsync(t.data(), d.tokens, sizeof(int64_t) * n_new * B, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < n_new; ++i) out_tokens[(int64_t)b * n_new + i] = t[(size_t)i * B + b];
  return 0;
}

}  // namespace gpt2
