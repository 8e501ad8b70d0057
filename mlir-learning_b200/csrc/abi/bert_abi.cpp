// bert_abi.cpp -- the BERT entry points of libgpt2_b200.so (include/bert_b200.h).
//
// _mlir_ciface_bert_model reproduces the function the reference's BERT host
// program links against (src/bert-base-uncased/call_bert.cpp:41-53): the
// model's position-id and token-type buffers, then input_ids, token_type_ids
// and attention_mask memrefs in; a result struct of two malloc'd FP32
// memrefs (last_hidden_state, pooler_output) out.  Nothing here aborts.
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "../../../include/bert_b200.h"
#include "../runtime/bert.h"

namespace gpt2 {
const char *last_error_text();
void clear_error();
}  // namespace gpt2

using namespace gpt2;

namespace {
std::mutex g_bert_mu;  // serialises every entry point that touches the BERT model

BertDims dims_of(const BertConfig *c) {
  BertDims m;
  m.n_layer = c->n_layer;
  m.n_embd = c->n_embd;
  m.n_head = c->n_head;
  m.n_inner = c->n_inner;
  m.vocab = c->vocab_size;
  m.n_pos = c->n_positions;
  m.type_vocab = c->type_vocab;
  m.eps = c->layer_norm_eps;
  return m;
}

bool valid_dims(const BertConfig *c) {
  return c && c->n_layer > 0 && c->n_embd > 0 && c->n_head > 0 && c->n_inner > 0 && c->vocab_size > 0 &&
         c->n_positions > 0 && c->type_vocab > 0;
}

int load_seeded_locked(uint64_t seed, int init_mode) {
  BertContext *c = bert_context();
  if (!c) {
    set_error("no BERT model: call bert_init first");
    return GPT2_ENOMODEL;
  }
  std::vector<float> blob(static_cast<size_t>(bert_blob_floats(c->dims)));
  bert_seeded_blob(c->dims, seed, init_mode, blob.data());
  return bert_load_blob(*c, blob.data());
}

// BERT-base (uncased) with seeded weights when no model exists; the
// reference's object carries bert-base-uncased's weights, this is the
// stand-in.
int ensure_default_model_locked() {
  BertContext *c = bert_context();
  if (c && c->loaded) return 0;
  if (!c) {
    int dtype = GPT2_DTYPE_F32;
    if (const char *e = getenv("BERT_DTYPE")) {
      if (!strcmp(e, "bf16")) dtype = GPT2_DTYPE_BF16;
      else if (strcmp(e, "f32") && strcmp(e, "fp32")) {
        set_error("BERT_DTYPE must be f32 or bf16, got '%s'", e);
        return GPT2_EINVAL;
      }
    }
    int r = bert_create_context(BertDims(), dtype, -1);
    if (r) return r;
  }
  uint64_t seed = 1234;
  if (const char *e = getenv("BERT_SEED")) seed = strtoull(e, nullptr, 10);
  return load_seeded_locked(seed, 0);
}

int read_status_locked(BertContext &c) {
  int h = 0;
  if (cudaMemcpy(&h, c.d_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (h) cudaMemset(c.d_status, 0, sizeof(int));
  return h;
}

int forward_host_locked(const int64_t *ids, const int64_t *tt, const int64_t *pos, const int64_t *mask, int B, int S,
                        float *hidden, float *pooled) {
  int r = ensure_default_model_locked();
  if (r) return r;
  BertContext &c = *bert_context();
  if (cudaSetDevice(c.device) != cudaSuccess) {
    set_error("cudaSetDevice(%d) failed", c.device);
    return GPT2_ECUDA;
  }
  const BertDims &m = c.dims;
  if (B < 1 || S < 1 || S > m.n_pos) {
    set_error("bad shape B=%d S=%d (max_position_embeddings %d)", B, S, m.n_pos);
    return GPT2_EINVAL;
  }
  const int64_t T = (int64_t)B * S;
  // Host-side range checks give a precise error; the embedding kernel also
  // checks and reports through the status word.
  for (int64_t i = 0; i < T; ++i) {
    if (ids[i] < 0 || ids[i] >= m.vocab) {
      set_error("token id %lld at position %lld outside [0, %d)", (long long)ids[i], (long long)i, m.vocab);
      return GPT2_EINVAL;
    }
    if (tt && (tt[i] < 0 || tt[i] >= m.type_vocab)) {
      set_error("token type %lld at position %lld outside [0, %d)", (long long)tt[i], (long long)i, m.type_vocab);
      return GPT2_EINVAL;
    }
  }
  for (int s = 0; pos && s < S; ++s)
    if (pos[s] < 0 || pos[s] >= m.n_pos) {
      set_error("position id %lld at %d outside [0, %d)", (long long)pos[s], s, m.n_pos);
      return GPT2_EINVAL;
    }
  r = bert_ensure_workspace(c, B, S);
  if (r) return r;
  BertWorkspace &w = c.ws;
  cudaStream_t st = c.stream;
  cudaError_t e = cudaMemcpyAsync(w.ids, ids, sizeof(int64_t) * T, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && tt) e = cudaMemcpyAsync(w.tt, tt, sizeof(int64_t) * T, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && pos) e = cudaMemcpyAsync(w.pos, pos, sizeof(int64_t) * S, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && mask) e = cudaMemcpyAsync(w.mask, mask, sizeof(int64_t) * T, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    set_error("host-to-device copy of the inputs failed: %s", cudaGetErrorString(e));
    return GPT2_ECUDA;
  }
  r = bert_forward_device(c, w.ids, tt ? w.tt : nullptr, pos ? w.pos : nullptr, mask ? w.mask : nullptr, B, S,
                          w.hidden, pooled ? w.pooled : nullptr, st);
  if (r) return r;
  const int64_t d = m.n_embd;
  e = cudaMemcpyAsync(hidden, w.hidden, sizeof(float) * T * d, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && pooled) e = cudaMemcpyAsync(pooled, w.pooled, sizeof(float) * B * d, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error("BERT forward failed: %s", cudaGetErrorString(e));
    return GPT2_ECUDA;
  }
  const int s = read_status_locked(c);
  if (s) {
    set_error("device status %d after the BERT forward", s);
    return GPT2_EDEVICE;
  }
  return 0;
}

// Gathers a strided memref<?x?xi64> into a contiguous [s0, s1] vector.
void gather_i64(const MemRef2D_i64 *m, std::vector<int64_t> &out) {
  out.resize(static_cast<size_t>(m->sizes[0] * m->sizes[1]));
  for (int64_t i = 0; i < m->sizes[0]; ++i)
    for (int64_t j = 0; j < m->sizes[1]; ++j)
      out[i * m->sizes[1] + j] = m->aligned[m->offset + i * m->strides[0] + j * m->strides[1]];
}

bool memref_ok(const MemRef2D_i64 *m) {
  return m && m->aligned && m->sizes[0] >= 1 && m->sizes[1] >= 1 && m->sizes[0] <= (1 << 20) &&
         m->sizes[1] <= (1 << 20);
}

void model_impl(BertOutput *result, const MemRef2D_i64 *pos_buf, const MemRef2D_i64 *tt_buf,
                const MemRef2D_i64 *input_ids, const MemRef2D_i64 *token_type_ids,
                const MemRef2D_i64 *attention_mask) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  if (!memref_ok(input_ids)) {
    set_error("_mlir_ciface_bert_model: bad input_ids memref");
    return;
  }
  const int64_t B = input_ids->sizes[0], S = input_ids->sizes[1];
  auto same_shape = [&](const MemRef2D_i64 *m) { return m->sizes[0] == B && m->sizes[1] == S; };
  std::vector<int64_t> ids, tt, pos, mask, tt_row;
  gather_i64(input_ids, ids);
  if (token_type_ids) {
    if (!memref_ok(token_type_ids) || !same_shape(token_type_ids)) {
      set_error("_mlir_ciface_bert_model: token_type_ids must have the shape of input_ids");
      return;
    }
    gather_i64(token_type_ids, tt);
  } else if (tt_buf) {
    // transformers' rule without token_type_ids: the registered buffer's
    // first S entries, the same for every sequence.
    if (!memref_ok(tt_buf) || tt_buf->sizes[1] < S) {
      set_error("_mlir_ciface_bert_model: token type buffer shorter than the sequence");
      return;
    }
    gather_i64(tt_buf, tt_row);
    tt.resize(static_cast<size_t>(B * S));
    for (int64_t b = 0; b < B; ++b)
      for (int64_t s = 0; s < S; ++s) tt[b * S + s] = tt_row[s];
  }
  if (pos_buf) {
    if (!memref_ok(pos_buf) || pos_buf->sizes[1] < S) {
      set_error("_mlir_ciface_bert_model: position buffer shorter than the sequence");
      return;
    }
    std::vector<int64_t> row;
    gather_i64(pos_buf, row);
    pos.assign(row.begin(), row.begin() + S);
  }
  bool has_mask = false;
  if (attention_mask) {
    if (!memref_ok(attention_mask) || !same_shape(attention_mask)) {
      set_error("_mlir_ciface_bert_model: attention_mask must have the shape of input_ids");
      return;
    }
    gather_i64(attention_mask, mask);
    for (int64_t v : mask)
      if (v == 0) {
        has_mask = true;
        break;
      }
  }
  if (ensure_default_model_locked()) return;
  const int64_t d = bert_context()->dims.n_embd;
  float *hidden = static_cast<float *>(malloc(sizeof(float) * B * S * d));
  float *pooled = static_cast<float *>(malloc(sizeof(float) * B * d));
  if (!hidden || !pooled) {
    free(hidden);
    free(pooled);
    set_error("_mlir_ciface_bert_model: malloc of the outputs failed");
    return;
  }
  // An all-ones mask is the unmasked computation; skip its kernels.
  const int r = forward_host_locked(ids.data(), tt.empty() ? nullptr : tt.data(), pos.empty() ? nullptr : pos.data(),
                                    has_mask ? mask.data() : nullptr, (int)B, (int)S, hidden, pooled);
  if (r) {
    free(hidden);
    free(pooled);
    return;
  }
  MemRef3D &h = result->last_hidden_state;
  h.allocated = h.aligned = hidden;
  h.offset = 0;
  h.sizes[0] = B;
  h.sizes[1] = S;
  h.sizes[2] = d;
  h.strides[0] = S * d;
  h.strides[1] = d;
  h.strides[2] = 1;
  MemRef2D_f32 &p = result->pooler_output;
  p.allocated = p.aligned = pooled;
  p.offset = 0;
  p.sizes[0] = B;
  p.sizes[1] = d;
  p.strides[0] = d;
  p.strides[1] = 1;
}
}  // namespace

extern "C" {

void _mlir_ciface_bert_model(BertOutput *result, MemRef2D_i64 *buffer_embeddings_position_ids,
                             MemRef2D_i64 *buffer_embeddings_token_type_ids, MemRef2D_i64 *input_ids,
                             MemRef2D_i64 *token_type_ids, MemRef2D_i64 *attention_mask) {
  if (!result) return;
  memset(result, 0, sizeof *result);
  model_impl(result, buffer_embeddings_position_ids, buffer_embeddings_token_type_ids, input_ids, token_type_ids,
             attention_mask);
}

int bert_init(const BertConfig *cfg, int device) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  if (!valid_dims(cfg)) {
    set_error("bert_init: invalid configuration");
    return GPT2_EINVAL;
  }
  return bert_create_context(dims_of(cfg), cfg->dtype, device);
}

int64_t bert_blob_floats(const BertConfig *cfg) {
  if (!valid_dims(cfg)) return GPT2_EINVAL;
  return bert_blob_floats(dims_of(cfg));
}

int bert_load_weights(const void *packed, size_t bytes, const char *manifest_json) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  BertContext *c = bert_context();
  if (!c) {
    set_error("bert_load_weights: no model, call bert_init first");
    return GPT2_ENOMODEL;
  }
  const size_t want = sizeof(float) * static_cast<size_t>(bert_blob_floats(c->dims));
  if (!packed || bytes != want) {
    set_error("bert_load_weights: expected %zu bytes of canonical FP32 blob, got %zu", want, bytes);
    return GPT2_EINVAL;
  }
  if (manifest_json && !strstr(manifest_json, "bert-canonical-f32-v1")) {
    set_error("bert_load_weights: manifest layout must be \"bert-canonical-f32-v1\"");
    return GPT2_EINVAL;
  }
  return bert_load_blob(*c, static_cast<const float *>(packed));
}

int bert_safetensors_to_blob(const char *path, const BertConfig *cfg, float *out) {
  clear_error();
  if (!path || !valid_dims(cfg) || !out) {
    set_error("bert_safetensors_to_blob: need a path, a valid configuration and an output buffer");
    return GPT2_EINVAL;
  }
  return bert_safetensors_blob(path, dims_of(cfg), out) ? GPT2_EINVAL : 0;
}

int bert_load_safetensors(const char *path) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  BertContext *c = bert_context();
  if (!c) {
    set_error("bert_load_safetensors: no model, call bert_init first");
    return GPT2_ENOMODEL;
  }
  if (!path) return GPT2_EINVAL;
  std::vector<float> blob(static_cast<size_t>(bert_blob_floats(c->dims)));
  if (bert_safetensors_blob(path, c->dims, blob.data())) return GPT2_EINVAL;
  return bert_load_blob(*c, blob.data());
}

int bert_init_seeded(uint64_t seed, int init_mode) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  if (init_mode != 0 && init_mode != 1) {
    set_error("bert_init_seeded: init_mode must be 0 or 1");
    return GPT2_EINVAL;
  }
  return load_seeded_locked(seed, init_mode);
}

int bert_seeded_blob(const BertConfig *cfg, uint64_t seed, int init_mode, float *out) {
  if (!valid_dims(cfg) || !out || (init_mode != 0 && init_mode != 1)) return GPT2_EINVAL;
  bert_seeded_blob(dims_of(cfg), seed, init_mode, out);
  return 0;
}

int bert_get_config(BertConfig *out) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  BertContext *c = bert_context();
  if (!c) {
    set_error("bert_get_config: no model");
    return GPT2_ENOMODEL;
  }
  if (!out) return GPT2_EINVAL;
  out->n_layer = c->dims.n_layer;
  out->n_embd = c->dims.n_embd;
  out->n_head = c->dims.n_head;
  out->n_inner = c->dims.n_inner;
  out->vocab_size = c->dims.vocab;
  out->n_positions = c->dims.n_pos;
  out->layer_norm_eps = c->dims.eps;
  out->type_vocab = c->dims.type_vocab;
  out->dtype = c->dtype;
  return 0;
}

void bert_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  bert_destroy_context();
}

const char *bert_last_error(void) { return last_error_text(); }

int bert_status(void) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  BertContext *c = bert_context();
  if (!c) return GPT2_ENOMODEL;
  cudaSetDevice(c->device);
  return read_status_locked(*c);
}

int bert_forward_device(const int64_t *d_ids, const int64_t *d_tt, const int64_t *d_pos, const int64_t *d_mask,
                        int B, int S, float *d_hidden, float *d_pooled, void *stream) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  BertContext *c = bert_context();
  if (!c || !c->loaded) {
    set_error("bert_forward_device: no model loaded");
    return GPT2_ENOMODEL;
  }
  cudaSetDevice(c->device);
  return bert_forward_device(*c, d_ids, d_tt, d_pos, d_mask, B, S, d_hidden, d_pooled,
                             static_cast<cudaStream_t>(stream));
}

int bert_forward_host(const int64_t *ids, const int64_t *tt, const int64_t *pos, const int64_t *mask, int B, int S,
                      float *hidden, float *pooled) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  clear_error();
  if (!ids || !hidden) {
    set_error("bert_forward_host: null ids or hidden");
    return GPT2_EINVAL;
  }
  return forward_host_locked(ids, tt, pos, mask, B, S, hidden, pooled);
}

int bert_forward_launches(int has_mask, int has_pooler) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  BertContext *c = bert_context();
  if (!c) return GPT2_ENOMODEL;
  return bert_forward_launch_count(*c, has_mask, has_pooler);
}

int bert_profile_begin(void) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  BertContext *c = bert_context();
  if (!c) return GPT2_ENOMODEL;
  return profile_begin(c->prof);
}

int bert_profile_end(double *ms_per_kind, int64_t *launches_per_kind, int n_kinds) {
  std::lock_guard<std::mutex> lk(g_bert_mu);
  BertContext *c = bert_context();
  if (!c) return GPT2_ENOMODEL;
  if (!ms_per_kind || !launches_per_kind || n_kinds < 0) return GPT2_EINVAL;
  cudaSetDevice(c->device);
  return profile_end(c->prof, ms_per_kind, launches_per_kind, n_kinds < K_NUM_KINDS ? n_kinds : K_NUM_KINDS);
}

}  // extern "C"
