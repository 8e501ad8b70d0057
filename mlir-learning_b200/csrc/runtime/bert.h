// bert.h -- host runtime of the BERT encoder in libgpt2_b200.so: model
// dimensions, canonical blob, the process-wide BERT context and its forward
// schedule.  Shares kernels, profiler and error reporting with the GPT-2
// runtime (runtime.h).
#pragma once

#include "runtime.h"

namespace gpt2 {

struct BertDims {
  int n_layer = 12, n_embd = 768, n_head = 12, n_inner = 3072, vocab = 30522, n_pos = 512, type_vocab = 2;
  float eps = 1e-12f;
};

// Per-layer tensor order inside the blob (transformers' state_dict order).
enum BertTensor {
  BQ_W, BQ_B, BK_W, BK_B, BV_W, BV_B, BAO_W, BAO_B, BAOLN_G, BAOLN_B, BI_W, BI_B, BO_W, BO_B, BOLN_G, BOLN_B,
  BERT_PER_LAYER
};

std::vector<TensorSpec> bert_blob_specs(const BertDims &m);
int64_t bert_blob_floats(const BertDims &m);
void bert_seeded_blob(const BertDims &m, uint64_t seed, int init_mode, float *blob);

struct BertLayer {
  float *qkv_w = nullptr, *qkv_b = nullptr;  // FP32 [3d, d] and [3d]: q, k, v stacked (owned)
  const float *ao_w, *ao_b, *aoln_g, *aoln_b, *i_w, *i_b, *o_w, *o_b, *oln_g, *oln_b;  // in the blob, [out, in]
  bf16 *qkv_h = nullptr, *ao_h = nullptr, *i_h = nullptr, *o_h = nullptr;             // BF16 [out, in]
  // BF16 forward with the LayerNorms folded: QKV with the previous layer's
  // output LayerNorm (layers after the first) and the intermediate layer with
  // this layer's attention-output LayerNorm, as gain-scaled weights and their
  // c1 / c2 vectors (see LnFold).
  bf16 *qkv_fold_h = nullptr, *i_fold_h = nullptr;
  float *qkv_c1 = nullptr, *qkv_c2 = nullptr, *i_c1 = nullptr, *i_c2 = nullptr;
};

struct BertWorkspace {
  int64_t T = 0;
  int B = 0;
  void *x = nullptr, *qkv = nullptr, *o = nullptr, *y = nullptr, *h = nullptr, *u = nullptr;
  float2 *stats_h = nullptr, *stats_y = nullptr;  // row statistics of h and y (BF16 forward, folded LayerNorms)
  int *first_valid = nullptr, *kv_end = nullptr;
  uint8_t *key_valid = nullptr;
  int64_t *ids = nullptr, *tt = nullptr, *pos = nullptr, *mask = nullptr;  // staging of the host entry points
  float *hidden = nullptr, *pooled = nullptr;                              // outputs of the host entry points
};

struct BertContext {
  BertDims dims;
  int dtype = 0;
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  int *d_status = nullptr;
  bool loaded = false;

  float *d_blob = nullptr;
  std::vector<TensorSpec> specs;
  const float *word = nullptr, *pos = nullptr, *type = nullptr, *emb_g = nullptr, *emb_b = nullptr;
  const float *pool_w = nullptr, *pool_b = nullptr;
  std::vector<BertLayer> layers;

  BertWorkspace ws;
  std::vector<TcGemmPlan> plans;  // per layer: qkv, attention output, intermediate, output
  int64_t plans_T = -1;
  AttnTcPlan attn_plan;

  Profiler prof;
  GraphCache graph;
  bool use_graphs = true;  // env GPT2_GRAPHS=0 turns graph replay off
};

BertContext *bert_context();
int bert_create_context(const BertDims &dims, int dtype, int device);
void bert_destroy_context();
int bert_load_blob(BertContext &c, const float *host_blob);
int bert_ensure_workspace(BertContext &c, int B, int S);
int bert_forward_device(BertContext &c, const int64_t *d_ids, const int64_t *d_tt, const int64_t *d_pos,
                        const int64_t *d_mask, int B, int S, float *d_hidden, float *d_pooled, cudaStream_t st);
int bert_forward_launch_count(const BertContext &c, int has_mask, int has_pooler);
int bert_safetensors_blob(const char *path, const BertDims &m, float *blob);

}  // namespace gpt2
