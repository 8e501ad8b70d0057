/*
 * bert_b200.h -- the BERT encoder entry points of libgpt2_b200.so: a B200
 * (sm_100a) implementation of the bert_model function that the reference
 * exports from transformers' BertModel (src/bert-base-uncased/
 * lower_bert_model.py:7-49) and calls from its host program
 * (src/bert-base-uncased/call_bert.cpp:41-53), built from the same kernels
 * as the GPT-2 forward (tcgen05 GEMMs and attention, fused LayerNorm).
 *
 * Error conventions are those of gpt2_b200.h: 0 or a negative GPT2_E* code,
 * bert_last_error() describing the failure; the ciface entry point zeroes
 * *result on failure.
 */
#ifndef BERT_B200_H
#define BERT_B200_H

#include "gpt2_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* memref<?x?xf32>: the pooler output. */
typedef struct MemRef2D_f32 {
  float *allocated;
  float *aligned;
  int64_t offset;
  int64_t sizes[2];
  int64_t strides[2];
} MemRef2D_f32;

/* The result struct of the exported function (call_bert.cpp:41-44):
 * last_hidden_state [B, S, d] and pooler_output [B, d], FP32. */
typedef struct BertOutput {
  MemRef3D last_hidden_state;
  MemRef2D_f32 pooler_output;
} BertOutput;

/* Replaces the compiled `_mlir_ciface_bert_model` declared at
 * src/bert-base-uncased/call_bert.cpp:46-53.  Operands are the model's two
 * registered buffers (embeddings.position_ids and
 * embeddings.token_type_ids, memref<1x512xi64>, call_bert.cpp:73-77), then
 * input_ids, token_type_ids and attention_mask (memref<?x?xi64>, any
 * strides).  Position s of every sequence uses
 * position_ids[0, s]; token_type_ids may be NULL, in which case the token
 * type buffer's first S entries apply to every sequence (transformers'
 * rule); attention_mask may be NULL (all ones).  The two outputs are
 * malloc'd by the callee (free `allocated`); what the caller placed in
 * *result beforehand is ignored, as with MLIR-generated code.  Without a
 * loaded model the first call creates BERT-base (uncased) with seeded
 * weights: env BERT_SEED (default 1234), BERT_DTYPE f32 (default) or bf16. */
void _mlir_ciface_bert_model(BertOutput *result, MemRef2D_i64 *buffer_embeddings_position_ids,
                             MemRef2D_i64 *buffer_embeddings_token_type_ids, MemRef2D_i64 *input_ids,
                             MemRef2D_i64 *token_type_ids, MemRef2D_i64 *attention_mask);

typedef struct BertConfig {
  int32_t n_layer;       /* 12 */
  int32_t n_embd;        /* 768; multiple of 64 */
  int32_t n_head;        /* 12; n_embd / n_head must be 64 */
  int32_t n_inner;       /* 3072 */
  int32_t vocab_size;    /* 30522 */
  int32_t n_positions;   /* 512 */
  float layer_norm_eps;  /* 1e-12 */
  int32_t type_vocab;    /* 2 */
  int32_t dtype;         /* GPT2_DTYPE_F32 or GPT2_DTYPE_BF16 */
} BertConfig;

/* Creates (or replaces) the process-wide BERT model on `device` (-1: the
 * current device); independent of the GPT-2 model. */
int bert_init(const BertConfig *cfg, int device);

/* Floats of the canonical FP32 blob, tensors in transformers' state_dict
 * order: embeddings word [V,d], position [P,d], token_type [TV,d],
 * LayerNorm weight, bias; per layer query, key, value, attention.output.dense
 * (weight [d,d], bias), attention.output.LayerNorm (weight, bias),
 * intermediate.dense (weight [ff,d], bias), output.dense (weight [d,ff],
 * bias), output.LayerNorm (weight, bias); pooler.dense (weight [d,d], bias).
 * Linear weights are [out, in]. */
int64_t bert_blob_floats(const BertConfig *cfg);

/* Loads a canonical blob (bytes == 4 * bert_blob_floats); manifest_json may
 * be NULL or name the layout "bert-canonical-f32-v1". */
int bert_load_weights(const void *packed, size_t bytes, const char *manifest_json);

/* HF safetensors checkpoint of a BERT model (transformers names with or
 * without "bert.", LayerNorm gamma / beta accepted; F32, F16 or BF16) into
 * the canonical blob (no GPU needed), or loaded into the current model.
 * Extra tensors (a pre-training head, position_ids buffers) are ignored. */
int bert_safetensors_to_blob(const char *path, const BertConfig *cfg, float *out);
int bert_load_safetensors(const char *path);

/* Seeded synthetic weights (Philox4x32-10 stream 0x20000 + tensor index;
 * init modes as gpt2_init_seeded), generated and loaded / written out. */
int bert_init_seeded(uint64_t seed, int init_mode);
int bert_seeded_blob(const BertConfig *cfg, uint64_t seed, int init_mode, float *out);

int bert_get_config(BertConfig *out);
void bert_shutdown(void);
const char *bert_last_error(void);
/* Device status word (as gpt2_status); reading clears it. */
int bert_status(void);

/* Device-resident forward: d_ids [B,S], d_tt [B,S] (NULL: type 0), d_pos [S]
 * (NULL: 0..S-1), d_mask [B,S] (NULL: all ones), contiguous int64 device
 * arrays; d_hidden FP32 [B,S,d] contiguous, d_pooled FP32 [B,d] (NULL: no
 * pooler).  Enqueued on `stream` (NULL = the CUDA default stream). */
int bert_forward_device(const int64_t *d_ids, const int64_t *d_tt, const int64_t *d_pos, const int64_t *d_mask,
                        int B, int S, float *d_hidden, float *d_pooled, void *stream);

/* The same with host buffers (copies in, runs, copies out, synchronises). */
int bert_forward_host(const int64_t *ids, const int64_t *tt, const int64_t *pos, const int64_t *mask, int B, int S,
                      float *hidden, float *pooled);

/* Kernel launches of one forward. */
int bert_forward_launches(int has_mask, int has_pooler);

/* Per-kernel timing as gpt2_profile_*; kinds: 0 seq_info, 1 embedding +
 * LayerNorm, 2 layernorm, 3 qkv GEMM, 4 attention, 5 masked-row fix-up,
 * 6 attention output GEMM, 7 intermediate GEMM, 8 output GEMM, 9 pooler. */
int bert_profile_begin(void);
int bert_profile_end(double *ms_per_kind, int64_t *launches_per_kind, int n_kinds);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* BERT_B200_H */
