// runtime.h -- host runtime of libgpt2_b200.so: model dimensions, the
// canonical weight blob, the per-process model context and the forward
// schedule.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <vector>

#include "../kernels.h"

namespace gpt2 {

struct ModelDims {
  int n_layer = 12, n_embd = 768, n_head = 12, n_inner = 3072, vocab = 50257, n_pos = 1024;
  float eps = 1e-5f;
};

// One tensor of the canonical FP32 blob.
struct TensorSpec {
  enum Kind { kMatrix = 0, kGain = 1, kBias = 2 };
  int64_t offset, numel;
  Kind kind;
};

// Per-layer tensor order inside the blob.
enum LayerTensor { LN1_G, LN1_B, QKV_W, QKV_B, PROJ_W, PROJ_B, LN2_G, LN2_B, FC_W, FC_B, MPROJ_W, MPROJ_B, PER_LAYER };

std::vector<TensorSpec> blob_specs(const ModelDims &m);
int64_t blob_floats(const ModelDims &m);

void seeded_normal(float *out, int64_t n, uint64_t seed, uint32_t stream, double mean, double stdv);
void seeded_ids(int64_t *ids, int64_t n, uint64_t seed, uint32_t stream, int64_t vocab);
void seeded_blob(const ModelDims &m, uint64_t seed, int init_mode, float *blob);

// Weight-only FP8: w [K, N] (Conv1D) -> q [N, K] E4M3 codes and scale [N].
uint8_t e4m3_encode(float x);
void fp8_quantize(const float *w, int K, int N, uint8_t *q, float *scale);

// Device copies of the weights, in the layouts the kernels read.
struct LayerWeights {
  const float *ln1_g, *ln1_b, *qkv_b, *proj_b, *ln2_g, *ln2_b, *fc_b, *mproj_b;  // FP32, in blob
  const float *qkv_w, *proj_w, *fc_w, *mproj_w;                                  // FP32 [in, out], in blob
  bf16 *qkv_wt, *proj_wt, *fc_wt, *mproj_wt;                                     // BF16 [out, in]
  // weight-only FP8: E4M3 codes [out, in] and per-output-channel scales
  uint8_t *qkv_q = nullptr, *proj_q = nullptr, *fc_q = nullptr, *mproj_q = nullptr;
  float *qkv_s = nullptr, *proj_s = nullptr, *fc_s = nullptr, *mproj_s = nullptr;
  // BF16 with ln_1 / ln_2 folded into the QKV and fc GEMMs (LnFold): the
  // gain-scaled weights [out, in] and the per-output vectors c1, c2
  bf16 *qkv_lnw = nullptr, *fc_lnw = nullptr;
  float *qkv_c1 = nullptr, *qkv_c2 = nullptr, *fc_c1 = nullptr, *fc_c2 = nullptr;
};

// Activation buffers of one forward, grown on demand.
struct Workspace {
  int64_t T = 0;  // tokens the buffers hold
  int B = 0;
  int S = 0;
  void *x = nullptr, *a = nullptr, *qkv = nullptr, *o = nullptr, *u = nullptr;
  float2 *stats = nullptr;  // [T][ceil(d / LN_SEG)] row statistics of x for a folded LayerNorm
  int *first_valid = nullptr;
  uint8_t *key_valid = nullptr;
  int64_t *ids = nullptr, *mask = nullptr;  // staging for host-side entry points
  float *logits = nullptr;                  // for host-side entry points
  int64_t logits_T = 0;
};

// Kernel kinds of the forward, for the per-kernel event profiler.
enum KernelKind : int {
  K_SEQ_INFO = 0, K_EMBED, K_LAYERNORM, K_GEMM_QKV, K_ATTENTION, K_MASKED_ROWS, K_GEMM_PROJ, K_GEMM_FC,
  K_GEMM_MPROJ, K_LM_HEAD, K_NUM_KINDS
};

// Optional CUDA-event pair around every launch of the forward (off by default).
struct Profiler {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<int> kinds;  // kind of record i; events 2i, 2i+1
};

// Incremental decoding: the key / value cache and the buffers of one step.
struct DecodeState {
  int B = 0, max_len = 0, len = 0;  // len = positions cached so far
  std::vector<void *> cache;        // per layer [B][max_len][2D], activation dtype
  void *x = nullptr, *a = nullptr, *qkv = nullptr, *o = nullptr, *u = nullptr, *a_last = nullptr;
  float *logits = nullptr;          // [B, ld_logits] for gpt2_generate
  int64_t ld_logits = 0;
  int64_t *tokens = nullptr;        // generated tokens [n_new][B] for gpt2_generate
  int64_t tokens_cap = 0;
  int64_t *cur = nullptr;           // the latest greedy tokens [B] (gpt2_generate)
  int *d_pos = nullptr;             // the next position, on the device (read by the step's kernels)
  std::vector<float *> wt;          // FP32 path: [out, in] copies of the Conv1D weights, 4 per layer
};

// The forward captured as one CUDA graph for a fixed set of arguments and
// buffers: replayed when a call repeats them (one graph launch instead of
// ~85 kernel launches).  Dropped whenever the workspace is reallocated.
struct GraphCache {
  cudaGraphExec_t exec = nullptr;
  uintptr_t key[12] = {};  // the call's pointers and sizes
  int nkey = 0;
  bool seen = false;  // the key has run once uncaptured (buffers, plans and kernel attributes set up)
};

void drop_graph(GraphCache &g);
int cuda_fail(cudaError_t e, const char *what);  // records the error text, returns -2

// Runs launch(stream) -- the enqueue of one forward whose buffers and
// descriptors are already prepared -- through the graph cache: the first
// call with a key runs uncaptured, the second captures on cap_stream and
// launches the graph on st, later ones replay it.  If capture or
// instantiation fails, *enabled is cleared and plain launches continue.
template <typename F>
int run_with_graph(GraphCache &g, bool *enabled, const uintptr_t *key, int nkey, cudaStream_t cap_stream,
                   cudaStream_t st, F launch) {
  if (!*enabled) return launch(st);
  bool same = g.nkey == nkey;
  for (int i = 0; same && i < nkey; ++i) same = g.key[i] == key[i];
  if (same && g.exec) return cudaGraphLaunch(g.exec, st) == cudaSuccess ? 0 : cuda_fail(cudaGetLastError(), "graph launch");
  if (!same || !g.seen) {
    drop_graph(g);
    for (int i = 0; i < nkey; ++i) g.key[i] = key[i];
    g.nkey = nkey;
    g.seen = true;
    return launch(st);
  }
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(cap_stream, cudaStreamCaptureModeThreadLocal);
  int r = e == cudaSuccess ? launch(cap_stream) : 0;
  if (e == cudaSuccess) e = cudaStreamEndCapture(cap_stream, &graph);
  if (r == 0 && e == cudaSuccess) e = cudaGraphInstantiate(&g.exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (r || e != cudaSuccess) {
    cudaGetLastError();
    g.exec = nullptr;
    drop_graph(g);
    *enabled = false;
    if (r) return r;
    return launch(st);
  }
  return cudaGraphLaunch(g.exec, st) == cudaSuccess ? 0 : cuda_fail(cudaGetLastError(), "graph launch");
}

struct Context {
  GraphCache dec_graph;  // the decode step (position read from the device, so one graph serves all)
  ModelDims dims;
  int dtype = 0;
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  int *d_status = nullptr;
  bool loaded = false;

  float *d_blob = nullptr;  // canonical FP32 blob
  std::vector<TensorSpec> specs;
  const float *wte = nullptr, *wpe = nullptr, *lnf_g = nullptr, *lnf_b = nullptr;
  bf16 *wte_h = nullptr, *wpe_h = nullptr;  // BF16 copies
  // BF16: ln_f folded into the lm_head (wte * ln_f gain, and its c1 / c2)
  bf16 *wte_ln = nullptr;
  float *head_c1 = nullptr, *head_c2 = nullptr;
  bool ln_fold = false;  // the BF16 forward folds every LayerNorm into the next GEMM
  std::vector<LayerWeights> layers;

  Workspace ws;
  // tcgen05 GEMM plans for the current workspace: 4 per layer + lm_head.
  std::vector<TcGemmPlan> plans;
  int64_t plans_T = -1;
  int head_tile = 0, head_bn = 0;  // lm_head tile choice, and the single-SM one for unaligned logits
  AttnTcPlan attn_plan;  // tcgen05 attention descriptor for (ws.qkv, B, S)

  Profiler prof;
  GraphCache graph;
  bool use_graphs = true;  // env GPT2_GRAPHS=0 turns graph replay off
  DecodeState dec;
  std::mutex mu;
};

Context *context();  // the process-wide model (null if none)
int create_context(const ModelDims &dims, int dtype, int device);
void destroy_context();
int load_blob(Context &c, const float *host_blob);
// Grows the activation / staging buffers to hold B sequences of S tokens.
int ensure_workspace(Context &c, int B, int S);

// Enqueues the forward on `st`; ids / mask are contiguous device arrays.
// logits_f32 = 1: FP32 logits; 0: bf16 logits (BF16 / FP8-weight models
// only), row stride ld_logits in elements of that type.
int forward_device(Context &c, const int64_t *d_ids, const int64_t *d_mask, int B, int S, void *d_logits,
                   int64_t ld_logits, int logits_f32, cudaStream_t st);
// A forward of at most this many tokens streams every weight for a handful
// of rows: it runs the split-K GEMV kernels of the decode step.
constexpr int64_t kFewRows = 16;
int forward_launch_count(const Context &c, int64_t T, int has_mask);
// The FP32 layer weights transposed to [out, in] for the GEMV kernels (once).
int ensure_nk_f32(Context &c);
int prepare_forward(Context &c, int B, int S, void *d_logits, int64_t ld_logits, int logits_f32 = 1);
int launch_forward(Context &c, const int64_t *d_ids, const int64_t *d_mask, int B, int S, void *d_logits,
                   int64_t ld_logits, cudaStream_t st, bool kv_fill, int logits_f32 = 1);
// Incremental decoding (B <= 16 sequences of up to max_len tokens).
int kv_reserve(Context &c, int B, int max_len);
// The forward over B x S ids that also fills the cache (positions 0 .. S-1)
// and writes only the last position's logits [B, ld].
int prefill(Context &c, const int64_t *d_ids, int B, int S, float *d_logits, int64_t ld, cudaStream_t st);
// One token per sequence at position c.dec.len; logits [B, ld].
int decode_step(Context &c, const int64_t *d_tokens, int B, float *d_logits, int64_t ld, cudaStream_t st);
int generate(Context &c, const int64_t *ids, int B, int S, int n_new, int64_t *out_tokens);
void free_decode(DecodeState &d);

// Fills the canonical blob of m from an HF safetensors checkpoint (F32 / F16 / BF16).
int gpt2_safetensors_blob(const char *path, const ModelDims &m, float *blob);
int profile_begin(Profiler &p);
int profile_end(Profiler &p, double *ms, int64_t *count, int n);
cudaEvent_t prof_event(Profiler &p);  // the next event of the pool (null if none can be created)

void set_error(const char *fmt, ...);

// Status-checked CUDA call inside a function returning int.
#define CK(call)                                          \
  do {                                                    \
    cudaError_t e_ = (call);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);   \
  } while (0)

// A kernel launch of kind K on stream `st` of context `c`, bracketed by
// profiler events when profiling is on.
#define CKP(K, call)                                      \
  do {                                                    \
    cudaEvent_t pa_ = nullptr, pb_ = nullptr;             \
    if (c.prof.on) {                                      \
      pa_ = prof_event(c.prof);                           \
      pb_ = prof_event(c.prof);                           \
      if (pa_ && pb_) cudaEventRecord(pa_, st);           \
    }                                                     \
    cudaError_t e_ = (call);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);   \
    if (pa_ && pb_) {                                     \
      cudaEventRecord(pb_, st);                           \
      c.prof.kinds.push_back(K);                          \
    }                                                     \
  } while (0)

}  // namespace gpt2
