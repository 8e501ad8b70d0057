// gpt2_abi.cpp -- the C ABI of libgpt2_b200.so (include/gpt2_b200.h).
//
// gpt2_decoder / _mlir_ciface_gpt2_decoder reproduce the entry points the
// reference's host program links against (src/gpt/gpt2_call.cpp:17-38,
// :62-64) and its CPU pipeline emits (src/gpt/run_mlir_pipeline.sh:7): ids and
// mask memrefs in, a malloc'd FP32 logits memref out (freed by the caller,
// src/gpt/gpt2_call.cpp:93-94).  Nothing here aborts: failures return a
// zeroed descriptor or a negative code plus gpt2_last_error().
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "../../../include/gpt2_b200.h"
#include "../runtime/hostcopy.h"
#include "../runtime/runtime.h"

namespace gpt2 {
const char *last_error_text();
void clear_error();
}  // namespace gpt2

using namespace gpt2;

namespace {
std::mutex g_api_mu;  // serialises every entry point that touches the model

ModelDims dims_of(const Gpt2Config *c) {
  ModelDims m;
  m.n_layer = c->n_layer;
  m.n_embd = c->n_embd;
  m.n_head = c->n_head;
  m.n_inner = c->n_inner;
  m.vocab = c->vocab_size;
  m.n_pos = c->n_positions;
  m.eps = c->layer_norm_eps;
  return m;
}

bool valid_dims(const Gpt2Config *c) {
  return c && c->n_layer > 0 && c->n_embd > 0 && c->n_head > 0 && c->n_inner > 0 && c->vocab_size > 0 &&
         c->n_positions > 0;
}

int load_seeded_locked(uint64_t seed, int init_mode) {
  Context *c = context();
  if (!c) {
    set_error("no model: call gpt2_init first");
    return GPT2_ENOMODEL;
  }
  std::vector<float> blob(static_cast<size_t>(blob_floats(c->dims)));
  seeded_blob(c->dims, seed, init_mode, blob.data());
  return load_blob(*c, blob.data());
}

// Creates GPT-2 small with seeded weights when no model exists (the
// reference's object file carries its weights; this is the stand-in).
int ensure_default_model_locked() {
  Context *c = context();
  if (c && c->loaded) return 0;
  if (!c) {
    int dtype = GPT2_DTYPE_F32;
    if (const char *e = getenv("GPT2_DTYPE")) {
      if (!strcmp(e, "bf16")) dtype = GPT2_DTYPE_BF16;
      else if (!strcmp(e, "fp8w")) dtype = GPT2_DTYPE_FP8W;
      else if (strcmp(e, "f32") && strcmp(e, "fp32")) {
        set_error("GPT2_DTYPE must be f32 or bf16, got '%s'", e);
        return GPT2_EINVAL;
      }
    }
    int r = create_context(ModelDims(), dtype, -1);
    if (r) return r;
  }
  uint64_t seed = 1234;
  if (const char *e = getenv("GPT2_SEED")) seed = strtoull(e, nullptr, 10);
  return load_seeded_locked(seed, 0);
}

int read_status_locked(Context &c) {
  int h = 0;
  if (cudaMemcpy(&h, c.d_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (h) cudaMemset(c.d_status, 0, sizeof(int));
  return h;
}

// Gathers a strided memref<?x?xi64> into a contiguous [B, S] vector.
void gather_i64(const int64_t *aligned, int64_t off, int64_t s0, int64_t s1, int64_t st0, int64_t st1,
                std::vector<int64_t> &out) {
  out.resize(static_cast<size_t>(s0 * s1));
  for (int64_t i = 0; i < s0; ++i)
    for (int64_t j = 0; j < s1; ++j) out[i * s1 + j] = aligned[off + i * st0 + j * st1];
}

int forward_host_locked(const int64_t *ids, const int64_t *mask, int B, int S, float *logits) {
  int r = ensure_default_model_locked();
  if (r) return r;
  Context &c = *context();
  if (cudaSetDevice(c.device) != cudaSuccess) {
    set_error("cudaSetDevice(%d) failed", c.device);
    return GPT2_ECUDA;
  }
  const int64_t T = (int64_t)B * S;
  if (B < 1 || S < 1 || S > c.dims.n_pos) {
    set_error("bad shape B=%d S=%d (n_positions %d)", B, S, c.dims.n_pos);
    return GPT2_EINVAL;
  }
  // Host-side check of the ids gives the caller a precise error; the embed
  // kernel also checks and reports through the status word.
  for (int64_t i = 0; i < T; ++i)
    if (ids[i] < 0 || ids[i] >= c.dims.vocab) {
      set_error("token id %lld at position %lld outside [0, %d)", (long long)ids[i], (long long)i, c.dims.vocab);
      return GPT2_EINVAL;
    }
  // Staging buffers and a device logits buffer, grown on demand.
  Workspace &w = c.ws;
  r = ensure_workspace(c, B, S);
  if (r) return r;
  const int64_t V = c.dims.vocab;
  // Device logits rows padded to a multiple of 4 floats (16 bytes) so the
  // lm_head epilogue can store them with TMA; the copy-out strips the pad.
  const int64_t ldl = (V + 3) / 4 * 4;
  if (!w.logits || w.logits_T < T) {
    if (w.logits) cudaFree(w.logits);
    w.logits = nullptr;
    w.logits_T = 0;
    if (cudaMalloc(&w.logits, sizeof(float) * T * ldl) != cudaSuccess) {
      set_error("cudaMalloc of %lld logits failed", (long long)(T * ldl));
      return GPT2_ENOMEM;
    }
    w.logits_T = T;
  }
  cudaStream_t st = c.stream;
  if (cudaMemcpyAsync(w.ids, ids, sizeof(int64_t) * T, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      (mask && cudaMemcpyAsync(w.mask, mask, sizeof(int64_t) * T, cudaMemcpyHostToDevice, st) != cudaSuccess)) {
    set_error("host-to-device copy of ids/mask failed");
    return GPT2_ECUDA;
  }
  r = forward_device(c, w.ids, mask ? w.mask : nullptr, B, S, w.logits, ldl, 1, st);
  if (r) return r;
  // Pinned destinations take one strided DMA; pageable ones (the drop-in's
  // malloc'd result) stream through pinned staging chunks.
  r = copy_rows_to_host(w.logits, ldl, T, V, logits, st);
  if (r) return r;
  const int s = read_status_locked(c);
  if (s) {
    set_error("device status %d after forward", s);
    return GPT2_EDEVICE;
  }
  return 0;
}

MemRef3D decoder_impl(const int64_t *ids_aligned, int64_t ids_off, int64_t is0, int64_t is1, int64_t ist0,
                      int64_t ist1, const int64_t *m_aligned, int64_t m_off, int64_t ms0, int64_t ms1, int64_t mst0,
                      int64_t mst1) {
  MemRef3D out;
  memset(&out, 0, sizeof out);
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  if (!ids_aligned || is0 < 1 || is1 < 1 || is0 > (1 << 20) || is1 > (1 << 20)) {
    set_error("gpt2_decoder: bad input_ids memref (sizes %lld x %lld)", (long long)is0, (long long)is1);
    return out;
  }
  std::vector<int64_t> ids, mask;
  gather_i64(ids_aligned, ids_off, is0, is1, ist0, ist1, ids);
  bool has_mask = false;
  if (m_aligned) {
    if (ms0 != is0 || ms1 != is1) {
      set_error("gpt2_decoder: attention_mask sizes %lld x %lld differ from input_ids %lld x %lld", (long long)ms0,
                (long long)ms1, (long long)is0, (long long)is1);
      return out;
    }
    gather_i64(m_aligned, m_off, ms0, ms1, mst0, mst1, mask);
    for (int64_t v : mask)
      if (v == 0) {
        has_mask = true;
        break;
      }
  }
  int r = ensure_default_model_locked();
  if (r) return out;
  const int64_t V = context()->dims.vocab;
  const int64_t n = is0 * is1 * V;
  // Released by the caller with free() (src/gpt/gpt2_call.cpp:94).
  float *buf = static_cast<float *>(alloc_host_output(sizeof(float) * n));
  if (!buf) {
    set_error("gpt2_decoder: allocation of %lld floats of host memory failed", (long long)n);
    return out;
  }
  // An all-ones mask is the unmasked computation; skip its kernels.
  r = forward_host_locked(ids.data(), has_mask ? mask.data() : nullptr, (int)is0, (int)is1, buf);
  if (r) {
    free(buf);
    return out;
  }
  out.allocated = buf;
  out.aligned = buf;
  out.offset = 0;
  out.sizes[0] = is0;
  out.sizes[1] = is1;
  out.sizes[2] = V;
  out.strides[0] = is1 * V;
  out.strides[1] = V;
  out.strides[2] = 1;
  return out;
}
}  // namespace

extern "C" {

MemRef3D gpt2_decoder(int64_t *in_alloc, int64_t *in_align, int64_t in_offs, int64_t in_s0, int64_t in_s1,
                      int64_t in_str0, int64_t in_str1, int64_t *mask_alloc, int64_t *mask_align,
                      int64_t mask_offs, int64_t mask_s0, int64_t mask_s1, int64_t mask_str0, int64_t mask_str1) {
  (void)in_alloc;
  (void)mask_alloc;
  return decoder_impl(in_align, in_offs, in_s0, in_s1, in_str0, in_str1, mask_align, mask_offs, mask_s0, mask_s1,
                      mask_str0, mask_str1);
}

void _mlir_ciface_gpt2_decoder(MemRef3D *result, MemRef2D_i64 *input_ids, MemRef2D_i64 *attention_mask) {
  if (!result) return;
  if (!input_ids) {
    memset(result, 0, sizeof *result);
    set_error("_mlir_ciface_gpt2_decoder: null input_ids");
    return;
  }
  const MemRef2D_i64 *m = attention_mask;
  *result = decoder_impl(input_ids->aligned, input_ids->offset, input_ids->sizes[0], input_ids->sizes[1],
                         input_ids->strides[0], input_ids->strides[1], m ? m->aligned : nullptr, m ? m->offset : 0,
                         m ? m->sizes[0] : 0, m ? m->sizes[1] : 0, m ? m->strides[0] : 0, m ? m->strides[1] : 0);
}

int gpt2_init(const Gpt2Config *cfg, int device) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  if (!valid_dims(cfg)) {
    set_error("gpt2_init: invalid configuration");
    return GPT2_EINVAL;
  }
  return create_context(dims_of(cfg), cfg->dtype, device);
}

int64_t gpt2_blob_floats(const Gpt2Config *cfg) {
  if (!valid_dims(cfg)) return GPT2_EINVAL;
  return blob_floats(dims_of(cfg));
}

int gpt2_load_weights(const void *packed, size_t bytes, const char *manifest_json) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  Context *c = context();
  if (!c) {
    set_error("gpt2_load_weights: no model, call gpt2_init first");
    return GPT2_ENOMODEL;
  }
  if (!packed || bytes != sizeof(float) * static_cast<size_t>(blob_floats(c->dims))) {
    set_error("gpt2_load_weights: expected %lld bytes of canonical FP32 blob, got %zu",
              (long long)(sizeof(float) * blob_floats(c->dims)), bytes);
    return GPT2_EINVAL;
  }
  if (manifest_json && !strstr(manifest_json, "gpt2-canonical-f32-v1")) {
    set_error("gpt2_load_weights: manifest layout must be \"gpt2-canonical-f32-v1\"");
    return GPT2_EINVAL;
  }
  return load_blob(*c, static_cast<const float *>(packed));
}

int gpt2_safetensors_to_blob(const char *path, const Gpt2Config *cfg, float *out) {
  clear_error();
  if (!path || !valid_dims(cfg) || !out) {
    set_error("gpt2_safetensors_to_blob: need a path, a valid configuration and an output buffer");
    return GPT2_EINVAL;
  }
  return gpt2_safetensors_blob(path, dims_of(cfg), out) ? GPT2_EINVAL : 0;
}

int gpt2_load_safetensors(const char *path) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  Context *c = context();
  if (!c) {
    set_error("gpt2_load_safetensors: no model, call gpt2_init first");
    return GPT2_ENOMODEL;
  }
  if (!path) return GPT2_EINVAL;
  std::vector<float> blob(static_cast<size_t>(blob_floats(c->dims)));
  if (gpt2_safetensors_blob(path, c->dims, blob.data())) return GPT2_EINVAL;
  return load_blob(*c, blob.data());
}

int gpt2_init_seeded(uint64_t seed, int init_mode) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  if (init_mode != 0 && init_mode != 1) {
    set_error("gpt2_init_seeded: init_mode must be 0 or 1");
    return GPT2_EINVAL;
  }
  return load_seeded_locked(seed, init_mode);
}

int gpt2_seeded_blob(const Gpt2Config *cfg, uint64_t seed, int init_mode, float *out) {
  if (!valid_dims(cfg) || !out || (init_mode != 0 && init_mode != 1)) return GPT2_EINVAL;
  seeded_blob(dims_of(cfg), seed, init_mode, out);
  return 0;
}

int gpt2_fp8_quantize(const float *w, int K, int N, uint8_t *q, float *scale) {
  if (!w || !q || !scale || K < 1 || N < 1) return GPT2_EINVAL;
  fp8_quantize(w, K, N, q, scale);
  return 0;
}

int gpt2_seeded_ids(int64_t *ids, int64_t n, uint64_t seed, uint32_t stream, int64_t vocab) {
  if (!ids || n < 0 || vocab < 1) return GPT2_EINVAL;
  seeded_ids(ids, n, seed, stream, vocab);
  return 0;
}

int gpt2_get_config(Gpt2Config *out) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  Context *c = context();
  if (!c) {
    set_error("gpt2_get_config: no model");
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
  out->dtype = c->dtype;
  return 0;
}

void gpt2_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  destroy_context();  // synchronises the device first
  release_host_staging();
}

const char *gpt2_last_error(void) { return last_error_text(); }

int gpt2_status(void) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  Context *c = context();
  if (!c) return GPT2_ENOMODEL;
  cudaSetDevice(c->device);
  return read_status_locked(*c);
}

int gpt2_forward_device(const int64_t *d_ids, const int64_t *d_mask, int B, int S, void *d_logits,
                        int64_t ld_logits, int logits_dtype, void *stream) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  Context *c = context();
  if (!c || !c->loaded) {
    set_error("gpt2_forward_device: no model loaded");
    return GPT2_ENOMODEL;
  }
  if ((logits_dtype != GPT2_DTYPE_F32 && logits_dtype != GPT2_DTYPE_BF16) || !d_ids || !d_logits) {
    set_error("gpt2_forward_device: need ids, logits and logits_dtype GPT2_DTYPE_F32 or GPT2_DTYPE_BF16");
    return GPT2_EINVAL;
  }
  cudaSetDevice(c->device);
  return forward_device(*c, d_ids, d_mask, B, S, d_logits, ld_logits, logits_dtype == GPT2_DTYPE_F32,
                        static_cast<cudaStream_t>(stream));
}

int gpt2_forward_host(const int64_t *ids, const int64_t *mask, int B, int S, float *logits) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  if (!ids || !logits) {
    set_error("gpt2_forward_host: null ids or logits");
    return GPT2_EINVAL;
  }
  return forward_host_locked(ids, mask, B, S, logits);
}

int gpt2_kv_reserve(int B, int max_len) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  Context *c = context();
  if (!c || !c->loaded) {
    set_error("gpt2_kv_reserve: no model loaded");
    return GPT2_ENOMODEL;
  }
  return kv_reserve(*c, B, max_len);
}

int gpt2_prefill(const int64_t *d_ids, int B, int S, float *d_logits, int64_t ld_logits, void *stream) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  Context *c = context();
  if (!c || !c->loaded) {
    set_error("gpt2_prefill: no model loaded");
    return GPT2_ENOMODEL;
  }
  if (!d_ids || !d_logits) return GPT2_EINVAL;
  cudaSetDevice(c->device);
  return prefill(*c, d_ids, B, S, d_logits, ld_logits, static_cast<cudaStream_t>(stream));
}

int gpt2_decode_step(const int64_t *d_tokens, int B, float *d_logits, int64_t ld_logits, void *stream) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  Context *c = context();
  if (!c || !c->loaded) {
    set_error("gpt2_decode_step: no model loaded");
    return GPT2_ENOMODEL;
  }
  if (!d_tokens || !d_logits) return GPT2_EINVAL;
  cudaSetDevice(c->device);
  return decode_step(*c, d_tokens, B, d_logits, ld_logits, static_cast<cudaStream_t>(stream));
}

int gpt2_kv_length(void) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  Context *c = context();
  return c ? c->dec.len : GPT2_ENOMODEL;
}

int gpt2_generate(const int64_t *ids, int B, int S, int n_new, int64_t *out_tokens) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  clear_error();
  if (!ids || !out_tokens) {
    set_error("gpt2_generate: null ids or output");
    return GPT2_EINVAL;
  }
  int r = ensure_default_model_locked();
  if (r) return r;
  Context &c = *context();
  cudaSetDevice(c.device);
  r = generate(c, ids, B, S, n_new, out_tokens);
  if (r) return r;
  const int s = read_status_locked(c);
  if (s) {
    set_error("device status %d after generation", s);
    return GPT2_EDEVICE;
  }
  return 0;
}

int gpt2_forward_launches(int B, int S, int has_mask) {
  Context *c = context();
  if (!c) return GPT2_ENOMODEL;
  return forward_launch_count(*c, (int64_t)B * S, has_mask);
}

int gpt2_profile_begin(void) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  Context *c = context();
  if (!c) return GPT2_ENOMODEL;
  return profile_begin(c->prof);
}

int gpt2_profile_end(double *ms_per_kind, int64_t *launches_per_kind, int n_kinds) {
  std::lock_guard<std::mutex> lk(g_api_mu);
  Context *c = context();
  if (!c) return GPT2_ENOMODEL;
  if (!ms_per_kind || !launches_per_kind || n_kinds < 0) return GPT2_EINVAL;
  cudaSetDevice(c->device);
  return profile_end(c->prof, ms_per_kind, launches_per_kind, n_kinds < K_NUM_KINDS ? n_kinds : K_NUM_KINDS);
}

// ---------------------------------------------------------------------------
// Kernel-level entry points
// ---------------------------------------------------------------------------
static int ck(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return 0;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorInvalidValue ? GPT2_EINVAL : GPT2_ECUDA;
}

int gpt2k_gemm_f32(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                   const float *bias, const float *resid, int epi, void *stream) {
  return ck(launch_gemm_f32(A, B, b_nk, C, M, N, K, ldc, bias, resid, epi, static_cast<cudaStream_t>(stream)),
            "gpt2k_gemm_f32");
}

int gpt2k_gemm_bf16(const void *A, const void *B, void *C, int M, int N, int K, int ldc, int out_f32,
                    const float *bias, const void *resid, int epi, int bn, void *stream) {
  TcGemmPlan plan;
  const int r = tc_gemm_plan(&plan, static_cast<const bf16 *>(A), static_cast<const bf16 *>(B), M, N, K, bn);
  if (r) {
    set_error("gpt2k_gemm_bf16: TMA descriptor creation failed (%d)", r);
    return GPT2_EINVAL;
  }
  tc_gemm_set_output(&plan, C, ldc, out_f32);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return ck(launch_gemm_tc(plan, C, ldc, out_f32, bias, static_cast<const bf16 *>(resid), epi, nullptr, sms,
                           static_cast<cudaStream_t>(stream)),
            "gpt2k_gemm_bf16");
}

int gpt2k_gemv_bf16(const void *x, const void *W, void *y, int M, int N, int K, int ldy, const float *bias,
                    const void *resid, int epi, const float *ln_gain, const float *ln_shift, float eps, int out_f32,
                    int impl, void *stream) {
  if (!x || !W || !y || M < 1 || M > 16 || N < 1 || K < 8 || ldy < N || (!ln_gain) != (!ln_shift)) {
    set_error("gpt2k_gemv_bf16: bad operands (M=%d N=%d K=%d ldy=%d)", M, N, K, ldy);
    return GPT2_EINVAL;
  }
  if (out_f32 && epi != GPT2_EPI_NONE) {
    set_error("gpt2k_gemv_bf16: an FP32 output takes no epilogue");
    return GPT2_EINVAL;
  }
  if (impl == 1 && !gemv_tc_supported(M, N, K, ldy)) {
    set_error("gpt2k_gemv_bf16: the tensor-core kernel needs K a multiple of 64 (K=%d)", K);
    return GPT2_EINVAL;
  }
  const GemvLn ln{ln_gain, ln_shift, eps};
  const GemvLn *lp = ln_gain ? &ln : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bf16 *xb = static_cast<const bf16 *>(x), *wb = static_cast<const bf16 *>(W);
  if (impl == 1) {
    if (out_f32) return ck(launch_gemv_tc_bf16_f32out(xb, wb, static_cast<float *>(y), M, N, K, ldy, nullptr, st, lp),
                           "gpt2k_gemv_bf16");
    return ck(launch_gemv_tc_bf16(xb, wb, static_cast<bf16 *>(y), M, N, K, ldy, bias,
                                  static_cast<const bf16 *>(resid), nullptr, epi, nullptr, st, lp),
              "gpt2k_gemv_bf16");
  }
  if (impl != 0) {
    set_error("gpt2k_gemv_bf16: impl must be 0 or 1");
    return GPT2_EINVAL;
  }
  if (out_f32) return ck(launch_gemv_bf16_f32out(xb, wb, static_cast<float *>(y), M, N, K, ldy, st, lp),
                         "gpt2k_gemv_bf16");
  return ck(launch_gemv_bf16(xb, wb, static_cast<bf16 *>(y), M, N, K, ldy, bias, static_cast<const bf16 *>(resid),
                             nullptr, epi, st, lp),
            "gpt2k_gemv_bf16");
}

int gpt2k_test_gemm_withheld_load(const void *A, const void *B, void *C, int M, int N, int K, int *d_status,
                                  void *stream) {
  if (!A || !B || !C || !d_status) {
    set_error("gpt2k_test_gemm_withheld_load: null operand or status");
    return GPT2_EINVAL;
  }
  TcGemmPlan plan;
  const int r = tc_gemm_plan(&plan, static_cast<const bf16 *>(A), static_cast<const bf16 *>(B), M, N, K, 128);
  if (r || N % 8) {
    set_error("gpt2k_test_gemm_withheld_load: bad operands (%d)", r);
    return GPT2_EINVAL;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return ck(launch_gemm_tc_withheld_load(plan, C, d_status, sms, static_cast<cudaStream_t>(stream)),
            "gpt2k_test_gemm_withheld_load");
}

int gpt2k_gemm_bf16_ln(const void *A, const void *B, void *C, int M, int N, int K, int ldc, int out_f32,
                       const float *bias, const void *resid, int epi, int bn, const float *c1, const float *c2,
                       const float *stats_in, float *stats_out, float eps, void *stream) {
  TcGemmPlan plan;
  const int r = tc_gemm_plan(&plan, static_cast<const bf16 *>(A), static_cast<const bf16 *>(B), M, N, K, bn);
  if (r) {
    set_error("gpt2k_gemm_bf16_ln: TMA descriptor creation failed (%d)", r);
    return GPT2_EINVAL;
  }
  tc_gemm_set_output(&plan, C, ldc, out_f32);
  LnFold ln;
  ln.c1 = c1;
  ln.c2 = c2;
  ln.stats_in = reinterpret_cast<const float2 *>(stats_in);
  ln.nseg_in = ln_segments(K);
  ln.k = K;
  ln.eps = eps;
  ln.stats_out = reinterpret_cast<float2 *>(stats_out);
  ln.nseg_out = ln_segments(N);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return ck(launch_gemm_tc(plan, C, ldc, out_f32, bias, static_cast<const bf16 *>(resid), epi, nullptr, sms,
                           static_cast<cudaStream_t>(stream), nullptr, &ln),
            "gpt2k_gemm_bf16_ln");
}

int gpt2k_ln_fold_pack(const float *W, int w_kn, const float *gain, const float *shift, const float *bias, void *B,
                       float *c1, float *c2, int N, int K, void *stream) {
  return ck(launch_ln_fold_pack(W, w_kn, gain, shift, bias, static_cast<bf16 *>(B), c1, c2, N, K,
                                static_cast<cudaStream_t>(stream)),
            "gpt2k_ln_fold_pack");
}

int gpt2k_ffma_peak(float *tflops, void *stream) {
  return ck(measure_ffma_peak(tflops, static_cast<cudaStream_t>(stream)), "gpt2k_ffma_peak");
}

int gpt2k_layernorm(const void *x, const float *gain, const float *shift, void *y, int T, int d, float eps,
                    int dtype, void *stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == GPT2_DTYPE_F32)
    return ck(launch_layernorm_f32(static_cast<const float *>(x), gain, shift, static_cast<float *>(y), T, d, eps, st),
              "gpt2k_layernorm");
  if (dtype == GPT2_DTYPE_BF16)
    return ck(launch_layernorm_bf16(static_cast<const bf16 *>(x), gain, shift, static_cast<bf16 *>(y), T, d, eps, st),
              "gpt2k_layernorm");
  set_error("gpt2k_layernorm: bad dtype");
  return GPT2_EINVAL;
}

namespace {
std::mutex g_blas_mu;
struct BlasStage {
  float *a = nullptr, *b = nullptr, *c = nullptr;
  size_t na = 0, nb = 0, nc = 0;
} g_blas;

bool is_device_ptr(const void *p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

int grow(float **p, size_t *cap, size_t n) {
  if (*cap >= n) return 0;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  if (cudaMalloc(p, n * sizeof(float)) != cudaSuccess) return -1;
  *cap = n;
  return 0;
}
}  // namespace

int gpt2_blas_sgemm(int order, int transA, int transB, int M, int N, int K, float alpha, const float *A, int lda,
                    const float *B, int ldb, float beta, float *C, int ldc) {
  clear_error();
  const bool b_nk = transB == 112;
  if (order != 101 || transA != 111 || (transB != 111 && transB != 112) || alpha != 1.0f || beta != 0.0f) {
    set_error("gpt2_blas_sgemm: only RowMajor, NoTrans A, NoTrans/Trans B, alpha 1, beta 0 (the lowering's call)");
    return GPT2_EINVAL;
  }
  if (M < 1 || N < 1 || K < 1 || !A || !B || !C || lda != K || ldb != (b_nk ? K : N) || ldc < N) {
    set_error("gpt2_blas_sgemm: bad sizes M=%d N=%d K=%d lda=%d ldb=%d ldc=%d", M, N, K, lda, ldb, ldc);
    return GPT2_EINVAL;
  }
  std::lock_guard<std::mutex> lk(g_blas_mu);
  // The SIMT kernel wants K % 8 == 0 and, for [K, N] B, N % 4 == 0; other
  // shapes (and host operands) go through zero-padded device copies.
  const int Kp = (K + 7) / 8 * 8, Np = b_nk ? N : (N + 3) / 4 * 4;
  const bool dev = is_device_ptr(A) && is_device_ptr(B) && is_device_ptr(C);
  cudaStream_t st = nullptr;
  cudaError_t e;
  if (dev && Kp == K && Np == N) {
    e = launch_gemm_f32(A, B, b_nk, C, M, N, K, ldc, nullptr, nullptr, EPI_NONE, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return ck(e, "gpt2_blas_sgemm");
  }
  const size_t brows = b_nk ? (size_t)N : (size_t)Kp, bcols = b_nk ? (size_t)Kp : (size_t)Np;
  if (grow(&g_blas.a, &g_blas.na, (size_t)M * Kp) || grow(&g_blas.b, &g_blas.nb, brows * bcols) ||
      grow(&g_blas.c, &g_blas.nc, (size_t)M * Np)) {
    set_error("gpt2_blas_sgemm: cannot allocate staging buffers");
    return GPT2_ENOMEM;
  }
  const cudaMemcpyKind in = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDefault;
  e = cudaMemsetAsync(g_blas.a, 0, sizeof(float) * (size_t)M * Kp, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(g_blas.b, 0, sizeof(float) * brows * bcols, st);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(g_blas.a, sizeof(float) * Kp, A, sizeof(float) * K, sizeof(float) * K, M, in, st);
  if (e == cudaSuccess)
    e = b_nk ? cudaMemcpy2DAsync(g_blas.b, sizeof(float) * Kp, B, sizeof(float) * K, sizeof(float) * K, N, in, st)
             : cudaMemcpy2DAsync(g_blas.b, sizeof(float) * Np, B, sizeof(float) * N, sizeof(float) * N, K, in, st);
  if (e == cudaSuccess)
    e = launch_gemm_f32(g_blas.a, g_blas.b, b_nk, g_blas.c, M, b_nk ? N : Np, Kp, Np, nullptr, nullptr, EPI_NONE, st);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(C, sizeof(float) * ldc, g_blas.c, sizeof(float) * Np, sizeof(float) * N, M,
                          dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDefault, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return ck(e, "gpt2_blas_sgemm");
}

size_t gpt2k_attention_workspace_bytes(int B, int S) {
  return 256 + sizeof(int) * (size_t)B + (size_t)B * S;
}

int gpt2k_attention(const void *qkv, const int64_t *d_mask, void *o, int B, int S, int H, int dtype, void *workspace,
                    void *stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int *first_valid = nullptr;
  uint8_t *key_valid = nullptr;
  if (d_mask) {
    if (!workspace) {
      set_error("gpt2k_attention: a mask needs a workspace");
      return GPT2_EINVAL;
    }
    first_valid = static_cast<int *>(workspace);
    key_valid = static_cast<uint8_t *>(workspace) + 256 + sizeof(int) * (size_t)B;
    int r = ck(launch_seq_info(d_mask, B, S, first_valid, key_valid, st), "gpt2k_attention");
    if (r) return r;
  }
  int r;
  if (dtype == GPT2_DTYPE_F32) {
    r = ck(launch_attention_f32(static_cast<const float *>(qkv), key_valid, static_cast<float *>(o), B, S, H, st),
           "gpt2k_attention");
    if (!r && d_mask)
      r = ck(launch_attn_masked_rows_f32(static_cast<const float *>(qkv), first_valid, static_cast<float *>(o), B, S,
                                         H, st),
             "gpt2k_attention");
  } else if (dtype == GPT2_DTYPE_BF16) {
    AttnTcPlan plan;
    if (attention_tc_plan(&plan, static_cast<const bf16 *>(qkv), B, S, H, static_cast<const bf16 *>(o))) {
      set_error("gpt2k_attention: TMA descriptor creation failed (qkv and o must be 16-byte aligned)");
      return GPT2_EINVAL;
    }
    r = ck(launch_attention_tc3(plan, key_valid, static_cast<bf16 *>(o), nullptr, st), "gpt2k_attention");
    if (!r && d_mask)
      r = ck(launch_attn_masked_rows_bf16(static_cast<const bf16 *>(qkv), first_valid, static_cast<bf16 *>(o), B, S,
                                          H, st),
             "gpt2k_attention");
  } else {
    set_error("gpt2k_attention: bad dtype");
    return GPT2_EINVAL;
  }
  return r;
}

size_t gpt2k_attention_ex_workspace_bytes(int B, int S) {
  return 256 + 2 * sizeof(int) * (size_t)B + (size_t)B * S;
}

int gpt2k_attention_ex(const void *qkv, const int64_t *d_mask, void *o, int B, int S, int H, int dtype, int causal,
                       void *workspace, void *stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int c = causal ? 1 : 0;
  int *first_valid = nullptr, *kv_end = nullptr;
  uint8_t *key_valid = nullptr;
  if (d_mask) {
    if (!workspace) {
      set_error("gpt2k_attention_ex: a mask needs a workspace");
      return GPT2_EINVAL;
    }
    first_valid = static_cast<int *>(workspace);
    kv_end = first_valid + B;
    key_valid = static_cast<uint8_t *>(workspace) + 256 + 2 * sizeof(int) * (size_t)B;
    int r = ck(launch_seq_info(d_mask, B, S, first_valid, key_valid, st, kv_end), "gpt2k_attention_ex");
    if (r) return r;
  }
  int r;
  if (dtype == GPT2_DTYPE_F32) {
    r = ck(launch_attention_f32(static_cast<const float *>(qkv), key_valid, static_cast<float *>(o), B, S, H, st, c),
           "gpt2k_attention_ex");
    if (!r && d_mask)
      r = ck(launch_attn_masked_rows_f32(static_cast<const float *>(qkv), first_valid, static_cast<float *>(o), B, S,
                                         H, st, c),
             "gpt2k_attention_ex");
    return r;
  }
  if (dtype == GPT2_DTYPE_BF16) {
    AttnTcPlan plan;
    if (attention_tc_plan(&plan, static_cast<const bf16 *>(qkv), B, S, H, static_cast<const bf16 *>(o))) {
      set_error("gpt2k_attention_ex: TMA descriptor creation failed (qkv and o must be 16-byte aligned)");
      return GPT2_EINVAL;
    }
    r = ck(launch_attention_tc3(plan, key_valid, static_cast<bf16 *>(o), nullptr, st, c, kv_end),
           "gpt2k_attention_ex");
  } else {
    set_error("gpt2k_attention_ex: bad dtype");
    return GPT2_EINVAL;
  }
  if (!r && d_mask)
    r = ck(launch_attn_masked_rows_bf16(static_cast<const bf16 *>(qkv), first_valid, static_cast<bf16 *>(o), B, S, H,
                                        st, c),
           "gpt2k_attention_ex");
  return r;
}

int gpt2k_embed(const int64_t *d_ids, const void *wte, const void *wpe, void *x, int T, int S, int d, int V, int dtype,
                int *d_status, void *stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == GPT2_DTYPE_F32)
    return ck(launch_embed_f32(d_ids, static_cast<const float *>(wte), static_cast<const float *>(wpe),
                               static_cast<float *>(x), T, S, d, V, d_status, st),
              "gpt2k_embed");
  if (dtype == GPT2_DTYPE_BF16)
    return ck(launch_embed_bf16(d_ids, static_cast<const bf16 *>(wte), static_cast<const bf16 *>(wpe),
                                static_cast<bf16 *>(x), T, S, d, V, d_status, st),
              "gpt2k_embed");
  set_error("gpt2k_embed: bad dtype");
  return GPT2_EINVAL;
}

}  // extern "C"
