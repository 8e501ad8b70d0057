// safetensors.cpp -- reads HF safetensors checkpoints into the canonical FP32
// weight blobs (GPT-2 and BERT), the ingestion path for real weights.
//
// The reference bakes its weights into the compiled object as dense_resource
// constants named after the HF state_dict (docs/Chapter3.md:167-175; the
// name mapping of lib/GPT2SliceAnalysis.cpp:94-113).  Here a checkpoint file
// is read instead: the safetensors layout is an 8-byte little-endian header
// length, a JSON header {name: {"dtype", "shape", "data_offsets": [b, e]},
// "__metadata__": {...}}, then the raw little-endian tensor bytes.  Tensors
// are found by their transformers names, with or without the model prefix
// ("transformer." / "bert."), and LayerNorm "gamma"/"beta" are accepted for
// "weight"/"bias" (older BERT checkpoints).  F32, F16 and BF16 tensors are
// widened to FP32 exactly.
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <string>
#include <vector>

#include "bert.h"
#include "runtime.h"

namespace gpt2 {

namespace {

struct StTensor {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;
};

// A minimal JSON reader for the header: objects, arrays, strings, integers,
// and skipping of any other value.
class Json {
 public:
  Json(const char *p, const char *e) : p_(p), e_(e) {}
  bool ok() const { return ok_; }

  bool parse_header(std::map<std::string, StTensor> &out) {
    ws();
    if (!eat('{')) return fail();
    ws();
    if (peek() == '}') return ++p_, true;
    for (;;) {
      std::string key;
      if (!str(key)) return fail();
      ws();
      if (!eat(':')) return fail();
      ws();
      if (key == "__metadata__") {
        if (!skip()) return fail();
      } else {
        StTensor t;
        if (!tensor(t)) return fail();
        out[key] = t;
      }
      ws();
      if (eat(',')) {
        ws();
        continue;
      }
      if (eat('}')) return true;
      return fail();
    }
  }

 private:
  const char *p_, *e_;
  bool ok_ = true;

  bool fail() { return ok_ = false; }
  char peek() const { return p_ < e_ ? *p_ : '\0'; }
  bool eat(char c) {
    if (peek() != c) return false;
    ++p_;
    return true;
  }
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool str(std::string &s) {
    if (!eat('"')) return false;
    s.clear();
    while (p_ < e_ && *p_ != '"') {
      if (*p_ == '\\') {
        if (++p_ >= e_) return false;
        const char c = *p_;
        if (c == 'u') {  // \uXXXX: names are ASCII; keep the escape text
          if (e_ - p_ < 5) return false;
          s.append(p_ - 1, 6);
          p_ += 5;
          continue;
        }
        s.push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c);
        ++p_;
        continue;
      }
      s.push_back(*p_++);
    }
    return eat('"');
  }
  bool integer(int64_t &v) {
    bool neg = eat('-');
    if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
    v = 0;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
      if (v > (INT64_MAX - 9) / 10) return false;
      v = v * 10 + (*p_++ - '0');
    }
    if (neg) v = -v;
    return true;
  }
  bool int_array(std::vector<int64_t> &a) {
    if (!eat('[')) return false;
    ws();
    a.clear();
    if (eat(']')) return true;
    for (;;) {
      int64_t v;
      ws();
      if (!integer(v)) return false;
      a.push_back(v);
      ws();
      if (eat(',')) continue;
      return eat(']');
    }
  }
  bool tensor(StTensor &t) {
    if (!eat('{')) return false;
    bool got_dtype = false, got_shape = false, got_off = false;
    for (;;) {
      ws();
      std::string k;
      if (!str(k)) return false;
      ws();
      if (!eat(':')) return false;
      ws();
      if (k == "dtype") {
        if (!str(t.dtype)) return false;
        got_dtype = true;
      } else if (k == "shape") {
        if (!int_array(t.shape)) return false;
        got_shape = true;
      } else if (k == "data_offsets") {
        std::vector<int64_t> o;
        if (!int_array(o) || o.size() != 2) return false;
        t.begin = o[0];
        t.end = o[1];
        got_off = true;
      } else if (!skip()) {
        return false;
      }
      ws();
      if (eat(',')) continue;
      if (eat('}')) return got_dtype && got_shape && got_off;
      return false;
    }
  }
  bool skip() {  // any JSON value
    ws();
    const char c = peek();
    if (c == '"') {
      std::string s;
      return str(s);
    }
    if (c == '{' || c == '[') {
      const char close = c == '{' ? '}' : ']';
      ++p_;
      ws();
      if (eat(close)) return true;
      for (;;) {
        ws();
        if (c == '{') {
          std::string k;
          if (!str(k)) return false;
          ws();
          if (!eat(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (eat(',')) continue;
        return eat(close);
      }
    }
    while (p_ < e_ && *p_ != ',' && *p_ != '}' && *p_ != ']' && *p_ != ' ' && *p_ != '\n') ++p_;
    return true;
  }
};

// IEEE binary16 -> binary32, exact.
float half_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {  // subnormal: normalise
    int e = -1;
    do {
      ++e;
      man <<= 1;
    } while ((man & 0x400u) == 0);
    bits = sign | ((112 - e) << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

class StFile {
 public:
  ~StFile() {
    if (map_ && map_ != MAP_FAILED) munmap(map_, size_);
    if (fd_ >= 0) close(fd_);
  }
  int open_file(const char *path) {
    fd_ = open(path, O_RDONLY);
    if (fd_ < 0) return err("cannot open %s", path);
    struct stat st;
    if (fstat(fd_, &st) != 0 || st.st_size < 8) return err("%s is not a safetensors file", path);
    size_ = static_cast<size_t>(st.st_size);
    map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (map_ == MAP_FAILED) return err("cannot map %s", path);
    const unsigned char *b = static_cast<const unsigned char *>(map_);
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | b[i];
    if (n > size_ - 8) return err("%s: header length %llu exceeds the file", path, (unsigned long long)n);
    Json js(reinterpret_cast<const char *>(b + 8), reinterpret_cast<const char *>(b + 8 + n));
    if (!js.parse_header(tensors_) || !js.ok()) return err("%s: malformed safetensors header", path);
    data_ = b + 8 + n;
    data_size_ = size_ - 8 - n;
    for (auto &kv : tensors_) {
      const StTensor &t = kv.second;
      if (t.begin < 0 || t.end < t.begin || static_cast<uint64_t>(t.end) > data_size_)
        return err("%s: tensor %s has offsets outside the data", path, kv.first.c_str());
    }
    return 0;
  }
  // Copies tensor `name` (tried as given, then with each prefix) into out as
  // FP32 after checking its element count.
  int read(const std::vector<std::string> &names, int64_t numel, const std::vector<int64_t> &shape, float *out) {
    const StTensor *t = nullptr;
    std::string found;
    for (const std::string &n : names) {
      auto it = tensors_.find(n);
      if (it != tensors_.end()) {
        t = &it->second;
        found = n;
        break;
      }
    }
    if (!t) return err("tensor %s missing from the checkpoint", names[0].c_str());
    int64_t cnt = 1;
    for (int64_t d : t->shape) cnt *= d;
    if (cnt != numel || (!shape.empty() && t->shape != shape)) {
      std::string want, got;
      for (int64_t d : shape) want += std::to_string(d) + " ";
      for (int64_t d : t->shape) got += std::to_string(d) + " ";
      return err("tensor %s has shape [%s], expected [%s]", found.c_str(), got.c_str(), want.c_str());
    }
    const unsigned char *src = data_ + t->begin;
    const int64_t bytes = t->end - t->begin;
    if (t->dtype == "F32") {
      if (bytes != numel * 4) return err("tensor %s: %lld bytes for %lld F32 values", found.c_str(), (long long)bytes,
                                         (long long)numel);
      memcpy(out, src, static_cast<size_t>(bytes));
    } else if (t->dtype == "F16" || t->dtype == "BF16") {
      if (bytes != numel * 2) return err("tensor %s: %lld bytes for %lld 16-bit values", found.c_str(),
                                         (long long)bytes, (long long)numel);
      const bool bf = t->dtype == "BF16";
      for (int64_t i = 0; i < numel; ++i) {
        const uint16_t h = static_cast<uint16_t>(src[2 * i] | (src[2 * i + 1] << 8));
        if (bf) {
          const uint32_t bits = static_cast<uint32_t>(h) << 16;
          memcpy(&out[i], &bits, 4);
        } else {
          out[i] = half_to_float(h);
        }
      }
    } else {
      return err("tensor %s has dtype %s (F32, F16 or BF16 expected)", found.c_str(), t->dtype.c_str());
    }
    return 0;
  }

 private:
  int fd_ = -1;
  void *map_ = nullptr;
  size_t size_ = 0;
  const unsigned char *data_ = nullptr;
  uint64_t data_size_ = 0;
  std::map<std::string, StTensor> tensors_;

  template <typename... A>
  int err(const char *fmt, A... a) {
    set_error(fmt, a...);
    return -1;
  }
};

std::vector<std::string> candidates(const std::string &name, const char *prefix) {
  std::vector<std::string> c = {name, std::string(prefix) + name};
  // older BERT checkpoints name LayerNorm parameters gamma / beta
  const size_t ln = name.find("LayerNorm.");
  if (ln != std::string::npos) {
    std::string alt = name;
    if (alt.compare(alt.size() - 6, 6, "weight") == 0) alt.replace(alt.size() - 6, 6, "gamma");
    else if (alt.compare(alt.size() - 4, 4, "bias") == 0) alt.replace(alt.size() - 4, 4, "beta");
    c.push_back(alt);
    c.push_back(std::string(prefix) + alt);
  }
  return c;
}
}  // namespace

// GPT-2: transformers' GPT2LMHeadModel names without / with "transformer.".
int gpt2_safetensors_blob(const char *path, const ModelDims &m, float *blob) {
  StFile f;
  if (int r = f.open_file(path)) return r;
  const std::vector<TensorSpec> specs = blob_specs(m);
  const int64_t d = m.n_embd, ff = m.n_inner;
  std::vector<std::pair<std::string, std::vector<int64_t>>> names;
  names.push_back({"wte.weight", {m.vocab, d}});
  names.push_back({"wpe.weight", {m.n_pos, d}});
  for (int l = 0; l < m.n_layer; ++l) {
    const std::string h = "h." + std::to_string(l) + ".";
    names.push_back({h + "ln_1.weight", {d}});
    names.push_back({h + "ln_1.bias", {d}});
    names.push_back({h + "attn.c_attn.weight", {d, 3 * d}});
    names.push_back({h + "attn.c_attn.bias", {3 * d}});
    names.push_back({h + "attn.c_proj.weight", {d, d}});
    names.push_back({h + "attn.c_proj.bias", {d}});
    names.push_back({h + "ln_2.weight", {d}});
    names.push_back({h + "ln_2.bias", {d}});
    names.push_back({h + "mlp.c_fc.weight", {d, ff}});
    names.push_back({h + "mlp.c_fc.bias", {ff}});
    names.push_back({h + "mlp.c_proj.weight", {ff, d}});
    names.push_back({h + "mlp.c_proj.bias", {d}});
  }
  names.push_back({"ln_f.weight", {d}});
  names.push_back({"ln_f.bias", {d}});
  if (names.size() != specs.size()) {
    set_error("internal: GPT-2 name table does not match the blob layout");
    return -1;
  }
  for (size_t i = 0; i < specs.size(); ++i)
    if (int r = f.read(candidates(names[i].first, "transformer."), specs[i].numel, names[i].second,
                       blob + specs[i].offset))
      return r;
  return 0;
}

// BERT: transformers' BertModel names without / with "bert.".
int bert_safetensors_blob(const char *path, const BertDims &m, float *blob) {
  StFile f;
  if (int r = f.open_file(path)) return r;
  const std::vector<TensorSpec> specs = bert_blob_specs(m);
  const int64_t d = m.n_embd, ff = m.n_inner;
  std::vector<std::pair<std::string, std::vector<int64_t>>> names;
  names.push_back({"embeddings.word_embeddings.weight", {m.vocab, d}});
  names.push_back({"embeddings.position_embeddings.weight", {m.n_pos, d}});
  names.push_back({"embeddings.token_type_embeddings.weight", {m.type_vocab, d}});
  names.push_back({"embeddings.LayerNorm.weight", {d}});
  names.push_back({"embeddings.LayerNorm.bias", {d}});
  for (int l = 0; l < m.n_layer; ++l) {
    const std::string e = "encoder.layer." + std::to_string(l) + ".";
    for (const char *p : {"attention.self.query.", "attention.self.key.", "attention.self.value.",
                          "attention.output.dense."}) {
      names.push_back({e + p + "weight", {d, d}});
      names.push_back({e + p + "bias", {d}});
    }
    names.push_back({e + "attention.output.LayerNorm.weight", {d}});
    names.push_back({e + "attention.output.LayerNorm.bias", {d}});
    names.push_back({e + "intermediate.dense.weight", {ff, d}});
    names.push_back({e + "intermediate.dense.bias", {ff}});
    names.push_back({e + "output.dense.weight", {d, ff}});
    names.push_back({e + "output.dense.bias", {d}});
    names.push_back({e + "output.LayerNorm.weight", {d}});
    names.push_back({e + "output.LayerNorm.bias", {d}});
  }
  names.push_back({"pooler.dense.weight", {d, d}});
  names.push_back({"pooler.dense.bias", {d}});
  if (names.size() != specs.size()) {
    set_error("internal: BERT name table does not match the blob layout");
    return -1;
  }
  for (size_t i = 0; i < specs.size(); ++i)
    if (int r = f.read(candidates(names[i].first, "bert."), specs[i].numel, names[i].second, blob + specs[i].offset))
      return r;
  return 0;
}

}  // namespace gpt2
