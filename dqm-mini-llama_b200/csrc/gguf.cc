// gguf.cc -- GGUF v3 model files into a dqmk_model (C++17).
//
// The reference loads a GGUF in two steps (src/gguf.cc, the container
// reader; src/gguf_loader.cc:202-364, LoadGgufModel): it builds a ModelConfig
// from the qwen2.* (else llama.*) metadata, maps llama.cpp tensor names onto
// its own ("blk.N.attn_q.weight" -> "layers.N.wq", src/gguf_loader.cc:21-59),
// swaps the two dims of 2-D shapes (GGUF lists the innermost first), and
// dequantizes the token embedding to F32 -- plus an F32 copy as the lm_head
// when the file has no output.weight (src/gguf_loader.cc:313-326,356-360),
// 2 x 544.5 MB for Qwen2-0.5B.  Here the file is parsed once on the host and
// every tensor goes to dqmk_model_upload as it is stored: quantized linears
// and the token embedding stay Q8_0 / Q4_0 blocks (the engine gathers
// embedding rows and runs the tied lm_head straight from those blocks), F32
// norms and biases stay F32.  The metadata rules are the reference's: qwen2
// architecture => NeoX RoPE, vocabulary = length of tokenizer.ggml.tokens,
// head_dim = dim / n_heads, defaults RoPE base 10000 and epsilon 1e-5.
//
// Container layout (GGUF version 3, little endian): "GGUF", u32 version, u64
// tensor count, u64 metadata count; metadata (string key, u32 type, value);
// tensor infos (string name, u32 n_dims, u64 dims, u32 ggml type, u64 offset
// from the data section); the data section starts at the next multiple of
// general.alignment (default 32).  Strings are a u64 length and bytes.
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "dqmk.h"
#include "internal.h"

namespace dqmk {
namespace {

const char* kApi = "LoadGgufModel";

enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
  kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12
};
enum : uint32_t { kGgmlF32 = 0, kGgmlQ40 = 2, kGgmlQ41 = 3, kGgmlQ80 = 8 };

constexpr uint64_t kMaxString = 16u << 20;
constexpr uint64_t kMaxEntries = 1u << 20;

struct Value {
  uint32_t type = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint32_t elem_type = 0;  // arrays
  uint64_t count = 0;
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // innermost first
  uint32_t type = 0;
  uint64_t offset = 0;
};

struct File {
  std::FILE* f = nullptr;
  std::map<std::string, Value> kv;
  std::vector<TensorInfo> tensors;
  uint64_t data_offset = 0;
  ~File() {
    if (f) std::fclose(f);
  }
};

bool read_bytes(std::FILE* f, void* dst, size_t n) { return std::fread(dst, 1, n, f) == n; }

template <typename T>
bool read_le(std::FILE* f, T* v) {
  return read_bytes(f, v, sizeof(T));
}

bool read_string(std::FILE* f, std::string* s) {
  uint64_t n = 0;
  if (!read_le(f, &n) || n > kMaxString) return false;
  s->resize(n);
  return n == 0 || read_bytes(f, &(*s)[0], n);
}

size_t scalar_bytes(uint32_t t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
  }
}

bool read_scalar(std::FILE* f, uint32_t t, Value* v) {
  unsigned char b[8] = {};
  const size_t n = scalar_bytes(t);
  if (!n || !read_bytes(f, b, n)) return false;
  switch (t) {
    case kU8: v->i = b[0]; break;
    case kI8: v->i = (int8_t)b[0]; break;
    case kBool: v->i = b[0] != 0; break;
    case kU16: { uint16_t x; std::memcpy(&x, b, 2); v->i = x; break; }
    case kI16: { int16_t x; std::memcpy(&x, b, 2); v->i = x; break; }
    case kU32: { uint32_t x; std::memcpy(&x, b, 4); v->i = x; break; }
    case kI32: { int32_t x; std::memcpy(&x, b, 4); v->i = x; break; }
    case kF32: { float x; std::memcpy(&x, b, 4); v->f = x; break; }
    case kU64: { uint64_t x; std::memcpy(&x, b, 8); v->i = (int64_t)x; break; }
    case kI64: { int64_t x; std::memcpy(&x, b, 8); v->i = x; break; }
    case kF64: { double x; std::memcpy(&x, b, 8); v->f = x; break; }
  }
  if (t != kF32 && t != kF64) v->f = (double)v->i;
  return true;
}

int bad(const std::string& what) { return fail(DQMK_ERR_INVALID, std::string(kApi) + ": " + what); }

int open_file(const char* path, File* g) {
  g->f = std::fopen(path, "rb");
  if (!g->f) return bad(std::string("cannot open ") + path);
  char magic[4];
  uint32_t version = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!read_bytes(g->f, magic, 4) || std::memcmp(magic, "GGUF", 4) != 0)
    return bad("not a GGUF file");
  if (!read_le(g->f, &version) || version != 3) return bad("GGUF version 3 expected");
  if (!read_le(g->f, &n_tensors) || !read_le(g->f, &n_kv) || n_tensors > kMaxEntries ||
      n_kv > kMaxEntries)
    return bad("truncated or oversized header");
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    Value v;
    if (!read_string(g->f, &key) || !read_le(g->f, &v.type)) return bad("truncated metadata");
    if (v.type == kString) {
      if (!read_string(g->f, &v.s)) return bad("truncated metadata string");
    } else if (v.type == kArray) {
      if (!read_le(g->f, &v.elem_type) || !read_le(g->f, &v.count) || v.count > (1ull << 32))
        return bad("truncated metadata array");
      for (uint64_t j = 0; j < v.count; ++j) {  // contents are not needed, only the count
        if (v.elem_type == kString) {
          std::string s;
          if (!read_string(g->f, &s)) return bad("truncated metadata array");
        } else {
          Value e;
          if (!read_scalar(g->f, v.elem_type, &e)) return bad("unsupported metadata array");
        }
      }
    } else if (!read_scalar(g->f, v.type, &v)) {
      return bad("unsupported metadata type for " + key);
    }
    g->kv[key] = std::move(v);
  }
  g->tensors.resize(n_tensors);
  for (auto& t : g->tensors) {
    uint32_t nd = 0;
    if (!read_string(g->f, &t.name) || !read_le(g->f, &nd) || nd == 0 || nd > 4)
      return bad("truncated tensor info");
    t.dims.resize(nd);
    for (auto& d : t.dims)
      if (!read_le(g->f, &d)) return bad("truncated tensor info");
    if (!read_le(g->f, &t.type) || !read_le(g->f, &t.offset)) return bad("truncated tensor info");
  }
  uint64_t align = 32;
  auto it = g->kv.find("general.alignment");
  if (it != g->kv.end() && it->second.type != kString && it->second.i > 0) align = it->second.i;
  const long pos = std::ftell(g->f);
  if (pos < 0) return bad("cannot tell position");
  g->data_offset = ((uint64_t)pos + align - 1) / align * align;
  return DQMK_OK;
}

int64_t get_int(const File& g, const std::string& arch, const std::string& key, int64_t dflt) {
  for (const std::string& k : {arch + "." + key, "llama." + key}) {
    auto it = g.kv.find(k);
    if (it != g.kv.end() && it->second.type != kString && it->second.type != kArray)
      return it->second.i;
  }
  return dflt;
}

double get_float(const File& g, const std::string& arch, const std::string& key, double dflt) {
  for (const std::string& k : {arch + "." + key, "llama." + key}) {
    auto it = g.kv.find(k);
    if (it != g.kv.end() && it->second.type != kString && it->second.type != kArray)
      return it->second.f;
  }
  return dflt;
}

// BuildConfig (src/gguf_loader.cc:202-273).
int build_config(const File& g, dqmk_model_config* c) {
  auto a = g.kv.find("general.architecture");
  const bool qwen2 = a != g.kv.end() && a->second.type == kString && a->second.s == "qwen2";
  const std::string arch = "qwen2";
  *c = dqmk_model_config{};
  c->n_layers = (int)get_int(g, arch, "block_count", 0);
  c->dim = (int)get_int(g, arch, "embedding_length", 0);
  c->hidden_dim = (int)get_int(g, arch, "feed_forward_length", 0);
  c->n_heads = (int)get_int(g, arch, "attention.head_count", 0);
  c->n_kv_heads = (int)get_int(g, arch, "attention.head_count_kv", 0);
  c->max_seq_len = (int)get_int(g, arch, "context_length", 0);
  c->rope_theta = (float)get_float(g, arch, "rope.freq_base", 10000.0);
  c->rms_norm_eps = (float)get_float(g, arch, "attention.layer_norm_rms_epsilon", 1e-5);
  auto tok = g.kv.find("tokenizer.ggml.tokens");
  c->vocab_size = tok != g.kv.end() && tok->second.type == kArray ? (int)tok->second.count : 0;
  c->rope_neox = qwen2 ? 1 : 0;
  if (c->n_layers <= 0 || c->dim <= 0 || c->hidden_dim <= 0 || c->n_heads <= 0 ||
      c->n_kv_heads <= 0 || c->max_seq_len <= 0 || c->vocab_size <= 0)
    return bad("incomplete GGUF model config");
  if (c->dim % c->n_heads != 0) return bad("GGUF dim not divisible by n_heads");
  if (c->n_heads % c->n_kv_heads != 0) return bad("GGUF n_heads not divisible by n_kv_heads");
  c->head_dim = c->dim / c->n_heads;
  return DQMK_OK;
}

// MapTensorName (src/gguf_loader.cc:21-59): llama.cpp names -> the engine's.
std::string map_name(const std::string& n) {
  if (n == "token_embd.weight") return "token_embedding";
  if (n == "output_norm.weight") return "final_norm";
  if (n == "output.weight") return "lm_head";
  if (n.rfind("blk.", 0) != 0) return "";
  const size_t d1 = n.find('.', 4);
  if (d1 == std::string::npos) return "";
  const size_t d2 = n.find('.', d1 + 1);
  if (d2 == std::string::npos) return "";
  const std::string layer = n.substr(4, d1 - 4), op = n.substr(d1 + 1, d2 - d1 - 1),
                    suffix = n.substr(d2 + 1);
  static const std::map<std::string, std::string> weights = {
      {"attn_norm", "attention_norm"}, {"attn_q", "wq"}, {"attn_k", "wk"}, {"attn_v", "wv"},
      {"attn_output", "wo"}, {"ffn_norm", "ffn_norm"}, {"ffn_gate", "w_gate"},
      {"ffn_up", "w_up"}, {"ffn_down", "w_down"}};
  static const std::map<std::string, std::string> biases = {
      {"attn_q", "bq"}, {"attn_k", "bk"}, {"attn_v", "bv"}};
  const auto& table = suffix == "weight" ? weights : biases;
  if (suffix != "weight" && suffix != "bias") return "";
  auto it = table.find(op);
  return it == table.end() ? "" : "layers." + layer + "." + it->second;
}

}  // namespace
}  // namespace dqmk

using namespace dqmk;

extern "C" int dqmk_gguf_read_config(const char* path, dqmk_model_config* out) {
  if (!path || !out) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null argument");
  File g;
  int rc = open_file(path, &g);
  if (rc) return rc;
  return build_config(g, out);
}

extern "C" int dqmk_model_load_gguf(const char* path, int max_seq_len, int device_id,
                                    dqmk_model** out) {
  if (!path || !out) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null argument");
  File g;
  int rc = open_file(path, &g);
  if (rc) return rc;
  dqmk_model_config c;
  if ((rc = build_config(g, &c))) return rc;
  if (max_seq_len > 0) c.max_seq_len = max_seq_len;
  dqmk_model* m = nullptr;
  if ((rc = dqmk_model_create(&c, device_id, &m))) return rc;
  std::unique_ptr<dqmk_model, int (*)(dqmk_model*)> hold(m, dqmk_model_destroy);
  std::vector<unsigned char> buf;
  for (const TensorInfo& t : g.tensors) {
    const std::string name = map_name(t.name);
    if (name.empty()) continue;  // tensors the forward pass does not use
    uint64_t n = 1;
    for (uint64_t d : t.dims) n *= d;
    int qtype;
    uint64_t bytes;
    switch (t.type) {
      case kGgmlF32: qtype = DQMK_F32; bytes = n * 4; break;
      case kGgmlQ80: qtype = DQMK_Q80; bytes = (n + 31) / 32 * 34; break;
      case kGgmlQ40: qtype = DQMK_Q40; bytes = (n + 31) / 32 * 18; break;
      default:
        return fail(DQMK_ERR_UNSUPPORTED,
                    std::string(kApi) + ": tensor " + t.name + " has an unsupported ggml type " +
                        std::to_string(t.type) + " (F32, Q8_0 and Q4_0 are loaded)");
    }
    // 2-D: GGUF [in, out] -> [out, in] (src/gguf_loader.cc:65-75)
    const int rows = t.dims.size() == 2 ? (int)t.dims[1] : 1;
    const int cols = (int)t.dims[0];
    if (t.dims.size() > 2) return bad("tensor " + t.name + " has more than 2 dims");
    buf.resize(bytes);
    if (std::fseek(g.f, (long)(g.data_offset + t.offset), SEEK_SET) != 0 ||
        !read_bytes(g.f, buf.data(), bytes))
      return bad("failed to read tensor data: " + t.name);
    if ((rc = dqmk_model_upload(m, name.c_str(), qtype, buf.data(), bytes, rows, cols)))
      return rc;
  }
  if ((rc = dqmk_model_finalize(m))) return rc;
  *out = hold.release();
  return DQMK_OK;
}
