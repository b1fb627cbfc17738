// ref_shim.cc -- extern "C" handle onto the reference's own CPU code.
//
// TEST INFRASTRUCTURE.  oracle/Makefile compiles this file together with the
// reference's src/*.cc (everything but main.cc, built exactly as the
// reference's CMake Release build does: -O3 -mavx2 -mfma, GNU C++17) into
// oracle/_ref/libdqmref.so.  It pins the C restatement in dqm_oracle.c and
// serves as the CPU baseline that bench.py times.  The product never loads
// it.
//
// A model is assembled in memory the way the reference's GGUF loader leaves
// it (src/gguf_loader.cc:279-364): quantized linears as QuantizedTensor
// blocks, norms / biases as F32 Tensors, token_embedding as the F32
// dequantization of the token_embd blocks, and -- for a tied embedding --
// lm_head as an F32 copy of that table (gguf_loader.cc:356-360).
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "dqm_llama/batch.h"
#include "dqm_llama/context.h"
#include "dqm_llama/forward.h"
#include "dqm_llama/gguf_loader.h"
#include "dqm_llama/matmul_dispatch.h"
#include "dqm_llama/model.h"
#include "dqm_llama/ops.h"
#include "dqm_llama/quant.h"
#include "dqm_llama/thread_pool.h"

using namespace dqm;

namespace {

thread_local std::string g_err;

Tensor MakeTensor(const float* p, std::vector<int> shape) {
  Tensor t(shape, 0.0f);
  if (p) std::memcpy(t.data.data(), p, t.data.size() * sizeof(float));
  return t;
}

// qtype: 0 = F32, 1 = Q8_0, 2 = Q4_0 (same codes as dqm_oracle.h)
QuantizedTensor MakeQuant(int qtype, const void* p, int rows, int cols) {
  QuantizedTensor q;
  q.shape = {rows, cols};
  const size_t nb = static_cast<size_t>(rows) * static_cast<size_t>((cols + 31) / 32);
  if (qtype == 1) {
    q.type = QuantType::kQ80;
    q.q8_0_data.resize(nb);
    std::memcpy(q.q8_0_data.data(), p, nb * sizeof(BlockQ80));
  } else if (qtype == 2) {
    q.type = QuantType::kQ40;
    q.q4_0_data.resize(nb);
    std::memcpy(q.q4_0_data.data(), p, nb * sizeof(BlockQ40));
  } else if (qtype == 3) {
    q.type = QuantType::kQ41;
    q.q4_1_data.resize(nb);
    std::memcpy(q.q4_1_data.data(), p, nb * sizeof(BlockQ41));
  } else {
    q.type = QuantType::kF32;
    q.f32_data.resize(static_cast<size_t>(rows) * cols);
    std::memcpy(q.f32_data.data(), p, q.f32_data.size() * sizeof(float));
  }
  return q;
}

Tensor Shaped(const float* x, int rows, int cols) {
  return rows <= 1 ? MakeTensor(x, {cols}) : MakeTensor(x, {rows, cols});
}

template <typename F>
int Guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

struct RefSession {
  MiniLlamaModel model;
  std::unique_ptr<MiniLlamaContext> ctx;
};

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }
void ref_set_threads(int n) { SetThreadCount(n); }
int ref_get_threads() { return GetThreadCount(); }

int ref_quantize_q80(const float* src, int rows, int cols, void* out) {
  return Guard([&] {
    auto b = QuantizeToQ80(Shaped(src, rows, cols));
    std::memcpy(out, b.data(), b.size() * sizeof(BlockQ80));
  });
}

int ref_quantize_q40(const float* src, int rows, int cols, void* out) {
  return Guard([&] {
    auto b = QuantizeToQ40(Shaped(src, rows, cols));
    std::memcpy(out, b.data(), b.size() * sizeof(BlockQ40));
  });
}

int ref_dequantize_q80(const void* blocks, int rows, int cols, float* out) {
  return Guard([&] {
    QuantizedTensor q = MakeQuant(1, blocks, rows, cols);
    Tensor t = DequantizeFromQ80(q.q8_0_data, rows <= 1 ? std::vector<int>{cols}
                                                        : std::vector<int>{rows, cols});
    std::memcpy(out, t.data.data(), t.data.size() * sizeof(float));
  });
}

int ref_dequantize_q40(const void* blocks, int rows, int cols, float* out) {
  return Guard([&] {
    QuantizedTensor q = MakeQuant(2, blocks, rows, cols);
    Tensor t = DequantizeFromQ40(q.q4_0_data, rows <= 1 ? std::vector<int>{cols}
                                                        : std::vector<int>{rows, cols});
    std::memcpy(out, t.data.data(), t.data.size() * sizeof(float));
  });
}

int ref_dequantize_q41(const void* blocks, int rows, int cols, float* out) {
  return Guard([&] {
    QuantizedTensor q = MakeQuant(3, blocks, rows, cols);
    Tensor t = DequantizeFromQ41(q.q4_1_data, rows <= 1 ? std::vector<int>{cols}
                                                        : std::vector<int>{rows, cols});
    std::memcpy(out, t.data.data(), t.data.size() * sizeof(float));
  });
}

// x: [rows, in] (rows == 1 -> 1-D input), weights [out, in] in blocks.
int ref_linear(int qtype, const float* x, int rows, int in, const void* w,
               int out, float* y) {
  return Guard([&] {
    QuantizedTensor q = MakeQuant(qtype, w, out, in);
    Tensor r = LinearDispatch(Shaped(x, rows, in), q, DefaultMatmulMode());
    std::memcpy(y, r.data.data(), r.data.size() * sizeof(float));
  });
}

int ref_rmsnorm(const float* x, const float* w, int dim, float eps, float* y) {
  return Guard([&] {
    Tensor r = RmsNorm(MakeTensor(x, {dim}), MakeTensor(w, {dim}), eps);
    std::memcpy(y, r.data.data(), r.data.size() * sizeof(float));
  });
}

int ref_rope(float* q, int n_heads, float* k, int n_kv_heads, int head_dim,
             int pos, float theta, int neox) {
  return Guard([&] {
    Tensor tq = MakeTensor(q, {n_heads, head_dim});
    Tensor tk = MakeTensor(k, {n_kv_heads, head_dim});
    Rope(tq, tk, pos, theta, neox ? RopeType::kNeoX : RopeType::kNormal);
    std::memcpy(q, tq.data.data(), tq.data.size() * sizeof(float));
    std::memcpy(k, tk.data.data(), tk.data.size() * sizeof(float));
  });
}

int ref_softmax(const float* x, int n, float* y) {
  return Guard([&] {
    Tensor r = Softmax(MakeTensor(x, {n}));
    std::memcpy(y, r.data.data(), r.data.size() * sizeof(float));
  });
}

int ref_swiglu(const float* g, const float* u, int n, float* y) {
  return Guard([&] {
    Tensor r = SwiGlu(MakeTensor(g, {n}), MakeTensor(u, {n}));
    std::memcpy(y, r.data.data(), r.data.size() * sizeof(float));
  });
}

int ref_argmax(const float* x, int n) { return ArgMax(MakeTensor(x, {n})); }

// ---- whole model ----------------------------------------------------------

void* ref_model_create(int vocab, int dim, int hidden, int n_layers,
                       int n_heads, int n_kv_heads, int max_seq,
                       float rope_theta, float eps, int rope_neox) {
  auto* s = new RefSession();
  ModelConfig& c = s->model.config;
  c.vocab_size = vocab;
  c.dim = dim;
  c.hidden_dim = hidden;
  c.n_layers = n_layers;
  c.n_heads = n_heads;
  c.n_kv_heads = n_kv_heads;
  c.head_dim = dim / n_heads;
  c.max_seq_len = max_seq;
  c.rope_theta = rope_theta;
  c.rms_norm_eps = eps;
  c.rope_type = rope_neox ? RopeType::kNeoX : RopeType::kNormal;
  s->model.layers.resize(static_cast<size_t>(n_layers));
  return s;
}

void ref_model_destroy(void* h) { delete static_cast<RefSession*>(h); }

// Token embedding given as quantized blocks (qtype 1/2) or F32 (qtype 0);
// stored F32 like load_f32 does (gguf_loader.cc:313-326).  When tied != 0,
// lm_head becomes an F32 copy (gguf_loader.cc:356-360).
int ref_model_set_embedding(void* h, int qtype, const void* data, int tied) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] {
    const ModelConfig& c = s->model.config;
    QuantizedTensor q = MakeQuant(qtype, data, c.vocab_size, c.dim);
    switch (q.type) {
      case QuantType::kQ80:
        s->model.token_embedding = DequantizeFromQ80(q.q8_0_data, q.shape);
        break;
      case QuantType::kQ40:
        s->model.token_embedding = DequantizeFromQ40(q.q4_0_data, q.shape);
        break;
      default:
        s->model.token_embedding = ToTensor(q);
        break;
    }
    if (tied) s->model.lm_head = ToQuantizedTensor(s->model.token_embedding);
  });
}

int ref_model_set_lm_head(void* h, int qtype, const void* data) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] {
    const ModelConfig& c = s->model.config;
    s->model.lm_head = MakeQuant(qtype, data, c.vocab_size, c.dim);
  });
}

int ref_model_set_final_norm(void* h, const float* w) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] { s->model.final_norm = MakeTensor(w, {s->model.config.dim}); });
}

// Biases may be NULL (models without attention bias).
int ref_model_set_layer(void* h, int layer, int qtype, const float* attn_norm,
                        const void* wq, const void* wk, const void* wv,
                        const float* bq, const float* bk, const float* bv,
                        const void* wo, const float* ffn_norm,
                        const void* w_gate, const void* w_up,
                        const void* w_down) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] {
    const ModelConfig& c = s->model.config;
    const int qd = c.n_heads * c.head_dim;
    const int kvd = c.n_kv_heads * c.head_dim;
    LayerWeights& lw = s->model.layers.at(static_cast<size_t>(layer));
    lw.attention_norm = MakeTensor(attn_norm, {c.dim});
    lw.wq = MakeQuant(qtype, wq, qd, c.dim);
    lw.wk = MakeQuant(qtype, wk, kvd, c.dim);
    lw.wv = MakeQuant(qtype, wv, kvd, c.dim);
    lw.bq = bq ? MakeTensor(bq, {qd}) : Tensor{};
    lw.bk = bk ? MakeTensor(bk, {kvd}) : Tensor{};
    lw.bv = bv ? MakeTensor(bv, {kvd}) : Tensor{};
    lw.wo = MakeQuant(qtype, wo, c.dim, qd);
    lw.ffn_norm = MakeTensor(ffn_norm, {c.dim});
    lw.w_gate = MakeQuant(qtype, w_gate, c.hidden_dim, c.dim);
    lw.w_up = MakeQuant(qtype, w_up, c.hidden_dim, c.dim);
    lw.w_down = MakeQuant(qtype, w_down, c.dim, c.hidden_dim);
  });
}

int ref_model_finish(void* h) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] {
    s->model.loaded = true;
    s->ctx = std::make_unique<MiniLlamaContext>(&s->model);
  });
}

// The reference's own GGUF path (src/gguf_loader.cc:279-364, LoadGgufModel):
// returns a session over the loaded model, or NULL with ref_last_error set.
// cfg_out (optional): vocab, dim, hidden, layers, heads, kv heads, max_seq,
// rope neox.
void* ref_model_load_gguf(const char* path, int* cfg_out) {
  auto* s = new RefSession();
  int rc = Guard([&] {
    s->model = LoadGgufModel(path);
    if (!s->model.loaded) throw std::runtime_error("LoadGgufModel: " + s->model.load_error);
    const ModelConfig& c = s->model.config;
    if (cfg_out) {
      const int v[8] = {c.vocab_size, c.dim, c.hidden_dim, c.n_layers, c.n_heads,
                        c.n_kv_heads, c.max_seq_len, c.rope_type == RopeType::kNeoX ? 1 : 0};
      std::memcpy(cfg_out, v, sizeof(v));
    }
    s->ctx = std::make_unique<MiniLlamaContext>(&s->model);
  });
  if (rc != 0) {
    delete s;
    return nullptr;
  }
  return s;
}

// Fresh context (empty KV cache, pos 0, empty history).
int ref_context_reset(void* h) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] { s->ctx = std::make_unique<MiniLlamaContext>(&s->model); });
}

// ForwardBatch over n tokens at positions start_pos.. (src/batch.cc:26-42);
// writes the last token's logits.
int ref_forward_batch(void* h, const int* tokens, int n, int start_pos,
                      float* logits) {
  auto* s = static_cast<RefSession*>(h);
  return Guard([&] {
    std::vector<int> toks(tokens, tokens + n);
    Tensor r = ForwardBatch(*s->ctx, s->model, MiniBatch::FromTokens(toks, start_pos));
    std::memcpy(logits, r.data.data(), r.data.size() * sizeof(float));
  });
}

int ref_context_pos(void* h) { return static_cast<RefSession*>(h)->ctx->pos; }

int ref_context_history(void* h, int* out, int cap) {
  auto* s = static_cast<RefSession*>(h);
  const auto& th = s->ctx->token_history;
  const int n = static_cast<int>(th.size());
  for (int i = 0; i < n && i < cap; ++i) out[i] = th[static_cast<size_t>(i)];
  return n;
}

}  // extern "C"
