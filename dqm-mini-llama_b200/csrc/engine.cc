// engine.cc -- device-resident decode engine behind the dqmk C ABI (C++17).
//
// Mirrors the reference's CUDA branch of ForwardToken (src/forward.cc:667-754)
// with the same inputs and outputs, restructured for the B200:
//   * weights are repacked once at finalize into planar fused layouts:
//     q|k|v rows concatenated and paired for RoPE, gate/up rows interleaved
//     for the SwiGLU epilogue, the tied token_embd blocks kept quantized and
//     reused as lm_head (the reference expands them to F32 twice,
//     src/gguf_loader.cc:313-326,356-360);
//   * one decode step is 1 + 5 * n_layers + 1 kernels on the context's own
//     stream (embed; per layer QKV, attention, O, gate/up, down; lm_head),
//     every kernel after the first launched with programmatic dependent
//     launch, and the whole step captured once into a CUDA graph;
//   * token and position live in device memory, so the graph replays for
//     every step; greedy decoding advances them on the device.
// Runtime counters follow the reference's per-logical-op accounting
// (src/forward.cc:97-165) so the engine's counter tests still hold.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "dqmk.h"
#include "internal.h"
#include "model.h"
#include "prefill.h"
#include "tp.h"

using namespace dqmk;

namespace {

// Per-context buffers of the batched prefill, allocated on first use.
struct PrefillBufs {
  int m_max = 0;  // rows per chunk
  float *x = nullptr, *q = nullptr, *att = nullptr, *f = nullptr;
  uint16_t *hi = nullptr, *lo = nullptr;  // fp16 activation planes [m_max][kp]
  float* rs = nullptr;                    // their row scales [m_max]
  float* partial = nullptr;               // split-K partial sums
  float* attn_part = nullptr;             // split causal attention: partial rows
  unsigned int* attn_tickets = nullptr;   // and per-block tickets (left zero by every launch)
  int* tokens = nullptr;
  CUtensorMap a_dim[2], a_qd[2], a_hid[2];  // {hi, lo} per K
};

}  // namespace

struct dqmk_context {
  dqmk_model* m = nullptr;
  cudaStream_t stream = nullptr;
  float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
  float* part = nullptr;        // tensor parallel: row-parallel partial sums [dim]
  float* logits_all = nullptr;  // tensor parallel: gathered logits [world][vocab_stride]
  // tensor parallel over peer memory: this rank's exchange buffer (its own
  // allocation, exported by IPC), the device array of every rank's mapping,
  // exchange counters [2] + the writers' CTA ticket; p2p once connected
  char* tp_buf = nullptr;
  char** peer_base = nullptr;
  unsigned int* tp_seq = nullptr;
  bool p2p = false;
  // a peer wait of this context ran out: the ranks' exchange counters and
  // parity slots may disagree from then on, so the context refuses to run
  bool tp_failed = false;
  // failure-detection hook: lm_head tile withheld in captured steps (-1: none)
  int lm_withhold = -1;
  std::vector<void*> ipc_opened;
  float *keys = nullptr, *values = nullptr, *partials = nullptr;
  // device state block: [argmax u64][lm ticket u32][token i32][pos i32][pad]
  //                     [attention tickets u32 x n_kv][pad]
  unsigned char* state = nullptr;
  int* history_dev = nullptr;
  int* pinned = nullptr;  // host staging: [token, pos]
  // host landing area of a greedy call: [max_seq tokens][3 error flag words],
  // and the device addresses of those flag words
  int* pinned_out = nullptr;
  unsigned int* flag_dev[3] = {nullptr, nullptr, nullptr};
  cudaEvent_t staged = nullptr;  // recorded after the last copy out of `pinned`
  int attn_splits = 1;
  PrefillBufs pf;
  cudaGraphExec_t graph = nullptr;
  int pos = 0;
  std::vector<int> history;
  std::vector<void*> allocs;

  unsigned long long* argmax_slot() { return reinterpret_cast<unsigned long long*>(state); }
  unsigned int* lm_ticket() { return reinterpret_cast<unsigned int*>(state + 8); }
  int* token_slot() { return reinterpret_cast<int*>(state + 12); }
  int* pos_slot() { return reinterpret_cast<int*>(state + 16); }
  unsigned int* attn_tickets() { return reinterpret_cast<unsigned int*>(state + 64); }

  ~dqmk_context() {
    cudaSetDevice(m ? m->device : 0);
    if (graph) cudaGraphExecDestroy(graph);
    for (void* p : ipc_opened) cudaIpcCloseMemHandle(p);
    if (staged) cudaEventDestroy(staged);
    if (stream) cudaStreamDestroy(stream);
    for (void* p : allocs) cudaFree(p);
    if (pinned) cudaFreeHost(pinned);
    if (pinned_out) cudaFreeHost(pinned_out);
  }
};

namespace dqmk {

// Reference float arithmetic for the RoPE angles (src/ops.cc:18-23 and
// :40-45): freq_i = 1 / pow(theta, (2i)/head_dim) in float, angle = pos *
// freq_i, then float cos / sin.  Compiled by the host compiler against the
// same libm as the reference, so the table matches it bit for bit.
void rope_table(float theta, int head_dim, int pos_begin, int pos_count, float2* out) {
  const int half = head_dim / 2;
  for (int p = 0; p < pos_count; ++p) {
    for (int i = 0; i < half; ++i) {
      const float freq =
          1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(head_dim));
      const float angle = static_cast<float>(pos_begin + p) * freq;
      out[(size_t)p * half + i] = make_float2(std::cos(angle), std::sin(angle));
    }
  }
}

}  // namespace dqmk

int dqmk::dev_alloc(std::vector<void*>& owner, size_t bytes, void** out, const char* api) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(api, e);
  owner.push_back(p);
  *out = p;
  return DQMK_OK;
}

namespace {

size_t block_bytes(int qtype) { return qtype == DQMK_Q80 ? 34 : 18; }

// Gather ggml rows from up to three sources (concatenated in order) through
// a row map into one packed weight.
int pack_rows(dqmk_model* m, const std::vector<const Raw*>& srcs, const std::vector<int>& map,
              Packed* out, const char* api) {
  const int qt = srcs[0]->qtype;
  const int cols = srcs[0]->cols;
  const int nb = (cols + 31) / 32;
  const size_t row_b = (size_t)nb * block_bytes(qt);
  int total = 0;
  for (const Raw* r : srcs) total += r->rows;
  // concatenate the sources in the map's order into one ggml buffer
  void* tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, row_b * map.size());
  if (e != cudaSuccess) return cuda_fail(api, e);
  std::vector<std::pair<const Raw*, int>> where(total);
  int off = 0;
  for (const Raw* r : srcs) {
    for (int i = 0; i < r->rows; ++i) where[off + i] = {r, i};
    off += r->rows;
  }
  // copy runs of consecutive rows with one memcpy each
  size_t i = 0;
  while (i < map.size()) {
    const Raw* src = where[map[i]].first;
    const int r0 = where[map[i]].second;
    size_t j = i + 1;
    while (j < map.size() && where[map[j]].first == src && where[map[j]].second == r0 + (int)(j - i))
      ++j;
    e = cudaMemcpy(static_cast<char*>(tmp) + i * row_b,
                   static_cast<const char*>(src->dev) + (size_t)r0 * row_b, (j - i) * row_b,
                   cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) {
      cudaFree(tmp);
      return cuda_fail(api, e);
    }
    i = j;
  }
  out->qtype = qt;
  out->rows = (int)map.size();
  out->k = cols;
  out->kp = nb * 32;
  out->bytes = packed_bytes(qt, out->rows, cols);
  void* p = nullptr;
  int rc = dev_alloc(m->allocs, out->bytes, &p, api);
  if (rc != DQMK_OK) {
    cudaFree(tmp);
    return rc;
  }
  out->base = static_cast<uint8_t*>(p);
  e = launch_pack(qt, tmp, out->rows, cols, out->base, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(tmp);
  if (e != cudaSuccess) return cuda_fail(api, e);
  m->memory_bytes += out->bytes;
  return DQMK_OK;
}

int upload_f32(dqmk_model* m, const std::vector<float>& host, float** out, const char* api) {
  void* p = nullptr;
  int rc = dev_alloc(m->allocs, host.size() * sizeof(float), &p, api);
  if (rc != DQMK_OK) return rc;
  cudaError_t e = cudaMemcpy(p, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(api, e);
  *out = static_cast<float*>(p);
  m->memory_bytes += host.size() * sizeof(float);
  return DQMK_OK;
}

std::vector<int> identity_map(int n) {
  std::vector<int> v(n);
  for (int i = 0; i < n; ++i) v[i] = i;
  return v;
}

// Row order of the fused q|k|v weight: each RoPE pair adjacent.  NeoX pairs
// (i, i + hd/2) of every head, Normal pairs (2i, 2i+1); V rows keep their
// natural adjacent pairs.  Only the heads of the tensor-parallel shard.
std::vector<int> qkv_map(const dqmk_model_config& c, const dqmk_tp_plan& tp) {
  const int hd = c.head_dim, half = hd / 2;
  std::vector<int> map;
  auto add_heads = [&](int base, int head0, int n_heads, bool rope) {
    for (int h = head0; h < head0 + n_heads; ++h)
      for (int i = 0; i < half; ++i) {
        if (rope && c.rope_neox) {
          map.push_back(base + h * hd + i);
          map.push_back(base + h * hd + i + half);
        } else {
          map.push_back(base + h * hd + 2 * i);
          map.push_back(base + h * hd + 2 * i + 1);
        }
      }
  };
  const int qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
  add_heads(0, tp.q_head0, tp.n_q_heads, true);
  add_heads(qd, tp.kv_head0, tp.n_kv_heads, true);
  add_heads(qd + kvd, tp.kv_head0, tp.n_kv_heads, false);
  return map;
}

// Columns [c0, c0 + n) of every row of a quantized weight (c0 and n multiples
// of 32) as a new temporary Raw whose device blocks the caller frees.
int slice_cols(const Raw& r, int c0, int n, Raw* out, const char* api) {
  const size_t bb = block_bytes(r.qtype);
  const int nb = (r.cols + 31) / 32, nbl = (n + 31) / 32;
  out->qtype = r.qtype;
  out->rows = r.rows;
  out->cols = n;
  cudaError_t e = cudaMalloc(&out->dev, (size_t)r.rows * nbl * bb);
  if (e != cudaSuccess) return cuda_fail(api, e);
  e = cudaMemcpy2D(out->dev, nbl * bb, static_cast<const char*>(r.dev) + (size_t)(c0 / 32) * bb,
                   nb * bb, nbl * bb, r.rows, cudaMemcpyDeviceToDevice);
  if (e != cudaSuccess) {
    cudaFree(out->dev);
    out->dev = nullptr;
    return cuda_fail(api, e);
  }
  return DQMK_OK;
}

// Rows [r0, r0 + n) map.
std::vector<int> range_map(int r0, int n) {
  std::vector<int> v(n);
  for (int i = 0; i < n; ++i) v[i] = r0 + i;
  return v;
}

int check_model(const dqmk_model* m, const char* api) {
  if (!m) return fail(DQMK_ERR_INVALID, std::string(api) + ": null model");
  return DQMK_OK;
}

}  // namespace

// ------------------------------------------------------------------ model
extern "C" int dqmk_model_create(const dqmk_model_config* config, int device_id,
                                 dqmk_model** out) {
  const char* api = "UploadModelWeightsToCuda";
  if (!config || !out) return fail(DQMK_ERR_INVALID, std::string(api) + ": null argument");
  const dqmk_model_config& c = *config;
  if (c.vocab_size <= 0 || c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 ||
      c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.max_seq_len <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid model config");
  if (c.n_heads % c.n_kv_heads != 0 || c.head_dim % 4 != 0 || c.head_dim > 256 ||
      c.n_heads / c.n_kv_heads > 8)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": unsupported head configuration");
  int n_dev = 0;
  cudaError_t e = cudaGetDeviceCount(&n_dev);
  if (e != cudaSuccess) return cuda_fail(api, e);
  if (device_id < 0 || device_id >= n_dev)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid device id");
  auto* m = new dqmk_model();
  m->cfg = c;
  m->device = device_id;
  m->tp = dqmk_tp_plan{0, 1, 0, c.n_heads, 0, c.n_kv_heads, 0, c.hidden_dim,
                       0, c.vocab_size, c.vocab_size};
  *out = m;
  return DQMK_OK;
}

extern "C" int dqmk_model_destroy(dqmk_model* model) {
  delete model;
  return DQMK_OK;
}

extern "C" int dqmk_model_set_tp(dqmk_model* m, int rank, int world, const unsigned char* id) {
  const char* api = "dqmk_model_set_tp";
  int rc = check_model(m, api);
  if (rc) return rc;
  if (m->finalized) return fail(DQMK_ERR_INVALID, std::string(api) + ": model already finalized");
  if (m->comm) return fail(DQMK_ERR_INVALID, std::string(api) + ": already set");
  dqmk_tp_plan plan;
  if ((rc = tp_plan(m->cfg, rank, world, &plan))) return rc;
  if (world > 1) {
    if (!id) return fail(DQMK_ERR_INVALID, std::string(api) + ": null NCCL id");
    cudaSetDevice(m->device);
    if ((rc = tp_comm_create(rank, world, id, &m->comm))) return rc;
  }
  m->tp = plan;
  return DQMK_OK;
}

extern "C" int dqmk_model_upload(dqmk_model* m, const char* name, int qtype, const void* data,
                                 size_t bytes, int rows, int cols) {
  const char* api = "UploadModelWeightsToCuda";
  int rc = check_model(m, api);
  if (rc) return rc;
  if (!name || !data) return fail(DQMK_ERR_INVALID, std::string(api) + ": null argument");
  if (m->finalized) return fail(DQMK_ERR_INVALID, std::string(api) + ": model already finalized");
  if (rows <= 0 || cols <= 0) return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape for " + name);
  cudaSetDevice(m->device);
  Raw r;
  r.qtype = qtype;
  r.rows = rows;
  r.cols = cols;
  if (qtype == DQMK_F32) {
    if (bytes != (size_t)rows * cols * sizeof(float))
      return fail(DQMK_ERR_INVALID, std::string(api) + ": size mismatch for " + name);
    r.host.resize((size_t)rows * cols);
    cudaError_t e = cudaMemcpy(r.host.data(), data, bytes, cudaMemcpyDefault);
    if (e != cudaSuccess) return cuda_fail(api, e);
  } else if (qtype == DQMK_Q80 || qtype == DQMK_Q40) {
    const size_t expected = (size_t)rows * ((cols + 31) / 32) * block_bytes(qtype);
    if (bytes != expected)
      return fail(DQMK_ERR_INVALID, std::string("CUDA weight upload: block count mismatch for ") +
                                        name + ", expected " +
                                        std::to_string(expected / block_bytes(qtype)) + ", got " +
                                        std::to_string(bytes / block_bytes(qtype)));
    if (m->qtype == 0 && std::string(name) != "token_embedding") m->qtype = qtype;
    cudaError_t e = cudaMalloc(&r.dev, bytes);
    if (e != cudaSuccess) return cuda_fail(api, e);
    e = cudaMemcpy(r.dev, data, bytes, cudaMemcpyDefault);
    if (e != cudaSuccess) {
      cudaFree(r.dev);
      return cuda_fail(api, e);
    }
  } else {
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": unsupported weight type for " + name);
  }
  auto it = m->raw.find(name);
  if (it != m->raw.end() && it->second.dev) cudaFree(it->second.dev);
  m->raw[name] = std::move(r);
  m->stats.uploaded_weight_count += 1;
  m->stats.uploaded_bytes += bytes;
  return DQMK_OK;
}

extern "C" int dqmk_model_finalize(dqmk_model* m) {
  const char* api = "UploadModelWeightsToCuda";
  int rc = check_model(m, api);
  if (rc) return rc;
  if (m->finalized) return DQMK_OK;
  cudaSetDevice(m->device);
  const dqmk_model_config& c = m->cfg;
  const int hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
  auto need = [&](const std::string& n, int qt_expect, int rows, int cols,
                  const Raw** out) -> int {
    auto it = m->raw.find(n);
    if (it == m->raw.end())
      return fail(DQMK_ERR_INVALID, "CUDA forward missing uploaded weight: " + n);
    const Raw& r = it->second;
    if (qt_expect >= 0 && ((qt_expect == DQMK_F32) != (r.qtype == DQMK_F32)))
      return fail(DQMK_ERR_INVALID, "CUDA forward unsupported weight type: " + n);
    if (r.rows * r.cols != rows * cols || (r.qtype != DQMK_F32 && (r.rows != rows || r.cols != cols)))
      return fail(DQMK_ERR_INVALID, "CUDA forward uploaded weight shape mismatch: " + n);
    *out = &r;
    return DQMK_OK;
  };
  const Raw* emb = nullptr;
  if ((rc = need("token_embedding", 1, c.vocab_size, c.dim, &emb))) return rc;
  if (m->qtype == 0) m->qtype = emb->qtype;
  const Raw* fn = nullptr;
  if ((rc = need("final_norm", DQMK_F32, 1, c.dim, &fn))) return rc;
  if ((rc = upload_f32(m, fn->host, &m->final_norm, api))) return rc;
  if ((rc = pack_rows(m, {emb}, identity_map(c.vocab_size), &m->embd, api))) return rc;
  const dqmk_tp_plan& tp = m->tp;
  auto lm = m->raw.find("lm_head");
  m->tied = lm == m->raw.end();
  if (!m->tied) {
    const Raw* l = nullptr;
    if ((rc = need("lm_head", 1, c.vocab_size, c.dim, &l))) return rc;
    if ((rc = pack_rows(m, {l}, range_map(tp.vocab0, tp.vocab), &m->lm_head, api))) return rc;
  } else if (tp.world > 1) {
    // vocabulary-parallel slice of the tied embedding blocks
    if ((rc = pack_rows(m, {emb}, range_map(tp.vocab0, tp.vocab), &m->lm_head, api))) return rc;
  } else {
    m->lm_head = m->embd;
  }
  m->layers.resize(c.n_layers);
  const std::vector<int> qmap = qkv_map(c, tp);
  std::vector<int> gmap(2 * tp.hidden);
  for (int o = 0; o < tp.hidden; ++o) {
    gmap[2 * o] = tp.hidden0 + o;
    gmap[2 * o + 1] = c.hidden_dim + tp.hidden0 + o;
  }
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    Layer& L = m->layers[l];
    const Raw *an, *wq, *wk, *wv, *wo, *ffn, *wg, *wu, *wd;
    if ((rc = need(p + "attention_norm", DQMK_F32, 1, c.dim, &an))) return rc;
    if ((rc = need(p + "wq", 1, qd, c.dim, &wq))) return rc;
    if ((rc = need(p + "wk", 1, kvd, c.dim, &wk))) return rc;
    if ((rc = need(p + "wv", 1, kvd, c.dim, &wv))) return rc;
    if ((rc = need(p + "wo", 1, c.dim, qd, &wo))) return rc;
    if ((rc = need(p + "ffn_norm", DQMK_F32, 1, c.dim, &ffn))) return rc;
    if ((rc = need(p + "w_gate", 1, c.hidden_dim, c.dim, &wg))) return rc;
    if ((rc = need(p + "w_up", 1, c.hidden_dim, c.dim, &wu))) return rc;
    if ((rc = need(p + "w_down", 1, c.dim, c.hidden_dim, &wd))) return rc;
    for (const Raw* r : {wq, wk, wv, wo, wg, wu, wd})
      if (r->qtype != m->qtype)
        return fail(DQMK_ERR_UNSUPPORTED, "CUDA forward: mixed quant types in " + p);
    if ((rc = upload_f32(m, an->host, &L.attn_norm, api))) return rc;
    if ((rc = upload_f32(m, ffn->host, &L.ffn_norm, api))) return rc;
    if ((rc = pack_rows(m, {wq, wk, wv}, qmap, &L.qkv, api))) return rc;
    if ((rc = pack_rows(m, {wg, wu}, gmap, &L.gate_up, api))) return rc;
    if (tp.world == 1) {
      if ((rc = pack_rows(m, {wo}, identity_map(c.dim), &L.wo, api))) return rc;
      if ((rc = pack_rows(m, {wd}, identity_map(c.dim), &L.down, api))) return rc;
    } else {  // row-parallel: this shard's K columns
      Raw so, sd;
      if ((rc = slice_cols(*wo, tp.q_head0 * hd, tp.n_q_heads * hd, &so, api))) return rc;
      rc = pack_rows(m, {&so}, identity_map(c.dim), &L.wo, api);
      cudaFree(so.dev);
      if (rc) return rc;
      if ((rc = slice_cols(*wd, tp.hidden0, tp.hidden, &sd, api))) return rc;
      rc = pack_rows(m, {&sd}, identity_map(c.dim), &L.down, api);
      cudaFree(sd.dev);
      if (rc) return rc;
    }
    // optional QKV bias, permuted like the rows
    auto bq = m->raw.find(p + "bq"), bk = m->raw.find(p + "bk"), bv = m->raw.find(p + "bv");
    const bool any = bq != m->raw.end() || bk != m->raw.end() || bv != m->raw.end();
    if (any) {
      std::vector<float> cat((size_t)qd + 2 * kvd, 0.0f);
      auto put = [&](decltype(bq) it, int off, int n, const char* nm) -> int {
        if (it == m->raw.end()) return DQMK_OK;
        if ((int)it->second.host.size() != n)
          return fail(DQMK_ERR_INVALID, "CUDA forward bias uploaded weight shape mismatch: " + p + nm);
        std::memcpy(cat.data() + off, it->second.host.data(), n * sizeof(float));
        return DQMK_OK;
      };
      if ((rc = put(bq, 0, qd, "bq"))) return rc;
      if ((rc = put(bk, qd, kvd, "bk"))) return rc;
      if ((rc = put(bv, qd + kvd, kvd, "bv"))) return rc;
      std::vector<float> perm(qmap.size());
      for (size_t i = 0; i < qmap.size(); ++i) perm[i] = cat[qmap[i]];
      if ((rc = upload_f32(m, perm, &L.qkv_bias, api))) return rc;
    }
  }
  // batched-prefill side tables (see prefill.cu) are built on the first
  // batched ForwardBatch; head sizes the prefill attention kernel does not
  // take, and tensor-parallel shards, prefill token by token
  m->prefill_eligible = (hd == 64 || hd == 128) && tp.world == 1 && c.dim % 4 == 0;

  // RoPE table for every cache position
  std::vector<float2> cs((size_t)c.max_seq_len * (hd / 2));
  rope_table(c.rope_theta, hd, 0, c.max_seq_len, cs.data());
  void* p = nullptr;
  if ((rc = dev_alloc(m->allocs, cs.size() * sizeof(float2), &p, api))) return rc;
  cudaError_t e = cudaMemcpy(p, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(api, e);
  m->rope_cs = static_cast<float2*>(p);
  // raw ggml copies are no longer needed
  for (auto& kv : m->raw)
    if (kv.second.dev) {
      cudaFree(kv.second.dev);
      kv.second.dev = nullptr;
    }
  m->finalized = true;
  return DQMK_OK;
}

// The batched prefill's side tables: per projection the exact two-term fp16
// planes of the dequantized weight (4 bytes per weight) and the per-row
// power-of-two scales.  Built once, on the first batched ForwardBatch, and
// counted in memory_bytes from then on, so an engine that only decodes holds
// (and reports) the block bytes plus the resident F32 tensors, the
// reference's accounting (src/model.cc:227-260).
int ensure_prefill_weights(dqmk_model* m, const char* api) {
  if (m->prefill_ready) return DQMK_OK;
  if (!m->prefill_eligible) return fail(DQMK_ERR_UNSUPPORTED, std::string(api) +
                                                                  ": no batched prefill for this model");
  auto side = [&](const Packed& w, float** cs, CUtensorMap* maps) -> int {
    void* p = nullptr;
    int r = dev_alloc(m->allocs, (size_t)w.rows * sizeof(float), &p, api);
    if (r) return r;
    *cs = static_cast<float*>(p);
    void* planes[2];
    for (int t = 0; t < 2; ++t) {
      if ((r = dev_alloc(m->allocs, (size_t)w.rows * w.kp * 2, &planes[t], api))) return r;
      if ((r = make_f16_tile_map(&maps[t], planes[t], w.rows, w.kp))) return r;
    }
    m->memory_bytes += (size_t)w.rows * sizeof(float) + (size_t)2 * w.rows * w.kp * 2;
    cudaError_t e = launch_weights_split(w.qtype, w.qs(), w.d(), w.rows, w.kp,
                                         static_cast<uint16_t*>(planes[0]),
                                         static_cast<uint16_t*>(planes[1]), *cs, nullptr);
    if (e != cudaSuccess) return cuda_fail(api, e);
    return DQMK_OK;
  };
  int rc;
  for (int l = 0; l < m->cfg.n_layers; ++l) {
    Layer& L = m->layers[l];
    if ((rc = side(L.qkv, &L.cs_qkv, L.map_qkv))) return rc;
    if ((rc = side(L.wo, &L.cs_o, L.map_o))) return rc;
    if ((rc = side(L.gate_up, &L.cs_gu, L.map_gu))) return rc;
    if ((rc = side(L.down, &L.cs_dn, L.map_dn))) return rc;
  }
  DQMK_CUDA_RET(api, cudaDeviceSynchronize());
  m->prefill_ready = true;
  return DQMK_OK;
}

extern "C" int dqmk_model_stats_get(const dqmk_model* m, dqmk_model_stats* out) {
  if (!m || !out) return fail(DQMK_ERR_INVALID, "ModelCudaStats: null argument");
  *out = m->stats;
  return DQMK_OK;
}

extern "C" int dqmk_model_stats_reset(dqmk_model* m) {
  if (!m) return fail(DQMK_ERR_INVALID, "ResetModelCudaRuntimeStats: null model");
  const uint64_t n = m->stats.uploaded_weight_count, b = m->stats.uploaded_bytes;
  m->stats = dqmk_model_stats{};
  m->stats.uploaded_weight_count = n;
  m->stats.uploaded_bytes = b;
  return DQMK_OK;
}

extern "C" size_t dqmk_model_memory_bytes(const dqmk_model* m) { return m ? m->memory_bytes : 0; }

// ------------------------------------------------------------------ context
// Programmatic dependent launch between the kernels of a step; DQMK_PDL=0 in
// the environment launches them plainly instead (diagnostics: same work).
bool dqmk::use_pdl() {
  static const bool on = [] {
    const char* v = std::getenv("DQMK_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

namespace {

PeerSet peer_set(const dqmk_context* x) {
  PeerSet ps{};
  ps.base = x->peer_base;
  ps.rank = x->m->tp.rank;
  ps.world = x->m->tp.world;
  ps.dim = x->m->cfg.dim;
  ps.seq = x->tp_seq;
  ps.ticket = x->tp_seq + 2;
  return ps;
}

int enqueue_lm_head(dqmk_context* x);

// The decode step: embedding, per layer QKV GEMV (RMSNorm, bias, RoPE, KV
// store), attention, O GEMV (+ residual), gate/up GEMV (RMSNorm, SwiGLU),
// down GEMV (+ residual); then the lm_head with the greedy advance.
int enqueue_step(dqmk_context* x) {
  const char* api = "ForwardToken";
  const bool pdl = use_pdl();
  dqmk_model* m = x->m;
  const dqmk_model_config& c = m->cfg;
  const dqmk_tp_plan& tp = m->tp;
  const bool tpar = tp.world > 1;
  const bool p2p = tpar && x->p2p;
  const PeerSet ps = peer_set(x);
  cudaStream_t s = x->stream;
  int rc;
  auto gemv_op = [&](const GemvArgs& a) { return launch_gemv(a, s, pdl); };
  auto attn_op = [&](const AttnArgs& a) { return launch_attention(a, s, pdl); };
  EmbedArgs ea = {};
  ea.qtype = m->embd.qtype;
  ea.qs = m->embd.qs();
  ea.d = m->embd.d();
  ea.vocab = c.vocab_size;
  ea.dim = c.dim;
  ea.kp = m->embd.kp;
  ea.token_dev = x->token_slot();
  ea.y = x->x;
  ea.argmax_slot = x->argmax_slot();
  DQMK_CUDA_RET(api, launch_embed_packed(ea, s));
  for (int l = 0; l < c.n_layers; ++l) {
    const Layer& L = m->layers[l];
    GemvArgs g = {};
    g.qtype = L.qkv.qtype;
    g.qs = L.qkv.qs();
    g.d = L.qkv.d();
    g.n_rows = L.qkv.rows;
    g.k = L.qkv.k;
    g.kp = L.qkv.kp;
    g.x = x->x;
    g.norm_w = L.attn_norm;
    g.eps = c.rms_norm_eps;
    g.epi = kEpiQkv;
    g.bias = L.qkv_bias;
    g.rope_cs = m->rope_cs;
    g.pos_dev = x->pos_slot();
    g.q_out = x->q;
    g.k_cache = x->keys;
    g.v_cache = x->values;
    g.layer = l;
    g.max_seq = c.max_seq_len;
    g.n_heads = tp.n_q_heads;
    g.n_kv_heads = tp.n_kv_heads;
    g.head_dim = c.head_dim;
    g.neox = c.rope_neox;
    DQMK_CUDA_RET(api, gemv_op(g));

    AttnArgs at = {};
    at.q = x->q;
    at.keys = x->keys;
    at.values = x->values;
    at.max_seq = c.max_seq_len;
    at.n_kv_heads = tp.n_kv_heads;
    at.head_dim = c.head_dim;
    at.layer = l;
    at.n_heads = tp.n_q_heads;
    at.pos_dev = x->pos_slot();
    at.out = x->att;
    at.partials = x->partials;
    at.tickets = x->attn_tickets();
    at.max_splits = x->attn_splits;
    at.min_chunk = decode_min_chunk(c.head_dim);
    DQMK_CUDA_RET(api, attn_op(at));

    GemvArgs o = {};
    o.qtype = L.wo.qtype;
    o.qs = L.wo.qs();
    o.d = L.wo.d();
    o.n_rows = L.wo.rows;
    o.k = L.wo.k;
    o.kp = L.wo.kp;
    o.x = x->att;
    o.epi = kEpiStore;
    o.residual = tpar ? nullptr : x->x;
    o.y = tpar ? x->part : x->x;
    if (p2p) {  // partial rows straight into every rank's slot
      o.epi = kEpiPeer;
      o.peer = ps;
    }
    DQMK_CUDA_RET(api, gemv_op(o));
    if (p2p) {
      DQMK_CUDA_RET(api, launch_tp_reduce(x->x, ps, s, pdl));
    } else if (tpar) {  // complete the row-parallel sum, then the residual add
      if ((rc = tp_allreduce_sum(m->comm, x->part, c.dim, s, api))) return rc;
      DQMK_CUDA_RET(api, launch_add(x->x, x->part, c.dim, x->x, s));
    }

    GemvArgs gu = {};
    gu.qtype = L.gate_up.qtype;
    gu.qs = L.gate_up.qs();
    gu.d = L.gate_up.d();
    gu.n_rows = L.gate_up.rows;
    gu.k = L.gate_up.k;
    gu.kp = L.gate_up.kp;
    gu.x = x->x;
    gu.norm_w = L.ffn_norm;
    gu.eps = c.rms_norm_eps;
    gu.epi = kEpiSwiGlu;
    gu.y = x->h;
    DQMK_CUDA_RET(api, gemv_op(gu));

    GemvArgs dn = {};
    dn.qtype = L.down.qtype;
    dn.qs = L.down.qs();
    dn.d = L.down.d();
    dn.n_rows = L.down.rows;
    dn.k = L.down.k;
    dn.kp = L.down.kp;
    dn.x = x->h;
    dn.epi = kEpiStore;
    dn.residual = tpar ? nullptr : x->x;
    dn.y = tpar ? x->part : x->x;
    if (p2p) {
      dn.epi = kEpiPeer;
      dn.peer = ps;
    }
    DQMK_CUDA_RET(api, gemv_op(dn));
    if (p2p) {
      DQMK_CUDA_RET(api, launch_tp_reduce(x->x, ps, s, pdl));
    } else if (tpar) {
      if ((rc = tp_allreduce_sum(m->comm, x->part, c.dim, s, api))) return rc;
      DQMK_CUDA_RET(api, launch_add(x->x, x->part, c.dim, x->x, s));
    }
  }
  return enqueue_lm_head(x);
}

int enqueue_lm_head(dqmk_context* x) {
  const char* api = "ForwardToken";
  const bool pdl = use_pdl();
  dqmk_model* m = x->m;
  const dqmk_model_config& c = m->cfg;
  const dqmk_tp_plan& tp = m->tp;
  const bool tpar = tp.world > 1;
  const bool p2p = tpar && x->p2p;
  const PeerSet ps = peer_set(x);
  cudaStream_t s = x->stream;
  int rc;
  GemvArgs lg = {};
  lg.qtype = m->lm_head.qtype;
  lg.qs = m->lm_head.qs();
  lg.d = m->lm_head.d();
  lg.n_rows = m->lm_head.rows;
  lg.k = m->lm_head.k;
  lg.kp = m->lm_head.kp;
  lg.x = x->x;
  lg.norm_w = m->final_norm;
  lg.eps = c.rms_norm_eps;
  lg.epi = kEpiLogits;
  lg.y = x->logits;
  lg.argmax_slot = x->argmax_slot();
  lg.row_offset = tp.vocab0;
  lg.ticket = tpar ? nullptr : x->lm_ticket();
  lg.token_slot = x->token_slot();
  lg.pos_slot = x->pos_slot();
  lg.history = x->history_dev;
  lg.history_cap = c.max_seq_len;
  if (x->lm_withhold != -1) {  // failure-detection hook (dqmk_context_withhold_lm_head)
    DQMK_CUDA_RET(api, launch_gemv_tma_skip(lg, s, x->lm_withhold));
  } else {
    DQMK_CUDA_RET(api, launch_gemv(lg, s, pdl));
  }
  if (p2p) {
    DQMK_CUDA_RET(api, launch_tp_argmax_advance(ps, x->argmax_slot(), x->token_slot(),
                                                x->pos_slot(), x->history_dev, c.max_seq_len,
                                                c.vocab_size, s, pdl));
  } else if (tpar) {  // global greedy choice: max over the ranks' (value, index) keys
    if ((rc = tp_allreduce_max_u64(m->comm, x->argmax_slot(), 1, s, api))) return rc;
    DQMK_CUDA_RET(api, launch_greedy_advance(x->argmax_slot(), x->token_slot(), x->pos_slot(),
                                             x->history_dev, c.max_seq_len, c.vocab_size, s));
  }
  return DQMK_OK;
}

// Host logits of the last step: the local vocabulary slice, or under tensor
// parallelism all slices gathered (every rank takes part).
int copy_logits(dqmk_context* x, float* logits, const char* api) {
  dqmk_model* m = x->m;
  const size_t bytes = (size_t)m->cfg.vocab_size * sizeof(float);
  const float* src = x->logits;
  if (m->tp.world > 1) {
    int rc = tp_allgather(m->comm, x->logits, x->logits_all, (size_t)m->tp.vocab_stride,
                          x->stream, api);
    if (rc) return rc;
    src = x->logits_all;
  }
  DQMK_CUDA_RET(api, cudaMemcpyAsync(logits, src, bytes, cudaMemcpyDeviceToHost, x->stream));
  m->stats.device_to_host_copies += 1;
  m->stats.device_to_host_bytes += bytes;
  return DQMK_OK;
}

int ensure_graph(dqmk_context* x) {
  const char* api = "ForwardToken";
  if (x->tp_failed)
    return fail(DQMK_ERR_TIMEOUT,
                std::string(api) + ": a peer-memory exchange of this context timed out earlier; "
                                   "destroy and recreate the contexts of every rank");
  if (x->graph) return DQMK_OK;
  cudaGraph_t g = nullptr;
  DQMK_CUDA_RET(api, cudaStreamBeginCapture(x->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue_step(x);
  cudaError_t e = cudaStreamEndCapture(x->stream, &g);
  if (rc != DQMK_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(api, e);
  e = cudaGraphInstantiate(&x->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return cuda_fail(api, e);
  return DQMK_OK;
}

void count_token(dqmk_context* x, int pos) {
  dqmk_model* m = x->m;
  const dqmk_model_config& c = m->cfg;
  const bool bias = !m->layers.empty() && m->layers[0].qkv_bias != nullptr;
  auto& st = m->stats;
  st.linear_calls += (uint64_t)7 * c.n_layers + 1;
  // per layer: 2 RMSNorm, 1 RoPE, 2 residual adds, SiLU + mul (+3 bias adds)
  st.activation_calls += (uint64_t)(bias ? 10 : 7) * c.n_layers + 1;
  st.attention_calls += c.n_layers;
  st.kv_cache_write_bytes += (uint64_t)c.n_layers * 2 * c.n_kv_heads * c.head_dim * sizeof(float);
  st.kv_cache_read_bytes +=
      (uint64_t)c.n_layers * (pos + 1) * c.n_heads * c.head_dim * sizeof(float) * 2;
}

// After a synchronizing call: a bounded device wait that ran out surfaces as
// DQMK_ERR_TIMEOUT (the flag is cleared so the context stays usable).
int check_device_error(const char* api, dqmk_context* x = nullptr) {
  unsigned int flags = 0, tp_flags = 0, ops_flags = 0;
  DQMK_CUDA_RET(api, read_device_error(&flags, true));
  DQMK_CUDA_RET(api, read_tp_error(&tp_flags, true));
  DQMK_CUDA_RET(api, read_ops_error(&ops_flags, true));
  if ((tp_flags & kErrTimeout) && x && x->p2p) x->tp_failed = true;
  return device_flags_status(api, flags | tp_flags | ops_flags);
}

// Synchronise the context's stream with the three error flag words read
// back behind the work already enqueued (asynchronous copies into pinned
// memory), then report: only a raised flag costs check_device_error's
// synchronous read-and-clear.
int sync_and_check(const char* api, dqmk_context* x) {
  unsigned int* flags = reinterpret_cast<unsigned int*>(x->pinned_out + x->m->cfg.max_seq_len);
  for (int i = 0; i < 3; ++i)
    DQMK_CUDA_RET(api, cudaMemcpyAsync(flags + i, x->flag_dev[i], sizeof(unsigned int),
                                       cudaMemcpyDeviceToHost, x->stream));
  DQMK_CUDA_RET(api, cudaStreamSynchronize(x->stream));
  if (flags[0] | flags[1] | flags[2]) return check_device_error(api, x);
  return DQMK_OK;
}

int validate_token(const dqmk_context* x, int token, int pos) {
  const dqmk_model_config& c = x->m->cfg;
  if (token < 0 || token >= c.vocab_size)
    return fail(DQMK_ERR_RANGE, "ForwardToken token id out of range");
  if (pos < 0 || pos >= c.max_seq_len)
    return fail(DQMK_ERR_RANGE, "ForwardToken position out of range");
  return DQMK_OK;
}

// Upload (token, pos) into the device state.  The pinned staging slot is
// reused, so wait until the previous copy out of it has executed.
int stage_token(dqmk_context* x, int token, int pos, const char* api) {
  DQMK_CUDA_RET(api, cudaEventSynchronize(x->staged));
  x->pinned[0] = token;
  x->pinned[1] = pos;
  DQMK_CUDA_RET(api, cudaMemcpyAsync(x->token_slot(), x->pinned, 2 * sizeof(int),
                                     cudaMemcpyHostToDevice, x->stream));
  DQMK_CUDA_RET(api, cudaEventRecord(x->staged, x->stream));
  return DQMK_OK;
}

int launch_token(dqmk_context* x, int token, int pos) {
  const char* api = "ForwardToken";
  int rc = stage_token(x, token, pos, api);
  if (rc) return rc;
  DQMK_CUDA_RET(api, cudaGraphLaunch(x->graph, x->stream));
  count_token(x, pos);
  return DQMK_OK;
}

// ------------------------------------------------------------ batched prefill
// A prompt of consecutive positions runs layer by layer over all its tokens
// (chunks of up to PrefillBufs::m_max rows): every projection is one int8
// tensor-core GEMM, attention is causal over the cache.  DQMK_PREFILL=0 in
// the environment replays the decode graph per token instead.
bool prefill_enabled() {
  const char* v = std::getenv("DQMK_PREFILL");
  return !(v && v[0] == '0');
}

int ensure_prefill(dqmk_context* x) {
  PrefillBufs& b = x->pf;
  if (b.m_max) return DQMK_OK;
  const char* api = "ForwardBatch";
  const dqmk_model* m = x->m;
  const dqmk_model_config& c = m->cfg;
  const Layer& L0 = m->layers[0];
  const int qd = c.n_heads * c.head_dim;
  const int kp_dim = L0.qkv.kp, kp_qd = L0.wo.kp, kp_hid = L0.down.kp;
  const int kp_max = std::max(kp_dim, std::max(kp_qd, kp_hid));
  const int m_max = std::min(1024, c.max_seq_len);
  size_t part = 0;
  const bool split_attn = c.head_dim == 64;  // the tensor-core attention's scratch
  for (const Packed* w : {&L0.qkv, &L0.wo, &L0.gate_up, &L0.down})
    part = std::max(part, partial_floats_bound(m_max, w->rows, w->kp));
  void* p = nullptr;
  int rc;
  struct {
    void** dst;
    size_t bytes;
  } bufs[] = {{(void**)&b.x, (size_t)m_max * c.dim * sizeof(float)},
              {(void**)&b.q, (size_t)m_max * qd * sizeof(float)},
              {(void**)&b.att, (size_t)m_max * qd * sizeof(float)},
              {(void**)&b.f, (size_t)m_max * c.hidden_dim * sizeof(float)},
              {(void**)&b.hi, (size_t)m_max * kp_max * 2},
              {(void**)&b.lo, (size_t)m_max * kp_max * 2},
              {(void**)&b.rs, (size_t)m_max * sizeof(float)},
              {(void**)&b.partial, part * sizeof(float)},
              {(void**)&b.attn_part, split_attn ? prefill_attn_part_floats(m_max, c.n_heads) * sizeof(float) : 0},
              {(void**)&b.attn_tickets, split_attn ? prefill_attn_tickets(m_max, c.n_heads) * sizeof(unsigned) : 0},
              {(void**)&b.tokens, (size_t)m_max * sizeof(int)}};
  for (auto& e : bufs) {
    if ((rc = dev_alloc(x->allocs, e.bytes, &p, api))) return rc;
    DQMK_CUDA_RET(api, cudaMemset(p, 0, e.bytes ? e.bytes : 16));
    *e.dst = p;
  }
  struct {
    CUtensorMap* maps;
    int kp;
  } ks[] = {{b.a_dim, kp_dim}, {b.a_qd, kp_qd}, {b.a_hid, kp_hid}};
  for (auto& k : ks) {
    if ((rc = make_f16_tile_map(&k.maps[0], b.hi, m_max, k.kp))) return rc;
    if ((rc = make_f16_tile_map(&k.maps[1], b.lo, m_max, k.kp))) return rc;
  }
  DQMK_CUDA_RET(api, prefill_prepare());
  b.m_max = m_max;
  return DQMK_OK;
}

// One chunk: tokens[0..n) at positions pos0 .. pos0+n-1 (n <= m_max).  With
// want_logits the final-norm lm_head runs on the last row into x->logits.
int prefill_chunk(dqmk_context* x, const int* tokens, int pos0, int n, bool want_logits) {
  const char* api = "ForwardBatch";
  dqmk_model* m = x->m;
  const dqmk_model_config& c = m->cfg;
  PrefillBufs& b = x->pf;
  cudaStream_t s = x->stream;
  const int qd = c.n_heads * c.head_dim;
  const float eps = c.rms_norm_eps;
  // a copy from pageable memory is staged by the driver before it returns
  DQMK_CUDA_RET(api, cudaMemcpyAsync(b.tokens, tokens, n * sizeof(int), cudaMemcpyHostToDevice, s));
  DQMK_CUDA_RET(api, launch_embed_rows(m->embd.qtype, m->embd.qs(), m->embd.d(), c.dim,
                                       m->embd.kp, c.vocab_size, b.tokens, n, b.x, s));
  for (int l = 0; l < c.n_layers; ++l) {
    const Layer& L = m->layers[l];
    // attention block: RMSNorm + fp16 split, fused QKV GEMM (bias, RoPE, cache
    // store), causal attention, O GEMM + residual
    DQMK_CUDA_RET(api, launch_split_rows(b.x, n, c.dim, L.qkv.kp, c.dim, L.attn_norm, eps, b.hi,
                                         b.lo, b.rs, s));
    PrefillGemm g = {};
    g.m = n;
    g.n = L.qkv.rows;
    g.kp = L.qkv.kp;
    g.rs = b.rs;
    g.partial = b.partial;
    g.plan = plan_gemm(n, L.qkv.rows, L.qkv.kp);
    g.cs = L.cs_qkv;
    g.epi = kEpiQkv;
    g.bias = L.qkv_bias;
    g.rope_cs = m->rope_cs;
    g.pos0 = pos0;
    g.q_out = b.q;
    g.ldq = qd;
    g.k_cache = x->keys;
    g.v_cache = x->values;
    g.layer = l;
    g.max_seq = c.max_seq_len;
    g.n_heads = c.n_heads;
    g.n_kv_heads = c.n_kv_heads;
    g.head_dim = c.head_dim;
    g.neox = c.rope_neox;
    DQMK_CUDA_RET(api, launch_prefill_gemm(b.a_dim[0], b.a_dim[1], L.map_qkv[0], L.map_qkv[1], g, s));

    PrefillAttn a = {};
    a.q = b.q;
    a.ldq = qd;
    a.keys = x->keys;
    a.values = x->values;
    a.out = b.att;
    a.ldo = qd;
    a.m = n;
    a.pos0 = pos0;
    a.layer = l;
    a.max_seq = c.max_seq_len;
    a.n_heads = c.n_heads;
    a.n_kv_heads = c.n_kv_heads;
    a.head_dim = c.head_dim;
    if (c.head_dim == 64) {
      a.part = b.attn_part;
      a.tickets = b.attn_tickets;
    }
    DQMK_CUDA_RET(api, launch_attention_prefill(a, s));

    DQMK_CUDA_RET(api, launch_split_rows(b.att, n, qd, L.wo.kp, qd, nullptr, eps, b.hi, b.lo,
                                         b.rs, s));
    PrefillGemm o = {};
    o.m = n;
    o.n = L.wo.rows;
    o.kp = L.wo.kp;
    o.rs = b.rs;
    o.partial = b.partial;
    o.plan = plan_gemm(n, L.wo.rows, L.wo.kp);
    o.cs = L.cs_o;
    o.epi = kEpiStore;
    o.residual = b.x;
    o.y = b.x;
    o.ldy = c.dim;
    DQMK_CUDA_RET(api, launch_prefill_gemm(b.a_qd[0], b.a_qd[1], L.map_o[0], L.map_o[1], o, s));

    // feed-forward block: RMSNorm + fp16 split, gate/up GEMM with SwiGLU,
    // down GEMM + residual
    DQMK_CUDA_RET(api, launch_split_rows(b.x, n, c.dim, L.gate_up.kp, c.dim, L.ffn_norm, eps,
                                         b.hi, b.lo, b.rs, s));
    PrefillGemm gu = {};
    gu.m = n;
    gu.n = L.gate_up.rows;
    gu.kp = L.gate_up.kp;
    gu.rs = b.rs;
    gu.partial = b.partial;
    gu.plan = plan_gemm(n, L.gate_up.rows, L.gate_up.kp);
    gu.cs = L.cs_gu;
    gu.epi = kEpiSwiGlu;
    gu.y = b.f;
    gu.ldy = c.hidden_dim;
    DQMK_CUDA_RET(api, launch_prefill_gemm(b.a_dim[0], b.a_dim[1], L.map_gu[0], L.map_gu[1], gu, s));

    DQMK_CUDA_RET(api, launch_split_rows(b.f, n, c.hidden_dim, L.down.kp, c.hidden_dim, nullptr,
                                         eps, b.hi, b.lo, b.rs, s));
    PrefillGemm dn = {};
    dn.m = n;
    dn.n = L.down.rows;
    dn.kp = L.down.kp;
    dn.rs = b.rs;
    dn.partial = b.partial;
    dn.plan = plan_gemm(n, L.down.rows, L.down.kp);
    dn.cs = L.cs_dn;
    dn.epi = kEpiStore;
    dn.residual = b.x;
    dn.y = b.x;
    dn.ldy = c.dim;
    DQMK_CUDA_RET(api, launch_prefill_gemm(b.a_hid[0], b.a_hid[1], L.map_dn[0], L.map_dn[1], dn, s));
  }
  if (!want_logits) return DQMK_OK;
  // lm_head on the last row; the greedy state then points past it
  int rc = stage_token(x, tokens[n - 1], pos0 + n - 1, api);
  if (rc) return rc;
  DQMK_CUDA_RET(api, cudaMemsetAsync(x->argmax_slot(), 0, sizeof(unsigned long long), s));
  GemvArgs lg = {};
  lg.qtype = m->lm_head.qtype;
  lg.qs = m->lm_head.qs();
  lg.d = m->lm_head.d();
  lg.n_rows = m->lm_head.rows;
  lg.k = m->lm_head.k;
  lg.kp = m->lm_head.kp;
  lg.x = b.x + (size_t)(n - 1) * c.dim;
  lg.norm_w = m->final_norm;
  lg.eps = c.rms_norm_eps;
  lg.epi = kEpiLogits;
  lg.y = x->logits;
  lg.argmax_slot = x->argmax_slot();
  lg.ticket = x->lm_ticket();
  lg.token_slot = x->token_slot();
  lg.pos_slot = x->pos_slot();
  lg.history = x->history_dev;
  lg.history_cap = c.max_seq_len;
  DQMK_CUDA_RET(api, launch_gemv(lg, s, false));
  return DQMK_OK;
}

int check_prefill_error(const char* api) {
  unsigned int flags = 0;
  DQMK_CUDA_RET(api, read_prefill_error(&flags, true));
  if (flags) return fail(DQMK_ERR_TIMEOUT, std::string(api) + ": a device-side wait timed out");
  return DQMK_OK;
}

}  // namespace

extern "C" int dqmk_context_create(dqmk_model* m, dqmk_context** out) {
  const char* api = "MiniLlamaContext";
  if (!m || !out) return fail(DQMK_ERR_INVALID, std::string(api) + ": null argument");
  if (!m->finalized) {
    int rc = dqmk_model_finalize(m);
    if (rc) return rc;
  }
  cudaSetDevice(m->device);
  const dqmk_model_config& c = m->cfg;
  std::unique_ptr<dqmk_context> x(new dqmk_context());
  x->m = m;
  DQMK_CUDA_RET(api, cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking));
  DQMK_CUDA_RET(api, cudaMallocHost(&x->pinned, 64));
  DQMK_CUDA_RET(api, cudaMallocHost(&x->pinned_out,
                                    ((size_t)m->cfg.max_seq_len + 4) * sizeof(int)));
  DQMK_CUDA_RET(api, device_error_address(&x->flag_dev[0]));
  DQMK_CUDA_RET(api, tp_error_address(&x->flag_dev[1]));
  DQMK_CUDA_RET(api, ops_error_address(&x->flag_dev[2]));
  DQMK_CUDA_RET(api, cudaEventCreateWithFlags(&x->staged, cudaEventDisableTiming));
  const dqmk_tp_plan& tp = m->tp;
  const size_t kv = (size_t)c.n_layers * c.max_seq_len * tp.n_kv_heads * c.head_dim;
  x->attn_splits = attention_splits(c.max_seq_len, tp.n_kv_heads, decode_min_chunk(c.head_dim));
  void* p = nullptr;
  int rc;
  const int hd = c.head_dim;
  struct {
    float** dst;
    size_t n;
  } bufs[] = {{&x->x, (size_t)c.dim},
              {&x->q, (size_t)tp.n_q_heads * hd},
              {&x->att, (size_t)tp.n_q_heads * hd},
              {&x->h, (size_t)tp.hidden},
              {&x->logits, (size_t)tp.vocab_stride},
              {&x->keys, kv},
              {&x->values, kv},
              {&x->partials, attention_partials_floats(tp.n_q_heads, hd, x->attn_splits)},
              {&x->part, (size_t)c.dim},
              {&x->logits_all, tp.world > 1 ? (size_t)tp.vocab_stride * tp.world : 1}};
  for (auto& b : bufs) {
    if ((rc = dev_alloc(x->allocs, b.n * sizeof(float), &p, api))) return rc;
    *b.dst = static_cast<float*>(p);
  }
  if (tp.world > 1) {
    const size_t tb = tp_buf_bytes(tp.world, c.dim);
    DQMK_CUDA_RET(api, cudaMalloc(reinterpret_cast<void**>(&x->tp_buf), tb));
    x->allocs.push_back(x->tp_buf);
    DQMK_CUDA_RET(api, cudaMemset(x->tp_buf, 0, tb));
    if ((rc = dev_alloc(x->allocs, (size_t)tp.world * sizeof(char*), &p, api))) return rc;
    x->peer_base = static_cast<char**>(p);
    if ((rc = dev_alloc(x->allocs, 4 * sizeof(unsigned int), &p, api))) return rc;
    x->tp_seq = static_cast<unsigned int*>(p);
    DQMK_CUDA_RET(api, cudaMemset(x->tp_seq, 0, 4 * sizeof(unsigned int)));
  }
  if ((rc = dev_alloc(x->allocs, 64 + 4 * (size_t)tp.n_kv_heads + 64, &p, api))) return rc;
  x->state = static_cast<unsigned char*>(p);
  if ((rc = dev_alloc(x->allocs, (size_t)c.max_seq_len * sizeof(int), &p, api))) return rc;
  x->history_dev = static_cast<int*>(p);
  DQMK_CUDA_RET(api, cudaMemset(x->state, 0, 64 + 4 * (size_t)tp.n_kv_heads + 64));
  DQMK_CUDA_RET(api, cudaMemset(x->keys, 0, kv * sizeof(float)));
  DQMK_CUDA_RET(api, cudaMemset(x->values, 0, kv * sizeof(float)));
  DQMK_CUDA_RET(api, gemv_prepare());
  DQMK_CUDA_RET(api, attention_prepare());
  DQMK_CUDA_RET(api, cudaDeviceSynchronize());
  *out = x.release();
  return DQMK_OK;
}

extern "C" int dqmk_context_destroy(dqmk_context* x) {
  delete x;
  return DQMK_OK;
}

extern "C" int dqmk_context_reset(dqmk_context* x) {
  const char* api = "MiniLlamaContext";
  if (!x) return fail(DQMK_ERR_INVALID, std::string(api) + ": null context");
  const dqmk_model_config& c = x->m->cfg;
  const size_t kv = (size_t)c.n_layers * c.max_seq_len * x->m->tp.n_kv_heads * c.head_dim;
  DQMK_CUDA_RET(api, cudaMemsetAsync(x->keys, 0, kv * sizeof(float), x->stream));
  DQMK_CUDA_RET(api, cudaMemsetAsync(x->values, 0, kv * sizeof(float), x->stream));
  DQMK_CUDA_RET(api, cudaStreamSynchronize(x->stream));
  x->pos = 0;
  x->history.clear();
  return DQMK_OK;
}

extern "C" int dqmk_context_pos(const dqmk_context* x) { return x ? x->pos : -1; }

extern "C" int dqmk_context_history(const dqmk_context* x, int* out, int cap) {
  if (!x) return -1;
  const int n = (int)x->history.size();
  for (int i = 0; i < n && i < cap && out; ++i) out[i] = x->history[i];
  return n;
}

extern "C" void* dqmk_context_stream(dqmk_context* x) { return x ? x->stream : nullptr; }

extern "C" int dqmk_context_tp_ipc_handle(dqmk_context* x, unsigned char* handle_out) {
  const char* api = "dqmk_context_tp_ipc_handle";
  if (!x || !handle_out) return fail(DQMK_ERR_INVALID, std::string(api) + ": null argument");
  if (!x->tp_buf) return fail(DQMK_ERR_INVALID, std::string(api) + ": not tensor parallel");
  cudaSetDevice(x->m->device);
  cudaIpcMemHandle_t h;
  DQMK_CUDA_RET(api, cudaIpcGetMemHandle(&h, x->tp_buf));
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  std::memcpy(handle_out, &h, 64);
  return DQMK_OK;
}

extern "C" int dqmk_context_tp_connect(dqmk_context* x, const unsigned char* handles) {
  const char* api = "dqmk_context_tp_connect";
  if (!x || !handles) return fail(DQMK_ERR_INVALID, std::string(api) + ": null argument");
  if (!x->tp_buf) return fail(DQMK_ERR_INVALID, std::string(api) + ": not tensor parallel");
  if (x->p2p) return fail(DQMK_ERR_INVALID, std::string(api) + ": already connected");
  cudaSetDevice(x->m->device);
  const dqmk_tp_plan& tp = x->m->tp;
  std::vector<char*> bases(tp.world, nullptr);
  for (int w = 0; w < tp.world; ++w) {
    if (w == tp.rank) {
      bases[w] = x->tp_buf;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + (size_t)w * 64, 64);
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(api, e);
    x->ipc_opened.push_back(ptr);
    bases[w] = static_cast<char*>(ptr);
  }
  DQMK_CUDA_RET(api, cudaMemcpy(x->peer_base, bases.data(), tp.world * sizeof(char*),
                                cudaMemcpyHostToDevice));
  if (x->graph) {  // the step is captured again with the peer-memory exchange
    cudaGraphExecDestroy(x->graph);
    x->graph = nullptr;
  }
  x->p2p = true;
  return DQMK_OK;
}

extern "C" int dqmk_context_withhold_lm_head(dqmk_context* x, int tile) {
  const char* api = "dqmk_context_withhold_lm_head";
  if (!x) return fail(DQMK_ERR_INVALID, std::string(api) + ": null context");
  if (tile < kSkipAllTiles) return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid tile");
  cudaSetDevice(x->m->device);
  DQMK_CUDA_RET(api, cudaStreamSynchronize(x->stream));
  if (x->graph) {  // the step is captured again with (or without) the hook
    cudaGraphExecDestroy(x->graph);
    x->graph = nullptr;
  }
  x->lm_withhold = tile;
  return DQMK_OK;
}

extern "C" int dqmk_forward_token(dqmk_context* x, int token, int pos, float* logits) {
  const char* api = "ForwardToken";
  if (!x) return fail(DQMK_ERR_INVALID, std::string(api) + " called with a null context");
  int rc = validate_token(x, token, pos);
  if (rc) return rc;
  cudaSetDevice(x->m->device);
  if ((rc = ensure_graph(x))) return rc;
  if ((rc = launch_token(x, token, pos))) return rc;
  if (logits && (rc = copy_logits(x, logits, api))) return rc;
  return sync_and_check(api, x);
}

extern "C" int dqmk_forward_batch(dqmk_context* x, const int* tokens, const int* positions, int n,
                                  float* logits) {
  const char* api = "ForwardBatch";
  if (!x) return fail(DQMK_ERR_INVALID, std::string(api) + ": null context");
  if (n <= 0 || !tokens) return fail(DQMK_ERR_INVALID, "ForwardBatch: empty token");
  if (!positions) return fail(DQMK_ERR_INVALID, "ForwardBatch: tokens and positions size mismatch");
  int rc;
  for (int i = 0; i < n; ++i)
    if ((rc = validate_token(x, tokens[i], positions[i]))) return rc;
  cudaSetDevice(x->m->device);
  bool consecutive = true;
  for (int i = 1; i < n && consecutive; ++i) consecutive = positions[i] == positions[0] + i;
  if (n > 1 && consecutive && x->m->prefill_eligible && prefill_enabled()) {
    if ((rc = ensure_prefill_weights(x->m, api))) return rc;
    if ((rc = ensure_prefill(x))) return rc;
    for (int i0 = 0; i0 < n; i0 += x->pf.m_max) {
      const int cnt = std::min(x->pf.m_max, n - i0);
      if ((rc = prefill_chunk(x, tokens + i0, positions[i0], cnt, i0 + cnt == n))) return rc;
    }
    for (int i = 0; i < n; ++i) {
      count_token(x, positions[i]);
      x->history.push_back(tokens[i]);
    }
    x->pos = positions[n - 1];
  } else {
    if ((rc = ensure_graph(x))) return rc;
    for (int i = 0; i < n; ++i) {
      x->pos = positions[i];
      if ((rc = launch_token(x, tokens[i], positions[i]))) return rc;
      x->history.push_back(tokens[i]);
    }
  }
  if (logits && (rc = copy_logits(x, logits, api))) return rc;
  DQMK_CUDA_RET(api, cudaStreamSynchronize(x->stream));
  if ((rc = check_prefill_error(api))) return rc;
  return check_device_error(api, x);
}

// Prefix reuse for a new prompt on a context that already holds a sequence
// (the chat path's reuse, src/main.cc:887-913, with the context's own token
// history as the source of truth): p = the longest common prefix of the
// history and the prompt.  p == 0 or p == n (nothing left to compute logits
// from) recomputes the whole prompt from position 0; otherwise the history
// is cut to p tokens, pos rolls back to p - 1, and only tokens[p..n) run,
// at positions p.. -- one batched prefill when the model has one.  KV rows
// past the kept prefix are simply overwritten as positions advance;
// attention never reads beyond the current position.
extern "C" int dqmk_forward_batch_prefix(dqmk_context* x, const int* tokens, int n,
                                         float* logits, int* reused) {
  const char* api = "ForwardBatch";
  if (!x) return fail(DQMK_ERR_INVALID, std::string(api) + ": null context");
  if (n <= 0 || !tokens) return fail(DQMK_ERR_INVALID, "ForwardBatch: empty token");
  size_t p = 0;
  while (p < x->history.size() && p < (size_t)n && x->history[p] == tokens[p]) ++p;
  if (p >= (size_t)n) p = 0;
  x->history.resize(p);
  x->pos = p ? (int)p - 1 : 0;
  std::vector<int> positions(n - p);
  for (size_t i = 0; i < positions.size(); ++i) positions[i] = (int)(p + i);
  if (reused) *reused = (int)p;
  return dqmk_forward_batch(x, tokens + p, positions.data(), (int)positions.size(), logits);
}

extern "C" int dqmk_decode_enqueue(dqmk_context* x, int token, int pos, int n_steps) {
  const char* api = "DecodeGreedy";
  if (!x) return fail(DQMK_ERR_INVALID, std::string(api) + ": null context");
  if (n_steps <= 0) return fail(DQMK_ERR_INVALID, std::string(api) + ": n_steps must be positive");
  int rc = validate_token(x, token, pos);
  if (rc) return rc;
  if (pos + n_steps > x->m->cfg.max_seq_len)
    return fail(DQMK_ERR_RANGE, std::string(api) + ": position out of range");
  cudaSetDevice(x->m->device);
  if ((rc = ensure_graph(x))) return rc;
  if ((rc = stage_token(x, token, pos, api))) return rc;
  for (int i = 0; i < n_steps; ++i) {
    DQMK_CUDA_RET(api, cudaGraphLaunch(x->graph, x->stream));
    count_token(x, pos + i);
  }
  return DQMK_OK;
}

extern "C" int dqmk_decode_greedy(dqmk_context* x, int token, int pos, int n_steps,
                                  int* tokens_out) {
  const char* api = "DecodeGreedy";
  int rc = dqmk_decode_enqueue(x, token, pos, n_steps);
  if (rc) return rc;
  // the tokens come back with the steps into pinned memory, behind the one
  // synchronisation of sync_and_check
  int* out = x->pinned_out;
  if (tokens_out) {
    DQMK_CUDA_RET(api, cudaMemcpyAsync(out, x->history_dev + pos, n_steps * sizeof(int),
                                       cudaMemcpyDeviceToHost, x->stream));
  }
  rc = sync_and_check(api, x);
  if (tokens_out) std::memcpy(tokens_out, out, n_steps * sizeof(int));
  x->history.push_back(token);
  for (int i = 0; i + 1 < n_steps && tokens_out; ++i) x->history.push_back(tokens_out[i]);
  x->pos = pos + n_steps - 1;
  return rc;
}
