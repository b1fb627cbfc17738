// batch_engine.cc -- multi-sequence decode behind the dqmk C ABI (C++17).
//
// The reference serves one sequence per context and one token per
// ForwardToken call (src/forward.cc:667-754).  A dqmk_batch holds n_slots
// independent sequences over one model, each with its own device KV cache,
// and runs a step over up to 64 columns at once -- column c feeds token[c] at
// position pos[c] of slot slot[c] -- so each weight is streamed once per step
// instead of once per token.  Per step, on the batch's own stream:
//   embed; per layer: RMSNorm + fp16 split, QKV GEMM (bias, RoPE, KV store),
//   attention per column, split, O GEMM (+ residual), RMSNorm + split,
//   gate/up GEMM (SwiGLU), split, down GEMM (+ residual);
//   final RMSNorm + split, lm_head GEMM with per-column argmax, greedy advance.
// Under tensor parallelism the row-parallel GEMMs produce partial sums that
// are all-reduced over NCCL before the residual add, and the vocabulary-
// parallel lm_head's argmax keys are max-reduced.  The whole step is captured
// once per column count into a CUDA graph; tokens, positions and slots live in
// device memory, so greedy decoding replays the graph with no host work.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "batch.h"
#include "dqmk.h"
#include "internal.h"
#include "model.h"
#include "prefill.h"
#include "tp.h"

using namespace dqmk;

struct dqmk_batch {
  dqmk_model* m = nullptr;
  int n_slots = 0, max_seq = 0;
  cudaStream_t stream = nullptr;
  size_t slot_stride = 0;               // floats per slot of keys / values
  float *keys = nullptr, *values = nullptr;  // [n_slots][layer][max_seq][kvd]
  // per-column activations [kBatchMaxCols][...]
  float *x = nullptr, *q = nullptr, *att = nullptr, *f = nullptr, *part = nullptr;
  float *logits = nullptr, *logits_all = nullptr;
  uint16_t *hi = nullptr, *lo = nullptr;  // fp16 activation planes [64][kp]
  float* rs = nullptr;                    // their column scales
  float* partial = nullptr;               // GEMM split-K sums
  float* attn_partials = nullptr;
  unsigned int* attn_tickets = nullptr;
  int* cols = nullptr;                    // device [3][64]: slot, token, pos
  unsigned long long* keys_arg = nullptr; // [64] argmax keys
  int* history = nullptr;                 // [n_slots][max_seq]: token after each position
  int* pinned = nullptr;                  // host staging [3][64]
  cudaEvent_t staged = nullptr;
  CUtensorMap x_dim[2], x_qd[2], x_hid[2];
  std::map<int, cudaGraphExec_t> graphs;  // key: columns * 2 + with_logits
  std::vector<void*> allocs;

  int* col_slot() { return cols; }
  int* col_token() { return cols + kBatchMaxCols; }
  int* col_pos() { return cols + 2 * kBatchMaxCols; }

  ~dqmk_batch() {
    cudaSetDevice(m ? m->device : 0);
    for (auto& g : graphs) cudaGraphExecDestroy(g.second);
    if (staged) cudaEventDestroy(staged);
    if (stream) cudaStreamDestroy(stream);
    for (void* p : allocs) cudaFree(p);
    if (pinned) cudaFreeHost(pinned);
  }
};

namespace {

const char* kApi = "DecodeBatch";

// Row scales and quant-plane tensor maps of every projection (once per model).
int ensure_batch_weights(dqmk_model* m) {
  if (m->batch_ready) return DQMK_OK;
  const int n_layers = m->cfg.n_layers;
  m->batch_layers.assign(n_layers, BatchLayer{});
  auto build = [&](const Packed& w, BatchWeight* out) -> int {
    void* p = nullptr;
    int rc = dev_alloc(m->allocs, (size_t)w.rows * sizeof(float), &p, kApi);
    if (rc) return rc;
    out->cs = static_cast<float*>(p);
    DQMK_CUDA_RET(kApi, launch_weight_row_scales(w.qtype, w.qs(), w.d(), w.rows, w.kp, out->cs,
                                                 nullptr));
    const size_t dp_bytes = (size_t)w.rows * scale_pitch(w.kp) * 2;
    if ((rc = dev_alloc(m->allocs, dp_bytes, &p, kApi))) return rc;
    out->d_pad = static_cast<uint16_t*>(p);
    DQMK_CUDA_RET(kApi, copy_scales_padded(w.d(), w.rows, w.kp, out->d_pad, nullptr));
    m->memory_bytes += (size_t)w.rows * sizeof(float) + dp_bytes;
    if ((rc = make_scale_map(&out->dmap, out->d_pad, w.rows, w.kp))) return rc;
    return make_quant_map(&out->map, w.qtype, w.qs(), w.rows, w.kp);
  };
  int rc;
  for (int l = 0; l < n_layers; ++l) {
    const Layer& L = m->layers[l];
    BatchLayer& B = m->batch_layers[l];
    if ((rc = build(L.qkv, &B.qkv)) || (rc = build(L.wo, &B.wo)) ||
        (rc = build(L.gate_up, &B.gate_up)) || (rc = build(L.down, &B.down)))
      return rc;
  }
  if ((rc = build(m->lm_head, &m->batch_lm))) return rc;
  DQMK_CUDA_RET(kApi, cudaDeviceSynchronize());
  m->batch_ready = true;
  return DQMK_OK;
}

int check_errors(const char* api) {
  unsigned int f0 = 0, f1 = 0, f2 = 0;
  DQMK_CUDA_RET(api, read_batch_error(&f0, true));
  DQMK_CUDA_RET(api, read_device_error(&f1, true));
  DQMK_CUDA_RET(api, read_prefill_error(&f2, true));
  return device_flags_status(api, f0 | f1 | f2);
}

BatchGemm gemm_args(const dqmk_batch* b, const Packed& w, const BatchWeight& bw, int n_cols,
                    int epi) {
  BatchGemm g = {};
  g.qtype = w.qtype;
  g.d = w.d();
  g.n = w.rows;
  g.kp = w.kp;
  g.cols = n_cols;
  g.rs = b->rs;
  g.cs = bw.cs;
  g.plan = plan_batch_gemm(w.rows, w.kp);
  g.partial = b->partial;
  g.epi = epi;
  g.col_slot = b->cols;
  g.col_pos = b->cols + 2 * kBatchMaxCols;
  return g;
}

// The step over columns 0..n-1 of the device column arrays, then the greedy
// advance (token, position, history).  With logits the lm_head also writes
// the per-column logits.
int enqueue_batch_step(dqmk_batch* b, int n, bool with_logits) {
  dqmk_model* m = b->m;
  const dqmk_model_config& c = m->cfg;
  const dqmk_tp_plan& tp = m->tp;
  const bool tpar = tp.world > 1;
  const bool pdl = use_pdl();
  cudaStream_t s = b->stream;
  const int hd = c.head_dim;
  const int qd = tp.n_q_heads * hd;
  const float eps = c.rms_norm_eps;
  int rc;
  DQMK_CUDA_RET(kApi, launch_embed_rows(m->embd.qtype, m->embd.qs(), m->embd.d(), c.dim,
                                        m->embd.kp, c.vocab_size, b->col_token(), n, b->x, s));
  const int splits = batch_attention_splits(n, tp.n_kv_heads, b->max_seq);
  for (int l = 0; l < c.n_layers; ++l) {
    const Layer& L = m->layers[l];
    const BatchLayer& B = m->batch_layers[l];
    DQMK_CUDA_RET(kApi, launch_split_rows(b->x, n, c.dim, L.qkv.kp, c.dim, L.attn_norm, eps,
                                          b->hi, b->lo, b->rs, s, pdl));
    BatchGemm g = gemm_args(b, L.qkv, B.qkv, n, kEpiQkv);
    g.bias = L.qkv_bias;
    g.rope_cs = m->rope_cs;
    g.q_out = b->q;
    g.ldq = qd;
    g.k_cache = b->keys;
    g.v_cache = b->values;
    g.slot_stride = b->slot_stride;
    g.layer = l;
    g.max_seq = b->max_seq;
    g.n_heads = tp.n_q_heads;
    g.n_kv_heads = tp.n_kv_heads;
    g.head_dim = hd;
    g.neox = c.rope_neox;
    DQMK_CUDA_RET(kApi, launch_batch_gemm(B.qkv.map, B.qkv.dmap, b->x_dim[0], b->x_dim[1], g, s, pdl));

    BatchAttn a = {};
    a.q = b->q;
    a.out = b->att;
    a.ldq = qd;
    a.keys = b->keys;
    a.values = b->values;
    a.slot_stride = b->slot_stride;
    a.cols = n;
    a.layer = l;
    a.max_seq = b->max_seq;
    a.n_heads = tp.n_q_heads;
    a.n_kv_heads = tp.n_kv_heads;
    a.head_dim = hd;
    a.col_slot = b->col_slot();
    a.col_pos = b->col_pos();
    a.partials = b->attn_partials;
    a.tickets = b->attn_tickets;
    a.max_splits = splits;
    DQMK_CUDA_RET(kApi, launch_attention_cols(a, s, pdl));

    DQMK_CUDA_RET(kApi, launch_split_rows(b->att, n, qd, L.wo.kp, qd, nullptr, eps, b->hi, b->lo,
                                          b->rs, s, pdl));
    BatchGemm o = gemm_args(b, L.wo, B.wo, n, kEpiStore);
    o.residual = tpar ? nullptr : b->x;
    o.y = tpar ? b->part : b->x;
    o.ldy = c.dim;
    DQMK_CUDA_RET(kApi, launch_batch_gemm(B.wo.map, B.wo.dmap, b->x_qd[0], b->x_qd[1], o, s, pdl));
    if (tpar) {  // complete the row-parallel sums, then the residual add
      if ((rc = tp_allreduce_sum(m->comm, b->part, (size_t)n * c.dim, s, kApi))) return rc;
      DQMK_CUDA_RET(kApi, launch_add(b->x, b->part, n * c.dim, b->x, s));
    }

    DQMK_CUDA_RET(kApi, launch_split_rows(b->x, n, c.dim, L.gate_up.kp, c.dim, L.ffn_norm, eps,
                                          b->hi, b->lo, b->rs, s, pdl));
    BatchGemm gu = gemm_args(b, L.gate_up, B.gate_up, n, kEpiSwiGlu);
    gu.y = b->f;
    gu.ldy = tp.hidden;
    DQMK_CUDA_RET(kApi, launch_batch_gemm(B.gate_up.map, B.gate_up.dmap, b->x_dim[0], b->x_dim[1], gu, s, pdl));

    DQMK_CUDA_RET(kApi, launch_split_rows(b->f, n, tp.hidden, L.down.kp, tp.hidden, nullptr, eps,
                                          b->hi, b->lo, b->rs, s, pdl));
    BatchGemm dn = gemm_args(b, L.down, B.down, n, kEpiStore);
    dn.residual = tpar ? nullptr : b->x;
    dn.y = tpar ? b->part : b->x;
    dn.ldy = c.dim;
    DQMK_CUDA_RET(kApi, launch_batch_gemm(B.down.map, B.down.dmap, b->x_hid[0], b->x_hid[1], dn, s, pdl));
    if (tpar) {
      if ((rc = tp_allreduce_sum(m->comm, b->part, (size_t)n * c.dim, s, kApi))) return rc;
      DQMK_CUDA_RET(kApi, launch_add(b->x, b->part, n * c.dim, b->x, s));
    }
  }
  DQMK_CUDA_RET(kApi, launch_split_rows(b->x, n, c.dim, m->lm_head.kp, c.dim, m->final_norm, eps,
                                        b->hi, b->lo, b->rs, s, pdl));
  BatchGemm lg = gemm_args(b, m->lm_head, m->batch_lm, n, kEpiLogits);
  lg.y = with_logits ? b->logits : nullptr;
  lg.ldy = tp.vocab_stride;
  lg.keys = b->keys_arg;
  lg.row_offset = tp.vocab0;
  DQMK_CUDA_RET(kApi, launch_batch_gemm(m->batch_lm.map, m->batch_lm.dmap, b->x_dim[0], b->x_dim[1], lg, s, pdl));
  if (tpar && (rc = tp_allreduce_max_u64(m->comm, b->keys_arg, n, s, kApi))) return rc;
  DQMK_CUDA_RET(kApi, launch_cols_advance(b->keys_arg, n, b->col_slot(), b->col_token(),
                                          b->col_pos(), b->history, b->max_seq, c.vocab_size, s,
                                          false));
  return DQMK_OK;
}

int ensure_graph(dqmk_batch* b, int n, bool with_logits) {
  const int key = n * 2 + (with_logits ? 1 : 0);
  if (b->graphs.count(key)) return DQMK_OK;
  cudaGraph_t g = nullptr;
  DQMK_CUDA_RET(kApi, cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue_batch_step(b, n, with_logits);
  cudaError_t e = cudaStreamEndCapture(b->stream, &g);
  if (rc != DQMK_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(kApi, e);
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return cuda_fail(kApi, e);
  b->graphs[key] = exec;
  return DQMK_OK;
}

// Copies the columns' (slot, token, position) into the device arrays; the
// pinned staging buffer is reused once the previous copy out of it ran.
int stage_cols(dqmk_batch* b, const int* slots, const int* tokens, const int* positions, int n) {
  DQMK_CUDA_RET(kApi, cudaEventSynchronize(b->staged));
  for (int i = 0; i < n; ++i) {
    b->pinned[i] = slots ? slots[i] : i;
    b->pinned[kBatchMaxCols + i] = tokens[i];
    b->pinned[2 * kBatchMaxCols + i] = positions[i];
  }
  DQMK_CUDA_RET(kApi, cudaMemcpyAsync(b->cols, b->pinned, 3 * kBatchMaxCols * sizeof(int),
                                      cudaMemcpyHostToDevice, b->stream));
  DQMK_CUDA_RET(kApi, cudaEventRecord(b->staged, b->stream));
  return DQMK_OK;
}

int validate_cols(const dqmk_batch* b, const int* slots, const int* tokens, const int* positions,
                  int n, int n_steps) {
  if (n < 1 || n > kBatchMaxCols)
    return fail(DQMK_ERR_INVALID, std::string(kApi) + ": 1 to 64 columns per step");
  if (!tokens || !positions) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null argument");
  const dqmk_model_config& c = b->m->cfg;
  std::vector<std::pair<int, int>> seen;
  for (int i = 0; i < n; ++i) {
    const int sl = slots ? slots[i] : i;
    if (sl < 0 || sl >= b->n_slots)
      return fail(DQMK_ERR_RANGE, std::string(kApi) + ": slot out of range");
    if (tokens[i] < 0 || tokens[i] >= c.vocab_size)
      return fail(DQMK_ERR_RANGE, std::string(kApi) + ": token id out of range");
    if (positions[i] < 0 || positions[i] + n_steps > b->max_seq)
      return fail(DQMK_ERR_RANGE, std::string(kApi) + ": position out of range");
    seen.emplace_back(sl, positions[i]);
  }
  // Each column writes KV and history at positions [pos, pos + n_steps) of
  // its slot; two columns of one slot must not share any of them.
  std::sort(seen.begin(), seen.end());
  for (size_t i = 1; i < seen.size(); ++i)
    if (seen[i].first == seen[i - 1].first && seen[i].second < seen[i - 1].second + n_steps)
      return fail(DQMK_ERR_INVALID,
                  std::string(kApi) + (n_steps > 1
                                           ? ": two columns of one slot would write the same "
                                             "positions over the decoded steps"
                                           : ": a (slot, position) appears twice"));
  return DQMK_OK;
}

}  // namespace

extern "C" int dqmk_batch_create(dqmk_model* m, int n_slots, int max_seq, dqmk_batch** out) {
  if (!m || !out) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null argument");
  if (n_slots < 1 || max_seq < 1)
    return fail(DQMK_ERR_INVALID, std::string(kApi) + ": n_slots and max_seq must be positive");
  if (!m->finalized) {
    int rc = dqmk_model_finalize(m);
    if (rc) return rc;
  }
  const dqmk_model_config& c = m->cfg;
  const dqmk_tp_plan& tp = m->tp;
  if (max_seq > c.max_seq_len)
    return fail(DQMK_ERR_RANGE, std::string(kApi) + ": max_seq above the model's max_seq_len");
  if (c.head_dim != 64 && c.head_dim != 128)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(kApi) + ": head_dim 64 or 128");
  if (m->qtype != DQMK_Q80 && m->qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(kApi) + ": Q8_0 or Q4_0 weights");
  cudaSetDevice(m->device);
  int rc = ensure_batch_weights(m);
  if (rc) return rc;
  std::unique_ptr<dqmk_batch> b(new dqmk_batch());
  b->m = m;
  b->n_slots = n_slots;
  b->max_seq = max_seq;
  DQMK_CUDA_RET(kApi, cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
  DQMK_CUDA_RET(kApi, cudaMallocHost(&b->pinned, 3 * kBatchMaxCols * sizeof(int)));
  DQMK_CUDA_RET(kApi, cudaEventCreateWithFlags(&b->staged, cudaEventDisableTiming));
  const int hd = c.head_dim, kvd = tp.n_kv_heads * hd, qd = tp.n_q_heads * hd;
  b->slot_stride = (size_t)c.n_layers * max_seq * kvd;
  const Layer& L0 = m->layers[0];
  const int kp_dim = L0.qkv.kp, kp_qd = L0.wo.kp, kp_hid = L0.down.kp;
  const int kp_max = std::max(std::max(kp_dim, kp_qd), std::max(kp_hid, m->lm_head.kp));
  size_t part = 0;
  const Packed* weights[] = {&L0.qkv, &L0.wo, &L0.gate_up, &L0.down, &m->lm_head};
  for (const Packed* w : weights) part = std::max(part, batch_partial_floats(w->rows, w->kp));
  size_t attn = 0;
  for (int n = 1; n <= kBatchMaxCols; ++n)
    attn = std::max(attn, batch_attention_partials_floats(
                              n, tp.n_q_heads, hd, batch_attention_splits(n, tp.n_kv_heads, max_seq)));
  const size_t C = kBatchMaxCols;
  struct {
    void** dst;
    size_t bytes;
  } bufs[] = {{(void**)&b->keys, b->slot_stride * n_slots * sizeof(float)},
              {(void**)&b->values, b->slot_stride * n_slots * sizeof(float)},
              {(void**)&b->x, C * c.dim * sizeof(float)},
              {(void**)&b->q, C * qd * sizeof(float)},
              {(void**)&b->att, C * qd * sizeof(float)},
              {(void**)&b->f, C * tp.hidden * sizeof(float)},
              {(void**)&b->part, C * c.dim * sizeof(float)},
              {(void**)&b->logits, C * tp.vocab_stride * sizeof(float)},
              {(void**)&b->logits_all, tp.world > 1 ? C * tp.vocab_stride * tp.world * sizeof(float) : 16},
              {(void**)&b->hi, C * kp_max * 2},
              {(void**)&b->lo, C * kp_max * 2},
              {(void**)&b->rs, C * sizeof(float)},
              {(void**)&b->partial, part * sizeof(float)},
              {(void**)&b->attn_partials, attn * sizeof(float)},
              {(void**)&b->attn_tickets, C * tp.n_kv_heads * sizeof(unsigned int)},
              {(void**)&b->cols, 3 * C * sizeof(int)},
              {(void**)&b->keys_arg, C * sizeof(unsigned long long)},
              {(void**)&b->history, (size_t)n_slots * max_seq * sizeof(int)}};
  for (auto& e : bufs) {
    void* p = nullptr;
    if ((rc = dev_alloc(b->allocs, e.bytes, &p, kApi))) return rc;
    DQMK_CUDA_RET(kApi, cudaMemset(p, 0, e.bytes ? e.bytes : 16));
    *e.dst = p;
  }
  struct {
    CUtensorMap* maps;
    int kp;
  } ks[] = {{b->x_dim, kp_dim}, {b->x_qd, kp_qd}, {b->x_hid, kp_hid}};
  for (auto& k : ks) {
    if ((rc = make_cols_map(&k.maps[0], b->hi, k.kp))) return rc;
    if ((rc = make_cols_map(&k.maps[1], b->lo, k.kp))) return rc;
  }
  if (m->lm_head.kp != kp_dim)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(kApi) + ": lm_head width differs from dim");
  DQMK_CUDA_RET(kApi, batch_prepare());
  DQMK_CUDA_RET(kApi, cudaDeviceSynchronize());
  *out = b.release();
  return DQMK_OK;
}

extern "C" int dqmk_batch_destroy(dqmk_batch* b) {
  delete b;
  return DQMK_OK;
}

extern "C" void* dqmk_batch_stream(dqmk_batch* b) { return b ? b->stream : nullptr; }

extern "C" int dqmk_batch_reset(dqmk_batch* b) {
  if (!b) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null batch");
  cudaSetDevice(b->m->device);
  const size_t kv = b->slot_stride * b->n_slots * sizeof(float);
  DQMK_CUDA_RET(kApi, cudaMemsetAsync(b->keys, 0, kv, b->stream));
  DQMK_CUDA_RET(kApi, cudaMemsetAsync(b->values, 0, kv, b->stream));
  DQMK_CUDA_RET(kApi, cudaStreamSynchronize(b->stream));
  return DQMK_OK;
}

extern "C" int dqmk_batch_step(dqmk_batch* b, const int* slots, const int* tokens,
                               const int* positions, int n, float* logits, int* next) {
  if (!b) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null batch");
  int rc = validate_cols(b, slots, tokens, positions, n, 1);
  if (rc) return rc;
  dqmk_model* m = b->m;
  cudaSetDevice(m->device);
  const bool with_logits = logits != nullptr;
  if ((rc = ensure_graph(b, n, with_logits))) return rc;
  if ((rc = stage_cols(b, slots, tokens, positions, n))) return rc;
  DQMK_CUDA_RET(kApi, cudaGraphLaunch(b->graphs[n * 2 + (with_logits ? 1 : 0)], b->stream));
  const dqmk_model_config& c = m->cfg;
  const dqmk_tp_plan& tp = m->tp;
  if (with_logits) {
    const size_t vs = (size_t)tp.vocab_stride;
    if (tp.world == 1) {
      DQMK_CUDA_RET(kApi, cudaMemcpy2DAsync(logits, c.vocab_size * sizeof(float), b->logits,
                                            vs * sizeof(float), c.vocab_size * sizeof(float), n,
                                            cudaMemcpyDeviceToHost, b->stream));
    } else {  // gather every rank's vocabulary slice, then place it per column
      if ((rc = tp_allgather(m->comm, b->logits, b->logits_all, kBatchMaxCols * vs, b->stream,
                             kApi)))
        return rc;
      for (int r = 0; r < tp.world; ++r) {
        dqmk_tp_plan pr{};
        if ((rc = tp_plan(c, r, tp.world, &pr))) return rc;
        DQMK_CUDA_RET(kApi, cudaMemcpy2DAsync(
                                logits + pr.vocab0, c.vocab_size * sizeof(float),
                                b->logits_all + (size_t)r * kBatchMaxCols * vs, vs * sizeof(float),
                                pr.vocab * sizeof(float), n, cudaMemcpyDeviceToHost, b->stream));
      }
    }
    m->stats.device_to_host_copies += 1;
    m->stats.device_to_host_bytes += (uint64_t)n * c.vocab_size * sizeof(float);
  }
  if (next)
    DQMK_CUDA_RET(kApi, cudaMemcpyAsync(next, b->col_token(), n * sizeof(int),
                                        cudaMemcpyDeviceToHost, b->stream));
  DQMK_CUDA_RET(kApi, cudaStreamSynchronize(b->stream));
  return check_errors(kApi);
}

extern "C" int dqmk_batch_decode_enqueue(dqmk_batch* b, const int* tokens, const int* positions,
                                         int n, int n_steps) {
  if (!b) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null batch");
  if (n_steps < 1) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": n_steps must be positive");
  if (n > b->n_slots) return fail(DQMK_ERR_RANGE, std::string(kApi) + ": more columns than slots");
  int rc = validate_cols(b, nullptr, tokens, positions, n, n_steps);
  if (rc) return rc;
  cudaSetDevice(b->m->device);
  if ((rc = ensure_graph(b, n, false))) return rc;
  if ((rc = stage_cols(b, nullptr, tokens, positions, n))) return rc;
  cudaGraphExec_t g = b->graphs[n * 2];
  for (int i = 0; i < n_steps; ++i) DQMK_CUDA_RET(kApi, cudaGraphLaunch(g, b->stream));
  return DQMK_OK;
}

extern "C" int dqmk_batch_history(dqmk_batch* b, int slot, int pos0, int count, int* out) {
  if (!b || !out) return fail(DQMK_ERR_INVALID, std::string(kApi) + ": null argument");
  if (slot < 0 || slot >= b->n_slots || pos0 < 0 || count < 0 || pos0 + count > b->max_seq)
    return fail(DQMK_ERR_RANGE, std::string(kApi) + ": history range out of range");
  cudaSetDevice(b->m->device);
  DQMK_CUDA_RET(kApi, cudaMemcpyAsync(out, b->history + (size_t)slot * b->max_seq + pos0,
                                      count * sizeof(int), cudaMemcpyDeviceToHost, b->stream));
  DQMK_CUDA_RET(kApi, cudaStreamSynchronize(b->stream));
  return check_errors(kApi);
}

extern "C" int dqmk_batch_decode_greedy(dqmk_batch* b, const int* tokens, const int* positions,
                                        int n, int n_steps, int* out) {
  int rc = dqmk_batch_decode_enqueue(b, tokens, positions, n, n_steps);
  if (rc) return rc;
  // out[step][column]: the token chosen after position positions[c] + step
  for (int col = 0; col < n && out; ++col) {
    std::vector<int> h(n_steps);
    if ((rc = dqmk_batch_history(b, col, positions[col], n_steps, h.data()))) return rc;
    for (int st = 0; st < n_steps; ++st) out[(size_t)st * n + col] = h[st];
  }
  DQMK_CUDA_RET(kApi, cudaStreamSynchronize(b->stream));
  return check_errors(kApi);
}
