// batch.h -- decode of many sequences in one step (batch.cu), shared with the
// engine (batch_engine.cc).
//
// A step runs C <= kBatchMaxCols columns; column c feeds token[c] at position
// pos[c] of KV slot slot[c].  Every projection is one tensor-core GEMM over
// the quantized weights (weight rows x columns), decode attention runs per
// (column, KV head, split), and the lm_head GEMM ends in a per-column argmax.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "internal.h"
#include "prefill.h"

namespace dqmk {

constexpr int kBatchMaxCols = 64;

// One projection of a step: Y[c][row] over packed weight rows.
struct BatchGemm {
  int qtype;
  const uint16_t* d;      // scale plane [n][kp/32]
  int n, kp;              // weight rows, padded in_features (multiple of 32)
  int cols;               // valid columns, 1..kBatchMaxCols
  const float* rs;        // [cols] power-of-two scales of the activation planes
  const float* cs;        // [n] power-of-two row scales of the weight (2^f)
  GemmPlan plan;          // K split; kb_per even
  float* partial;         // plan.splits > 1: [splits][kBatchMaxCols][n] raw sums
  int epi;                // kEpiStore / kEpiSwiGlu / kEpiQkv / kEpiLogits
  const float* bias;      // by packed row (may be null)
  const float* residual;  // kEpiStore: [cols][ldy], may alias y
  float* y;               // [cols][ldy] (kEpiSwiGlu: n/2 outputs; kEpiLogits: may be null)
  int ldy;
  // kEpiQkv: rows paired for RoPE like the decode GEMV; caches [slot][layer][pos][kvd]
  const float2* rope_cs;
  float* q_out;
  int ldq;
  float* k_cache;
  float* v_cache;
  size_t slot_stride;     // floats from one slot's cache to the next
  int layer, max_seq, n_heads, n_kv_heads, head_dim, neox;
  const int* col_slot;    // [cols]
  const int* col_pos;     // [cols]
  // kEpiLogits: per-column argmax keys (value, first index), max-combined
  unsigned long long* keys;
  int row_offset;         // vocabulary index of packed row 0
};

// Decode attention of every column: q [cols][ldq], out [cols][ldq].
struct BatchAttn {
  const float* q;
  float* out;
  int ldq;
  const float* keys;
  const float* values;
  size_t slot_stride;
  int cols, layer, max_seq, n_heads, n_kv_heads, head_dim;
  const int* col_slot;
  const int* col_pos;
  float* partials;        // [cols][n_heads][max_splits][head_dim + 4]
  unsigned int* tickets;  // [cols][n_kv_heads], zero at rest
  int max_splits;
};

GemmPlan plan_batch_gemm(int n, int kp);
// Floats of the split-K partial buffer of plan_batch_gemm(n, kp).
size_t batch_partial_floats(int n, int kp);
int batch_row_tiles(int n);
// Tensor map of a packed quant plane [rows][kp (Q8_0) or kp/2 (Q4_0) bytes].
int make_quant_map(CUtensorMap* map, int qtype, const uint8_t* qs, int rows, int kp);
// Tensor map of an activation plane [kBatchMaxCols][kp] fp16.
int make_cols_map(CUtensorMap* map, const uint16_t* plane, int kp);
// Block scales of a weight copied into rows of scale_pitch(kp) (a multiple
// of 8, zero-padded) so TMA can fetch them, and the tensor map of the copy.
int scale_pitch(int kp);
cudaError_t copy_scales_padded(const uint16_t* d, int rows, int kp, uint16_t* d_pad,
                               cudaStream_t s);
int make_scale_map(CUtensorMap* map, const uint16_t* d_pad, int rows, int kp);
cudaError_t batch_prepare();
// The GEMM, plus the split-K reduce kernel when p.plan.splits > 1.
cudaError_t launch_batch_gemm(const CUtensorMap& wq, const CUtensorMap& wd,
                              const CUtensorMap& xhi, const CUtensorMap& xlo, const BatchGemm& p,
                              cudaStream_t s, bool pdl);
// cs[row] = 2^f with max |d q| 2^-f of the row in [2^14, 2^15) (1 for a zero row).
cudaError_t launch_weight_row_scales(int qtype, const uint8_t* qs, const uint16_t* d, int rows,
                                     int kp, float* cs, cudaStream_t s);
int batch_attention_splits(int cols, int n_kv_heads, int max_seq);
size_t batch_attention_partials_floats(int cols, int n_heads, int head_dim, int max_splits);
cudaError_t launch_attention_cols(const BatchAttn& a, cudaStream_t s, bool pdl);
// Greedy step of every column: token[c] = argmax from keys[c] (keys reset),
// history[slot][pos] = token, pos[c] += 1; a column without a valid key in
// [0, vocab) keeps its state and the batch error flag records kErrNoToken.
cudaError_t launch_cols_advance(unsigned long long* keys, int cols, const int* col_slot,
                                int* col_token, int* col_pos, int* history, int max_seq, int vocab,
                                cudaStream_t s, bool pdl);

}  // namespace dqmk
