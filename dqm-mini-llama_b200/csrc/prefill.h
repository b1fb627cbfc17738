// prefill.h -- batched prefill (tcgen05 GEMM, causal attention) shared between
// prefill.cu and the engine.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace dqmk {

// Split of the K dimension of one GEMM across CTAs.
struct GemmPlan {
  int splits;  // CTAs along K; > 1 adds a deterministic reduce + epilogue kernel
  int kb_per;  // 32-value scale blocks per split (even)
};

// One projection of a prompt chunk: C[m][n] over weight rows n (packed order).
struct PrefillGemm {
  int m;                  // valid token rows
  int n;                  // weight rows
  int kp;                 // padded in_features (multiple of 32)
  const float* rs;        // power-of-two row scales of the fp16 activation planes [m]
  const float* cs;        // power-of-two row scales of the fp16 weight planes [n]
  GemmPlan plan;
  float* partial;         // plan.splits > 1: [splits][m][n] raw sums
  int epi;                // kEpiStore / kEpiSwiGlu / kEpiQkv
  const float* bias;      // by packed row (may be null)
  const float* residual;  // kEpiStore: y = residual + (acc + bias) (may alias y)
  float* y;               // kEpiStore: [m][ldy]; kEpiSwiGlu: [m][ldy] with n/2 columns
  int ldy;
  // kEpiQkv: rows paired for RoPE like the decode GEMV
  const float2* rope_cs;
  int pos0;               // position of token row 0
  float* q_out;           // [m][ldq]
  int ldq;
  float* k_cache;
  float* v_cache;
  int layer, max_seq, n_heads, n_kv_heads, head_dim, neox;
};

struct PrefillAttn {
  const float* q;  // [m][ldq] after RoPE
  int ldq;
  const float* keys;
  const float* values;
  float* out;  // [m][ldo]
  int ldo;
  int m, pos0, layer, max_seq, n_heads, n_kv_heads, head_dim;
  // Tensor-core kernel (head_dim 64): scratch that lets several CTAs share
  // one 128-row query block's cache range (prefill_attn_part_floats and
  // prefill_attn_tickets entries for the chunk size; tickets zeroed once,
  // every launch leaves them zero).  Null: one CTA per query block.
  float* part;
  unsigned int* tickets;
  int tiles_per_split;  // target 64-position tiles per CTA (set by the launcher)
};

// 2D tiled tensor map over a row-major [outer][inner] array (no multicast
// anywhere); base, row pitch and box inner extent 16-byte multiples.
int make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                uint32_t box_outer, CUtensorMapSwizzle swizzle);
// Tensor map of an fp16 [rows][kp] plane in box_rows x 64-element boxes with
// the 128-byte swizzle of the tensor-core operand tiles.
int make_f16_tile_map(CUtensorMap* map, const void* base, int rows, int kp, int box_rows = 128);
GemmPlan plan_gemm(int m, int n, int kp);
// Largest splits * m * n over every m <= m_max (floats of the partial buffer).
size_t partial_floats_bound(int m_max, int n, int kp);
// Scratch of the split causal attention for chunks of up to m_max rows.
size_t prefill_attn_part_floats(int m_max, int n_heads);
size_t prefill_attn_tickets(int m_max, int n_heads);
cudaError_t prefill_prepare();
cudaError_t launch_prefill_gemm(const CUtensorMap& a_hi, const CUtensorMap& a_lo,
                                const CUtensorMap& b_hi, const CUtensorMap& b_lo,
                                const PrefillGemm& p, cudaStream_t s);
// x [m][ldx] (optionally RMS-normalised with norm_w) -> fp16 planes hi, lo
// [m][kp] with x * 2^-e ~= hi + lo, and rs[row] = 2^e.
// With pdl the launch may start while the previous kernel of the stream
// drains (programmatic dependent launch); the kernel waits before reading x.
cudaError_t launch_split_rows(const float* x, int m, int k, int kp, int ldx, const float* norm_w,
                              float eps, uint16_t* hi, uint16_t* lo, float* rs, cudaStream_t st,
                              bool pdl = false);
// Token ids outside [0, vocab) gather a zero row and set kErrBadToken.
cudaError_t launch_embed_rows(int qtype, const uint8_t* qs, const uint16_t* d, int dim, int kp,
                              int vocab, const int* tokens, int m, float* y, cudaStream_t st);
cudaError_t launch_attention_prefill(const PrefillAttn& a, cudaStream_t st);
// Packed Q8_0 / Q4_0 weight [rows][kp] -> exact two-term fp16 planes of
// d * q * 2^-f and the row scales cs[row] = 2^f.
cudaError_t launch_weights_split(int qtype, const uint8_t* qs, const uint16_t* d, int rows, int kp,
                                 uint16_t* bhi, uint16_t* blo, float* cs, cudaStream_t st);
cudaError_t read_prefill_error(unsigned int* flags, bool clear);

}  // namespace dqmk
