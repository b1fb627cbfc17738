// prefill.h -- batched prefill (tcgen05 int8 GEMM, causal attention) shared
// between prefill.cu and the engine.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace dqmk {

// One projection of a prompt chunk: C[m][n] over weight rows n (packed order).
struct PrefillGemm {
  int m;                  // valid token rows
  int m_pad;              // rows of the activation buffers (multiple of 128)
  int n;                  // weight rows
  int kp;                 // padded in_features (multiple of 32)
  const float* sx;        // activation term scales [2][m_pad][kp/32]
  const float* dwt;       // weight scales, transposed [kp/32][n], fp32
  int epi;                // kEpiStore / kEpiSwiGlu / kEpiQkv
  const float* bias;      // by packed row (may be null)
  const float* residual;  // kEpiStore: y = residual + acc (may alias y)
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
};

int make_i8_tile_map(CUtensorMap* map, const void* base, int rows, int kp);
size_t prefill_gemm_smem();
cudaError_t prefill_prepare();
cudaError_t launch_prefill_gemm(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b,
                                const PrefillGemm& p, cudaStream_t s);
cudaError_t launch_quantize_rows(const float* x, int m, int k, int kp, int ldx,
                                 const float* norm_w, float eps, int m_pad, int8_t* q, float* s,
                                 cudaStream_t st);
cudaError_t launch_embed_rows(int qtype, const uint8_t* qs, const uint16_t* d, int dim, int kp,
                              const int* tokens, int m, float* y, cudaStream_t st);
cudaError_t launch_attention_prefill(const PrefillAttn& a, cudaStream_t st);
cudaError_t launch_transpose_scales(const uint16_t* d, int n, int nbk, float* out,
                                    cudaStream_t st);
cudaError_t read_prefill_error(unsigned int* flags, bool clear);

}  // namespace dqmk
