/*
 * dqm_oracle.h -- CPU restatement of dqm-mini-llama's quantized-matmul hot
 * path.  Test infrastructure: the checker for the CUDA path, never part of
 * it.  See dqm_oracle.c for the reference citations.
 */
#ifndef DQM_ORACLE_H_
#define DQM_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml block layouts, include/dqm_llama/quantized_tensor.h:25-42 */
typedef struct {
  uint16_t d;
  int8_t qs[32];
} orc_block_q80; /* 34 bytes */

typedef struct {
  uint16_t d;
  uint8_t qs[16];
} orc_block_q40; /* 18 bytes */

typedef struct {
  uint16_t d;
  uint16_t m;
  uint8_t qs[16];
} orc_block_q41; /* 20 bytes: x = d * q + m, q an unsigned nibble */

enum { ORC_F32 = 0, ORC_Q80 = 1, ORC_Q40 = 2 };

float orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float v);

void orc_quantize_q80(const float* src, int64_t n_rows, int64_t row_size,
                      orc_block_q80* dst);
void orc_quantize_q40(const float* src, int64_t n_rows, int64_t row_size,
                      orc_block_q40* dst);
void orc_dequantize_q80(const orc_block_q80* blocks, int64_t n_rows,
                        int64_t row_size, float* dst);
void orc_dequantize_q40(const orc_block_q40* blocks, int64_t n_rows,
                        int64_t row_size, float* dst);

void orc_linear_q80(const float* x, int rows, int in_features,
                    const orc_block_q80* w, int out_features, float* y);
void orc_linear_q40(const float* x, int rows, int in_features,
                    const orc_block_q40* w, int out_features, float* y);
void orc_dequantize_q41(const orc_block_q41* blocks, int64_t n_rows,
                        int64_t row_size, float* dst);
void orc_linear_q41(const float* x, int rows, int in_features,
                    const orc_block_q41* w, int out_features, float* y);
void orc_linear_f32_simd(const float* x, int in_features, const float* w,
                         int out_features, float* y);

void orc_rmsnorm(const float* x, const float* w, int dim, float eps, float* y);
void orc_rope(float* q, int n_heads, float* k, int n_kv_heads, int head_dim,
              int pos, float theta, int neox);
void orc_softmax(const float* x, int n, float* y);
void orc_swiglu(const float* gate, const float* up, int n, float* y);
int orc_argmax(const float* x, int n);

void orc_kv_write(float* keys, float* values, int max_seq, int n_kv_heads,
                  int head_dim, int layer, int pos, const float* k,
                  const float* v);
/* scratch: 2*(pos+1) floats */
void orc_attention(const float* q, const float* keys, const float* values,
                   int max_seq, int n_kv_heads, int head_dim, int layer,
                   int pos, int n_heads, float* out, float* scratch);

typedef struct {
  const float* attention_norm;
  const void* wq;
  const void* wk;
  const void* wv;
  const float* bq; /* NULL when the model has no attention bias */
  const float* bk;
  const float* bv;
  const void* wo;
  const float* ffn_norm;
  const void* w_gate;
  const void* w_up;
  const void* w_down;
} orc_layer;

typedef struct {
  int vocab, dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, max_seq;
  float rope_theta, eps;
  int rope_neox;
  int qtype;         /* ORC_Q80 / ORC_Q40 / ORC_F32 for the layer linears */
  int lm_head_qtype; /* ORC_F32 for a tied embedding (F32 copy) */
  const float* token_embedding; /* [vocab][dim] F32 */
  const float* final_norm;
  const void* lm_head;
  const orc_layer* layers;
} orc_model;

int64_t orc_forward_scratch_floats(const orc_model* m);
void orc_forward_token(const orc_model* m, float* keys, float* values,
                       int pos, int token, float* logits, float* scratch);

#ifdef __cplusplus
}
#endif

#endif /* DQM_ORACLE_H_ */
