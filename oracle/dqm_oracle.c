/*
 * dqm_oracle.c -- CPU restatement of dqm-mini-llama's block-quantized
 * matmul hot path.  TEST INFRASTRUCTURE ONLY: this file is the checker for
 * the CUDA kernels.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it; the product never does.
 *
 * Every function restates one reference routine and cites it as
 * path:line inside the dqm-mini-llama project.  Parity of this restatement
 * is pinned bit-for-bit against the reference's own CPU code compiled from
 * its sources (oracle/_ref, built by oracle/Makefile) and against the
 * known-answer values of the reference's tests/quant_test.cc.
 *
 * Floating-point contraction: the reference is built with -O3 -mavx2 -mfma
 * in GNU C++ mode, where GCC contracts `sum += a * b` into one fused
 * multiply-add.  This file is compiled with -ffp-contract=off and spells
 * every contraction out with fmaf(), so the rounding sequence is written
 * down instead of left to the compiler.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "dqm_oracle.h"

/* ------------------------------------------------------------------ */
/* fp16 <-> fp32, src/quant.cc:19-90                                   */
/* ------------------------------------------------------------------ */

/* src/quant.cc:19-50.  Exact widening, subnormals normalised. */
float orc_fp16_to_fp32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      /* normalise: shift the mantissa up until the implicit bit appears */
      int32_t exp = 1;
      while ((m & 0x400u) == 0) {
        m <<= 1;
        exp -= 1;
      }
      m &= 0x3ffu;
      bits = sign | ((uint32_t)(exp + 112) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* src/quant.cc:53-90.  NOT round-to-nearest-even: the result is bumped
 * whenever bit 12 of the (shifted) mantissa is set, i.e. ties round away
 * from zero in magnitude and sticky bits below bit 12 are ignored.
 * Overflow saturates to infinity; NaN inputs also map to infinity. */
uint16_t orc_fp32_to_fp16(float v) {
  uint32_t bits;
  memcpy(&bits, &v, sizeof bits);
  uint32_t sign = (bits >> 16) & 0x8000u;
  int32_t exp = (int32_t)((bits >> 23) & 0xffu) - 112;
  uint32_t m = bits & 0x7fffffu;
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    m |= 0x800000u;
    uint32_t sh = m >> (uint32_t)(1 - exp);
    if (sh & 0x1000u) sh += 0x2000u;
    return (uint16_t)(sign | (sh >> 13));
  }
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  if (m & 0x1000u) {
    m += 0x2000u;
    if (m & 0x800000u) {
      m = 0;
      exp += 1;
      if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    }
  }
  return (uint16_t)(sign | ((uint32_t)exp << 10) | (m >> 13));
}

/* ------------------------------------------------------------------ */
/* Quantize / dequantize, src/quant.cc:117-190, 372-476                */
/* A tensor is split into rows of `row_size` (its last dimension); each */
/* row is cut into ceil(row_size/32) blocks, the last one zero-padded.  */
/* ------------------------------------------------------------------ */

static int64_t blocks_per_row(int64_t row_size) { return (row_size + 31) / 32; }

/* src/quant.cc:372-418 */
void orc_quantize_q80(const float* src, int64_t n_rows, int64_t row_size,
                      orc_block_q80* dst) {
  const int64_t nb = blocks_per_row(row_size);
  for (int64_t r = 0; r < n_rows; ++r) {
    const float* row = src + r * row_size;
    for (int64_t b = 0; b < nb; ++b) {
      orc_block_q80* blk = dst + r * nb + b;
      memset(blk, 0, sizeof *blk);
      const int64_t k0 = b * 32;
      const int64_t len = (row_size - k0) < 32 ? (row_size - k0) : 32;
      float amax = 0.0f;
      for (int64_t i = 0; i < len; ++i) {
        float a = fabsf(row[k0 + i]);
        if (a > amax) amax = a;
      }
      if (amax > 0.0f) {
        blk->d = orc_fp32_to_fp16(amax / 127.0f);
        float stored = orc_fp16_to_fp32(blk->d);
        float inv = stored == 0.0f ? 0.0f : 1.0f / stored;
        for (int64_t i = 0; i < len; ++i) {
          int q = (int)roundf(row[k0 + i] * inv);
          if (q > 127) q = 127;
          if (q < -127) q = -127;
          blk->qs[i] = (int8_t)q;
        }
      }
    }
  }
}

/* src/quant.cc:420-476.  Scale absmax/7, offset 8, clamp to [0,15];
 * element j goes to the low nibble of byte j, element j+16 to its high
 * nibble. */
void orc_quantize_q40(const float* src, int64_t n_rows, int64_t row_size,
                      orc_block_q40* dst) {
  const int64_t nb = blocks_per_row(row_size);
  for (int64_t r = 0; r < n_rows; ++r) {
    const float* row = src + r * row_size;
    for (int64_t b = 0; b < nb; ++b) {
      orc_block_q40* blk = dst + r * nb + b;
      memset(blk, 0, sizeof *blk);
      const int64_t k0 = b * 32;
      const int64_t len = (row_size - k0) < 32 ? (row_size - k0) : 32;
      float amax = 0.0f;
      for (int64_t i = 0; i < len; ++i) {
        float a = fabsf(row[k0 + i]);
        if (a > amax) amax = a;
      }
      if (amax > 0.0f) {
        blk->d = orc_fp32_to_fp16(amax / 7.0f);
        float stored = orc_fp16_to_fp32(blk->d);
        float inv = stored == 0.0f ? 0.0f : 1.0f / stored;
        for (int j = 0; j < 16; ++j) {
          float x0 = j < len ? row[k0 + j] * inv : 0.0f;
          float x1 = (j + 16) < len ? row[k0 + j + 16] * inv : 0.0f;
          int q0 = (int)roundf(x0 + 8.0f);
          int q1 = (int)roundf(x1 + 8.0f);
          q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
          q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
          blk->qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
      }
    }
  }
}

/* src/quant.cc:117-148 */
void orc_dequantize_q80(const orc_block_q80* blocks, int64_t n_rows,
                        int64_t row_size, float* dst) {
  const int64_t nb = blocks_per_row(row_size);
  for (int64_t r = 0; r < n_rows; ++r) {
    for (int64_t k = 0; k < row_size; ++k) {
      const orc_block_q80* blk = blocks + r * nb + k / 32;
      dst[r * row_size + k] = orc_fp16_to_fp32(blk->d) * (float)blk->qs[k % 32];
    }
  }
}

/* src/quant.cc:150-190 */
void orc_dequantize_q40(const orc_block_q40* blocks, int64_t n_rows,
                        int64_t row_size, float* dst) {
  const int64_t nb = blocks_per_row(row_size);
  for (int64_t r = 0; r < n_rows; ++r) {
    for (int64_t k = 0; k < row_size; ++k) {
      const orc_block_q40* blk = blocks + r * nb + k / 32;
      int j = (int)(k % 32);
      int q = j < 16 ? (blk->qs[j] & 0x0f) : (blk->qs[j - 16] >> 4);
      dst[r * row_size + k] = orc_fp16_to_fp32(blk->d) * (float)(q - 8);
    }
  }
}

/* ------------------------------------------------------------------ */
/* Quantized Linear, src/quant.cc:243-346                              */
/* y[r][j] = one sequential fused-multiply-add chain over k ascending   */
/* of (d * q_k) * x_k, where d * q_k is rounded first (it is exact: an  */
/* fp16 times an int8 fits a float significand).                        */
/* ------------------------------------------------------------------ */

/* src/quant.cc:244-246 (DequantQ80) and :326-344 (the k loop) */
void orc_linear_q80(const float* x, int rows, int in_features,
                    const orc_block_q80* w, int out_features, float* y) {
  const int nb = (int)blocks_per_row(in_features);
  for (int64_t flat = 0; flat < (int64_t)rows * out_features; ++flat) {
    const int r = (int)(flat / out_features);
    const int j = (int)(flat % out_features);
    const float* xr = x + (int64_t)r * in_features;
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b) {
      const orc_block_q80* blk = w + (int64_t)j * nb + b;
      const float d = orc_fp16_to_fp32(blk->d);
      const int k0 = b * 32;
      const int k1 = k0 + 32 < in_features ? k0 + 32 : in_features;
      for (int k = k0; k < k1; ++k) {
        sum = fmaf(d * (float)blk->qs[k - k0], xr[k], sum);
      }
    }
    y[flat] = sum;
  }
}

/* src/quant.cc:249-254 (DequantQ40) and :326-344 */
void orc_linear_q40(const float* x, int rows, int in_features,
                    const orc_block_q40* w, int out_features, float* y) {
  const int nb = (int)blocks_per_row(in_features);
  for (int64_t flat = 0; flat < (int64_t)rows * out_features; ++flat) {
    const int r = (int)(flat / out_features);
    const int j = (int)(flat % out_features);
    const float* xr = x + (int64_t)r * in_features;
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b) {
      const orc_block_q40* blk = w + (int64_t)j * nb + b;
      const float d = orc_fp16_to_fp32(blk->d);
      const int k0 = b * 32;
      const int k1 = k0 + 32 < in_features ? k0 + 32 : in_features;
      for (int k = k0; k < k1; ++k) {
        const int i = k - k0;
        const int q = i < 16 ? (blk->qs[i] & 0x0f) : (blk->qs[i - 16] >> 4);
        sum = fmaf(d * (float)(q - 8), xr[k], sum);
      }
    }
    y[flat] = sum;
  }
}

/* src/quant.cc:256-262 (DequantQ41, d * q + m: contracted to one fused
 * multiply-add in the -O3 -mfma build) and :326-344 (the k loop) */
static float dequant_q41(const orc_block_q41* blk, int i) {
  const int q = i < 16 ? (blk->qs[i] & 0x0f) : (blk->qs[i - 16] >> 4);
  return fmaf(orc_fp16_to_fp32(blk->d), (float)q, orc_fp16_to_fp32(blk->m));
}

void orc_linear_q41(const float* x, int rows, int in_features,
                    const orc_block_q41* w, int out_features, float* y) {
  const int nb = (int)blocks_per_row(in_features);
  for (int64_t flat = 0; flat < (int64_t)rows * out_features; ++flat) {
    const int r = (int)(flat / out_features);
    const int j = (int)(flat % out_features);
    const float* xr = x + (int64_t)r * in_features;
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b) {
      const orc_block_q41* blk = w + (int64_t)j * nb + b;
      const int k0 = b * 32;
      const int k1 = k0 + 32 < in_features ? k0 + 32 : in_features;
      for (int k = k0; k < k1; ++k) sum = fmaf(dequant_q41(blk, k - k0), xr[k], sum);
    }
    y[flat] = sum;
  }
}

/* src/quant.cc:192-235 (DequantizeFromQ41): the same d * q + m per value as
 * the Linear's dequantization, low nibbles values 0-15, high 16-31 */
void orc_dequantize_q41(const orc_block_q41* blocks, int64_t n_rows, int64_t row_size,
                        float* dst) {
  const int64_t nb = blocks_per_row(row_size);
  for (int64_t r = 0; r < n_rows; ++r)
    for (int64_t k = 0; k < row_size; ++k)
      dst[r * row_size + k] = dequant_q41(blocks + r * nb + k / 32, (int)(k % 32));
}

/* F32 Linear in the reference's default "threaded-simd" mode:
 * src/matmul_dispatch.cc:208-222 (LinearThreadedSimd) over
 * src/matmul_dispatch.cc:153-173 (DotSimdAvx2).  Eight lane accumulators
 * take k = 8i + lane with fused multiply-adds; the lanes are then folded
 * (l + l+4), (0+1), (2+3), and the two pair sums added; a scalar fused
 * tail finishes k >= 8*floor(n/8). */
void orc_linear_f32_simd(const float* x, int in_features, const float* w,
                         int out_features, float* y) {
  for (int j = 0; j < out_features; ++j) {
    const float* wr = w + (int64_t)j * in_features;
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k + 8 <= in_features; k += 8) {
      for (int l = 0; l < 8; ++l) lane[l] = fmaf(x[k + l], wr[k + l], lane[l]);
    }
    float s0 = lane[0] + lane[4];
    float s1 = lane[1] + lane[5];
    float s2 = lane[2] + lane[6];
    float s3 = lane[3] + lane[7];
    float r = (s0 + s1) + (s2 + s3);
    /* Tail: GCC vectorises the first four remaining products (rounded
     * multiplies added in order) and fuses the rest one by one. */
    if (in_features - k >= 4) {
      for (int t = 0; t < 4; ++t, ++k) r = r + x[k] * wr[k];
    }
    for (; k < in_features; ++k) r = fmaf(x[k], wr[k], r);
    y[j] = r;
  }
}

/* ------------------------------------------------------------------ */
/* Memory-bound ops, src/ops.cc                                        */
/* ------------------------------------------------------------------ */

/* src/ops.cc:68-90.  The sum of squares is NOT fused in the reference
 * build: GCC vectorises the squares (rounded multiplies) and adds them in
 * order, so each square is rounded before it is accumulated. */
void orc_rmsnorm(const float* x, const float* w, int dim, float eps, float* y) {
  float mean = 0.0f;
  for (int i = 0; i < dim; ++i) mean = mean + x[i] * x[i];
  mean /= (float)dim;
  const float scale = 1.0f / sqrtf(mean + eps);
  for (int i = 0; i < dim; ++i) y[i] = (x[i] * scale) * w[i];
}

/* Rotation of one pair: x0' = x0*c - x1*s, x1' = x0*s + x1*c.
 * NeoX pairs (ops.cc:46-49) are rotated with the left product fused; the
 * adjacent Normal pairs (ops.cc:24-27) are SLP-vectorised by GCC in the
 * reference build and come out with every product rounded. */
static void rot_fused(float* a, float* b, float c, float s) {
  const float x0 = *a, x1 = *b;
  *a = fmaf(x0, c, -(x1 * s));
  *b = fmaf(x0, s, x1 * c);
}

static void rot_plain(float* a, float* b, float c, float s) {
  const float x0 = *a, x1 = *b;
  *a = x0 * c - x1 * s;
  *b = x0 * s + x1 * c;
}

/* Frequency of pair i (exponent numerator e = 2i for both variants):
 * src/ops.cc:18-20 and :40-42. */
static float rope_freq(float theta, int e, int head_dim) {
  return 1.0f / powf(theta, (float)e / (float)head_dim);
}

/* src/ops.cc:13-52 (ApplyRopeNormalToHeads / ApplyRopeNeoXToHeads) */
static void rope_heads(float* x, int n_heads, int head_dim, int pos,
                       float theta, int neox) {
  const int half = head_dim / 2;
  for (int h = 0; h < n_heads; ++h) {
    float* base = x + (int64_t)h * head_dim;
    for (int i = 0; i < half; ++i) {
      const float freq = rope_freq(theta, 2 * i, head_dim);
      const float angle = (float)pos * freq;
      const float c = cosf(angle), s = sinf(angle);
      if (neox) {
        rot_fused(base + i, base + half + i, c, s);
      } else {
        rot_plain(base + 2 * i, base + 2 * i + 1, c, s);
      }
    }
  }
}

/* src/ops.cc:153-180 */
void orc_rope(float* q, int n_heads, float* k, int n_kv_heads, int head_dim,
              int pos, float theta, int neox) {
  rope_heads(q, n_heads, head_dim, pos, theta, neox);
  rope_heads(k, n_kv_heads, head_dim, pos, theta, neox);
}

/* src/ops.cc:92-118 */
void orc_softmax(const float* x, int n, float* y) {
  float mx = x[0];
  for (int i = 1; i < n; ++i)
    if (x[i] > mx) mx = x[i];
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    y[i] = expf(x[i] - mx);
    sum += y[i];
  }
  for (int i = 0; i < n; ++i) y[i] /= sum;
}

/* src/ops.cc:140-151 */
void orc_swiglu(const float* gate, const float* up, int n, float* y) {
  for (int i = 0; i < n; ++i) {
    const float g = gate[i];
    const float sig = 1.0f / (1.0f + expf(-g));
    y[i] = (g * sig) * up[i];
  }
}

/* src/ops.cc:182-195: first maximum wins. */
int orc_argmax(const float* x, int n) {
  int best = 0;
  float bv = x[0];
  for (int i = 1; i < n; ++i)
    if (x[i] > bv) {
      bv = x[i];
      best = i;
    }
  return best;
}

/* ------------------------------------------------------------------ */
/* KV cache + decode attention, src/kv_cache.cc:25-53 and              */
/* src/forward.cc:426-507.  Cache layout [layer][max_seq][n_kv][hd].   */
/* ------------------------------------------------------------------ */

void orc_kv_write(float* keys, float* values, int max_seq, int n_kv_heads,
                  int head_dim, int layer, int pos, const float* k,
                  const float* v) {
  const int64_t stride = (int64_t)n_kv_heads * head_dim;
  const int64_t base = ((int64_t)layer * max_seq + pos) * stride;
  memcpy(keys + base, k, (size_t)stride * sizeof(float));
  memcpy(values + base, v, (size_t)stride * sizeof(float));
}

/* src/forward.cc:461-506 (CPU branch of AttentionForward). */
void orc_attention(const float* q, const float* keys, const float* values,
                   int max_seq, int n_kv_heads, int head_dim, int layer,
                   int pos, int n_heads, float* out, float* scratch) {
  const float scale = 1.0f / sqrtf((float)head_dim);
  const int group = n_heads / n_kv_heads; /* forward.cc:427-430 */
  const int64_t pos_stride = (int64_t)n_kv_heads * head_dim;
  const int64_t layer_base = (int64_t)layer * max_seq * pos_stride;
  float* scores = scratch;
  float* probs = scratch + (pos + 1);
  for (int h = 0; h < n_heads; ++h) {
    const int kvh = h / group;
    const float* qh = q + (int64_t)h * head_dim;
    for (int t = 0; t <= pos; ++t) {
      const float* kp = keys + layer_base + t * pos_stride + (int64_t)kvh * head_dim;
      float dot = 0.0f;
      /* each product rounded, then added in order: the reference build
       * does not fuse this loop (forward.cc:476-479) */
      for (int d = 0; d < head_dim; ++d) dot = dot + qh[d] * kp[d];
      scores[t] = dot * scale;
    }
    orc_softmax(scores, pos + 1, probs);
    for (int d = 0; d < head_dim; ++d) {
      float acc = 0.0f;
      for (int t = 0; t <= pos; ++t) {
        const float* vp =
            values + layer_base + t * pos_stride + (int64_t)kvh * head_dim;
        acc = acc + probs[t] * vp[d]; /* not fused either (:487-492) */
      }
      out[(int64_t)h * head_dim + d] = acc;
    }
  }
}

/* ------------------------------------------------------------------ */
/* One decode token through the whole model:                            */
/* src/forward.cc:729-754 (ForwardToken, CPU branch), :574-628          */
/* (ForwardLayer), :60-73 (AddOptionalBias), :344-366 (ForwardAdd),     */
/* :528-557 (FfnForward), :709-714 (ComputeLogits), :400-407            */
/* (EmbedToken).                                                        */
/* ------------------------------------------------------------------ */

static void linear_any(int qtype, const void* w, const float* x, int in,
                       int out, float* y) {
  if (qtype == ORC_Q80) {
    orc_linear_q80(x, 1, in, (const orc_block_q80*)w, out, y);
  } else if (qtype == ORC_Q40) {
    orc_linear_q40(x, 1, in, (const orc_block_q40*)w, out, y);
  } else {
    orc_linear_f32_simd(x, in, (const float*)w, out, y);
  }
}

static void add_bias(float* x, const float* b, int n) {
  if (!b) return;
  for (int i = 0; i < n; ++i) x[i] = x[i] + b[i];
}

int64_t orc_forward_scratch_floats(const orc_model* m) {
  const int64_t qd = (int64_t)m->n_heads * m->head_dim;
  const int64_t kvd = (int64_t)m->n_kv_heads * m->head_dim;
  return 4 * (int64_t)m->dim + qd * 2 + 2 * kvd + 3 * (int64_t)m->hidden_dim +
         2 * (int64_t)m->max_seq;
}

void orc_forward_token(const orc_model* m, float* keys, float* values,
                       int pos, int token, float* logits, float* scratch) {
  const int dim = m->dim, hd = m->head_dim, nh = m->n_heads,
            nkv = m->n_kv_heads, hid = m->hidden_dim;
  const int qd = nh * hd, kvd = nkv * hd;
  float* x = scratch;
  float* h = x + dim;
  float* tmp = h + dim;
  float* x2 = tmp + dim;
  float* q = x2 + dim;
  float* att = q + qd;
  float* k = att + qd;
  float* v = k + kvd;
  float* g = v + kvd;
  float* u = g + hid;
  float* f = u + hid;
  float* attn_scratch = f + hid;

  memcpy(x, m->token_embedding + (int64_t)token * dim, (size_t)dim * sizeof(float));
  for (int l = 0; l < m->n_layers; ++l) {
    const orc_layer* L = &m->layers[l];
    orc_rmsnorm(x, L->attention_norm, dim, m->eps, h);
    linear_any(m->qtype, L->wq, h, dim, qd, q);
    linear_any(m->qtype, L->wk, h, dim, kvd, k);
    linear_any(m->qtype, L->wv, h, dim, kvd, v);
    add_bias(q, L->bq, qd);
    add_bias(k, L->bk, kvd);
    add_bias(v, L->bv, kvd);
    orc_rope(q, nh, k, nkv, hd, pos, m->rope_theta, m->rope_neox);
    orc_kv_write(keys, values, m->max_seq, nkv, hd, l, pos, k, v);
    orc_attention(q, keys, values, m->max_seq, nkv, hd, l, pos, nh, att,
                  attn_scratch);
    linear_any(m->qtype, L->wo, att, qd, dim, tmp);
    for (int i = 0; i < dim; ++i) x2[i] = x[i] + tmp[i];
    orc_rmsnorm(x2, L->ffn_norm, dim, m->eps, h);
    linear_any(m->qtype, L->w_gate, h, dim, hid, g);
    linear_any(m->qtype, L->w_up, h, dim, hid, u);
    orc_swiglu(g, u, hid, f);
    linear_any(m->qtype, L->w_down, f, hid, dim, tmp);
    for (int i = 0; i < dim; ++i) x[i] = x2[i] + tmp[i];
  }
  orc_rmsnorm(x, m->final_norm, dim, m->eps, h);
  linear_any(m->lm_head_qtype, m->lm_head, h, dim, m->vocab, logits);
}
