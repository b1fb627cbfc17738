/*
 * dqmk.h -- C ABI of the B200 (sm_100a) block-quantized matmul path for the
 * dqm-mini-llama engine.
 *
 * Every entry point takes plain pointers and sizes, returns a dqmk_status and
 * never throws.  On failure dqmk_last_error() returns a message that starts
 * with the name of the reference API the entry point replaces (for example
 * "CudaQ80Linear: block count mismatch ..."), so the engine's C++ shim can
 * rethrow it unchanged.  DQMK_ERR_RANGE maps to std::out_of_range, every
 * other non-zero status to std::runtime_error.
 *
 * Pointers named *_dev are device pointers (cudaMalloc, or any pointer the
 * device can dereference); `stream` is a cudaStream_t passed as void*
 * (NULL = legacy default stream).  Calls are asynchronous on `stream` unless
 * stated otherwise.
 *
 * Block layouts are ggml's (include/dqm_llama/quantized_tensor.h:25-42):
 * Q8_0 = { uint16 d (fp16); int8 qs[32] } (34 bytes), Q4_0 = { uint16 d;
 * uint8 qs[16] } (18 bytes, element j in the low nibble of qs[j], element
 * j+16 in the high nibble).  A [rows, cols] tensor is rows * ceil(cols/32)
 * blocks, row-major.
 *
 * Citations are path:line inside the dqm-mini-llama project.
 */
#ifndef DQMK_H_
#define DQMK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dqmk_status {
  DQMK_OK = 0,
  DQMK_ERR_INVALID = 1,     /* bad shape / null pointer / count mismatch -> runtime_error */
  DQMK_ERR_RANGE = 2,       /* layer, pos or token out of range -> out_of_range */
  DQMK_ERR_CUDA = 3,        /* CUDA runtime error (message has cudaGetErrorString) */
  DQMK_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up */
  DQMK_ERR_UNSUPPORTED = 5, /* shape or type this build does not handle */
  DQMK_ERR_NOMEM = 6        /* device allocation failed */
} dqmk_status;

enum { DQMK_F32 = 0, DQMK_Q80 = 1, DQMK_Q40 = 2, DQMK_Q41 = 3 };

/* Message of the last failed call on this host thread ("" if none). */
const char* dqmk_last_error(void);

/* 1: kernels built for sm_100a.  Replaces CudaQuantBuilt / CudaOpsBuilt /
 * CudaAttentionBuilt / CudaKvCacheBuilt (include/dqm_llama/cuda_quant.h:15,
 * cuda_ops.h:13, cuda_attention.h:11, cuda_kv_cache.h:12). */
int dqmk_built(void);

/* ------------------------------------------------------------------ */
/* Block quantization (bit-exact with the reference's CPU routines)     */
/* ------------------------------------------------------------------ */

/* QuantizeToQ80 (src/quant.cc:372-418): src_dev [n_rows, row_size] f32 ->
 * n_rows*ceil(row_size/32) Q8_0 blocks.  Scale = fp16(absmax/127) with the
 * reference's fp16 rounding, inverse of the STORED scale, round half away
 * from zero, clamp to +-127, tail lanes zero. */
int dqmk_quantize_q80(const float* src_dev, int64_t n_rows, int64_t row_size,
                      void* blocks_dev, void* stream);

/* QuantizeToQ40 (src/quant.cc:420-476): scale absmax/7, q = clamp(round(x/d
 * + 8), 0, 15). */
int dqmk_quantize_q40(const float* src_dev, int64_t n_rows, int64_t row_size,
                      void* blocks_dev, void* stream);

/* DequantizeFromQ80 / DequantizeFromQ40 (src/quant.cc:117-190). */
int dqmk_dequantize_q80(const void* blocks_dev, int64_t n_rows, int64_t row_size,
                        float* dst_dev, void* stream);
int dqmk_dequantize_q40(const void* blocks_dev, int64_t n_rows, int64_t row_size,
                        float* dst_dev, void* stream);

/* ------------------------------------------------------------------ */
/* Quantized Linear on ggml blocks (drop-in)                            */
/* ------------------------------------------------------------------ */

/* y_dev[rows, out] = x_dev[rows, in] * W^T (+ bias_dev[out] if non-NULL),
 * W = [out_features, in_features] as ggml blocks, block_count must equal
 * out_features * ceil(in_features/32).  Replaces CudaQ80LinearDeviceInput
 * (include/dqm_llama/cuda_quant.h:27-31; src/cuda_quant.cu:487) and the bias
 * form of CudaQ80Linear / CudaQ80LinearDeviceWeight (cuda_quant.h:17-25). */
int dqmk_q80_linear(const float* x_dev, int rows, int in_features, const void* blocks_dev,
                    size_t block_count, int out_features, const float* bias_dev,
                    float* y_dev, void* stream);

/* Q4_0 twin: CudaQ40LinearDeviceInput / CudaQ40Linear(DeviceWeight)
 * (include/dqm_llama/cuda_quant.h:33-47). */
int dqmk_q40_linear(const float* x_dev, int rows, int in_features, const void* blocks_dev,
                    size_t block_count, int out_features, const float* bias_dev,
                    float* y_dev, void* stream);

/* Q4_1 twin (20-byte blocks { fp16 d; fp16 m; uint8 qs[16] }, value d * q + m
 * with an unsigned nibble q): CudaQ41LinearDeviceInput / CudaQ41Linear
 * (DeviceWeight) (include/dqm_llama/cuda_quant.h:49-63; src/cuda_quant.cu:
 * 105-127). */
int dqmk_q41_linear(const float* x_dev, int rows, int in_features, const void* blocks_dev,
                    size_t block_count, int out_features, const float* bias_dev,
                    float* y_dev, void* stream);

/* F32-weight Linear: y_dev[rows, out] = x_dev[rows, in] * W^T (+ bias) for
 * W_dev [out_features, in_features] float.  Replaces CudaLinear /
 * CudaLinearDeviceWeight / CudaLinearDeviceInput (include/dqm_llama/
 * cuda_matmul.h:25-41; src/cuda_matmul.cc:60-64,167,209,251: a cuBLAS SGEMM
 * with a handle created per call).  A bandwidth-bound warp-per-row kernel. */
int dqmk_f32_linear(const float* x_dev, int rows, int in_features, const float* w_dev,
                    int out_features, const float* bias_dev, float* y_dev, void* stream);

/* ------------------------------------------------------------------ */
/* Planar ("packed") weights: the layout the engine keeps in HBM        */
/* ------------------------------------------------------------------ */
/* A packed [out, in] weight is the same bytes as its ggml blocks, split
 * into two planes: quants first (Q8_0: int8 [out][kp], Q4_0: uint8
 * [out][kp/2] with ggml's nibble order inside each 16-byte block; kp =
 * 32*ceil(in/32), tail values zero), then scales (fp16 [out][kp/32]).
 * Every quant row starts 16-byte aligned, so rows stream with 128-bit loads
 * and tile cleanly for TMA.  Replaces the verbatim block upload of
 * UploadQuantizedLinearWeight (src/model.cc:97-137). */
size_t dqmk_packed_bytes(int qtype, int out_features, int in_features);
int dqmk_pack_weight(int qtype, const void* blocks_dev, size_t block_count, int out_features,
                     int in_features, void* packed_dev, void* stream);

/* Batch-1 decode GEMV on a packed weight: y[o] = residual[o] + bias[o] +
 * sum_k W[o][k] x[k] (residual_dev / bias_dev may be NULL; y_dev may equal
 * residual_dev).  The kernel behind every projection of the decode step. */
int dqmk_gemv_packed(int qtype, const float* x_dev, int in_features, const void* packed_dev,
                     int out_features, const float* bias_dev, const float* residual_dev,
                     float* y_dev, void* stream);

/* The decode step's GEMV as the step launches it, for measurement: RMSNorm
 * of x by norm_dev (NULL: none) in the prologue, y = W x (swiglu == 0) or the
 * SwiGLU of interleaved gate/up rows (swiglu != 0; y has out_features / 2
 * values), launched with programmatic dependent launch so back-to-back calls
 * overlap like the kernels of the captured step.  No reference counterpart. */
int dqmk_gemv_packed_chained(int qtype, const float* x_dev, int in_features,
                             const void* packed_dev, int out_features, const float* norm_dev,
                             float eps, int swiglu, float* y_dev, void* stream);

/* Batched (prefill) linear on a packed weight, on the tensor cores:
 * y[m][o] = residual[m][o] + bias[o] + sum_k W[o][k] x[m][k] for `m` rows
 * (residual_dev / bias_dev may be NULL; y_dev may equal residual_dev).  The
 * batched form of LinearQ80 / LinearQ40 (src/quant.cc:350-360, rows of x
 * times the block-dequantized weight) and of the reference's per-token
 * Linear calls inside ForwardBatch (src/batch.cc:35-40).  Every
 * dequantized weight is exact as two fp16 terms once its row is scaled by a
 * power of two; each row of x is scaled likewise and split into two fp16
 * terms (relative error <= 2^-22); the tensor cores accumulate the products
 * in fp32 over all of K, so results match the F32 product to fp32
 * summation-order differences.  Scratch (including the weight's fp16 planes)
 * is allocated stream-ordered on `stream`; the engine keeps its weights'
 * planes resident instead. */
int dqmk_linear_batch_packed(int qtype, const float* x_dev, int m, int in_features,
                             const void* packed_dev, int out_features, const float* bias_dev,
                             const float* residual_dev, float* y_dev, void* stream);

/* Multi-sequence decode linear: the same product for 1..64 columns of x
 * (one per sequence), computed the way a dqmk_batch step runs its
 * projections -- the packed Q8_0 / Q4_0 blocks are streamed from HBM once and
 * turned into exact two-term fp16 tensor-core operands on chip (no fp16
 * weight planes are kept).  y[c][o] = residual[c][o] + bias[o] +
 * sum_k W[o][k] x[c][k]; results match the F32 product to fp32
 * summation-order differences.  Scratch is stream-ordered on `stream`. */
int dqmk_linear_cols_packed(int qtype, const float* x_dev, int cols, int in_features,
                            const void* packed_dev, int out_features, const float* bias_dev,
                            const float* residual_dev, float* y_dev, void* stream);

/* Failure detection.  Kernels that wait on asynchronous copies bound every
 * wait (about one second); a wait that runs out records a flag in device
 * memory and the kernel exits instead of hanging.  dqmk_device_error returns
 * the flags (bit 0: a bounded wait timed out; -1 if the read itself failed)
 * and clears them when `clear` != 0.  The engine's synchronous calls check
 * the flag and return DQMK_ERR_TIMEOUT.  No reference counterpart: the
 * reference has no device-side waits. */
int dqmk_device_error(int clear);

/* Test hook for the above: dqmk_gemv_packed with the shared-memory copies of
 * one row tile (tile index `tile`, 8-32 rows) withheld, so that tile's wait
 * runs out.  Outputs are undefined; the device error flag is set. */
int dqmk_gemv_packed_withhold_tile(int qtype, const float* x_dev, int in_features,
                                   const void* packed_dev, int out_features, float* y_dev,
                                   int tile, void* stream);

/* Test hook exposing the integer arithmetic of the TMA-staged GEMV (the
 * lm_head form): x_dev (in_features floats) is split into three int8 terms
 * per 32-value block, x ~= s1 q1 + s2 q2 + s3 q3, and every block b of every
 * row of the packed weight is summed exactly against each term with dp4a:
 * sums_dev[row][t][b] = sum_j w_j q_t[j] (Q4_0: nibble - 8).  Outputs:
 * q_terms_dev [3][nb][32] int8, scales_dev [3][nb] float, sums_dev
 * [out_features][3][nb] int32 (nb = ceil(in_features/32)).  One CTA; for
 * checking against an integer restatement on the host, not for speed.  No
 * reference counterpart: the reference's Linear has no integer dot product. */
int dqmk_lm_head_block_sums(int qtype, const float* x_dev, int in_features,
                            const void* packed_dev, int out_features, int8_t* q_terms_dev,
                            float* scales_dev, int32_t* sums_dev, void* stream);

/* ------------------------------------------------------------------ */
/* Memory-bound ops                                                     */
/* ------------------------------------------------------------------ */

/* CudaRmsNormDeviceWeight (include/dqm_llama/cuda_ops.h:35-38; reference
 * math src/ops.cc:68-90): y = x * (1/sqrt(mean(x^2) + eps)) * w. */
int dqmk_rmsnorm(const float* x_dev, const float* w_dev, int dim, float eps, float* y_dev,
                 void* stream);

/* CudaSiluDeviceInput + CudaElementwiseMulDeviceInput (cuda_ops.h:39-44),
 * reference SwiGlu (src/ops.cc:140-151): y = silu(gate) * up. */
int dqmk_silu_mul(const float* gate_dev, const float* up_dev, int n, float* y_dev, void* stream);

/* CudaSiluDeviceInput (cuda_ops.h:39-40): y = x * sigmoid(x);
 * CudaElementwiseMulDeviceInput (cuda_ops.h:41-44): y = a * b;
 * CudaSoftmax (cuda_ops.h:24): y = softmax(x) over n values.  The decode step
 * fuses these into its kernels; the standalone forms serve the per-op API. */
int dqmk_silu(const float* x_dev, int n, float* y_dev, void* stream);
int dqmk_mul(const float* a_dev, const float* b_dev, int n, float* y_dev, void* stream);
int dqmk_softmax(const float* x_dev, int n, float* y_dev, void* stream);

/* CudaElementwiseAddDeviceInput / DeviceWeight (cuda_ops.h:45-53): y = a + b. */
int dqmk_add(const float* a_dev, const float* b_dev, int n, float* y_dev, void* stream);

/* CudaRopeDeviceInput (cuda_ops.h:57-61; reference src/ops.cc:13-52,153-180):
 * rotates q [n_heads, head_dim] and k [n_kv_heads, head_dim] in place at
 * position pos.  neox != 0 pairs (i, i+head_dim/2), else (2i, 2i+1).  The
 * cos/sin table is computed on the host with the reference's float
 * expressions, so the rotation angles are the reference's bit for bit. */
int dqmk_rope(float* q_dev, float* k_dev, int n_heads, int n_kv_heads, int head_dim, int pos,
              float theta, int neox, void* stream);

/* CudaEmbeddingLookupDeviceWeight (cuda_ops.h:28-31): y = table[token]. */
int dqmk_embedding_lookup(const float* table_dev, int vocab, int dim, int token, float* y_dev,
                          void* stream);

/* Embedding row gathered straight from Q8_0 / Q4_0 token_embd blocks: the
 * same values the reference's F32 table holds after DequantizeFromQ80/Q40
 * (src/gguf_loader.cc:313-326). */
int dqmk_embedding_lookup_blocks(int qtype, const void* blocks_dev, int vocab, int dim,
                                 int token, float* y_dev, void* stream);

/* ArgMax (src/ops.cc:182-195) on the device: first maximum wins.  The index
 * is written to *index_dev. */
int dqmk_argmax(const float* x_dev, int n, int* index_dev, void* stream);

/* ------------------------------------------------------------------ */
/* KV cache and decode attention                                        */
/* ------------------------------------------------------------------ */
/* Cache layout is the reference's: f32 [n_layers][max_seq][n_kv_heads]
 * [head_dim] for keys and for values (src/cuda_kv_cache.cc:63-96). */

/* CudaKvCache::WriteDevice (include/dqm_llama/cuda_kv_cache.h:41-42,
 * src/cuda_kv_cache.cc:134-164). */
int dqmk_kv_write(float* keys_dev, float* values_dev, int n_layers, int max_seq, int n_kv_heads,
                  int head_dim, int layer, int pos, const float* k_dev, const float* v_dev,
                  void* stream);

/* CudaAttentionDecodeDeviceInput (include/dqm_llama/cuda_attention.h:19-23,
 * src/cuda_attention.cu:272-311; CPU math src/forward.cc:435-507): GQA
 * decode attention of q [n_heads, head_dim] over cache positions 0..pos of
 * `layer`, out [n_heads, head_dim].  Split over positions with an in-kernel
 * combine; the split partials live in a per-device scratch buffer the
 * library allocates once and reuses. */
int dqmk_attention_decode(const float* q_dev, const float* keys_dev, const float* values_dev,
                          int n_layers, int max_seq, int n_kv_heads, int head_dim, int layer,
                          int pos, int n_heads, float* out_dev, void* stream);

/* Allocation-free form of dqmk_attention_decode.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they run attention (an engine that reserves its whole device budget at
 * start-up and treats later cudaMalloc calls as failures, or a host that
 * forbids allocations outside its own allocator).  Same arguments, results
 * and errors as dqmk_attention_decode; it calls no cudaMalloc, cudaFree or
 * other allocating routine.  The split partials and tickets live in one
 * fixed 2 MiB device buffer compiled into the library (every GPU that loads
 * it holds the 2 MiB until the process exits): n_heads * splits *
 * (head_dim + 4) * 4 bytes + 256 must fit, where splits = min(ceil(max_seq /
 * 128), SM count / n_kv_heads) -- on a 148-SM B200 every supported shape
 * (at most 8 query heads per KV head, head_dim <= 256) needs at most
 * 1.23 MB; on a GPU where a shape does not fit it is rejected with
 * DQMK_ERR_UNSUPPORTED and a message giving both sizes.  All calls share the
 * buffer: each call zeroes the tickets first, and calls that overlap on the
 * GPU (for example on two streams) race.  The first call on a device looks
 * up the buffer's device address (cudaGetSymbolAddress, no allocation) with
 * that device current; make that first call before any stream capture. */
int dqmk_attention_decode_noalloc(const float* q_dev, const float* keys_dev,
                                  const float* values_dev, int n_layers, int max_seq,
                                  int n_kv_heads, int head_dim, int layer, int pos, int n_heads,
                                  float* out_dev, void* stream);

/* ------------------------------------------------------------------ */
/* Engine: device-resident model + context (ForwardToken / ForwardBatch)*/
/* ------------------------------------------------------------------ */

typedef struct dqmk_model dqmk_model;
typedef struct dqmk_context dqmk_context;

/* ModelConfig (include/dqm_llama/model.h:23-35). */
typedef struct dqmk_model_config {
  int vocab_size;
  int dim;
  int hidden_dim;
  int n_layers;
  int n_heads;
  int n_kv_heads;
  int head_dim;
  int max_seq_len;
  float rope_theta;
  float rms_norm_eps;
  int rope_neox; /* 1 = RopeType::kNeoX (qwen2), 0 = kNormal */
} dqmk_model_config;

/* CudaModelWeights runtime counters (include/dqm_llama/model.h:64-79),
 * counted per logical op as the reference's RecordCuda* helpers do
 * (src/forward.cc:97-165). */
typedef struct dqmk_model_stats {
  uint64_t uploaded_weight_count;
  uint64_t uploaded_bytes;
  uint64_t linear_calls;
  uint64_t activation_calls;
  uint64_t attention_calls;
  uint64_t kv_cache_write_bytes;
  uint64_t kv_cache_read_bytes;
  uint64_t host_to_device_copies;
  uint64_t device_to_host_copies;
  uint64_t host_to_device_bytes;
  uint64_t device_to_host_bytes;
} dqmk_model_stats;

int dqmk_model_create(const dqmk_model_config* config, int device_id, dqmk_model** out);
int dqmk_model_destroy(dqmk_model* model);

/* UploadModelWeightsToCuda (include/dqm_llama/model.h:103, src/model.cc:227-260)
 * one tensor at a time, under the reference's names: "token_embedding",
 * "final_norm", "lm_head", "layers.<i>.{attention_norm,wq,wk,wv,bq,bk,bv,wo,
 * ffn_norm,w_gate,w_up,w_down}".  qtype is DQMK_F32 for norms / biases and
 * DQMK_Q80 / DQMK_Q40 for linears and the token embedding.  `data` may be a
 * host or a device pointer; `bytes` is its size.  Without "lm_head" the
 * token embedding blocks are reused as a tied lm_head. */
int dqmk_model_upload(dqmk_model* model, const char* name, int qtype, const void* data,
                      size_t bytes, int rows, int cols);

/* Validates that every tensor is present and builds the fused layouts. */
int dqmk_model_finalize(dqmk_model* model);

/* GGUF v3 model files (LoadGgufModel, src/gguf_loader.cc:279-364, with the
 * configuration rules of BuildConfig, :202-273).  dqmk_gguf_read_config
 * parses the metadata only (no device work).  dqmk_model_load_gguf creates,
 * uploads and finalizes a model on device_id: quantized tensors (Q8_0,
 * Q4_0) are uploaded as stored -- the token embedding stays quantized and a
 * file without output.weight gets the tied lm_head over those blocks, where
 * the reference expands both to F32 (:313-326, 356-360) -- and F32 norms and
 * biases as F32.  max_seq_len > 0 overrides the file's context length.
 * Other ggml types fail with DQMK_ERR_UNSUPPORTED. */
int dqmk_gguf_read_config(const char* path, dqmk_model_config* out);
int dqmk_model_load_gguf(const char* path, int max_seq_len, int device_id, dqmk_model** out);

/* Tensor parallelism (Megatron split; no reference counterpart -- the
 * reference runs one device).  A rank's share of the model: */
typedef struct dqmk_tp_plan {
  int rank, world;
  int q_head0, n_q_heads;   /* query heads: columns of wq, rows of wo's K */
  int kv_head0, n_kv_heads; /* key/value heads: wk, wv rows; the KV cache shard */
  int hidden0, hidden;      /* FFN: w_gate / w_up rows, w_down's K columns */
  int vocab0, vocab;        /* lm_head rows (vocabulary-parallel) */
  int vocab_stride;         /* ceil(vocab_size / world): rows per rank slot */
} dqmk_tp_plan;
/* Host-only: the plan of `rank` in a `world`-way group (DQMK_ERR_UNSUPPORTED
 * when heads, key/value heads, or the FFN / query widths at 32-value blocks
 * do not split evenly). */
int dqmk_tp_plan_get(const dqmk_model_config* config, int rank, int world, dqmk_tp_plan* out);
/* NCCL unique id (128 bytes) for dqmk_model_set_tp; created on one rank and
 * passed to the others out of band (e.g. a torch.distributed broadcast). */
int dqmk_nccl_unique_id(unsigned char* id_out);
/* Before dqmk_model_finalize, with the full weights uploaded: the model keeps
 * only rank `rank`'s shard, and its decode step all-reduces the row-parallel
 * projections over NCCL.  Collective: every rank of the group calls it with
 * the same id, each on its own device. */
int dqmk_model_set_tp(dqmk_model* model, int rank, int world, const unsigned char* nccl_id);

/* Peer-memory exchange for a tensor-parallel context (optional; without it
 * the decode step all-reduces over NCCL).  Each rank's context owns one
 * exchange buffer; dqmk_context_tp_ipc_handle exports it (64-byte CUDA IPC
 * handle), the host gathers the handles of all ranks in rank order, and
 * dqmk_context_tp_connect maps the peers' buffers.  From then on the O and
 * down GEMVs store their partial rows straight into every rank's buffer over
 * NVLink and raise a flag there, a one-CTA kernel waits (bounded, ~2 s; a
 * timeout sets the device error flag) for all ranks' flags and sums the
 * partials in rank order, and the greedy argmax is exchanged the same way.
 * Every rank connects its context before the next step. */
int dqmk_context_tp_ipc_handle(dqmk_context* ctx, unsigned char* handle_out);
int dqmk_context_tp_connect(dqmk_context* ctx, const unsigned char* handles);

/* Test hook for the decode step: the context's lm_head runs as the
 * TMA-staged GEMV with row tile `tile` withheld (tile >= 0), every tile
 * withheld (tile == -2) or nothing withheld (tile == -1, the default); the
 * step is captured again.  A step whose lm_head rows were all withheld finds
 * no scored token: the greedy state (token, position, history) is kept and the
 * call returns DQMK_ERR_TIMEOUT, so no invalid token id reaches the next
 * embedding.  No reference counterpart. */
int dqmk_context_withhold_lm_head(dqmk_context* ctx, int tile);
int dqmk_model_stats_get(const dqmk_model* model, dqmk_model_stats* out);
int dqmk_model_stats_reset(dqmk_model* model);
/* ModelCudaMemoryBytes (include/dqm_llama/model.h:119). */
size_t dqmk_model_memory_bytes(const dqmk_model* model);

/* MiniLlamaContext (include/dqm_llama/context.h:14-31): KV cache, position,
 * token history, its own CUDA stream and captured decode graph. */
int dqmk_context_create(dqmk_model* model, dqmk_context** out);
int dqmk_context_destroy(dqmk_context* ctx);
/* Clears the KV cache, pos = 0, empty history. */
int dqmk_context_reset(dqmk_context* ctx);
int dqmk_context_pos(const dqmk_context* ctx);
/* Copies up to `cap` history tokens into `out`; returns the history length. */
int dqmk_context_history(const dqmk_context* ctx, int* out, int cap);

/* ForwardToken (include/dqm_llama/forward.h:11-12, src/forward.cc:729-754):
 * one token at position pos through the model; the vocab_size logits are
 * copied to the host buffer logits (may be NULL to skip the copy).  Does
 * not touch pos or history, like the reference.  Synchronous. */
int dqmk_forward_token(dqmk_context* ctx, int token, int pos, float* logits);

/* ForwardBatch (include/dqm_llama/forward.h:16-17, src/batch.cc:26-42):
 * runs tokens[i] at positions[i] in order, sets ctx pos to the last position,
 * appends every token to the history, writes the last token's logits.
 * Synchronous. */
int dqmk_forward_batch(dqmk_context* ctx, const int* tokens, const int* positions, int n,
                       float* logits);

/* ForwardBatch with prefix reuse, the reference chat loop's step before its
 * prefill (src/main.cc:887-913): the longest common prefix p of the
 * context's token history and `tokens` is kept (history cut to p tokens, pos
 * rolled back to p - 1) and only tokens[p..n) run, from position p, as a
 * batched prefill.  p == 0, or p == n (no token left to give logits), runs
 * the whole prompt from position 0.  *reused (if non-NULL) receives p.  The
 * reference intersects this with its RadixTree registry of cached prompts;
 * here the context's own history is the registry.  Synchronous. */
int dqmk_forward_batch_prefix(dqmk_context* ctx, const int* tokens, int n, float* logits,
                              int* reused);

/* Greedy decode on the device: feeds `token` at `pos`, then n_steps-1 more
 * tokens chosen by the device argmax, replaying the captured decode graph
 * with no host round trip per step.  tokens_out[i] receives the argmax after
 * step i.  Synchronous. */
int dqmk_decode_greedy(dqmk_context* ctx, int token, int pos, int n_steps, int* tokens_out);

/* Timing hook: enqueue n_steps greedy decode steps (same as above) without
 * synchronizing; returns the context stream for event timing. */
int dqmk_decode_enqueue(dqmk_context* ctx, int token, int pos, int n_steps);
void* dqmk_context_stream(dqmk_context* ctx);

/* ---------------------------------------------------- multi-sequence decode
 * The reference serves one sequence per MiniLlamaContext and one token per
 * ForwardToken (src/forward.cc:667-754); serving many sequences means many
 * contexts, each re-reading every weight per token.  A dqmk_batch holds
 * n_slots independent sequences (each its own KV cache of max_seq
 * positions, fp32 [layer][pos][kv_head][head_dim] like CudaKvCache) over one
 * model and runs a step over up to 64 columns at once: column c feeds
 * tokens[c] at positions[c] of slot slots[c].  Each column computes exactly
 * what ForwardToken computes for that sequence (within fp32 summation-order
 * differences); the weights are streamed once per step.  Works on tensor-
 * parallel models (dqmk_model_set_tp): every rank calls the same functions
 * with the same arguments.  Head sizes 64 and 128, Q8_0 / Q4_0 weights. */
typedef struct dqmk_batch dqmk_batch;
int dqmk_batch_create(dqmk_model* model, int n_slots, int max_seq, dqmk_batch** out);
int dqmk_batch_destroy(dqmk_batch* batch);
/* Zeroes every slot's KV cache. */
int dqmk_batch_reset(dqmk_batch* batch);
/* One step over n columns (1..64; slots NULL means slot c for column c; a
 * (slot, position) pair at most once; a slot may take several positions in
 * one step, e.g. a prompt chunk, since every column's K/V is stored before
 * attention runs).  logits: NULL or [n][vocab_size] on the host; next: NULL
 * or the n greedy tokens.  Synchronous. */
int dqmk_batch_step(dqmk_batch* batch, const int* slots, const int* tokens, const int* positions,
                    int n, float* logits, int* next);
/* Greedy decoding of slots 0..n-1 together: slot c starts from tokens[c] at
 * positions[c]; n_steps steps, each one replay of the captured step graph
 * with the argmax, token and position advanced on the device.  out:
 * [n_steps][n], out[i][c] = the token chosen after position positions[c] + i.
 * Synchronous. */
int dqmk_batch_decode_greedy(dqmk_batch* batch, const int* tokens, const int* positions, int n,
                             int n_steps, int* out);
/* Timing hook: the same steps enqueued without synchronizing, and the batch
 * stream to time them on. */
int dqmk_batch_decode_enqueue(dqmk_batch* batch, const int* tokens, const int* positions, int n,
                              int n_steps);
void* dqmk_batch_stream(dqmk_batch* batch);
/* out[i] = the greedy token chosen after position pos0 + i of `slot`.
 * Synchronous. */
int dqmk_batch_history(dqmk_batch* batch, int slot, int pos0, int count, int* out);

#ifdef __cplusplus
}
#endif

#endif /* DQMK_H_ */
