// internal.h -- launchers shared by the kernel files and the C++ engine.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <string>

// Returns the dqmk status of a failed CUDA call from the enclosing function.
#define DQMK_CUDA_RET(api, expr)                                \
  do {                                                          \
    cudaError_t _e = (expr);                                    \
    if (_e != cudaSuccess) return ::dqmk::cuda_fail(api, _e);   \
  } while (0)

namespace dqmk {

// --------------------------------------------------------------- status
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_fail(const char* api, cudaError_t err);
const char* last_error_cstr();
// SM count of the current device (cached per device).
int sm_count();
// Programmatic dependent launch between chained kernels (off with DQMK_PDL=0).
bool use_pdl();

// Kernel attributes (cudaFuncSetAttribute) and occupancy figures belong to
// the device that is current when they are set or queried, so every one-time
// set-up runs once per device: fn() with that device current.
constexpr int kMaxDevices = 64;
class DeviceOnce {
 public:
  template <typename F>
  cudaError_t run(F fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    e = fn();
    if (e == cudaSuccess) done_[dev].store(true, std::memory_order_release);
    return e;
  }

 private:
  std::mutex mu_;
  std::atomic<bool> done_[kMaxDevices] = {};
};

// Device error flags, per kernel family; every flag word uses the same bits.
constexpr unsigned int kErrTimeout = 1u;   // a bounded wait ran out
constexpr unsigned int kErrNoToken = 2u;   // greedy step without a valid argmax (state kept)
constexpr unsigned int kErrBadToken = 4u;  // embedding of a token id outside [0, vocab)
// DQMK_OK when no flag is set, else DQMK_ERR_TIMEOUT with a message prefixed
// by `api` that names what the flags record.
int device_flags_status(const char* api, unsigned int flags);
// Library-owned per-device scratch (grown on demand, zero-filled when
// (re)allocated).  Callers that use it from several streams at once race.
cudaError_t device_scratch(size_t bytes, void** out);

// --------------------------------------------------------------- quant
size_t packed_bytes(int qtype, int out_features, int in_features);
cudaError_t launch_pack(int qtype, const void* blocks, int out_features, int in_features,
                        void* packed, cudaStream_t stream);
cudaError_t launch_quantize(int qtype, const float* src, int64_t n_rows, int64_t row_size,
                            void* blocks, cudaStream_t stream);
cudaError_t launch_dequantize(int qtype, const void* blocks, int64_t n_rows, int64_t row_size,
                              float* dst, cudaStream_t stream);

// --------------------------------------------------------------- GEMV
// Epilogues of the packed GEMV.
enum GemvEpilogue : int {
  kEpiStore = 0,   // y[o] = residual[o] + (acc + bias[o])
  kEpiSwiGlu = 1,  // rows interleaved (gate_o, up_o): y[o] = silu(gate) * up
  kEpiQkv = 2,     // rows paired for RoPE: bias, rotate, write q / K / V cache
  kEpiLogits = 3,  // y[o] = acc; device argmax + greedy advance
  kEpiPeer = 4,    // tensor parallel: row o of the partial sum goes to every rank's slot
};

// Tensor-parallel exchange over peer memory.  Every rank owns one
// communication buffer (mapped into the other ranks' address spaces):
//   vector slots [2 parities][world][dim] fp32, key slots [2][world] u64,
//   flags [2 channels][world] u32 (channel 0: vectors, 1: argmax keys).
// Exchange number s (1, 2, ...) of a channel uses parity s & 1; its writers
// store into slot [s & 1][own rank] of every rank, then raise flag
// [channel][own rank] to s everywhere; a reader waits for all flags >= s.
struct PeerSet {
  char* const* base;   // device array [world]: each rank's buffer (own included)
  int rank, world, dim;
  unsigned int* seq;   // this rank's completed exchanges per channel [2]
  unsigned int* ticket;  // CTA completion counter of the writing kernel
};
__host__ __device__ __forceinline__ size_t tp_round256(size_t b) { return (b + 255) / 256 * 256; }
__host__ __device__ __forceinline__ size_t tp_vec_off(int parity, int rank, int world, int dim) {
  return ((size_t)(parity * world + rank) * dim) * sizeof(float);
}
__host__ __device__ __forceinline__ size_t tp_keys_off(int world, int dim) {
  return tp_round256((size_t)2 * world * dim * sizeof(float));
}
__host__ __device__ __forceinline__ size_t tp_flags_off(int world, int dim) {
  return tp_keys_off(world, dim) + tp_round256((size_t)2 * world * 8);
}
__host__ __device__ __forceinline__ size_t tp_buf_bytes(int world, int dim) {
  return tp_flags_off(world, dim) + tp_round256((size_t)2 * world * 4);
}

struct GemvArgs {
  int qtype;
  const uint8_t* qs;    // quant plane
  const uint16_t* d;    // scale plane
  int n_rows;           // packed rows
  int k;                // in_features
  int kp;               // in_features rounded up to 32
  const float* x;       // input [k]
  const float* norm_w;  // fused RMSNorm weight (nullptr: none)
  float eps;
  int epi;
  const float* bias;      // by packed row
  const float* residual;  // kEpiStore
  float* y;
  // kEpiQkv
  const float2* rope_cs;  // [max_seq][head_dim/2] (cos, sin)
  const int* pos_dev;     // device position (engine); nullptr -> pos_arg
  int pos_arg;
  float* q_out;
  float* k_cache;
  float* v_cache;
  int layer, max_seq, n_heads, n_kv_heads, head_dim, neox;
  // kEpiLogits
  unsigned long long* argmax_slot;  // packed (value, index) max
  int row_offset;                   // index of packed row 0 in the full vocabulary
  unsigned int* ticket;             // CTA completion counter (reset by the last CTA);
                                    // nullptr: no greedy advance in the kernel
  int* token_slot;                  // greedy: next token
  int* pos_slot;                    // greedy: next position (incremented)
  int* history;                     // greedy: token written at history[pos+1]
  int history_cap;
  // kEpiPeer: where the partial rows go
  PeerSet peer;
};

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);
// Register-GEMV variant the dispatcher picks for a shape (-1: the TMA form).
int gemv_variant_id(const GemvArgs& a);
// Sets kernel attributes of every GEMV / attention instantiation; call
// outside stream capture.
cudaError_t gemv_prepare();
// Failure-detection hook: the TMA GEMV with the copies of one tile withheld
// (skip_tile >= 0) or of every tile (kSkipAllTiles), so those bounded waits
// run out and set the device error flag.
constexpr int kSkipAllTiles = -2;
cudaError_t launch_gemv_tma_skip(const GemvArgs& a, cudaStream_t stream, int skip_tile);
// Device error flags set by bounded waits (bit 0: timeout); optionally cleared.
cudaError_t read_device_error(unsigned int* flags, bool clear);
// Device addresses (current device) of the three error flag words -- this
// file's, the peer exchange's and the standalone ops' -- for asynchronous
// reads of all three with a step's results.
cudaError_t device_error_address(unsigned int** p);
cudaError_t tp_error_address(unsigned int** p);
cudaError_t ops_error_address(unsigned int** p);
cudaError_t attention_prepare();

// ggml-layout Linear (compatibility entry point), rows >= 1.
cudaError_t launch_linear_blocks(int qtype, const float* x, int rows, int in_features,
                                 const void* blocks, int out_features, const float* bias,
                                 float* y, cudaStream_t stream);

// --------------------------------------------------------------- ops
cudaError_t launch_rmsnorm(const float* x, const float* w, int dim, float eps, float* y,
                           cudaStream_t stream);
cudaError_t launch_silu_mul(const float* g, const float* u, int n, float* y, cudaStream_t s);
cudaError_t launch_add(const float* a, const float* b, int n, float* y, cudaStream_t s);
cudaError_t launch_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim,
                        const float2* cs, int neox, cudaStream_t s);
cudaError_t launch_embed_f32(const float* table, int dim, int token, float* y, cudaStream_t s);

// Embedding gather from packed Q8_0/Q4_0 rows.  Token from *token_dev when
// non-null (graph replay), else `token`.  Also resets *argmax_slot.
struct EmbedArgs {
  int qtype;
  const uint8_t* qs;
  const uint16_t* d;
  int vocab, dim, kp;
  const int* token_dev;
  int token;
  float* y;
  unsigned long long* argmax_slot;
};
cudaError_t launch_embed_packed(const EmbedArgs& a, cudaStream_t s);
cudaError_t launch_embed_blocks(int qtype, const void* blocks, int dim, int token, float* y,
                                cudaStream_t s);
cudaError_t launch_argmax(const float* x, int n, unsigned long long* slot, int* index,
                          cudaStream_t s);
// Flags of the embedding and greedy-advance kernels (ops.cu).
cudaError_t read_ops_error(unsigned int* flags, bool clear);
// Peer-memory tensor parallelism (tp_p2p.cu): wait for every rank's partial
// of exchange seq[0] + 1, x += their sum (fixed rank order); and the greedy
// step after a vocabulary-parallel lm_head (max over the ranks' keys).
cudaError_t launch_tp_reduce(float* x, const PeerSet& ps, cudaStream_t s, bool pdl);
cudaError_t launch_tp_argmax_advance(const PeerSet& ps, const unsigned long long* local_key,
                                     int* token, int* pos, int* history, int cap, int vocab,
                                     cudaStream_t s, bool pdl);
cudaError_t read_tp_error(unsigned int* flags, bool clear);
// Multi-sequence decode GEMM (batch.cu): bounded-wait flag.
cudaError_t read_batch_error(unsigned int* flags, bool clear);
cudaError_t launch_greedy_advance(const unsigned long long* slot, int* token, int* pos,
                                  int* history, int cap, int vocab, cudaStream_t s);
cudaError_t launch_kv_write(float* keys, float* values, int max_seq, int n_kv_heads,
                            int head_dim, int layer, int pos, const float* k, const float* v,
                            cudaStream_t s);

// --------------------------------------------------------------- attention
struct AttnArgs {
  const float* q;        // [n_heads][hd]
  const float* keys;     // cache base
  const float* values;
  int max_seq, n_kv_heads, head_dim, layer, n_heads;
  const int* pos_dev;    // device position; nullptr -> pos_arg
  int pos_arg;
  float* out;            // [n_heads][hd]
  float* partials;       // [n_heads][max_splits][hd + 4]: sums, m, l, pad
  unsigned int* tickets; // [n_kv_heads], zero at rest
  int max_splits;        // gridDim.y
  int min_chunk;         // shortest split in positions (0: 128)
};
// Shortest split of the batch-1 decode attention for a head size: 64
// positions at head_dim 128 (Qwen2-7B batch-1 step 2.62 -> 2.56 ms against
// 128), 128 below it (Qwen2-0.5B at 2048 positions: 0.714 vs 0.743 ms at 64).
int decode_min_chunk(int head_dim);
// Splits (CTAs per KV head along the sequence) used for a cache of max_seq.
int attention_splits(int max_seq, int n_kv_heads, int min_chunk = 128);
size_t attention_partials_floats(int n_heads, int head_dim, int max_splits);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t stream, bool pdl);
int attention_chunk_cap(int max_seq, int max_splits);

// host-side RoPE table in the reference's float arithmetic (src/ops.cc:18-23,
// :40-45): entry [p][i] = (cos, sin) of p * 1/theta^(2i/head_dim).
void rope_table(float theta, int head_dim, int pos_begin, int pos_count, float2* out);

}  // namespace dqmk
