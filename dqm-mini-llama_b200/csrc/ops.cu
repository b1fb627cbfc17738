// ops.cu -- memory-bound ops of the decode path, standalone forms.
//
// Inside the engine these are fused into the GEMV prologues/epilogues
// (gemv.cu); the standalone kernels here back the reference's per-op device
// entry points (include/dqm_llama/cuda_ops.h) and the tests.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace dqmk {

// --------------------------------------------------------------- errors
namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

const char* last_error_cstr() { return g_last_error.c_str(); }

int cuda_fail(const char* api, cudaError_t err) {
  g_last_error = std::string(api) + ": CUDA error: " + cudaGetErrorString(err);
  return err == cudaErrorMemoryAllocation ? DQMK_ERR_NOMEM : DQMK_ERR_CUDA;
}

int device_flags_status(const char* api, unsigned int flags) {
  if (!flags) return DQMK_OK;
  std::string msg = std::string(api) + ": a device-side wait timed out";
  if (flags & kErrNoToken) msg += "; a greedy step found no scored token and kept its state";
  if (flags & kErrBadToken) msg += "; an embedding was asked for a token id outside the vocabulary";
  return fail(DQMK_ERR_TIMEOUT, msg);
}

int sm_count() {
  static std::atomic<int> cached[kMaxDevices];  // zero-initialized: not yet queried
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n = v > 0 ? v : 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

namespace {

__device__ unsigned int g_ops_error;  // kErrNoToken / kErrBadToken

constexpr int kMaxRopeHalf = 128;

struct RopeTableArg {
  float2 cs[kMaxRopeHalf];
};

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, int dim,
                               float eps, float* __restrict__ y) {
  __shared__ float red[32];
  __shared__ float scale_s;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    scale_s = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)dim), eps)));
  }
  __syncthreads();
  const float sc = scale_s;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], sc), w[i]);
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, int n,
                                float* __restrict__ y) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = g[i];
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
    y[i] = __fmul_rn(__fmul_rn(v, sig), u[i]);
  }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, int n,
                           float* __restrict__ y) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[i] = __fadd_rn(a[i], b[i]);
}

__global__ void rope_kernel(float* q, float* k, int n_heads, int n_kv_heads, int head_dim,
                            int neox, const RopeTableArg tab) {
  const int half = head_dim / 2;
  const int total = (n_heads + n_kv_heads) * half;
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < total; p += gridDim.x * blockDim.x) {
    const int h = p / half, i = p % half;
    float* base = h < n_heads ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
    const int o0 = neox ? i : 2 * i;
    const int o1 = neox ? i + half : 2 * i + 1;
    const float a = base[o0], b = base[o1];
    const float c = tab.cs[i].x, s = tab.cs[i].y;
    if (neox) {
      base[o0] = __fmaf_rn(a, c, -__fmul_rn(b, s));
      base[o1] = __fmaf_rn(a, s, __fmul_rn(b, c));
    } else {
      base[o0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
      base[o1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
  }
}

__global__ void embed_f32_kernel(const float* __restrict__ table, int dim, int token,
                                 float* __restrict__ y) {
  for (int i = threadIdx.x; i < dim; i += blockDim.x) y[i] = table[(size_t)token * dim + i];
}

// Packed (planar) table row gather; also clears the greedy argmax slot for
// the step this kernel opens.  A token id outside [0, vocab) (possible only
// on the device, where the host cannot validate it) gathers nothing: the row
// is zeroed and kErrBadToken recorded.
__global__ void embed_packed_kernel(const EmbedArgs a) {
  const int token = a.token_dev ? *a.token_dev : a.token;
  if (token < 0 || token >= a.vocab) {
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) a.y[i] = 0.0f;
    if (threadIdx.x == 0) {
      atomicOr(&g_ops_error, kErrBadToken);
      if (a.argmax_slot) *a.argmax_slot = 0ull;
    }
    pdl_trigger();
    return;
  }
  const int nbk = a.kp / 32;
  const size_t row_bytes = a.qtype == DQMK_Q80 ? (size_t)a.kp : (size_t)a.kp / 2;
  const uint8_t* q = a.qs + (size_t)token * row_bytes;
  const uint16_t* d = a.d + (size_t)token * nbk;
  for (int i = threadIdx.x; i < a.dim; i += blockDim.x) {
    const float s = h2f(d[i / 32]);
    float v;
    if (a.qtype == DQMK_Q80) {
      v = (float)(int8_t)q[i];
    } else {
      const int j = i % 32;
      const uint8_t byte = q[(i / 32) * 16 + (j & 15)];
      v = (float)((j < 16 ? (byte & 0x0f) : (byte >> 4)) - 8);
    }
    a.y[i] = __fmul_rn(s, v);
  }
  if (threadIdx.x == 0 && a.argmax_slot) *a.argmax_slot = 0ull;
  pdl_trigger();
}

__global__ void embed_blocks_kernel(int qtype, const uint8_t* __restrict__ blocks, int dim,
                                    int token, float* __restrict__ y) {
  const int nb = (dim + 31) / 32;
  const int bytes = qtype == DQMK_Q80 ? 34 : 18;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const uint8_t* p = blocks + ((size_t)token * nb + i / 32) * bytes;
    const float s = h2f((uint16_t)(p[0] | (p[1] << 8)));
    const int j = i % 32;
    float v;
    if (qtype == DQMK_Q80) {
      v = (float)(int8_t)p[2 + j];
    } else {
      v = (float)((j < 16 ? (p[2 + j] & 0x0f) : (p[2 + j - 16] >> 4)) - 8);
    }
    y[i] = __fmul_rn(s, v);
  }
}

__global__ void argmax_kernel(const float* __restrict__ x, int n, unsigned long long* slot) {
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = argmax_key(x[i], (uint32_t)i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(slot, best);
}

__global__ void argmax_finish_kernel(unsigned long long* slot, int n, int* index) {
  int idx = 0;
  if (!argmax_token(*slot, n, &idx)) atomicOr(&g_ops_error, kErrNoToken);
  *index = idx;
  *slot = 0ull;
}

__global__ void kv_write_kernel(float* keys, float* values, int max_seq, int n_kv_heads,
                                int head_dim, int layer, int pos, const float* k,
                                const float* v) {
  const int n = n_kv_heads * head_dim;
  const size_t base = ((size_t)layer * max_seq + pos) * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    keys[base + i] = k[i];
    values[base + i] = v[i];
  }
}

// y = x * sigmoid(x) (SiluKernel, src/cuda_ops.cu:52-58) and y = a * b
// (ElementwiseMulKernel, :60-66): the standalone forms of the SwiGLU pieces.
__global__ void silu_kernel(const float* __restrict__ x, int n, float* __restrict__ y) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
  }
}

__global__ void mul_kernel(const float* __restrict__ a, const float* __restrict__ b, int n,
                           float* __restrict__ y) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[i] = __fmul_rn(a[i], b[i]);
}

// One-dimensional softmax (src/ops.cc:92-118; the reference's three-kernel
// CUDA form, src/cuda_ops.cu:84-136): one CTA, max, sum of exp(x - max),
// divide.
__global__ void softmax_kernel(const float* __restrict__ x, int n, float* __restrict__ y) {
  __shared__ float red[32];
  __shared__ float bc;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
    bc = t;
  }
  __syncthreads();
  m = bc;
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += expf(x[i] - m);
  s = warp_sum(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    bc = t;
  }
  __syncthreads();
  const float inv = bc;
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fdiv_rn(expf(x[i] - m), inv);
}

int grid1d(int n, int threads) {
  int g = (n + threads - 1) / threads;
  const int cap = sm_count() * 8;
  return g < 1 ? 1 : (g > cap ? cap : g);
}

}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* w, int dim, float eps, float* y,
                           cudaStream_t s) {
  rmsnorm_kernel<<<1, 1024, 0, s>>>(x, w, dim, eps, y);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float* g, const float* u, int n, float* y, cudaStream_t s) {
  silu_mul_kernel<<<grid1d(n, 256), 256, 0, s>>>(g, u, n, y);
  return cudaGetLastError();
}

cudaError_t launch_add(const float* a, const float* b, int n, float* y, cudaStream_t s) {
  add_kernel<<<grid1d(n, 256), 256, 0, s>>>(a, b, n, y);
  return cudaGetLastError();
}

cudaError_t launch_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim,
                        const float2* cs, int neox, cudaStream_t s) {
  RopeTableArg tab;
  for (int i = 0; i < head_dim / 2; ++i) tab.cs[i] = cs[i];
  const int total = (n_heads + n_kv_heads) * (head_dim / 2);
  rope_kernel<<<grid1d(total, 128), 128, 0, s>>>(q, k, n_heads, n_kv_heads, head_dim, neox, tab);
  return cudaGetLastError();
}

cudaError_t launch_embed_f32(const float* table, int dim, int token, float* y, cudaStream_t s) {
  embed_f32_kernel<<<1, 256, 0, s>>>(table, dim, token, y);
  return cudaGetLastError();
}

cudaError_t launch_embed_packed(const EmbedArgs& a, cudaStream_t s) {
  embed_packed_kernel<<<1, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_embed_blocks(int qtype, const void* blocks, int dim, int token, float* y,
                                cudaStream_t s) {
  embed_blocks_kernel<<<1, 256, 0, s>>>(qtype, static_cast<const uint8_t*>(blocks), dim, token,
                                        y);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* x, int n, unsigned long long* slot, int* index,
                          cudaStream_t s) {
  argmax_kernel<<<grid1d(n, 256), 256, 0, s>>>(x, n, slot);
  argmax_finish_kernel<<<1, 1, 0, s>>>(slot, n, index);
  return cudaGetLastError();
}

// Greedy decode state after a tensor-parallel lm_head: the all-reduced
// (value, index) key names the next token; record it, advance the position.
// Without a valid key (an lm_head wait ran out) the state is kept and
// kErrNoToken recorded.
__global__ void greedy_advance_kernel(const unsigned long long* slot, int* token, int* pos,
                                      int* history, int cap, int vocab) {
  int idx = 0;
  if (!argmax_token(*slot, vocab, &idx)) {
    atomicOr(&g_ops_error, kErrNoToken);
    return;
  }
  const int p = *pos;
  if (history && p >= 0 && p < cap) history[p] = idx;
  *token = idx;
  *pos = p + 1;
}

cudaError_t launch_greedy_advance(const unsigned long long* slot, int* token, int* pos,
                                  int* history, int cap, int vocab, cudaStream_t s) {
  greedy_advance_kernel<<<1, 1, 0, s>>>(slot, token, pos, history, cap, vocab);
  return cudaGetLastError();
}

cudaError_t ops_error_address(unsigned int** p) {
  return cudaGetSymbolAddress(reinterpret_cast<void**>(p), g_ops_error);
}

cudaError_t read_ops_error(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_ops_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *flags) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_ops_error, &zero, sizeof(unsigned int));
  }
  return e;
}

cudaError_t launch_kv_write(float* keys, float* values, int max_seq, int n_kv_heads,
                            int head_dim, int layer, int pos, const float* k, const float* v,
                            cudaStream_t s) {
  kv_write_kernel<<<grid1d(n_kv_heads * head_dim, 128), 128, 0, s>>>(
      keys, values, max_seq, n_kv_heads, head_dim, layer, pos, k, v);
  return cudaGetLastError();
}

// Per-device scratch owned by the library: attention split partials,
// completion tickets and the argmax slot of the standalone entry points.
// Grown (never shrunk) under a lock; the zero-at-rest counters live at the
// front and are cleared whenever the buffer is (re)allocated.
struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};

static std::mutex g_scratch_mu;
static std::vector<Scratch> g_scratch;

cudaError_t device_scratch(size_t bytes, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((int)g_scratch.size() <= dev) g_scratch.resize(dev + 1);
  Scratch& s = g_scratch[dev];
  if (s.bytes < bytes) {
    if (s.ptr) {
      e = cudaDeviceSynchronize();  // the old buffer may still be in use
      if (e != cudaSuccess) return e;
      cudaFree(s.ptr);
      s.ptr = nullptr;
      s.bytes = 0;
    }
    const size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    e = cudaMalloc(&s.ptr, want);
    if (e != cudaSuccess) return e;
    e = cudaMemset(s.ptr, 0, want);
    if (e != cudaSuccess) return e;
    s.bytes = want;
  }
  *out = s.ptr;
  return cudaSuccess;
}

}  // namespace dqmk

// ------------------------------------------------------------------ C ABI
using namespace dqmk;

extern "C" const char* dqmk_last_error(void) { return last_error_cstr(); }

extern "C" int dqmk_built(void) { return 1; }

extern "C" int dqmk_rmsnorm(const float* x, const float* w, int dim, float eps, float* y,
                            void* stream) {
  if (dim <= 0) return fail(DQMK_ERR_INVALID, "ops: RmsNorm: dim must be positive");
  if (!x || !w || !y) return fail(DQMK_ERR_INVALID, "ops: RmsNorm: null pointer");
  DQMK_CUDA_RET("CudaRmsNorm", launch_rmsnorm(x, w, dim, eps, y, (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_silu_mul(const float* g, const float* u, int n, float* y, void* stream) {
  if (n < 0) return fail(DQMK_ERR_INVALID, "SwiGlu: shape mismatch");
  if (n == 0) return DQMK_OK;
  if (!g || !u || !y) return fail(DQMK_ERR_INVALID, "SwiGlu: null pointer");
  DQMK_CUDA_RET("CudaSilu", launch_silu_mul(g, u, n, y, (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_silu(const float* x, int n, float* y, void* stream) {
  if (n < 0) return fail(DQMK_ERR_INVALID, "CudaSilu: shape mismatch");
  if (n == 0) return DQMK_OK;
  if (!x || !y) return fail(DQMK_ERR_INVALID, "CudaSilu: null pointer");
  silu_kernel<<<grid1d(n, 256), 256, 0, (cudaStream_t)stream>>>(x, n, y);
  DQMK_CUDA_RET("CudaSilu", cudaGetLastError());
  return DQMK_OK;
}

extern "C" int dqmk_mul(const float* a, const float* b, int n, float* y, void* stream) {
  if (n < 0) return fail(DQMK_ERR_INVALID, "CudaElementwiseMul: shape mismatch");
  if (n == 0) return DQMK_OK;
  if (!a || !b || !y) return fail(DQMK_ERR_INVALID, "CudaElementwiseMul: null pointer");
  mul_kernel<<<grid1d(n, 256), 256, 0, (cudaStream_t)stream>>>(a, b, n, y);
  DQMK_CUDA_RET("CudaElementwiseMul", cudaGetLastError());
  return DQMK_OK;
}

extern "C" int dqmk_softmax(const float* x, int n, float* y, void* stream) {
  if (n <= 0) return fail(DQMK_ERR_INVALID, "CudaSoftmax: empty input");
  if (!x || !y) return fail(DQMK_ERR_INVALID, "CudaSoftmax: null pointer");
  softmax_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, n, y);
  DQMK_CUDA_RET("CudaSoftmax", cudaGetLastError());
  return DQMK_OK;
}

extern "C" int dqmk_add(const float* a, const float* b, int n, float* y, void* stream) {
  if (n < 0) return fail(DQMK_ERR_INVALID, "CudaElementwiseAdd: shape mismatch");
  if (n == 0) return DQMK_OK;
  if (!a || !b || !y) return fail(DQMK_ERR_INVALID, "CudaElementwiseAdd: null pointer");
  DQMK_CUDA_RET("CudaElementwiseAdd", launch_add(a, b, n, y, (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos,
                         float theta, int neox, void* stream) {
  if (pos < 0) return fail(DQMK_ERR_RANGE, "Rope: position must be non-negative");
  if (!(theta > 0.0f) || theta != theta || theta > 3.4e38f)
    return fail(DQMK_ERR_INVALID, "Rope: theta must be finite and positive");
  if (head_dim <= 0 || head_dim % 2 != 0)
    return fail(DQMK_ERR_INVALID, "Rope: head_dim must be positive and even");
  if (head_dim / 2 > kMaxRopeHalf)
    return fail(DQMK_ERR_UNSUPPORTED, "Rope: head_dim larger than 256");
  if (n_heads < 0 || n_kv_heads < 0) return fail(DQMK_ERR_INVALID, "Rope: expected 2D tensors");
  if (!q || !k) return fail(DQMK_ERR_INVALID, "Rope: null pointer");
  std::vector<float2> cs(head_dim / 2);
  rope_table(theta, head_dim, pos, 1, cs.data());
  DQMK_CUDA_RET("CudaRope", launch_rope(q, k, n_heads, n_kv_heads, head_dim, cs.data(), neox,
                                        (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_embedding_lookup(const float* table, int vocab, int dim, int token,
                                     float* y, void* stream) {
  if (token < 0 || token >= vocab)
    return fail(DQMK_ERR_RANGE, "CudaEmbeddingLookup: token id out of range");
  if (dim <= 0 || !table || !y) return fail(DQMK_ERR_INVALID, "CudaEmbeddingLookup: invalid argument");
  DQMK_CUDA_RET("CudaEmbeddingLookup", launch_embed_f32(table, dim, token, y, (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_embedding_lookup_blocks(int qtype, const void* blocks, int vocab, int dim,
                                            int token, float* y, void* stream) {
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, "CudaEmbeddingLookup: unsupported quant type");
  if (token < 0 || token >= vocab)
    return fail(DQMK_ERR_RANGE, "CudaEmbeddingLookup: token id out of range");
  if (dim <= 0 || !blocks || !y) return fail(DQMK_ERR_INVALID, "CudaEmbeddingLookup: invalid argument");
  DQMK_CUDA_RET("CudaEmbeddingLookup",
                launch_embed_blocks(qtype, blocks, dim, token, y, (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_argmax(const float* x, int n, int* index, void* stream) {
  if (n <= 0) return fail(DQMK_ERR_INVALID, "ArgMax: empty tensor");
  if (!x || !index) return fail(DQMK_ERR_INVALID, "ArgMax: null pointer");
  void* scratch = nullptr;
  DQMK_CUDA_RET("ArgMax", device_scratch(4096, &scratch));
  auto* slot = static_cast<unsigned long long*>(scratch);
  DQMK_CUDA_RET("ArgMax", launch_argmax(x, n, slot, index, (cudaStream_t)stream));
  return DQMK_OK;
}

extern "C" int dqmk_kv_write(float* keys, float* values, int n_layers, int max_seq,
                             int n_kv_heads, int head_dim, int layer, int pos, const float* k,
                             const float* v, void* stream) {
  if (layer < 0 || layer >= n_layers)
    return fail(DQMK_ERR_RANGE, "CudaKvCache::WriteDevice: layer out of range");
  if (pos < 0 || pos >= max_seq)
    return fail(DQMK_ERR_RANGE, "CudaKvCache::WriteDevice: pos out of range");
  if (n_kv_heads <= 0 || head_dim <= 0 || !keys || !values || !k || !v)
    return fail(DQMK_ERR_INVALID, "CudaKvCache::WriteDevice: invalid argument");
  DQMK_CUDA_RET("CudaKvCache::WriteDevice",
                launch_kv_write(keys, values, max_seq, n_kv_heads, head_dim, layer, pos, k, v,
                                (cudaStream_t)stream));
  return DQMK_OK;
}
