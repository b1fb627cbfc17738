// dqmk_backend.cc -- dqm-mini-llama's CUDA backend functions over libdqmk.
//
// The engine's CUDA backend is a set of free functions declared in its
// include/dqm_llama/cuda_quant.h, cuda_ops.h, cuda_attention.h and
// cuda_matmul.h, implemented by src/cuda_quant.cu, src/cuda_ops.cu,
// src/cuda_attention.cu (SIMT kernels) and src/cuda_matmul.cc (cuBLAS).
// This file is the drop-in replacement a maintainer compiles in their place:
// every function keeps its signature, argument checks and exception types,
// and its body calls the C ABI of include/dqmk.h.  Everything else of the
// engine -- CudaTensor, CudaKvCache, the weight upload, ForwardToken's device
// branch -- is the engine's own code, unchanged.
//
// Conventions kept from the engine: outputs are freshly allocated CudaTensor
// / Tensor objects on device_id, work runs on the legacy default stream
// (the engine's CudaTensor copies are synchronous), status codes become
// std::out_of_range (DQMK_ERR_RANGE) or std::runtime_error with the message
// dqmk_last_error() gives, which starts with the engine API's name.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "dqm_llama/cuda_attention.h"
#include "dqm_llama/cuda_kv_cache.h"
#include "dqm_llama/cuda_matmul.h"
#include "dqm_llama/cuda_ops.h"
#include "dqm_llama/cuda_quant.h"
#include "dqm_llama/cuda_tensor.h"
#include "dqmk.h"

namespace dqm {
namespace {

void Check(int status) {
  if (status == DQMK_OK) return;
  const char* msg = dqmk_last_error();
  if (status == DQMK_ERR_RANGE) throw std::out_of_range(msg);
  throw std::runtime_error(msg);
}

void SetDevice(int device_id, const char* api) {
  const cudaError_t e = cudaSetDevice(device_id);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(api) + ": CUDA error: " + cudaGetErrorString(e));
}

size_t Numel(const std::vector<int>& shape) {
  size_t n = 1;
  for (int d : shape) n *= static_cast<size_t>(d);
  return n;
}

const float* F(const CudaTensor& t) { return static_cast<const float*>(t.data()); }
float* F(CudaTensor& t) { return static_cast<float*>(t.data()); }

// x [in] or [rows, in] against a weight [out, in]: rows and the output shape.
int RowsOf(const std::vector<int>& x_shape, const std::vector<int>& w_shape, const char* api,
           std::vector<int>* y_shape) {
  if (w_shape.size() != 2) throw std::runtime_error(std::string(api) + ": expected 2D weight shape");
  if (x_shape.empty() || x_shape.size() > 2)
    throw std::runtime_error(std::string(api) + ": expected 1D or 2D input");
  if (x_shape.back() != w_shape[1])
    throw std::runtime_error(std::string(api) + ": dimension mismatch");
  const int rows = x_shape.size() == 1 ? 1 : x_shape[0];
  *y_shape = x_shape.size() == 1 ? std::vector<int>{w_shape[0]}
                                 : std::vector<int>{rows, w_shape[0]};
  return rows;
}

using BlockLinear = int (*)(const float*, int, int, const void*, size_t, int, const float*,
                            float*, void*);

CudaTensor QuantDeviceInput(BlockLinear fn, const char* api, const CudaTensor& x,
                            const void* blocks, size_t block_count,
                            const std::vector<int>& w_shape, const float* bias_dev,
                            int device_id) {
  SetDevice(device_id, api);
  std::vector<int> y_shape;
  const int rows = RowsOf(x.shape(), w_shape, api, &y_shape);
  CudaTensor y(y_shape, device_id);
  Check(fn(F(x), rows, w_shape[1], blocks, block_count, w_shape[0], bias_dev, F(y), nullptr));
  return y;
}

Tensor QuantDeviceWeight(BlockLinear fn, const char* api, const Tensor& x, const void* blocks,
                         size_t block_count, const std::vector<int>& w_shape, const Tensor* bias,
                         int device_id) {
  CudaTensor xd = CudaTensorFromHost(x, device_id);
  CudaTensor bd;
  if (bias) {
    if (bias->data.size() != static_cast<size_t>(w_shape.at(0)))
      throw std::runtime_error(std::string(api) + ": bias shape mismatch");
    bd = CudaTensorFromHost(*bias, device_id);
  }
  return QuantDeviceInput(fn, api, xd, blocks, block_count, w_shape, bias ? F(bd) : nullptr,
                          device_id)
      .Download();
}

template <typename Block>
Tensor QuantHost(BlockLinear fn, const char* api, const Tensor& x,
                 const std::vector<Block>& weight, const std::vector<int>& w_shape,
                 const Tensor* bias, int device_id) {
  SetDevice(device_id, api);
  CudaDeviceBuffer w(weight.size() * sizeof(Block), device_id);
  if (!weight.empty()) {
    const cudaError_t e = cudaMemcpy(w.data(), weight.data(), weight.size() * sizeof(Block),
                                     cudaMemcpyHostToDevice);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string(api) + ": CUDA error: " + cudaGetErrorString(e));
  }
  return QuantDeviceWeight(fn, api, x, w.data(), weight.size(), w_shape, bias, device_id);
}

Tensor Run1(const Tensor& x, int device_id, const char* api,
            int (*fn)(const float*, int, float*, void*)) {
  SetDevice(device_id, api);
  CudaTensor xd = CudaTensorFromHost(x, device_id);
  CudaTensor y(x.shape, device_id);
  Check(fn(F(xd), static_cast<int>(x.data.size()), F(y), nullptr));
  return y.Download();
}

Tensor Run2(const Tensor& a, const Tensor& b, int device_id, const char* api,
            int (*fn)(const float*, const float*, int, float*, void*)) {
  if (a.data.size() != b.data.size())
    throw std::runtime_error(std::string(api) + ": shape mismatch");
  SetDevice(device_id, api);
  CudaTensor ad = CudaTensorFromHost(a, device_id), bd = CudaTensorFromHost(b, device_id);
  CudaTensor y(a.shape, device_id);
  Check(fn(F(ad), F(bd), static_cast<int>(a.data.size()), F(y), nullptr));
  return y.Download();
}

}  // namespace

// ---------------------------------------------------------------- cuda_quant.h
Tensor CudaQ80Linear(const Tensor& x, const std::vector<BlockQ80>& weight,
                     const std::vector<int>& weight_shape, const Tensor* bias, int device_id) {
  return QuantHost(dqmk_q80_linear, "CudaQ80Linear", x, weight, weight_shape, bias, device_id);
}
Tensor CudaQ80LinearDeviceWeight(const Tensor& x, const void* q8_0_device, size_t q8_0_block_count,
                                 const std::vector<int>& weight_shape, const Tensor* bias,
                                 int device_id) {
  return QuantDeviceWeight(dqmk_q80_linear, "CudaQ80Linear", x, q8_0_device, q8_0_block_count,
                           weight_shape, bias, device_id);
}
CudaTensor CudaQ80LinearDeviceInput(const CudaTensor& x, const void* q8_0_device,
                                    size_t q8_0_block_count, const std::vector<int>& weight_shape,
                                    int device_id) {
  return QuantDeviceInput(dqmk_q80_linear, "CudaQ80Linear", x, q8_0_device, q8_0_block_count,
                          weight_shape, nullptr, device_id);
}
Tensor CudaQ40Linear(const Tensor& x, const std::vector<BlockQ40>& weight,
                     const std::vector<int>& weight_shape, const Tensor* bias, int device_id) {
  return QuantHost(dqmk_q40_linear, "CudaQ40Linear", x, weight, weight_shape, bias, device_id);
}
Tensor CudaQ40LinearDeviceWeight(const Tensor& x, const void* q4_0_device, size_t q4_0_block_count,
                                 const std::vector<int>& weight_shape, const Tensor* bias,
                                 int device_id) {
  return QuantDeviceWeight(dqmk_q40_linear, "CudaQ40Linear", x, q4_0_device, q4_0_block_count,
                           weight_shape, bias, device_id);
}
CudaTensor CudaQ40LinearDeviceInput(const CudaTensor& x, const void* q4_0_device,
                                    size_t q4_0_block_count, const std::vector<int>& weight_shape,
                                    int device_id) {
  return QuantDeviceInput(dqmk_q40_linear, "CudaQ40Linear", x, q4_0_device, q4_0_block_count,
                          weight_shape, nullptr, device_id);
}
Tensor CudaQ41Linear(const Tensor& x, const std::vector<BlockQ41>& weight,
                     const std::vector<int>& weight_shape, const Tensor* bias, int device_id) {
  return QuantHost(dqmk_q41_linear, "CudaQ41Linear", x, weight, weight_shape, bias, device_id);
}
Tensor CudaQ41LinearDeviceWeight(const Tensor& x, const void* q4_1_device, size_t q4_1_block_count,
                                 const std::vector<int>& weight_shape, const Tensor* bias,
                                 int device_id) {
  return QuantDeviceWeight(dqmk_q41_linear, "CudaQ41Linear", x, q4_1_device, q4_1_block_count,
                           weight_shape, bias, device_id);
}
CudaTensor CudaQ41LinearDeviceInput(const CudaTensor& x, const void* q4_1_device,
                                    size_t q4_1_block_count, const std::vector<int>& weight_shape,
                                    int device_id) {
  return QuantDeviceInput(dqmk_q41_linear, "CudaQ41Linear", x, q4_1_device, q4_1_block_count,
                          weight_shape, nullptr, device_id);
}

// ---------------------------------------------------------------- cuda_ops.h
Tensor CudaRmsNorm(const Tensor& x, const Tensor& weight, float eps, int device_id) {
  if (x.data.size() != weight.data.size())
    throw std::runtime_error("CudaRmsNorm: weight shape mismatch");
  SetDevice(device_id, "CudaRmsNorm");
  CudaTensor xd = CudaTensorFromHost(x, device_id), wd = CudaTensorFromHost(weight, device_id);
  CudaTensor y(x.shape, device_id);
  Check(dqmk_rmsnorm(F(xd), F(wd), static_cast<int>(x.data.size()), eps, F(y), nullptr));
  return y.Download();
}
Tensor CudaSilu(const Tensor& x, int device_id) { return Run1(x, device_id, "CudaSilu", dqmk_silu); }
Tensor CudaElementwiseMul(const Tensor& a, const Tensor& b, int device_id) {
  return Run2(a, b, device_id, "CudaElementwiseMul", dqmk_mul);
}
Tensor CudaElementwiseAdd(const Tensor& a, const Tensor& b, int device_id) {
  return Run2(a, b, device_id, "CudaElementwiseAdd", dqmk_add);
}
Tensor CudaSoftmax(const Tensor& x, int device_id) {
  return Run1(x, device_id, "CudaSoftmax", dqmk_softmax);
}
CudaTensor CudaEmbeddingLookupDeviceWeight(const void* embedding_data,
                                           const std::vector<int>& embedding_shape, int token_id,
                                           int device_id) {
  if (embedding_shape.size() != 2)
    throw std::runtime_error("CudaEmbeddingLookup: expected 2D embedding shape");
  if (token_id < 0 || token_id >= embedding_shape[0])
    throw std::out_of_range("CudaEmbeddingLookup: token id out of range");
  SetDevice(device_id, "CudaEmbeddingLookup");
  CudaTensor y({embedding_shape[1]}, device_id);
  Check(dqmk_embedding_lookup(static_cast<const float*>(embedding_data), embedding_shape[0],
                              embedding_shape[1], token_id, F(y), nullptr));
  return y;
}
CudaTensor CudaRmsNormDeviceInput(const CudaTensor& x, const Tensor& weight, float eps,
                                  int device_id) {
  CudaTensor wd = CudaTensorFromHost(weight, device_id);
  return CudaRmsNormDeviceWeight(x, wd.data(), weight.shape, eps, device_id);
}
CudaTensor CudaRmsNormDeviceWeight(const CudaTensor& x, const void* weight_data,
                                   const std::vector<int>& weight_shape, float eps,
                                   int device_id) {
  if (Numel(weight_shape) != x.size())
    throw std::runtime_error("CudaRmsNorm: weight shape mismatch");
  SetDevice(device_id, "CudaRmsNorm");
  CudaTensor y(x.shape(), device_id);
  Check(dqmk_rmsnorm(F(x), static_cast<const float*>(weight_data), static_cast<int>(x.size()), eps,
                     F(y), nullptr));
  return y;
}
CudaTensor CudaSiluDeviceInput(const CudaTensor& x, int device_id) {
  SetDevice(device_id, "CudaSilu");
  CudaTensor y(x.shape(), device_id);
  Check(dqmk_silu(F(x), static_cast<int>(x.size()), F(y), nullptr));
  return y;
}
CudaTensor CudaElementwiseMulDeviceInput(const CudaTensor& a, const CudaTensor& b, int device_id) {
  if (a.size() != b.size()) throw std::runtime_error("CudaElementwiseMul: shape mismatch");
  SetDevice(device_id, "CudaElementwiseMul");
  CudaTensor y(a.shape(), device_id);
  Check(dqmk_mul(F(a), F(b), static_cast<int>(a.size()), F(y), nullptr));
  return y;
}
CudaTensor CudaElementwiseAddDeviceInput(const CudaTensor& a, const CudaTensor& b, int device_id) {
  if (a.size() != b.size()) throw std::runtime_error("CudaElementwiseAdd: shape mismatch");
  SetDevice(device_id, "CudaElementwiseAdd");
  CudaTensor y(a.shape(), device_id);
  Check(dqmk_add(F(a), F(b), static_cast<int>(a.size()), F(y), nullptr));
  return y;
}
CudaTensor CudaElementwiseAddDeviceWeight(const CudaTensor& a, const void* b_data,
                                          const std::vector<int>& b_shape, int device_id) {
  if (Numel(b_shape) != a.size()) throw std::runtime_error("CudaElementwiseAdd: shape mismatch");
  SetDevice(device_id, "CudaElementwiseAdd");
  CudaTensor y(a.shape(), device_id);
  Check(dqmk_add(F(a), static_cast<const float*>(b_data), static_cast<int>(a.size()), F(y),
                 nullptr));
  return y;
}
void CudaRope(Tensor& q, Tensor& k, int pos, float theta, RopeType rope_type, int device_id) {
  if (q.shape.size() != 2 || k.shape.size() != 2 || q.shape[1] != k.shape[1])
    throw std::runtime_error("CudaRope: expected q [n_heads, head_dim], k [n_kv_heads, head_dim]");
  CudaTensor qd = CudaTensorFromHost(q, device_id), kd = CudaTensorFromHost(k, device_id);
  CudaRopeDeviceInput(qd, kd, q.shape[0], k.shape[0], q.shape[1], pos, theta, rope_type,
                      device_id);
  qd.DownloadTo(q);
  kd.DownloadTo(k);
}
void CudaRopeDeviceInput(CudaTensor& q, CudaTensor& k, int n_heads, int n_kv_heads, int head_dim,
                         int pos, float theta, RopeType rope_type, int device_id) {
  if (q.size() != static_cast<size_t>(n_heads) * head_dim ||
      k.size() != static_cast<size_t>(n_kv_heads) * head_dim)
    throw std::runtime_error("CudaRope: shape mismatch");
  SetDevice(device_id, "CudaRope");
  Check(dqmk_rope(F(q), F(k), n_heads, n_kv_heads, head_dim, pos, theta,
                  rope_type == RopeType::kNeoX ? 1 : 0, nullptr));
}

// ---------------------------------------------------------------- cuda_attention.h
CudaTensor CudaAttentionDecodeDeviceInput(const CudaTensor& q, const CudaKvCache& kv_cache,
                                          int layer, int pos, int n_heads, int n_kv_heads,
                                          int head_dim, int device_id) {
  if (kv_cache.empty()) throw std::runtime_error("CudaAttentionDecode: empty KV cache");
  if (kv_cache.n_kv_heads() != n_kv_heads || kv_cache.head_dim() != head_dim)
    throw std::runtime_error("CudaAttentionDecode: cache shape mismatch");
  if (q.size() != static_cast<size_t>(n_heads) * head_dim)
    throw std::runtime_error("CudaAttentionDecode: q shape mismatch");
  SetDevice(device_id, "CudaAttentionDecode");
  // The device-resident result is flat [n_heads * head_dim], ready for the O projection.
  CudaTensor out({n_heads * head_dim}, device_id);
  Check(dqmk_attention_decode(F(q), static_cast<const float*>(kv_cache.keys_data()),
                              static_cast<const float*>(kv_cache.values_data()),
                              kv_cache.n_layers(), kv_cache.max_seq_len(), n_kv_heads, head_dim,
                              layer, pos, n_heads, F(out), nullptr));
  return out;
}
Tensor CudaAttentionDecode(const Tensor& q, const CudaKvCache& kv_cache, int layer, int pos,
                           int n_heads, int n_kv_heads, int head_dim, int device_id) {
  CudaTensor qd = CudaTensorFromHost(q, device_id);
  Tensor out = CudaAttentionDecodeDeviceInput(qd, kv_cache, layer, pos, n_heads, n_kv_heads,
                                              head_dim, device_id)
                   .Download();
  out.shape = {n_heads, head_dim};
  return out;
}

// ---------------------------------------------------------------- cuda_matmul.h
bool CudaMatmulBuilt() { return true; }

CudaTensor CudaLinearDeviceInput(const CudaTensor& x, const void* w_device,
                                 const std::vector<int>& w_shape, int device_id) {
  SetDevice(device_id, "CudaLinear");
  std::vector<int> y_shape;
  const int rows = RowsOf(x.shape(), w_shape, "CudaLinear", &y_shape);
  CudaTensor y(y_shape, device_id);
  Check(dqmk_f32_linear(F(x), rows, w_shape[1], static_cast<const float*>(w_device), w_shape[0],
                        nullptr, F(y), nullptr));
  return y;
}
Tensor CudaLinearDeviceWeight(const Tensor& x, const void* w_device,
                              const std::vector<int>& w_shape, const Tensor* bias,
                              int device_id) {
  SetDevice(device_id, "CudaLinear");
  CudaTensor xd = CudaTensorFromHost(x, device_id);
  std::vector<int> y_shape;
  const int rows = RowsOf(x.shape, w_shape, "CudaLinear", &y_shape);
  CudaTensor bd;
  if (bias) {
    if (bias->data.size() != static_cast<size_t>(w_shape[0]))
      throw std::runtime_error("CudaLinear: bias shape mismatch");
    bd = CudaTensorFromHost(*bias, device_id);
  }
  CudaTensor y(y_shape, device_id);
  Check(dqmk_f32_linear(F(xd), rows, w_shape[1], static_cast<const float*>(w_device), w_shape[0],
                        bias ? F(bd) : nullptr, F(y), nullptr));
  return y.Download();
}
Tensor CudaLinear(const Tensor& x, const Tensor& weight, const Tensor* bias, int device_id) {
  if (weight.shape.size() != 2) throw std::runtime_error("CudaLinear: expected 2D weight");
  CudaTensor wd = CudaTensorFromHost(weight, device_id);
  return CudaLinearDeviceWeight(x, wd.data(), weight.shape, bias, device_id);
}
// C = A B for A [m, k], B [k, n]: the F32 Linear against B transposed.
Tensor CudaMatmul(const Tensor& a, const Tensor& b, int device_id) {
  if (a.shape.size() != 2 || b.shape.size() != 2 || a.shape[1] != b.shape[0])
    throw std::runtime_error("CudaMatmul: shape mismatch");
  const int k = b.shape[0], n = b.shape[1];
  Tensor bt({n, k}, 0.0f);
  for (int i = 0; i < k; ++i)
    for (int j = 0; j < n; ++j) bt.data[static_cast<size_t>(j) * k + i] = b.data[static_cast<size_t>(i) * n + j];
  return CudaLinear(a, bt, nullptr, device_id);
}

}  // namespace dqm
