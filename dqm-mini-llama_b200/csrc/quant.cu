// quant.cu -- Q8_0 / Q4_0 quantize, dequantize and repack on the device.
//
// Quantizers are bit-exact restatements of the reference's CPU routines
// (src/quant.cc:372-476): one warp owns one 32-value block, lane i holds
// element i.  Every float operation is spelled with an explicit _rn
// intrinsic so the compiler cannot fuse a multiply into an add where the
// reference rounds twice.
#include "common.cuh"
#include "internal.h"

namespace dqmk {
namespace {

constexpr int kQ80Bytes = 34;
constexpr int kQ40Bytes = 18;

__global__ void quantize_q80_kernel(const float* __restrict__ src, int64_t n_rows,
                                    int64_t row_size, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nb = (row_size + 31) / 32;
  const int64_t total = n_rows * nb;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t blk = warp; blk < total; blk += nwarps) {
    const int64_t r = blk / nb, b = blk % nb;
    const int64_t k = b * 32 + lane;
    const bool valid = k < row_size;
    const float v = valid ? src[r * row_size + k] : 0.0f;
    // absmax over the block (src/quant.cc:388-394); NaN never wins.
    float amax = warp_max(valid ? fabsf(v) : 0.0f);
    uint8_t* o = out + blk * kQ80Bytes;
    uint16_t d = 0;
    int q = 0;
    if (amax > 0.0f) {
      d = f2h_ref(__fdiv_rn(amax, 127.0f));
      const float stored = h2f(d);
      const float inv = stored == 0.0f ? 0.0f : __fdiv_rn(1.0f, stored);
      if (valid) {
        q = (int)roundf(__fmul_rn(v, inv));
        q = q > 127 ? 127 : (q < -127 ? -127 : q);
      }
    }
    if (lane == 0) {
      o[0] = (uint8_t)(d & 0xff);
      o[1] = (uint8_t)(d >> 8);
    }
    o[2 + lane] = (uint8_t)(int8_t)q;
  }
}

__global__ void quantize_q40_kernel(const float* __restrict__ src, int64_t n_rows,
                                    int64_t row_size, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nb = (row_size + 31) / 32;
  const int64_t total = n_rows * nb;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t blk = warp; blk < total; blk += nwarps) {
    const int64_t r = blk / nb, b = blk % nb;
    const int64_t k = b * 32 + lane;
    const bool valid = k < row_size;
    const float v = valid ? src[r * row_size + k] : 0.0f;
    float amax = warp_max(valid ? fabsf(v) : 0.0f);
    uint8_t* o = out + blk * kQ40Bytes;
    uint16_t d = 0;
    int q = 0;  // nibble for this lane's element; whole block zero when amax == 0
    if (amax > 0.0f) {
      d = f2h_ref(__fdiv_rn(amax, 7.0f));
      const float stored = h2f(d);
      const float inv = stored == 0.0f ? 0.0f : __fdiv_rn(1.0f, stored);
      // src/quant.cc:453-468: x*id (0 past the row end), then round(x + 8).
      const float xs = valid ? __fmul_rn(v, inv) : 0.0f;
      q = (int)roundf(__fadd_rn(xs, 8.0f));
      q = q < 0 ? 0 : (q > 15 ? 15 : q);
    }
    const int hi = __shfl_down_sync(0xffffffffu, q, 16);
    if (lane == 0) {
      o[0] = (uint8_t)(d & 0xff);
      o[1] = (uint8_t)(d >> 8);
    }
    if (lane < 16) o[2 + lane] = (uint8_t)(q | (hi << 4));
  }
}

__global__ void dequantize_kernel(int qtype, const uint8_t* __restrict__ blocks, int64_t n_rows,
                                  int64_t row_size, float* __restrict__ dst) {
  const int64_t nb = (row_size + 31) / 32;
  const int64_t total = n_rows * row_size;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / row_size, k = e % row_size;
    const int64_t blk = r * nb + k / 32;
    const int j = (int)(k % 32);
    if (qtype == DQMK_Q80) {
      const uint8_t* p = blocks + blk * kQ80Bytes;
      const float d = h2f((uint16_t)(p[0] | (p[1] << 8)));
      dst[e] = __fmul_rn(d, (float)(int8_t)p[2 + j]);
    } else {
      const uint8_t* p = blocks + blk * kQ40Bytes;
      const float d = h2f((uint16_t)(p[0] | (p[1] << 8)));
      const int q = j < 16 ? (p[2 + j] & 0x0f) : (p[2 + j - 16] >> 4);
      dst[e] = __fmul_rn(d, (float)(q - 8));
    }
  }
}

// ggml blocks -> planar weight (quants plane, then scales plane).  One thread
// per block.  Q8_0 quants past in_features are zeroed.
__global__ void pack_kernel(int qtype, const uint8_t* __restrict__ blocks, int out_features,
                            int in_features, uint8_t* __restrict__ packed) {
  const int nb = (in_features + 31) / 32;
  const int64_t total = (int64_t)out_features * nb;
  const size_t qbytes_row = qtype == DQMK_Q80 ? (size_t)nb * 32 : (size_t)nb * 16;
  uint8_t* qplane = packed;
  uint16_t* dplane = reinterpret_cast<uint16_t*>(packed + qbytes_row * out_features);
  for (int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; blk < total;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = blk / nb;
    const int b = (int)(blk % nb);
    if (qtype == DQMK_Q80) {
      const uint8_t* p = blocks + blk * kQ80Bytes;
      uint8_t* q = qplane + r * qbytes_row + (size_t)b * 32;
      const int valid = min(32, in_features - b * 32);
      for (int j = 0; j < 32; ++j) q[j] = j < valid ? p[2 + j] : 0;
      dplane[blk] = (uint16_t)(p[0] | (p[1] << 8));
    } else {
      const uint8_t* p = blocks + blk * kQ40Bytes;
      uint8_t* q = qplane + r * qbytes_row + (size_t)b * 16;
      for (int j = 0; j < 16; ++j) q[j] = p[2 + j];
      dplane[blk] = (uint16_t)(p[0] | (p[1] << 8));
    }
  }
}

int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

size_t packed_bytes(int qtype, int out_features, int in_features) {
  const size_t nb = (size_t)((in_features + 31) / 32);
  const size_t per_block = qtype == DQMK_Q80 ? 34 : 18;
  return (size_t)out_features * nb * per_block;
}

cudaError_t launch_pack(int qtype, const void* blocks, int out_features, int in_features,
                        void* packed, cudaStream_t stream) {
  const int64_t total = (int64_t)out_features * ((in_features + 31) / 32);
  pack_kernel<<<grid_for(total, 256), 256, 0, stream>>>(
      qtype, static_cast<const uint8_t*>(blocks), out_features, in_features,
      static_cast<uint8_t*>(packed));
  return cudaGetLastError();
}

cudaError_t launch_quantize(int qtype, const float* src, int64_t n_rows, int64_t row_size,
                            void* blocks, cudaStream_t stream) {
  const int64_t total = n_rows * ((row_size + 31) / 32);
  const int g = grid_for(total, 8);
  if (qtype == DQMK_Q80)
    quantize_q80_kernel<<<g, 256, 0, stream>>>(src, n_rows, row_size,
                                               static_cast<uint8_t*>(blocks));
  else
    quantize_q40_kernel<<<g, 256, 0, stream>>>(src, n_rows, row_size,
                                               static_cast<uint8_t*>(blocks));
  return cudaGetLastError();
}

cudaError_t launch_dequantize(int qtype, const void* blocks, int64_t n_rows, int64_t row_size,
                              float* dst, cudaStream_t stream) {
  dequantize_kernel<<<grid_for(n_rows * row_size, 256), 256, 0, stream>>>(
      qtype, static_cast<const uint8_t*>(blocks), n_rows, row_size, dst);
  return cudaGetLastError();
}

}  // namespace dqmk

// ------------------------------------------------------------------ C ABI
using namespace dqmk;

namespace {
int quant_common(const char* api, int qtype, const float* src, int64_t n_rows, int64_t row_size,
                 void* blocks, void* stream) {
  if (n_rows < 0 || row_size < 0) return fail(DQMK_ERR_INVALID, std::string(api) + ": negative shape");
  if (n_rows == 0 || row_size == 0) return DQMK_OK;  // empty tensor -> no blocks
  if (!src || !blocks) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  DQMK_CUDA_RET(api, launch_quantize(qtype, src, n_rows, row_size, blocks,
                                     static_cast<cudaStream_t>(stream)));
  return DQMK_OK;
}
int dequant_common(const char* api, int qtype, const void* blocks, int64_t n_rows,
                   int64_t row_size, float* dst, void* stream) {
  if (n_rows < 0 || row_size < 0) return fail(DQMK_ERR_INVALID, std::string(api) + ": negative shape");
  if (n_rows == 0 || row_size == 0) return DQMK_OK;
  if (!blocks || !dst) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  DQMK_CUDA_RET(api, launch_dequantize(qtype, blocks, n_rows, row_size, dst,
                                       static_cast<cudaStream_t>(stream)));
  return DQMK_OK;
}
}  // namespace

extern "C" int dqmk_quantize_q80(const float* src, int64_t n_rows, int64_t row_size,
                                 void* blocks, void* stream) {
  return quant_common("QuantizeToQ80", DQMK_Q80, src, n_rows, row_size, blocks, stream);
}
extern "C" int dqmk_quantize_q40(const float* src, int64_t n_rows, int64_t row_size,
                                 void* blocks, void* stream) {
  return quant_common("QuantizeToQ40", DQMK_Q40, src, n_rows, row_size, blocks, stream);
}
extern "C" int dqmk_dequantize_q80(const void* blocks, int64_t n_rows, int64_t row_size,
                                   float* dst, void* stream) {
  return dequant_common("DequantizeFromQ80", DQMK_Q80, blocks, n_rows, row_size, dst, stream);
}
extern "C" int dqmk_dequantize_q40(const void* blocks, int64_t n_rows, int64_t row_size,
                                   float* dst, void* stream) {
  return dequant_common("DequantizeFromQ40", DQMK_Q40, blocks, n_rows, row_size, dst, stream);
}

extern "C" size_t dqmk_packed_bytes(int qtype, int out_features, int in_features) {
  if ((qtype != DQMK_Q80 && qtype != DQMK_Q40) || out_features <= 0 || in_features <= 0) return 0;
  return packed_bytes(qtype, out_features, in_features);
}

extern "C" int dqmk_pack_weight(int qtype, const void* blocks, size_t block_count,
                                int out_features, int in_features, void* packed, void* stream) {
  const char* api = "CUDA weight upload";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": unsupported quant type");
  if (out_features <= 0 || in_features <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": expected 2D quantized weight");
  const size_t expected = (size_t)out_features * (size_t)((in_features + 31) / 32);
  if (block_count != expected)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": block count mismatch, expected " +
                                      std::to_string(expected) + ", got " +
                                      std::to_string(block_count));
  if (!blocks || !packed) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  DQMK_CUDA_RET(api, launch_pack(qtype, blocks, out_features, in_features, packed,
                                 static_cast<cudaStream_t>(stream)));
  return DQMK_OK;
}
