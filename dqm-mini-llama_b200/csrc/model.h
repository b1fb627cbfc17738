// model.h -- the device-resident model shared by the engine files
// (engine.cc: single-sequence context; batch_engine.cc: multi-sequence batch).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "dqmk.h"
#include "internal.h"
#include "tp.h"

namespace dqmk {

struct Packed {
  int qtype = 0;
  int rows = 0, k = 0, kp = 0;
  uint8_t* base = nullptr;  // owns qs plane followed by d plane
  size_t bytes = 0;
  const uint8_t* qs() const { return base; }
  const uint16_t* d() const {
    const size_t qb = (size_t)rows * (qtype == DQMK_Q80 ? kp : kp / 2);
    return reinterpret_cast<const uint16_t*>(base + qb);
  }
};

struct Raw {
  int qtype = 0;
  int rows = 0, cols = 0;
  void* dev = nullptr;           // quantized blocks on the device
  std::vector<float> host;       // F32 tensors (small) kept on the host
};

struct Layer {
  Packed qkv, wo, gate_up, down;
  float* qkv_bias = nullptr;  // packed (paired) row order
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  // batched prefill: each weight as two exact fp16 planes (TMA maps {hi, lo})
  // of its dequantized values scaled per row by 2^-f, and the 2^f
  float *cs_qkv = nullptr, *cs_o = nullptr, *cs_gu = nullptr, *cs_dn = nullptr;
  CUtensorMap map_qkv[2], map_o[2], map_gu[2], map_dn[2];
};

// Weight-side tables of the multi-sequence decode GEMM (batch.cu), built on
// the first batch: per weight its power-of-two row scales, a copy of its block
// scales in 16-byte-padded rows, and the tensor maps of both planes.
struct BatchWeight {
  float* cs = nullptr;
  uint16_t* d_pad = nullptr;  // block scales in 16-byte-padded rows
  CUtensorMap map, dmap;      // quant plane, padded scales
};
struct BatchLayer {
  BatchWeight qkv, wo, gate_up, down;
};

int dev_alloc(std::vector<void*>& owner, size_t bytes, void** out, const char* api);
bool use_pdl();

}  // namespace dqmk


struct dqmk_model {
  dqmk_model_config cfg{};
  int device = 0;
  int qtype = 0;
  bool finalized = false;
  std::map<std::string, dqmk::Raw> raw;
  std::vector<dqmk::Layer> layers;
  dqmk::Packed embd, lm_head;
  bool tied = true;
  bool prefill_eligible = false;  // batched prefill possible (head size, no TP)
  bool prefill_ready = false;     // its two-term weight planes and TMA maps built
  bool batch_ready = false;    // multi-sequence GEMM tables built
  std::vector<dqmk::BatchLayer> batch_layers;
  dqmk::BatchWeight batch_lm;
  dqmk_tp_plan tp{};           // this model's shard (world 1: everything)
  void* comm = nullptr;        // NCCL communicator when tp.world > 1
  float* final_norm = nullptr;
  float2* rope_cs = nullptr;
  std::vector<void*> allocs;
  size_t memory_bytes = 0;
  dqmk_model_stats stats{};

  ~dqmk_model() {
    cudaSetDevice(device);
    for (void* p : allocs) cudaFree(p);
    for (auto& kv : raw)
      if (kv.second.dev) cudaFree(kv.second.dev);
    dqmk::tp_comm_destroy(comm);
  }
};

