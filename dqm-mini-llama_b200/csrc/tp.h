// tp.h -- tensor-parallel shard plan and NCCL collectives (tp.cc).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstring>

#include "dqmk.h"

namespace dqmk {

int tp_plan(const dqmk_model_config& c, int rank, int world, dqmk_tp_plan* out);
// Collective over all ranks of the group: every rank calls it with the same id.
int tp_comm_create(int rank, int world, const unsigned char id[128], void** comm);
void tp_comm_destroy(void* comm);
// In-place all-reduces and an all-gather of `count` elements per rank, enqueued
// on `s` (capturable into a CUDA graph).
int tp_allreduce_sum(void* comm, float* buf, size_t count, cudaStream_t s, const char* api);
int tp_allreduce_max_u64(void* comm, unsigned long long* buf, size_t count, cudaStream_t s,
                         const char* api);
int tp_allgather(void* comm, const float* send, float* recv, size_t count, cudaStream_t s,
                 const char* api);

}  // namespace dqmk
