// common.cuh -- shared device/host helpers for the dqmk kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "dqmk.h"
#include "internal.h"

namespace dqmk {

// ---------------------------------------------------------------- errors
// The C-ABI never throws: each entry point returns a dqmk_status and leaves a
// message (prefixed with the reference API name it replaces) in a
// thread-local buffer read back by dqmk_last_error().


// ---------------------------------------------------------------- launch
// Every kernel after the first of a dependent chain is launched with
// programmatic stream serialization (PDL): its CTAs may start while the
// previous kernel drains, prefetch their weights, then block in
// griddepcontrol.wait until the producer grid has completed and flushed.
template <typename Kern, typename... Args>
cudaError_t launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------- device
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// fp16 bits -> float: exact widening (same value as src/quant.cc:19-50).
__device__ __forceinline__ float h2f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// float -> fp16 bits with the reference's rounding (src/quant.cc:53-90):
// bump by one fp16 ulp whenever bit 12 of the dropped mantissa is set (ties
// and above round away from zero in magnitude, sticky bits ignored);
// overflow and NaN saturate to infinity.
__device__ __forceinline__ uint16_t f2h_ref(float v) {
  uint32_t bits = __float_as_uint(v);
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

// Packed fp32x2 arithmetic (sm_100): one instruction, two lanes of work.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(unsigned long long v) {
  return __uint_as_float((uint32_t)(v >> 32));
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Byte k of `w` as a float 2^23 + byte: one PRMT, no int->float unit.
__device__ __forceinline__ float magic_byte(uint32_t w, int k) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + (uint32_t)k));
}

// 128-bit streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 128-bit streaming load of four floats (read once, no L1 allocation).
__device__ __forceinline__ float4 ldg_f4_stream(const float* p) {
  const uint4 r = ldg_stream(p);
  return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z),
                     __uint_as_float(r.w));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Total-order key for a float so that unsigned max == float max; among equal
// values the smaller index wins (the reference's ArgMax keeps the first max,
// src/ops.cc:182-195).
// System-scope release store / acquire load (flags exchanged with peer GPUs).
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int* tp_flag(char* base, int world, int dim, int channel,
                                                 int rank) {
  return reinterpret_cast<unsigned int*>(base + tp_flags_off(world, dim)) + channel * world + rank;
}

// After every thread of the CTA stored its share of exchange s: the last CTA
// of the grid raises flag [channel][own rank] to s on every rank.  Called by
// all threads of every CTA.  One system-scope fence per CTA: the barrier
// orders the CTA's stores before thread 0's fence, and release cumulativity
// carries them to any rank that acquires the flag.
__device__ __forceinline__ void peer_signal(const PeerSet& ps, int channel, unsigned int s,
                                            int n_ctas) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int done = atomicAdd(ps.ticket, 1u);
    if (done == (unsigned int)n_ctas - 1) {
      __threadfence_system();
      for (int w = 0; w < ps.world; ++w)
        st_release_sys(tp_flag(ps.base[w], ps.world, ps.dim, channel, ps.rank), s);
      *ps.ticket = 0u;
    }
  }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xffffffffu - idx);
}

// The token id a folded argmax key names; false when nothing was folded in
// (key 0: the lm_head's bounded wait ran out before its rows were scored) or
// the id lies outside [0, limit).  Greedy steps keep their state then, so a
// timed-out step never feeds an invalid id to the next embedding.
__device__ __forceinline__ bool argmax_token(unsigned long long key, int limit, int* token) {
  if (key == 0ull) return false;
  const int idx = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffu));
  if (idx < 0 || idx >= limit) return false;
  *token = idx;
  return true;
}

}  // namespace dqmk
