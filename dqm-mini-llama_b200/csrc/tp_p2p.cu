// tp_p2p.cu -- the reading side of the tensor-parallel exchange over peer
// memory (NVLink / NVSwitch), which replaces an NCCL all-reduce per
// row-parallel GEMV in the decode step.
//
// The writing side of the vector exchange lives in the row-parallel GEMV
// (gemv.cu, kEpiPeer): each rank stores its partial rows straight into slot
// [parity][own rank] of every rank's buffer and raises its flag there with a
// system-scope release.  The argmax exchange is one kernel here.  Here a rank waits until every rank's flag for the
// exchange has arrived (acquire loads on its own memory, bounded to about two
// seconds), then sums the slots in fixed rank order -- the same order on
// every rank, so all ranks hold bit-identical sums -- and adds the residual.
// Two parities suffice: a rank can only write exchange s + 2 after reading
// exchange s + 1, which every rank wrote after finishing its read of s.
#include "common.cuh"
#include "internal.h"

namespace dqmk {
namespace {

constexpr unsigned long long kPeerWaitNs = 2000000000ull;

__device__ unsigned int g_tp_error;  // kErrTimeout: a peer wait ran out; kErrNoToken

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread-level: true once flag [channel][w] >= s for every rank w.  After one
// wait has run out (flag set, not yet cleared by the host) later waits give up
// at once, so a lost rank costs one timeout, not one per exchange.
__device__ bool wait_flags(const PeerSet& ps, int channel, unsigned int s) {
  char* own = ps.base[ps.rank];
  const unsigned long long t0 = now_ns();
  while (true) {
    if (*(volatile unsigned int*)&g_tp_error) return false;
    bool all = true;
    for (int w = 0; w < ps.world; ++w)
      all = all && ld_acquire_sys(tp_flag(own, ps.world, ps.dim, channel, w)) >= s;
    if (all) return true;
    if (now_ns() - t0 > kPeerWaitNs) {
      atomicOr(&g_tp_error, 1u);
      return false;
    }
  }
}

__global__ void __launch_bounds__(256) tp_reduce_kernel(float* __restrict__ x, const PeerSet ps) {
  __shared__ int ok;
  pdl_trigger();
  pdl_wait();
  const unsigned int s = ps.seq[0] + 1;
  if (threadIdx.x == 0) ok = wait_flags(ps, 0, s);
  __syncthreads();
  if (ok) {
    const float4* slots = reinterpret_cast<const float4*>(
        ps.base[ps.rank] + tp_vec_off((int)(s & 1u), 0, ps.world, ps.dim));
    const int n4 = ps.dim / 4;
    float4* x4 = reinterpret_cast<float4*>(x);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      float4 acc = __ldcv(slots + i);
      for (int w = 1; w < ps.world; ++w) {
        const float4 v = __ldcv(slots + (size_t)w * n4 + i);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
      }
      const float4 r = x4[i];
      x4[i] = make_float4(__fadd_rn(r.x, acc.x), __fadd_rn(r.y, acc.y), __fadd_rn(r.z, acc.z),
                          __fadd_rn(r.w, acc.w));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ps.seq[0] = s;
}

// One thread: send this rank's argmax key (from the vocabulary-parallel
// lm_head) to every rank, wait for all ranks' keys, take the max -- first
// maximum wins through the packed index -- and advance the greedy state.
__global__ void tp_argmax_advance_kernel(const PeerSet ps, const unsigned long long* local_key,
                                         int* token, int* pos, int* history, int cap, int vocab) {
  pdl_trigger();
  pdl_wait();
  const unsigned int s = ps.seq[1] + 1;
  const unsigned long long mine = *local_key;
  for (int w = 0; w < ps.world; ++w)
    reinterpret_cast<unsigned long long*>(ps.base[w] + tp_keys_off(ps.world, ps.dim))
        [(s & 1u) * ps.world + ps.rank] = mine;
  __threadfence_system();
  for (int w = 0; w < ps.world; ++w)
    st_release_sys(tp_flag(ps.base[w], ps.world, ps.dim, 1, ps.rank), s);
  unsigned long long best = 0ull;
  if (wait_flags(ps, 1, s)) {
    const unsigned long long* keys = reinterpret_cast<const unsigned long long*>(
        ps.base[ps.rank] + tp_keys_off(ps.world, ps.dim)) + (s & 1u) * ps.world;
    for (int w = 0; w < ps.world; ++w) {
      const unsigned long long k = __ldcv(keys + w);
      best = k > best ? k : best;
    }
  }
  ps.seq[1] = s;
  // no valid key (a wait ran out here or in the lm_head): keep the state
  int idx = 0;
  if (!argmax_token(best, vocab, &idx)) {
    atomicOr(&g_tp_error, kErrNoToken);
    return;
  }
  const int p = *pos;
  if (history && p >= 0 && p < cap) history[p] = idx;
  *token = idx;
  *pos = p + 1;
}

}  // namespace

cudaError_t launch_tp_reduce(float* x, const PeerSet& ps, cudaStream_t s, bool pdl) {
  if (ps.dim % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u)) return cudaErrorInvalidValue;
  return launch(tp_reduce_kernel, dim3(1), dim3(256), 0, s, pdl, x, ps);
}

cudaError_t launch_tp_argmax_advance(const PeerSet& ps, const unsigned long long* local_key,
                                     int* token, int* pos, int* history, int cap, int vocab,
                                     cudaStream_t s, bool pdl) {
  return launch(tp_argmax_advance_kernel, dim3(1), dim3(1), 0, s, pdl, ps, local_key, token, pos,
                history, cap, vocab);
}

cudaError_t tp_error_address(unsigned int** p) {
  return cudaGetSymbolAddress(reinterpret_cast<void**>(p), g_tp_error);
}

cudaError_t read_tp_error(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_tp_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *flags) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_tp_error, &zero, sizeof(unsigned int));
  }
  return e;
}

}  // namespace dqmk
