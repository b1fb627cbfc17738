// step.cu -- the decode step as one persistent kernel (sm_100a).
//
// The multi-kernel decode step is 1 + 5 L kernels chained by programmatic
// dependent launch; at batch 1 every kernel is short and the chain's per-link
// latency, not HBM, sets the step time.  Here the same work runs as phases of
// one cooperative kernel (every CTA resident; the launch fails rather than
// hangs if they cannot all be): embedding, then per layer the fused QKV
// GEMV, attention, the O GEMV, the gate/up GEMV and the down GEMV, with a
// grid barrier between phases.  A GEMV phase loads its first weight tile and
// RMSNorm weight into registers BEFORE the barrier -- they do not depend on
// the previous phase -- so the barrier wait overlaps its weight stream, which
// is what programmatic dependent launch gives the multi-kernel chain.  The
// phases run the same device code as the standalone kernels (gemv_dev.cuh,
// attention_dev.cuh), so results are bit-identical to the multi-kernel path.
// The lm_head (TMA-staged GEMV, its own CTA shape) follows as a second launch.
// Measured on Qwen2-0.5B Q8_0 decode: 773 tok/s against 1357 for the chain --
// a grid barrier costs 2.5-3.5 us with 148-592 CTAs, and the step has 121 of
// them, each followed by a phase that starts cold; so the engine uses this
// kernel only when asked (DQMK_STEP_KERNEL=1).
//
// Grid barrier: one arrival counter and one generation word in device
// memory; the last CTA to arrive resets the counter and bumps the generation
// (release); the others wait for the bump (acquire), bounded to about a
// second.  A wait that runs out records a flag (read by dqmk_device_error and
// the engine's synchronous calls) and every later wait of the kernel gives up
// at once, so a fault elsewhere costs one timeout, not a hang.
#include "attention_dev.cuh"
#include "common.cuh"
#include "gemv_dev.cuh"
#include "internal.h"

namespace dqmk {
namespace {

using namespace gv;

constexpr unsigned long long kSyncWaitNs = 1000000000ull;

__device__ unsigned int g_step_error;  // bit 0: a grid-barrier wait timed out

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void grid_sync(const StepSync& s, int n_ctas) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int g = ld_acquire_gpu(s.gen);
    __threadfence();
    if (atomicAdd(s.count, 1u) == (unsigned int)n_ctas - 1) {
      atomicExch(s.count, 0u);
      __threadfence();
      st_release_gpu(s.gen, g + 1);
    } else {
      const unsigned long long t0 = now_ns();
      while (ld_acquire_gpu(s.gen) == g) {
        if (*(volatile unsigned int*)&g_step_error) break;
        if (now_ns() - t0 > kSyncWaitNs) {
          atomicOr(&g_step_error, 1u);
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
}

// Embedding gather of the device token from the packed token_embd rows
// (values d * q, exact in float) and the argmax slot reset; CTA 0 only.
__device__ __forceinline__ void embed_phase(const EmbedArgs& a) {
  const int token = a.token_dev ? __ldcg(a.token_dev) : a.token;
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
}

template <int HD>
__device__ __forceinline__ void attention_phase(const AttnArgs& a, int chunk_cap, int cta,
                                                int n_ctas, float* sm) {
  const int items = a.n_kv_heads * a.max_splits;
  for (int w = cta; w < items; w += n_ctas)
    at::attention_hd_body<HD, kWarps * 32>(a, chunk_cap, w % a.n_kv_heads, w / a.n_kv_heads,
                                           a.max_splits, sm);
}

// Compile-time shape of a GEMV variant id.
template <int ID>
struct VariantOf;
#define DQMK_VARIANT_TRAITS(ID, QT_, RPW_, CPL_, GW_)                          \
  template <>                                                                 \
  struct VariantOf<ID> {                                                      \
    static constexpr int QT = QT_, RPW = RPW_, CPL = CPL_, GW = GW_;          \
  };
#pragma nv_diag_suppress 177  // traits of the ids no step set uses
DQMK_GEMV_VARIANT_IDS(DQMK_VARIANT_TRAITS)
#pragma nv_diag_default 177
#undef DQMK_VARIANT_TRAITS

// One GEMV phase: prefetch, barrier, math (see the file comment).
template <int ID>
__device__ __forceinline__ void gemv_phase(const GemvArgs& a, float4* smem, int cta, int n,
                                           const StepSync& sync) {
  using V = VariantOf<ID>;
  GemvPhase<V::QT, V::RPW, V::CPL, V::GW> ph;
  ph.prefetch(a, cta, n);
  grid_sync(sync, n);
  gemv_run<V::QT, V::RPW, V::CPL, V::GW, false>(ph, a, smem, n);
}

// Instantiated per set of GEMV variants a model's layers use (at most three):
// a kernel holding every variant of a quant type spills heavily, one holding
// the few a model needs does not.  Unused slots are -1.
template <int V0, int V1, int V2>
__global__ void __launch_bounds__(kWarps * 32, 1) decode_step_kernel(const StepPhase* __restrict__ phases,
                                                                     int n_phases,
                                                                     const StepSync sync) {
  extern __shared__ float4 smem[];
  const int cta = blockIdx.x, n = gridDim.x;
  for (int i = 0; i < n_phases; ++i) {
    const int kind = phases[i].kind;
    if (kind == kPhaseEmbed) {
      if (cta == 0) embed_phase(phases[i].e);
    } else if (kind == kPhaseAttn) {
      const AttnArgs& at = phases[i].at;
      const int cap = phases[i].chunk_cap;
      grid_sync(sync, n);
      if (at.head_dim == 64)
        attention_phase<64>(at, cap, cta, n, reinterpret_cast<float*>(smem));
      else
        attention_phase<128>(at, cap, cta, n, reinterpret_cast<float*>(smem));
    } else {
      const GemvArgs& a = phases[i].g;
      const int v = phases[i].variant;
      if (v == V0) {
        gemv_phase<V0>(a, smem, cta, n, sync);
      } else if constexpr (V1 >= 0) {
        if (v == V1) {
          gemv_phase<V1>(a, smem, cta, n, sync);
        } else if constexpr (V2 >= 0) {
          if (v == V2) gemv_phase<V2>(a, smem, cta, n, sync);
          else grid_sync(sync, n);
        } else {
          grid_sync(sync, n);
        }
      } else {
        grid_sync(sync, n);
      }
    }
  }
  pdl_trigger();
}

// The variant sets with a step kernel: Qwen2-0.5B Q8_0 (QKV / O / gate-up,
// down), Qwen2-0.5B Q4_0 (QKV / O / gate-up, down), Qwen2-7B Q4_0 (QKV / O,
// gate-up, down).
#define DQMK_STEP_SETS(X) X(1, 4, -1) X(14, 11, -1) X(10, 8, 13)

}  // namespace

namespace {

// The step kernel for a set of variant ids (sorted as in DQMK_STEP_SETS), or
// nullptr.
const void* step_kernel_for(const int (&v)[3]) {
#define DQMK_STEP_PICK(A, B, C) \
  if (v[0] == A && v[1] == B && v[2] == C) return (const void*)decode_step_kernel<A, B, C>;
  DQMK_STEP_SETS(DQMK_STEP_PICK)
#undef DQMK_STEP_PICK
  return nullptr;
}

}  // namespace

bool step_kernel_variants(const int* ids, int n, int out[3]) {
  int v[3] = {-1, -1, -1};
  int k = 0;
  for (int i = 0; i < n; ++i) {
    bool seen = false;
    for (int j = 0; j < k; ++j) seen = seen || v[j] == ids[i];
    if (seen) continue;
    if (k == 3) return false;
    v[k++] = ids[i];
  }
  // try every order of the distinct ids against the instantiated sets
  const int perm[6][3] = {{0, 1, 2}, {0, 2, 1}, {1, 0, 2}, {1, 2, 0}, {2, 0, 1}, {2, 1, 0}};
  for (const auto& p : perm) {
    const int c[3] = {v[p[0]], v[p[1]], v[p[2]]};
    if (step_kernel_for(c)) {
      for (int j = 0; j < 3; ++j) out[j] = c[j];
      return true;
    }
  }
  return false;
}

cudaError_t step_kernel_grid(const int set[3], size_t smem, int* grid) {
  const void* fn = step_kernel_for(*reinterpret_cast<const int(*)[3]>(set));
  if (!fn) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kWarps * 32, smem);
  if (e != cudaSuccess) return e;
  *grid = per_sm * sm_count();
  return *grid > 0 ? cudaSuccess : cudaErrorInvalidConfiguration;
}

cudaError_t launch_step_kernel(const int set[3], const StepPhase* phases, int n_phases,
                               const StepSync& sync, int grid, size_t smem, cudaStream_t s) {
  const void* fn = step_kernel_for(*reinterpret_cast<const int(*)[3]>(set));
  if (!fn) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  StepSync sy = sync;
  void* args[] = {(void*)&phases, (void*)&n_phases, (void*)&sy};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

size_t step_attention_smem(int head_dim, int chunk_cap, int max_splits) {
  return at::smem_bytes_hd(head_dim, chunk_cap, max_splits, kWarps * 32);
}

cudaError_t read_step_error(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_step_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *flags) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_step_error, &zero, sizeof(unsigned int));
  }
  return e;
}

}  // namespace dqmk
