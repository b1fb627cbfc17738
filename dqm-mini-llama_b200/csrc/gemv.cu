// gemv.cu -- batch-1 decode GEMV over Q8_0 / Q4_0 weights (sm_100a).
//
// The kernel behind every projection of the decode step, with the
// memory-bound neighbours fused in:
//   prologue  x staged once per CTA into shared memory (bank-swizzled),
//             optionally RMS-normalised on the fly (src/ops.cc:68-90);
//   main loop each warp owns RPW weight rows; each lane streams 16-byte
//             chunks of them with 128-bit no-L1-allocate loads, converts
//             bytes to floats with a PRMT "magic number" (no int->float
//             unit), and accumulates with packed f32x2 FMAs; one fp16 scale
//             multiply per 32-value block;
//   epilogue  warp-shuffle reduction, then bias / residual add, SwiGLU of
//             interleaved gate/up rows, QKV bias + RoPE + KV-cache store, or
//             logits + device argmax.
// Weights for the warp's first rows are loaded BEFORE griddepcontrol.wait,
// so under programmatic dependent launch the weight stream of this kernel
// overlaps the tail of the previous kernel in the decode chain.
//
// Reference semantics: LinearQuantizedImpl (src/quant.cc:278-346) computes
// y[j] = sum_k (d*q_k) * x_k as one sequential FMA chain in k.  Here the sum
// is split across lanes and the scale is applied per block, so results agree
// to float rounding (checked against the oracle), not bit for bit.
#include <algorithm>

#include "common.cuh"
#include "gemv_dev.cuh"
#include "internal.h"
#include "prefill.h"
#include "tc_dev.cuh"

namespace dqmk {
namespace {

using namespace gv;

__device__ unsigned int g_device_error;  // kErrTimeout / kErrNoToken

template <int QT, int RPW, int CPL, int GW, bool PEER>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const GemvArgs a) {
  extern __shared__ float4 xs[];
  // Weights and norm weights do not depend on the previous kernel: fetch
  // them before the programmatic-dependency wait.
  GemvPhase<QT, RPW, CPL, GW> ph;
  ph.prefetch(a, blockIdx.x, gridDim.x, xs + (a.kp >> 2));
  pdl_trigger();
  pdl_wait();
  gemv_run<QT, RPW, CPL, GW, PEER>(ph, a, xs, gridDim.x, &g_device_error);
}

// ------------------------------------------------------------ launch table
// One-time kernel attributes and the resident-CTA cap for the grid-stride
// case.  Run before any stream capture (context creation does).
template <int QT, int RPW, int CPL, int GW, bool PEER>
cudaError_t prepare_t(int* max_ctas_out) {
  static DeviceOnce once;
  static int max_ctas[kMaxDevices];  // written under once's lock, per device
  cudaError_t e = once.run([] {
    int dev = 0;
    cudaError_t r = cudaGetDevice(&dev);
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(gemv_kernel<QT, RPW, CPL, GW, PEER>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    int per_sm = 0;
    if (r == cudaSuccess)
      r = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &per_sm, gemv_kernel<QT, RPW, CPL, GW, PEER>, kWarps * 32, 4096 * sizeof(float));
    if (r == cudaSuccess) max_ctas[dev] = (per_sm > 0 ? per_sm : 1) * sm_count();
    return r;
  });
  if (e != cudaSuccess) return e;
  if (max_ctas_out) {
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    *max_ctas_out = max_ctas[dev];
  }
  return cudaSuccess;
}

template <int QT, int RPW, int CPL, int GW, bool PEER>
cudaError_t launch_impl(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  int max_ctas = 0;
  cudaError_t e = prepare_t<QT, RPW, CPL, GW, PEER>(&max_ctas);
  if (e != cudaSuccess) return e;
  // x, then (RMSNorm kernels) the norm weight
  const size_t smem = (size_t)a.kp * sizeof(float) * (a.norm_w ? 2 : 1);
  const int n_groups = (a.n_rows + RPW - 1) / RPW;
  constexpr int GPC = kWarps / GW;
  int grid = (n_groups + GPC - 1) / GPC;
  if (grid > max_ctas) grid = max_ctas;
  if (grid < 1) grid = 1;
  return launch(gemv_kernel<QT, RPW, CPL, GW, PEER>, dim3(grid), dim3(kWarps * 32), smem,
                stream, pdl, a);
}

// kEpiPeer takes its own instantiation of the variant (see epilogue).
template <int QT, int RPW, int CPL, int GW>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  if (a.epi == kEpiPeer) return launch_impl<QT, RPW, CPL, GW, true>(a, stream, pdl);
  return launch_impl<QT, RPW, CPL, GW, false>(a, stream, pdl);
}

// ============================================================ TMA-staged GEMV
// Weights stream through a ring of shared-memory stages filled by bulk
// asynchronous copies (cp.async.bulk, completion counted on an mbarrier), so
// the bytes in flight cost shared memory instead of registers.  A CTA owns
// tiles of TR = 8 warps x RPW contiguous rows; its first `nstage` tiles are
// requested before griddepcontrol.wait, so under programmatic dependent
// launch they arrive while the previous kernel of the chain still runs.
// Every wait on a stage is bounded (about a second of %globaltimer); on
// timeout the CTA records DQMK_ERR_TIMEOUT in a device flag, stops issuing,
// waits (bounded) for its copies still in flight, and exits.
constexpr int kTmaWarps = 8;                        // consumer warps
constexpr int kTmaConsumers = kTmaWarps * 32;
constexpr int kTmaThreads = kTmaConsumers + 32;     // + the producer warp
constexpr int kMaxStages = 4;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// global -> shared bulk copy completing on `bar`; 16-byte aligned, size % 16 == 0
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

struct TmaGeo {
  int chunks, row_bytes, nbk, n_tiles, my_tiles;
  size_t q_stage, stage_bytes;  // bytes of one stage's quants, of the whole stage
};

// Issue the copies of local tile i into stage s (thread 0 only).  Returns
// whether the stage now has a copy in flight.
template <int QT, int RPW>
__device__ __forceinline__ bool tma_issue(const GemvArgs& a, const TmaGeo& g, unsigned char* stages,
                                          uint64_t* full, int i, int s, uint64_t policy,
                                          int skip_tile) {
  constexpr int TR = kTmaWarps * RPW;
  const int tile = blockIdx.x + i * gridDim.x;
  const int r0 = tile * TR;
  const int rows = min(TR, a.n_rows - r0);
  const uint32_t qbytes = (uint32_t)rows * g.row_bytes;
  const uint32_t dbytes = (uint32_t)rows * g.nbk * 2;
  const uint32_t dbulk = (dbytes & 15u) == 0 ? dbytes : 0u;  // ragged tail: scales read directly
  // failure-detection hook: nothing arrives for the withheld tile (or tiles)
  if (tile == skip_tile || skip_tile == kSkipAllTiles) return false;
  unsigned char* st = stages + (size_t)s * g.stage_bytes;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_expect_tx(&full[s], qbytes + dbulk);
  bulk_g2s(st, a.qs + (size_t)r0 * g.row_bytes, qbytes, &full[s], policy);
  if (dbulk)
    bulk_g2s(st + g.q_stage, reinterpret_cast<const unsigned char*>(a.d) + (size_t)r0 * g.nbk * 2,
             dbulk, &full[s], policy);
  return true;
}

// x staged linearly (fp32), RMS-normalised when norm_w is set.  Same single
// round trip as stage_x; the float values are identical.
template <int NWARPS, int NR>
__device__ __forceinline__ void stage_x_linear(const GemvArgs& a, float* xf, const float4 (&nw)[NR],
                                               bool norm_pref, float* red, float* bcast) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int NT = NWARPS * 32;
  const bool active = tid < NT;  // threads beyond NT only join the barriers
  const int nf4 = a.kp >> 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) && ((a.k & 3) == 0);
  float4* xf4 = reinterpret_cast<float4*>(xf);
  float ss = 0.0f;
  if (!active) {
  } else if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const int k4 = a.k >> 2;
    for (int base = 0; base < nf4; base += 8 * NT) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i4 = base + u * NT + tid;
        v[u] = i4 < k4 ? __ldcg(x4 + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i4 = base + u * NT + tid;
        if (i4 < nf4) {
          ss = __fadd_rn(ss, __fmul_rn(v[u].x, v[u].x));
          ss = __fadd_rn(ss, __fmul_rn(v[u].y, v[u].y));
          ss = __fadd_rn(ss, __fmul_rn(v[u].z, v[u].z));
          ss = __fadd_rn(ss, __fmul_rn(v[u].w, v[u].w));
          xf4[i4] = v[u];
        }
      }
    }
  } else {
    for (int e = tid; e < a.kp; e += NT) {
      const float v = e < a.k ? __ldcg(a.x + e) : 0.0f;
      xf[e] = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  }
  if (a.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0 && active) red[wid] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < NWARPS; ++w) t += red[w];
      *bcast = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)a.k), a.eps)));
    }
    __syncthreads();
    const float scale = *bcast;
    if (!active) {
    } else if (vec && norm_pref) {
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        const int i4 = u * NT + tid;
        if (i4 < (a.k >> 2)) {
          float4 v = xf4[i4];
          v.x = __fmul_rn(__fmul_rn(v.x, scale), nw[u].x);
          v.y = __fmul_rn(__fmul_rn(v.y, scale), nw[u].y);
          v.z = __fmul_rn(__fmul_rn(v.z, scale), nw[u].z);
          v.w = __fmul_rn(__fmul_rn(v.w, scale), nw[u].w);
          xf4[i4] = v;
        }
      }
    } else {
      for (int e = tid; e < a.k; e += NT) xf[e] = __fmul_rn(__fmul_rn(xf[e], scale), a.norm_w[e]);
    }
  }
  __syncthreads();
}

// Each 32-value block of x as three int8 terms, x ~= s1 q1 + s2 q2 + s3 q3
// with s1 = absmax/127, s2 = s1/254, s3 = s2/254: every residual fits the next
// term, and what is left is below 6e-8 of the block's absmax -- float
// precision.  Eight threads own a block (four values each, one packed int8x4
// store per term).  Planes [term][half][block][16 bytes] keep the 16-byte
// reads of a lane-per-block loop conflict-free.  Each term's scale is stored,
// and for Q4_0 the sum of its 32 values (for the nibble offset of 8).
template <int NWARPS, bool SUMS>
__device__ __forceinline__ void quantize_x_terms(const float* xf, int nbk, int8_t* q, float* sc,
                                                 int* sum) {
  constexpr int NT = NWARPS * 32;
  const int tid = threadIdx.x;
  const int sub = tid & 7;  // which 4 values of the block
  for (int base = 0; base < nbk * 8; base += NT) {
    const int b = (base + tid) >> 3;
    const bool valid = b < nbk;  // uniform per group of 8 lanes
    float4 v = valid ? reinterpret_cast<const float4*>(xf)[b * 8 + sub]
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    float r[4] = {v.x, v.y, v.z, v.w};
    float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 0.0f;
    const int h = sub >> 2, word = sub & 3;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      const float inv = s > 0.0f ? __frcp_rn(s) : 0.0f;
      uint32_t packed = 0;
      int tsum = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int qq = __float2int_rn(__fmul_rn(r[e], inv));
        qq = qq > 127 ? 127 : (qq < -127 ? -127 : qq);
        r[e] = __fmaf_rn(-s, (float)qq, r[e]);
        packed |= ((uint32_t)qq & 0xffu) << (8 * e);
        tsum += qq;
      }
      if (valid) {
        reinterpret_cast<uint32_t*>(q)[((size_t)(t * 2 + h) * nbk + b) * 4 + word] = packed;
        if (sub == 0) sc[t * nbk + b] = s;
      }
      if constexpr (SUMS) {
        tsum += __shfl_xor_sync(0xffffffffu, tsum, 1);
        tsum += __shfl_xor_sync(0xffffffffu, tsum, 2);
        tsum += __shfl_xor_sync(0xffffffffu, tsum, 4);
        if (valid && sub == 0) sum[t * nbk + b] = tsum;
      }
      s = __fmul_rn(s, 1.0f / 254.0f);
    }
  }
}

// The 32 weights of block b of a packed row as eight int8x4 words in the
// order of the x-term planes: Q8_0 bytes as stored (signed); Q4_0 nibbles
// unpacked to unsigned bytes 0..15, words 0-3 the low nibbles (values
// 4j..4j+3), words 4-7 the high nibbles (values 16+4j..).
template <int QT>
__device__ __forceinline__ void block_words(const unsigned char* row, int b, int (&w)[8]) {
  if constexpr (QT == DQMK_Q80) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(row + b * 32);
    const uint4 w1 = *reinterpret_cast<const uint4*>(row + b * 32 + 16);
    w[0] = (int)w0.x; w[1] = (int)w0.y; w[2] = (int)w0.z; w[3] = (int)w0.w;
    w[4] = (int)w1.x; w[5] = (int)w1.y; w[6] = (int)w1.z; w[7] = (int)w1.w;
  } else {
    const uint4 p = *reinterpret_cast<const uint4*>(row + b * 16);
    const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      w[j] = (int)(pw[j] & 0x0f0f0f0fu);
      w[4 + j] = (int)((pw[j] >> 4) & 0x0f0f0f0fu);
    }
  }
}

// Exact int32 sums of one block against the three x terms:
// S[t] = sum_j q_w[j] q_t[j] (Q4_0: nibbles minus 8, via sm8[t] = 8 sum_j q_t[j]).
// xv[2t], xv[2t+1]: values 0-15 and 16-31 of term t as int8x4 words.
__device__ __forceinline__ void block_term_sums(const int (&w)[8], const int4 (&xv)[6],
                                                const int (&sm8)[3], int (&S)[3]) {
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const int4 lo = xv[t * 2], hi = xv[t * 2 + 1];
    int v = __dp4a(w[0], lo.x, 0);
    v = __dp4a(w[1], lo.y, v);
    v = __dp4a(w[2], lo.z, v);
    v = __dp4a(w[3], lo.w, v);
    v = __dp4a(w[4], hi.x, v);
    v = __dp4a(w[5], hi.y, v);
    v = __dp4a(w[6], hi.z, v);
    v = __dp4a(w[7], hi.w, v);
    S[t] = v - sm8[t];
  }
}

__host__ __device__ __forceinline__ size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

// Shared-memory layout of the staged x: fp32 copy, int8 term planes, term
// scales, term sums; the weight stages follow.
struct XLayout {
  size_t q, sc, sum, stages;
};
__host__ __device__ __forceinline__ XLayout x_layout(int kp) {
  const size_t nbk = (size_t)kp / 32;
  XLayout l;
  l.q = ((size_t)kp * 4 + 15) & ~(size_t)15;
  l.sc = l.q + ((3 * (size_t)kp + 15) & ~(size_t)15);
  l.sum = l.sc + ((12 * nbk + 15) & ~(size_t)15);
  l.stages = l.sum + ((12 * nbk + 15) & ~(size_t)15);
  return l;
}

// Warp roles: warps 0..kTmaWarps-1 consume row tiles, warp kTmaWarps (one
// lane) keeps the ring full.  Each stage has a "full" mbarrier (the copies'
// bytes) and an "empty" one (one arrival per consumer warp), so a consumer
// warp moves on to the next tile as soon as its own rows are done and the
// producer refills a stage as soon as the last warp has left it -- no
// CTA-wide barrier inside the tile loop.  When x has at most 32 blocks (K <=
// 1024, the lm_head) lane b keeps block b's three int8 terms in registers
// for the whole kernel.  The arithmetic (and its order) is per lane and per
// row exactly that of the per-tile loop, so results do not depend on the
// schedule.  Every wait is bounded; a wait that runs out sets the device
// error flag and the CTA's abort flag, every role leaves its loop, and the
// producer lets the copies it issued land before the CTA exits.
template <int QT, int RPW>
__global__ void __launch_bounds__(kTmaThreads) gemv_tma_kernel(const GemvArgs a, int nstage,
                                                              int skip_tile) {
  constexpr int TR = kTmaWarps * RPW;
  constexpr int NR = 4;  // float4 of RMSNorm weight prefetched per consumer thread
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ float red[kTmaWarps];
  __shared__ float bcast;
  __shared__ unsigned long long best_w[kTmaWarps];
  __shared__ int s_abort;

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const bool producer = wid == kTmaWarps;
  TmaGeo g;
  g.chunks = a.kp / Fmt<QT>::kElems;
  g.row_bytes = QT == DQMK_Q80 ? a.kp : a.kp / 2;
  g.nbk = a.kp / 32;
  g.n_tiles = (a.n_rows + TR - 1) / TR;
  g.my_tiles = (int)blockIdx.x < g.n_tiles
                   ? (g.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                   : 0;
  g.q_stage = (size_t)TR * g.row_bytes;
  g.stage_bytes = g.q_stage + align16((size_t)TR * g.nbk * 2);
  const XLayout xl = x_layout(a.kp);
  float* xf = reinterpret_cast<float*>(smem);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + xl.q);
  float* xsc = reinterpret_cast<float*>(smem + xl.sc);
  int* xsum = reinterpret_cast<int*>(smem + xl.sum);
  unsigned char* stages = smem + xl.stages;
  volatile int* abort = &s_abort;

  if (producer && lane == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTmaWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  __syncthreads();
  // producer bookkeeping (lane 0 of the producer warp): last tile issued into
  // each stage, -1 for none
  __shared__ int last_issued[kMaxStages];
  uint64_t policy = 0;
  if (producer && lane == 0) {
    for (int s = 0; s < kMaxStages; ++s) last_issued[s] = -1;
    policy = evict_first_policy();
    const int pre = min(nstage, g.my_tiles);
    for (int i = 0; i < pre; ++i)
      if (tma_issue<QT, RPW>(a, g, stages, full, i, i, policy, skip_tile)) last_issued[i] = i;
  }
  float4 nw[NR];
  const bool norm_pref = a.norm_w && (a.kp >> 2) <= NR * kTmaConsumers && ((a.k & 3) == 0) &&
                         ((reinterpret_cast<uintptr_t>(a.norm_w) & 15u) == 0);
  if (norm_pref && !producer) {
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      const int i4 = u * kTmaConsumers + tid;
      nw[u] = i4 < (a.k >> 2) ? __ldg(reinterpret_cast<const float4*>(a.norm_w) + i4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_trigger();
  pdl_wait();

  // x staging by the consumer threads; the producer warp only joins the
  // CTA barriers inside
  stage_x_linear<kTmaWarps, NR>(a, xf, nw, norm_pref, red, &bcast);
  if (!producer) quantize_x_terms<kTmaWarps, QT == DQMK_Q40>(xf, g.nbk, xq, xsc, xsum);
  __syncthreads();

  unsigned long long best = 0ull;
  if (producer) {
    if (lane == 0) {
      for (int i = nstage; i < g.my_tiles; ++i) {
        const int s = i % nstage;
        const uint32_t parity = (uint32_t)(i / nstage - 1) & 1u;
        if (!tc::bar_wait(&empty[s], parity, abort, &g_device_error, 32)) break;
        if (tma_issue<QT, RPW>(a, g, stages, full, i, s, policy, skip_tile)) last_issued[s] = i;
      }
    }
    __syncwarp();
  } else {
    int pos = 0;
    if (a.epi == kEpiQkv) pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
    const int4* xq4 = reinterpret_cast<const int4*>(xq);
    const bool xreg = g.nbk <= 32;
    int4 xv[6];  // [term][half] of block `lane` when xreg
    float sc[3];
    int sm8[3];
    if (xreg && lane < g.nbk) {
#pragma unroll
      for (int t = 0; t < 6; ++t) xv[t] = xq4[(size_t)t * g.nbk + lane];
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        sc[t] = xsc[t * g.nbk + lane];
        sm8[t] = QT == DQMK_Q40 ? 8 * xsum[t * g.nbk + lane] : 0;
      }
    }
    for (int i = 0; i < g.my_tiles; ++i) {
      const int s = i % nstage;
      const uint32_t phase = (uint32_t)(i / nstage) & 1u;
      const bool ok = tc::bar_wait(&full[s], phase, abort, &g_device_error);
      if (!__all_sync(0xffffffffu, ok)) {
        *abort = 1;
        break;
      }
      const int tile = blockIdx.x + i * gridDim.x;
      const int r0 = tile * TR;
      const int rows = min(TR, a.n_rows - r0);
      const bool d_smem = (((uint32_t)rows * g.nbk * 2) & 15u) == 0;
      const unsigned char* sq = stages + (size_t)s * g.stage_bytes;
      const uint16_t* sd = reinterpret_cast<const uint16_t*>(sq + g.q_stage);
      float acc[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) acc[r] = 0.0f;
      for (int b = lane; b < g.nbk; b += 32) {
        if (!xreg) {
#pragma unroll
          for (int t = 0; t < 6; ++t) xv[t] = xq4[(size_t)t * g.nbk + b];
#pragma unroll
          for (int t = 0; t < 3; ++t) {
            sc[t] = xsc[t * g.nbk + b];
            sm8[t] = QT == DQMK_Q40 ? 8 * xsum[t * g.nbk + b] : 0;
          }
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const int rl = wid * RPW + r;
          if (rl < rows) {
            int w[8];
            block_words<QT>(sq + (size_t)rl * g.row_bytes, b, w);
            const uint16_t dv =
                d_smem ? sd[rl * g.nbk + b] : __ldg(a.d + (size_t)(r0 + rl) * g.nbk + b);
            int S[3];
            block_term_sums(w, xv, sm8, S);
            float blk = 0.0f;
#pragma unroll
            for (int t = 0; t < 3; ++t) blk = __fmaf_rn(sc[t], (float)S[t], blk);
            acc[r] = __fmaf_rn(h2f(dv), blk, acc[r]);
          }
        }
      }
      // every shared-memory read of stage s has returned (its values fed the
      // sums above): hand the stage back
      __syncwarp();
      if (lane == 0) tc::bar_arrive(&empty[s]);
#pragma unroll
      for (int r = 0; r < RPW; ++r) acc[r] = warp_sum(acc[r]);
      epilogue<RPW, false>(a, tile * kTmaWarps + wid, lane, acc, pos, best);
    }
  }
  if (a.epi == kEpiLogits && !producer) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) best_w[wid] = best;
  }
  __syncthreads();
  if (*abort && producer && lane == 0) {
    // every role has stopped; let each copy still in flight land before the
    // CTA's shared memory goes away
    volatile int never = 0;
    for (int s = 0; s < nstage; ++s)
      if (last_issued[s] >= 0)
        tc::bar_wait(&full[s], (uint32_t)(last_issued[s] / nstage) & 1u, &never,
                     &g_device_error);
  }
  // Every CTA, aborted or not, folds in what it scored and takes its
  // completion ticket exactly once, so the last CTA's greedy step and the
  // ticket reset always happen (a step whose rows were all withheld finds no
  // key and keeps the greedy state).
  if (a.epi == kEpiLogits && tid == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kTmaWarps; ++w) b = best_w[w] > b ? best_w[w] : b;
    logits_finish(a, b, gridDim.x, &g_device_error);
  }
}

// ============================================================= ring GEMV
// Wide rows (K >= 2048: the Qwen2-7B-class projections).  Two things decide
// the bandwidth there: bytes in flight per SM and instructions per block.
//  * Row tiles of TR rows arrive by cp.async.bulk in a ring of up to six
//    shared-memory stages filled by one producer lane (full / empty
//    mbarriers, as in gemv_tma_kernel); the first stages are requested
//    before griddepcontrol.wait, and 100-170 KB stay in flight per SM.
//  * x stays in registers: consumer warp w owns the 32-block chunk
//    c = w % nch for the whole kernel (lane l: block 32c + l) and row set
//    w / nch of every tile.  Each lane loads its block of x once, applies the
//    fused RMSNorm (one CTA reduction of sum(x^2)), and splits it into the
//    three int8 terms of quantize_x_terms (same arithmetic, same terms).  A
//    (row, block) product is then the exact int32 dp4a sums of
//    block_term_sums scaled by the term scales: no per-row x traffic.
// Per tile each warp sums its rows over its lanes, the chunk partials meet
// in shared memory (double-buffered by tile parity, one named barrier of the
// consumer warps per tile) and are added in chunk order, and the group's
// epilogue runs on the totals.  Every wait is bounded (as in
// gemv_tma_kernel); a consumer that gives up marks the tile in a flag that the
// consumers read after that tile's barrier, so they all leave together.
constexpr int kRingMaxStages = 6;

// Barrier `id` (1..15) over the first n threads that reach it (n a multiple
// of 32): the consumer warps of a CTA without its producer warp.
__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

struct RingDims {
  int W;         // consumer warps
  int nch;       // 32-block chunks of a row
  int TR;        // rows per tile = row sets x RW
  int nstage;    // ring stages
  int rows_cap;  // rows a CTA holds partial sums for: TR x its most tiles
};

// Sums R per-lane values of R rows over the 32 lanes of a warp with 31
// fewer shuffles than R separate reductions: each halving stage trades half
// of the values with the partner lane, so lane l ends with the total of row
// (l >> (5 - log2 R)) & (R - 1) (every lane of that row alike).
template <int R>
__device__ __forceinline__ float transpose_sum(float (&v)[R], int lane) {
#pragma unroll
  for (int m = 16, n = R; n > 1; m >>= 1, n >>= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int k = 0; k < n / 2; ++k) {
      const float send = upper ? v[k] : v[k + n / 2];
      const float keep = upper ? v[k + n / 2] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
#pragma unroll
  for (int m = 32 / R / 2; m >= 1; m >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
  return v[0];
}
template <int R>
__host__ __device__ constexpr int log2i() {
  return R <= 1 ? 0 : 1 + log2i<R / 2>();
}

// The three int8 terms of one 32-value block of x, as quantize_x_terms
// computes them, by one thread: xv[2t], xv[2t+1] = values 0-15 / 16-31 of
// term t; sc[t] its scale; sm8[t] = 8 * sum of its values (Q4_0 offset).
__device__ __forceinline__ void block_x_terms(const float (&v)[32], int4 (&xv)[6], float (&sc)[3],
                                              int (&sm8)[3]) {
  float m = 0.0f;
#pragma unroll
  for (int e = 0; e < 32; ++e) m = fmaxf(m, fabsf(v[e]));
  float r[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) r[e] = v[e];
  float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 0.0f;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const float inv = s > 0.0f ? __frcp_rn(s) : 0.0f;
    uint32_t wd[8];
    int tsum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t packed = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int qq = __float2int_rn(__fmul_rn(r[4 * j + e], inv));
        qq = qq > 127 ? 127 : (qq < -127 ? -127 : qq);
        r[4 * j + e] = __fmaf_rn(-s, (float)qq, r[4 * j + e]);
        packed |= ((uint32_t)qq & 0xffu) << (8 * e);
        tsum += qq;
      }
      wd[j] = packed;
    }
    xv[2 * t] = make_int4((int)wd[0], (int)wd[1], (int)wd[2], (int)wd[3]);
    xv[2 * t + 1] = make_int4((int)wd[4], (int)wd[5], (int)wd[6], (int)wd[7]);
    sc[t] = s;
    sm8[t] = 8 * tsum;
    s = __fmul_rn(s, 1.0f / 254.0f);
  }
}

template <int QT, int RW, int WMAX, bool PEER>
__global__ void __launch_bounds__((WMAX + 1) * 32) gemv_ring_kernel(const GemvArgs a,
                                                                   const RingDims dm) {
  constexpr int EG = RW >= 8 ? 8 : 4;  // rows per epilogue group
  constexpr int BB = QT == DQMK_Q80 ? 32 : 16;  // quant bytes of a block
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kRingMaxStages];
  __shared__ __align__(8) uint64_t empty[kRingMaxStages];
  __shared__ int last_issued[kRingMaxStages];
  __shared__ float red_norm[WMAX];
  __shared__ unsigned long long best_w[WMAX];
  __shared__ int s_abort;
  __shared__ int c_abort[2];

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int W = dm.W, nch = dm.nch, TR = dm.TR, nstage = dm.nstage;
  const bool producer = wid == W;
  const int nbk = a.kp / 32;
  const size_t row_bytes = (size_t)nbk * BB;
  const size_t q_stage = (size_t)TR * row_bytes;
  const size_t stage_bytes = q_stage + align16((size_t)TR * nbk * 2);
  const int n_tiles = (a.n_rows + TR - 1) / TR;
  const int my_tiles =
      (int)blockIdx.x < n_tiles ? (n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                                : 0;
  float* red = reinterpret_cast<float*>(smem);  // [nch][rows_cap] partial row sums
  unsigned char* stages = smem + align16((size_t)nch * dm.rows_cap * 4);
  volatile int* abort = &s_abort;

  if (producer && lane == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
      last_issued[s] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    c_abort[0] = c_abort[1] = 0;
  }
  __syncthreads();

  // Issue the copies of local tile i into stage s (producer lane 0).
  auto issue = [&](int i, int s, uint64_t policy) {
    const int tile = blockIdx.x + i * gridDim.x;
    const int r0 = tile * TR;
    const int rows = min(TR, a.n_rows - r0);
    const uint32_t qbytes = (uint32_t)((size_t)rows * row_bytes);
    const uint32_t dbytes = (uint32_t)rows * nbk * 2;
    const uint32_t dbulk = (dbytes & 15u) == 0 ? dbytes : 0u;  // ragged: read in place
    unsigned char* st = stages + (size_t)s * stage_bytes;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(&full[s], qbytes + dbulk);
    bulk_g2s(st, a.qs + (size_t)r0 * row_bytes, qbytes, &full[s], policy);
    if (dbulk)
      bulk_g2s(st + q_stage, reinterpret_cast<const unsigned char*>(a.d) + (size_t)r0 * nbk * 2,
               dbulk, &full[s], policy);
    last_issued[s] = i;
  };

  uint64_t policy = 0;
  if (producer && lane == 0) {
    policy = evict_first_policy();
    const int pre = min(nstage, my_tiles);
    for (int i = 0; i < pre; ++i) issue(i, i, policy);
  }
  // consumer lane: its block of x, and of the RMSNorm weight (constant:
  // fetched before the dependency wait)
  const int c = producer ? 0 : wid % nch, rs = producer ? 0 : wid / nch;
  const int b = c * 32 + lane;
  const bool bok = !producer && b < nbk;
  float4 nw[8];
  if (a.norm_w && bok) {
#pragma unroll
    for (int u = 0; u < 8; ++u) nw[u] = __ldg(reinterpret_cast<const float4*>(a.norm_w) + b * 8 + u);
  }
  pdl_trigger();
  pdl_wait();

  unsigned long long best = 0ull;
  if (producer) {
    if (lane == 0) {
      for (int i = nstage; i < my_tiles; ++i) {
        const int s = i % nstage;
        const uint32_t parity = (uint32_t)(i / nstage - 1) & 1u;
        if (!tc::bar_wait(&empty[s], parity, abort, &g_device_error, 32)) break;
        issue(i, s, policy);
      }
    }
    __syncwarp();
  } else {
    // ---- x: this lane's block, RMS-normalised, as three int8 terms
    float v[32];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float4 t4 = bok ? __ldcg(reinterpret_cast<const float4*>(a.x) + b * 8 + u)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * u] = t4.x;
      v[4 * u + 1] = t4.y;
      v[4 * u + 2] = t4.z;
      v[4 * u + 3] = t4.w;
    }
    if (a.norm_w) {
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < 32; ++e) ss = __fadd_rn(ss, __fmul_rn(v[e], v[e]));
      ss = warp_sum(ss);
      if (rs == 0 && lane == 0) red_norm[c] = ss;
      named_bar(1, W * 32);
      float tot = 0.0f;
      for (int k = 0; k < nch; ++k) tot += red_norm[k];
      const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)a.k), a.eps)));
      if (bok) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          v[4 * u] = __fmul_rn(__fmul_rn(v[4 * u], scale), nw[u].x);
          v[4 * u + 1] = __fmul_rn(__fmul_rn(v[4 * u + 1], scale), nw[u].y);
          v[4 * u + 2] = __fmul_rn(__fmul_rn(v[4 * u + 2], scale), nw[u].z);
          v[4 * u + 3] = __fmul_rn(__fmul_rn(v[4 * u + 3], scale), nw[u].w);
        }
      }
    }
    int4 xv[6];
    float sc[3];
    int sm8[3];
    block_x_terms(v, xv, sc, sm8);
    if constexpr (QT == DQMK_Q80) sm8[0] = sm8[1] = sm8[2] = 0;
    int pos = 0;
    if (a.epi == kEpiQkv) pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;

    for (int i = 0; i < my_tiles; ++i) {
      const int s = i % nstage;
      const uint32_t phase = (uint32_t)(i / nstage) & 1u;
      bool ok = tc::bar_wait(&full[s], phase, abort, &g_device_error);
      ok = __all_sync(0xffffffffu, ok);
      const int tile = blockIdx.x + i * gridDim.x;
      const int r0 = tile * TR;
      const int rows = min(TR, a.n_rows - r0);
      float acc[RW];
#pragma unroll
      for (int j = 0; j < RW; ++j) acc[j] = 0.0f;
      if (ok && bok) {
        const unsigned char* sq = stages + (size_t)s * stage_bytes;
        const uint16_t* sd = reinterpret_cast<const uint16_t*>(sq + q_stage);
        const bool d_smem = (((uint32_t)rows * nbk * 2) & 15u) == 0;
#pragma unroll
        for (int j = 0; j < RW; ++j) {
          const int rl = rs * RW + j;
          if (rl < rows) {
            const unsigned char* p = sq + (size_t)rl * row_bytes + (size_t)b * BB;
            int w[8];
            if constexpr (QT == DQMK_Q80) {
              const uint4 w0 = *reinterpret_cast<const uint4*>(p);
              const uint4 w1 = *reinterpret_cast<const uint4*>(p + 16);
              w[0] = (int)w0.x; w[1] = (int)w0.y; w[2] = (int)w0.z; w[3] = (int)w0.w;
              w[4] = (int)w1.x; w[5] = (int)w1.y; w[6] = (int)w1.z; w[7] = (int)w1.w;
            } else {
              const uint4 pq = *reinterpret_cast<const uint4*>(p);
              const uint32_t pw[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                w[k] = (int)(pw[k] & 0x0f0f0f0fu);
                w[4 + k] = (int)((pw[k] >> 4) & 0x0f0f0f0fu);
              }
            }
            const uint16_t dv =
                d_smem ? sd[rl * nbk + b] : __ldg(a.d + (size_t)(r0 + rl) * nbk + b);
            // the three terms' sums as six independent dp4a chains of four
            // (values 0-15 and 16-31 apart), the integer results of
            // block_term_sums
            int lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
#pragma unroll
              for (int k = 0; k < 3; ++k) {
                const int4 xl = xv[2 * k], xh = xv[2 * k + 1];
                lo[k] = __dp4a(w[q], q == 0 ? xl.x : q == 1 ? xl.y : q == 2 ? xl.z : xl.w, lo[k]);
                hi[k] = __dp4a(w[4 + q], q == 0 ? xh.x : q == 1 ? xh.y : q == 2 ? xh.z : xh.w,
                               hi[k]);
              }
            }
            float blk = 0.0f;
#pragma unroll
            for (int k = 0; k < 3; ++k) blk = __fmaf_rn(sc[k], (float)(lo[k] + hi[k] - sm8[k]), blk);
            acc[j] = __fmaf_rn(h2f(dv), blk, acc[j]);
          }
        }
      }
      // every shared-memory read of stage s has returned: hand it back
      __syncwarp();
      if (!ok) {
        if (lane == 0) c_abort[0] = 1;
        break;
      }
      if (lane == 0) tc::bar_arrive(&empty[s]);
      // this warp's chunk of the tile's rows: lane l ends with row j(l)
      const float tot = transpose_sum<RW>(acc, lane);
      if ((lane & (32 / RW - 1)) == 0) {
        const int j = (lane >> (5 - log2i<RW>())) & (RW - 1);
        red[(size_t)c * dm.rows_cap + i * TR + rs * RW + j] = tot;
      }
    }
    // ---- every partial is in: chunks added in order, epilogues by groups
    named_bar(1, W * 32);
    if (!c_abort[0]) {
      for (int gg = wid; gg < my_tiles * TR / EG; gg += W) {
        const int i = gg * EG / TR;
        const int row0 = (blockIdx.x + i * gridDim.x) * TR + (gg * EG) % TR;
        float e8[EG];
#pragma unroll
        for (int r = 0; r < EG; ++r) {
          float t = 0.0f;
          for (int k = 0; k < nch; ++k) t += red[(size_t)k * dm.rows_cap + gg * EG + r];
          e8[r] = t;
        }
        epilogue<EG, PEER>(a, row0 / EG, lane, e8, pos, best);
      }
    }
  }
  if (a.epi == kEpiLogits && !producer) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) best_w[wid] = best;
  }
  __syncthreads();
  if (*abort && producer && lane == 0) {
    // every role has stopped; let each copy still in flight land before the
    // CTA's shared memory goes away
    volatile int never = 0;
    for (int s = 0; s < nstage; ++s)
      if (last_issued[s] >= 0)
        tc::bar_wait(&full[s], (uint32_t)(last_issued[s] / nstage) & 1u, &never,
                     &g_device_error);
  }
  if (a.epi == kEpiLogits && tid == 0) {
    unsigned long long bb = 0ull;
    for (int w = 0; w < W; ++w) bb = best_w[w] > bb ? best_w[w] : bb;
    logits_finish(a, bb, gridDim.x, &g_device_error);
  }
}

// ====================================================== tensor-core GEMV
// Tall weights with rows of 2048-4096 values (the Qwen2-7B gate/up and
// lm_head shapes).  The per-block integer dot products that cost the other
// forms ~90-160 instructions per (row, 32-value block) run on the tensor
// cores: tcgen05.mma kind::i8 with A = 128 weight rows x one block (Q8_0:
// the bytes as TMA brought them; Q4_0: nibbles unpacked to bytes by the row
// threads into tensor memory), B = the three int8 terms of x's block
// (quantize_x_terms' arithmetic) as N = 16 columns (only 0-2 are read), and
// one D slot of 16 s32 columns per block in tensor memory.  One thread per
// weight row then reads its three sums per block (tcgen05.ld) and applies
// the term scales and the block scale -- the exact int32 sums of
// block_term_sums, combined in the same order per block, and added over the
// blocks in order by one thread per row.
//
// Warp roles: 0 TMA producer (one lane), 1 MMA issuer (one elected lane;
// also allocates tensor memory), 2-5 row warps (row 32 * (warp % 4) + lane
// of the tile: the tensor-memory lane quarter the warp may access).  Raw
// tiles of 128 rows x 8 blocks (quants, 128-byte swizzle, and their scales)
// stream through kTcStages shared-memory stages filled before the
// dependency wait; the row threads build x's terms for all of K once per
// CTA.  Per chunk of 8 blocks the row threads unpack (Q4_0) and read the
// scales, the MMA warp issues 8 MMAs into one of two D buffers, and the row
// threads fold the previous chunk's D.  Every wait is bounded (an abort flag
// unwinds every role; the producer lets its copies land before exit).
constexpr int kTcRows = 128;                        // M: weight rows per tile
constexpr int kTcKB = 8;                            // 32-value blocks per chunk
constexpr int kTcStages = 4;
constexpr int kTcRowWarps = 4;
constexpr int kTcThreads = (2 + kTcRowWarps) * 32;
constexpr uint32_t kTcDCols = kTcKB * 16;           // D columns of one chunk
constexpr uint32_t kTcACols = kTcKB * 8;            // A columns of one chunk (Q4_0)
constexpr uint32_t kTcTmemCols = 512;               // 2 x (128 + 64) used

template <int QT>
struct TcLayout {
  static constexpr int QB = QT == DQMK_Q80 ? 32 : 16;          // quant bytes per block
  static constexpr size_t kQuant = (size_t)kTcRows * kTcKB * QB;  // 32 / 16 KB
  static constexpr size_t kScale = (size_t)kTcRows * kTcKB * 2;   // 2 KB
  static constexpr size_t kStage = kQuant + kScale;
  // B operand: one 1 KB 128-byte-swizzled atom (8 rows x 128 K bytes, only
  // rows 0-2 meaningful) per 4 blocks, plus one more for the last atom's
  // rows 8-15; per block the three term scales and 8 x the three term sums
  __host__ __device__ static size_t b_bytes(int nbk) { return ((size_t)nbk / 4 + 1) * 1024; }
  __host__ __device__ static size_t c_bytes(int nbk) { return (size_t)nbk * 32; }
  static size_t smem(int nbk) {
    return 1024 + kTcStages * kStage + b_bytes(nbk) + c_bytes(nbk);
  }
};

// x (k = kp floats, 16-byte aligned), RMS-normalised when norm_w is set,
// as the three int8 terms of each 32-value block written into the B atoms
// (term t = row t; block b at K bytes 32 (b % 4).. of atom b / 4, 16-byte
// chunks XOR-swizzled by the row as TMA's 128-byte swizzle lays them out),
// and per block the term scales {s0, s1, s2} and, for Q4_0 (nibbles offset
// by 8), {8 sum(q0), 8 sum(q1), 8 sum(q2)}.  The 128 row threads; eight
// threads per block, four values each (quantize_x_terms' arithmetic).
template <int QT>
__device__ __forceinline__ void tc_build_x(const GemvArgs& a, int t, int nbk, unsigned char* batoms,
                                           float4* scales, int4* sums8, float* red, float* bcast,
                                           const float4 (&nw)[8]) {
  constexpr int NT = kTcRowWarps * 32;
  const int lane = t & 31, w = t >> 5;
  const float4* x4 = reinterpret_cast<const float4*>(a.x);
  const int nf4 = a.kp >> 2;
  float4 v[8];  // float4 i4 = t + u * NT (8 * NT >= kp / 4: kp <= 4096)
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i4 = t + u * NT;
    v[u] = i4 < nf4 ? __ldcg(x4 + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
    ss = __fadd_rn(ss, __fmul_rn(v[u].x, v[u].x));
    ss = __fadd_rn(ss, __fmul_rn(v[u].y, v[u].y));
    ss = __fadd_rn(ss, __fmul_rn(v[u].z, v[u].z));
    ss = __fadd_rn(ss, __fmul_rn(v[u].w, v[u].w));
  }
  if (a.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) red[w] = ss;
    named_bar(1, NT);
    if (t == 0) {
      float tot = 0.0f;
      for (int i = 0; i < kTcRowWarps; ++i) tot += red[i];
      *bcast = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)a.k), a.eps)));
    }
    named_bar(1, NT);
    const float scale = *bcast;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      v[u].x = __fmul_rn(__fmul_rn(v[u].x, scale), nw[u].x);
      v[u].y = __fmul_rn(__fmul_rn(v[u].y, scale), nw[u].y);
      v[u].z = __fmul_rn(__fmul_rn(v[u].z, scale), nw[u].z);
      v[u].w = __fmul_rn(__fmul_rn(v[u].w, scale), nw[u].w);
    }
  }
  const int sub = t & 7;  // which 4 values of the block
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i4 = t + u * NT;
    const int b = i4 >> 3;
    const bool valid = i4 < nf4;  // uniform per group of 8 lanes
    float m = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    float r[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
    float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 0.0f;
    float sc[3];
    int s8[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float inv = s > 0.0f ? __frcp_rn(s) : 0.0f;
      uint32_t packed = 0;
      int tsum = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int qq = __float2int_rn(__fmul_rn(r[e], inv));
        qq = qq > 127 ? 127 : (qq < -127 ? -127 : qq);
        r[e] = __fmaf_rn(-s, (float)qq, r[e]);
        packed |= ((uint32_t)qq & 0xffu) << (8 * e);
        tsum += qq;
      }
      tsum += __shfl_xor_sync(0xffffffffu, tsum, 1);
      tsum += __shfl_xor_sync(0xffffffffu, tsum, 2);
      tsum += __shfl_xor_sync(0xffffffffu, tsum, 4);
      if (valid) {
        // row k, K byte 32 (b % 4) + 4 sub of atom b / 4, 128-byte swizzle
        const int kb = 32 * (b & 3) + 4 * sub;
        unsigned char* atom = batoms + (size_t)(b >> 2) * 1024;
        *reinterpret_cast<uint32_t*>(atom + k * 128 + (((kb >> 4) ^ k) << 4) + (kb & 15)) = packed;
      }
      sc[k] = s;
      s8[k] = QT == DQMK_Q40 ? 8 * tsum : 0;
      s = __fmul_rn(s, 1.0f / 254.0f);
    }
    if (valid && sub == 0) {
      scales[b] = make_float4(sc[0], sc[1], sc[2], 0.0f);
      sums8[b] = make_int4(s8[0], s8[1], s8[2], 0);
    }
  }
}

template <int QT>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_d, const GemvArgs a) {
  using L = TcLayout<QT>;
  extern __shared__ unsigned char smem_tc[];
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages];
  __shared__ __align__(8) uint64_t a_full[2], a_empty[2], d_full[2], d_empty[2];
  __shared__ __align__(8) uint64_t b_ready, mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_abort;
  __shared__ int last_issued[kTcStages];
  __shared__ float red[kTcRowWarps];
  __shared__ float bcast;
  __shared__ unsigned long long best_w[kTcRowWarps];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbk = a.kp / 32;
  const int nch = nbk / kTcKB;  // chunks per tile
  const int n_tiles = (a.n_rows + kTcRows - 1) / kTcRows;
  const int my_tiles = (int)blockIdx.x < n_tiles
                           ? (n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                           : 0;
  const int total = my_tiles * nch;  // chunks of this CTA
  unsigned char* stages = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_tc) + 1023) & ~(uintptr_t)1023);
  unsigned char* batoms = stages + (size_t)kTcStages * L::kStage;
  float4* scales = reinterpret_cast<float4*>(batoms + L::b_bytes(nbk));
  int4* sums8 = reinterpret_cast<int4*>(scales + nbk);
  volatile int* abort = &s_abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      tc::bar_init(&full[s], 1);
      tc::bar_init(&empty[s], QT == DQMK_Q80 ? kTcRowWarps + 1 : kTcRowWarps);
      last_issued[s] = -1;
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&a_full[b], kTcRowWarps);
      tc::bar_init(&a_empty[b], 1);
      tc::bar_init(&d_full[b], 1);
      tc::bar_init(&d_empty[b], kTcRowWarps);
    }
    tc::bar_init(&b_ready, kTcRowWarps);
    tc::bar_init(&mma_done, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::tma_prefetch_desc(&map_q);
    tc::tma_prefetch_desc(&map_d);
  }
  if (warp == 1) tc::tmem_alloc(&tmem_slot, kTcTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_slot;

  // weights are read once: evict them from L2 first
  uint64_t policy = 0;
  if (warp == 0 && lane == 0) policy = evict_first_policy();
  // chunk g of this CTA into stage s (producer lane)
  auto issue = [&](int g, int s) {
    const int tile = (int)blockIdx.x + (g / nch) * (int)gridDim.x, c = g % nch;
    unsigned char* st = stages + (size_t)s * L::kStage;
    tc::bar_expect_tx(&full[s], (uint32_t)L::kStage);
    if constexpr (QT == DQMK_Q80) {
      tc::tma_load_2d_hint(st, &map_q, c * 256, tile * kTcRows, &full[s], policy);
      tc::tma_load_2d_hint(st + 16384, &map_q, c * 256 + 128, tile * kTcRows, &full[s], policy);
    } else {
      tc::tma_load_2d_hint(st, &map_q, c * 128, tile * kTcRows, &full[s], policy);
    }
    tc::tma_load_2d_hint(st + L::kQuant, &map_d, c * kTcKB, tile * kTcRows, &full[s], policy);
    last_issued[s] = g;
  };
  // before the dependency: the first stages of weights (constant), the
  // row threads' RMSNorm weights
  if (warp == 0 && lane == 0)
    for (int g = 0; g < total && g < kTcStages; ++g) issue(g, g);
  const int t = 32 * (warp & 3) + lane;  // row of the tile (row warps)
  float4 nw[8];
  if (warp >= 2) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i4 = t + u * kTcRowWarps * 32;
      nw[u] = a.norm_w && i4 < (a.kp >> 2)
                  ? __ldg(reinterpret_cast<const float4*>(a.norm_w) + i4)
                  : make_float4(1.f, 1.f, 1.f, 1.f);
    }
  }
  pdl_trigger();
  pdl_wait();

  unsigned long long best = 0ull;
  if (warp == 0) {  // ----------------------------------------- TMA producer
    if (lane == 0) {
      for (int g = kTcStages; g < total; ++g) {
        const int s = g % kTcStages;
        if (!tc::bar_wait(&empty[s], (uint32_t)((g / kTcStages - 1) & 1), abort, &g_device_error,
                          32))
          break;
        issue(g, s);
      }
    }
    __syncwarp();
  } else if (warp == 1) {  // ------------------------------------ MMA issue
    const uint32_t idesc = tc::idesc_i8(kTcRows, 16, QT == DQMK_Q80 ? 1 : 0, 1);
    bool ok = __all_sync(0xffffffffu, tc::bar_wait(&b_ready, 0u, abort, &g_device_error));
    for (int g = 0; g < total && ok; ++g) {
      const int s = g % kTcStages, buf = g & 1;
      bool w = QT == DQMK_Q80
                   ? tc::bar_wait(&full[s], (uint32_t)((g / kTcStages) & 1), abort, &g_device_error)
                   : tc::bar_wait(&a_full[buf], (uint32_t)((g >> 1) & 1), abort, &g_device_error);
      if (w && g >= 2)
        w = tc::bar_wait(&d_empty[buf], (uint32_t)(((g >> 1) - 1) & 1), abort, &g_device_error);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc::tc_fence_after();
      if (tc::elect_one()) {
        const unsigned char* st = stages + (size_t)s * L::kStage;
#pragma unroll
        for (int j = 0; j < kTcKB; ++j) {
          const int b = (g % nch) * kTcKB + j;  // block of the row
          const uint64_t bdesc = tc::smem_desc(tc::su32(batoms + (size_t)(b >> 2) * 1024)) +
                                 2u * (uint32_t)(b & 3);
          const uint32_t d = tmem + (uint32_t)buf * kTcDCols + 16u * (uint32_t)j;
          if constexpr (QT == DQMK_Q80) {
            const uint64_t adesc = tc::smem_desc(tc::su32(st + (j >> 2) * 16384)) +
                                   2u * (uint32_t)(j & 3);
            tc::mma_i8(d, adesc, bdesc, idesc, 0u);
          } else {
            tc::mma_i8_ts(d, tmem + 2u * kTcDCols + (uint32_t)buf * kTcACols + 8u * (uint32_t)j,
                          bdesc, idesc, 0u);
          }
        }
        tc::mma_commit(&d_full[buf]);
        tc::mma_commit(QT == DQMK_Q80 ? &empty[s] : &a_empty[buf]);
      }
      __syncwarp();
    }
    // every MMA issued has finished before tensor memory is freed
    if (tc::elect_one()) tc::mma_commit(&mma_done);
    __syncwarp();
    volatile int never = 0;
    tc::bar_wait(&mma_done, 0u, &never, &g_device_error);
  } else {  // ------------------------------------------------- row warps
    tc_build_x<QT>(a, t, nbk, batoms, scales, sums8, red, &bcast, nw);
    tc::fence_proxy_async_smem();  // the B atoms are read by the tensor core
    named_bar(1, kTcRowWarps * 32);
    if (lane == 0) tc::bar_arrive(&b_ready);
    int pos = 0;
    if (a.epi == kEpiQkv) pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    uint4 dsw[2];  // the 8 block scales (fp16) of the two chunks in flight
    float acc = 0.0f;
    for (int g = 0; g <= total; ++g) {
      if (g < total) {  // ---- chunk g: scales, and the Q4_0 expansion
        const int s = g % kTcStages, buf = g & 1;
        // waits are voted: the tcgen05 loads and stores below are warp-wide
        if (!__all_sync(0xffffffffu, tc::bar_wait(&full[s], (uint32_t)((g / kTcStages) & 1),
                                                  abort, &g_device_error)))
          break;
        const unsigned char* st = stages + (size_t)s * L::kStage;
        dsw[buf] = *reinterpret_cast<const uint4*>(st + L::kQuant + (size_t)t * 16);
        if constexpr (QT == DQMK_Q40) {
          uint32_t r[64];
#pragma unroll
          for (int c = 0; c < kTcKB; ++c) {
            const uint4 p = *reinterpret_cast<const uint4*>(st + (size_t)t * 128 +
                                                            (((c ^ (t & 7))) << 4));
            const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              r[8 * c + k] = pw[k] & 0x0f0f0f0fu;
              r[8 * c + 4 + k] = (pw[k] >> 4) & 0x0f0f0f0fu;
            }
          }
          if (g >= 2 && !__all_sync(0xffffffffu,
                                    tc::bar_wait(&a_empty[buf], (uint32_t)(((g >> 1) - 1) & 1),
                                                 abort, &g_device_error)))
            break;
          tc::tc_fence_after();
          const uint32_t acol = tmem + lane_base + 2u * kTcDCols + (uint32_t)buf * kTcACols;
          uint32_t (&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
          uint32_t (&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
          tc::tmem_st32(acol, r0);
          tc::tmem_st32(acol + 32, r1);
          tc::tmem_wait_st();
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::bar_arrive(&a_full[buf]);
        }
        // this thread's reads of stage s are done before the next TMA write
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::bar_arrive(&empty[s]);
      }
      if (g >= 1) {  // ---- chunk g - 1: fold its D into the row's sum
        const int pg = g - 1, pb = pg & 1;
        if (!__all_sync(0xffffffffu, tc::bar_wait(&d_full[pb], (uint32_t)((pg >> 1) & 1), abort,
                                                  &g_device_error)))
          break;
        tc::tc_fence_after();
        uint32_t dv[kTcKB][4];
#pragma unroll
        for (int j = 0; j < kTcKB; ++j)
          tc::tmem_ld4(tmem + lane_base + (uint32_t)pb * kTcDCols + 16u * (uint32_t)j, dv[j]);
        tc::tmem_wait_ld();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::bar_arrive(&d_empty[pb]);
        const int cg = pg % nch;
        const uint32_t hw[4] = {dsw[pb].x, dsw[pb].y, dsw[pb].z, dsw[pb].w};
#pragma unroll
        for (int j = 0; j < kTcKB; ++j) {
          const int b = cg * kTcKB + j;
          const float4 sc = scales[b];
          const int4 s8 = sums8[b];
          float blk = __fmul_rn(sc.x, (float)((int)dv[j][0] - s8.x));
          blk = __fmaf_rn(sc.y, (float)((int)dv[j][1] - s8.y), blk);
          blk = __fmaf_rn(sc.z, (float)((int)dv[j][2] - s8.z), blk);
          const uint16_t h = (uint16_t)((hw[j >> 1] >> (16 * (j & 1))) & 0xffffu);
          acc = __fmaf_rn(h2f(h), blk, acc);
        }
        if (cg == nch - 1) {  // the tile's rows are complete
          const int row = ((int)blockIdx.x + (pg / nch) * (int)gridDim.x) * kTcRows + t;
          const float other = __shfl_xor_sync(0xffffffffu, acc, 1);
          const float pr[2] = {(lane & 1) ? other : acc, (lane & 1) ? acc : other};
          epilogue<2, false>(a, row >> 1, lane & 1, pr, pos, best);
          acc = 0.0f;
        }
      }
    }
    if (a.epi == kEpiLogits) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      if (lane == 0) best_w[warp - 2] = best;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (*abort && warp == 0 && lane == 0) {
    // every role has stopped; let each copy still in flight land before the
    // CTA's shared memory goes away
    volatile int never = 0;
    for (int s = 0; s < kTcStages; ++s)
      if (last_issued[s] >= 0)
        tc::bar_wait(&full[s], (uint32_t)((last_issued[s] / kTcStages) & 1), &never,
                     &g_device_error);
  }
  if (a.epi == kEpiLogits && threadIdx.x == 64) {
    unsigned long long bb = 0ull;
    for (int w = 0; w < kTcRowWarps; ++w) bb = best_w[w] > bb ? best_w[w] : bb;
    logits_finish(a, bb, gridDim.x, &g_device_error);
  }
  if (warp == 1) tc::tmem_free(tmem, kTcTmemCols);
}

// Test hook behind dqmk_lm_head_block_sums: x (k floats) split into the three
// int8 terms by quantize_x_terms, then every (row, block) of a packed weight
// summed against them with block_term_sums -- the integer arithmetic of
// gemv_tma_kernel, exposed so it can be checked exactly.  One CTA of
// kTmaConsumers threads; x staged in shared memory (zero past k).
template <int QT>
__global__ void __launch_bounds__(kTmaConsumers) block_sums_kernel(
    const float* __restrict__ x, int k, int kp, const uint8_t* __restrict__ qs, int n_rows,
    int8_t* __restrict__ q_terms, float* __restrict__ scales, int* __restrict__ sums) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int nbk = kp / 32;
  float* xf = reinterpret_cast<float*>(smem);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + (size_t)kp * 4);
  float* xsc = reinterpret_cast<float*>(smem + (size_t)kp * 4 + (size_t)3 * kp);
  int* xsum = reinterpret_cast<int*>(xsc + 3 * nbk);
  for (int e = threadIdx.x; e < kp; e += blockDim.x) xf[e] = e < k ? x[e] : 0.0f;
  __syncthreads();
  quantize_x_terms<kTmaWarps, QT == DQMK_Q40>(xf, nbk, xq, xsc, xsum);
  __syncthreads();
  // terms out as [term][block][32 values]: plane [t][half][block][16 bytes]
  for (int i = threadIdx.x; i < 3 * nbk * 32; i += blockDim.x) {
    const int t = i / (nbk * 32), b = (i / 32) % nbk, j = i % 32;
    q_terms[i] = xq[((size_t)(t * 2 + j / 16) * nbk + b) * 16 + (j % 16)];
  }
  for (int i = threadIdx.x; i < 3 * nbk; i += blockDim.x) scales[i] = xsc[i];
  const int4* xq4 = reinterpret_cast<const int4*>(xq);
  const size_t row_bytes = QT == DQMK_Q80 ? (size_t)kp : (size_t)kp / 2;
  for (int i = threadIdx.x; i < n_rows * nbk; i += blockDim.x) {
    const int row = i / nbk, b = i % nbk;
    int4 xv[6];
    int sm8[3];
#pragma unroll
    for (int t = 0; t < 6; ++t) xv[t] = xq4[(size_t)t * nbk + b];
#pragma unroll
    for (int t = 0; t < 3; ++t) sm8[t] = QT == DQMK_Q40 ? 8 * xsum[t * nbk + b] : 0;
    int w[8];
    block_words<QT>(qs + (size_t)row * row_bytes, b, w);
    int S[3];
    block_term_sums(w, xv, sm8, S);
#pragma unroll
    for (int t = 0; t < 3; ++t) sums[((size_t)row * 3 + t) * nbk + b] = S[t];
  }
}

struct TmaPlan {
  int rpw, stages, grid;
  size_t smem;
};

size_t tma_stage_bytes(int qtype, int rpw, int kp) {
  const size_t tr = (size_t)kTmaWarps * rpw;
  const size_t row = qtype == DQMK_Q80 ? (size_t)kp : (size_t)kp / 2;
  return tr * row + ((tr * (kp / 32) * 2 + 15) & ~(size_t)15);
}

// Rows per warp by shape; stages so that (when the grid fits on the GPU at
// once) every tile of a CTA is requested before the dependency wait; a
// persistent ring for the very tall lm_head.
TmaPlan tma_plan(const GemvArgs& a) {
  TmaPlan p;
  const bool paired = a.epi == kEpiSwiGlu || a.epi == kEpiQkv;
  if (paired || a.n_rows >= 4096) p.rpw = 2;
  else p.rpw = 1;
  const int tr = kTmaWarps * p.rpw;
  const int n_tiles = (a.n_rows + tr - 1) / tr;
  const size_t stage = tma_stage_bytes(a.qtype, p.rpw, a.kp);
  const size_t xbytes = x_layout(a.kp).stages;
  const size_t budget = 200 * 1024;
  const int sms = sm_count();
  auto per_sm = [&](int stages) {
    const size_t sm_bytes = xbytes + stages * stage + 1024;
    int c = (int)(220 * 1024 / sm_bytes);
    return c < 8 ? c : 8;
  };
  p.stages = 1;
  p.grid = n_tiles;
  while (p.stages < kMaxStages && p.grid > sms * per_sm(p.stages) &&
         xbytes + (p.stages + 1) * stage <= budget) {
    ++p.stages;
    p.grid = (n_tiles + p.stages - 1) / p.stages;
  }
  const int cap = sms * (per_sm(p.stages) > 0 ? per_sm(p.stages) : 1);
  if (p.grid > cap) p.grid = cap;
  if (p.grid < 1) p.grid = 1;
  p.smem = xbytes + p.stages * stage;
  return p;
}

template <int QT, int RPW>
cudaError_t tma_prepare() {
  static DeviceOnce once;
  return once.run([] {
    return cudaFuncSetAttribute(gemv_tma_kernel<QT, RPW>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024);
  });
}

template <int QT, int RPW>
cudaError_t tma_launch(const GemvArgs& a, const TmaPlan& p, cudaStream_t stream, bool pdl,
                       int skip_tile) {
  cudaError_t e = tma_prepare<QT, RPW>();
  if (e != cudaSuccess) return e;
  // the plan counts CTAs per SM by shared memory; registers may allow fewer,
  // and a grid beyond what is resident at once would run as a second wave
  // (the figure is cached per device and shared-memory size)
  static std::mutex mu;
  static size_t occ_smem[kMaxDevices];
  static int occ[kMaxDevices];
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int resident = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (occ_smem[dev] != p.smem) {
      int n = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_tma_kernel<QT, RPW>,
                                                        kTmaThreads, p.smem);
      if (e != cudaSuccess) return e;
      occ[dev] = n > 0 ? n : 1;
      occ_smem[dev] = p.smem;
    }
    resident = occ[dev];
  }
  const int grid = std::min(p.grid, sm_count() * resident);
  return launch(gemv_tma_kernel<QT, RPW>, dim3(grid), dim3(kTmaThreads), p.smem, stream, pdl, a,
                p.stages, skip_tile);
}

#define DQMK_TMA_VARIANTS(X) \
  X(DQMK_Q80, 1) X(DQMK_Q80, 2) X(DQMK_Q80, 4) X(DQMK_Q40, 1) X(DQMK_Q40, 2) X(DQMK_Q40, 4)

cudaError_t tma_dispatch(const GemvArgs& a, cudaStream_t stream, bool pdl, int skip_tile) {
  const TmaPlan p = tma_plan(a);
#define DQMK_TMA_CASE(QT, RPW) \
  if (a.qtype == QT && p.rpw == RPW) return tma_launch<QT, RPW>(a, p, stream, pdl, skip_tile);
  DQMK_TMA_VARIANTS(DQMK_TMA_CASE)
#undef DQMK_TMA_CASE
  return cudaErrorInvalidValue;
}

// The TMA form streams the very tall Q8_0 weights (lm_head): there bandwidth
// decides, and the shared-memory ring keeps more bytes in flight than
// registers can.  For Q4_0 the register form with 4 rows per warp measured
// faster at every tall shape (the consumer work per byte doubles), and the
// per-layer projections are latency-bound links of the decode chain where the
// register form, whose weights are already in registers when the dependency
// resolves, finishes sooner.
bool tma_eligible(const GemvArgs& a) {
  return a.qtype == DQMK_Q80 && a.kp <= 8192 && a.n_rows >= 32768 && a.epi != kEpiPeer;
}

// ------------------------------------------------ tensor-core GEMV launches
template <int QT>
cudaError_t tc_prepare() {
  static DeviceOnce once;
  return once.run([] {
    return cudaFuncSetAttribute(gemv_tc_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
  });
}

// Tall Q8_0 weights (16384 rows or more) with rows of 2048-4096 values in
// whole 256-value chunks, x and the RMSNorm weight 16-byte aligned; not the
// peer-memory epilogue.  Measured on a B200 at the Qwen2-7B shapes, weights
// HBM-cold: Q8_0 gate/up 37888 x 3584 0.74 of HBM (TMA form 0.66), and the
// Qwen2-7B Q8_0 batch-1 decode step 2.60 vs 2.69 ms.  Q4_0 stays with the
// register / ring forms: the kernel is faster there alone (gate/up 0.42 vs
// 0.37) but made the Q4_0 decode step slower (3.2-3.4 vs 2.62 ms), with the
// down projection on the register or on the ring form alike, under early or
// late dependent-launch triggers, and with evict-first weight copies; the
// cause is not found.
bool tc_eligible(const GemvArgs& a) {
  if (a.epi == kEpiPeer || a.qtype != DQMK_Q80) return false;
  if (a.n_rows < 16384 || a.k != a.kp || a.kp % 256 != 0 || a.kp < 2048 || a.kp > 4096)
    return false;
  if (a.qtype == DQMK_Q80 ? TcLayout<DQMK_Q80>::smem(a.kp / 32) > 200 * 1024
                          : TcLayout<DQMK_Q40>::smem(a.kp / 32) > 200 * 1024)
    return false;
  return ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.norm_w) |
           reinterpret_cast<uintptr_t>(a.qs) | reinterpret_cast<uintptr_t>(a.d)) & 15u) == 0;
}

template <int QT>
cudaError_t tc_launch(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  cudaError_t e = tc_prepare<QT>();
  if (e != cudaSuccess) return e;
  const int nbk = a.kp / 32;
  const uint64_t row_bytes = QT == DQMK_Q80 ? (uint64_t)a.kp : (uint64_t)a.kp / 2;
  CUtensorMap mq, md;
  if (make_map_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.qs, row_bytes, (uint64_t)a.n_rows,
                  row_bytes, 128, kTcRows, CU_TENSOR_MAP_SWIZZLE_128B) != DQMK_OK ||
      make_map_2d(&md, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.d, (uint64_t)nbk, (uint64_t)a.n_rows,
                  (uint64_t)nbk * 2, kTcKB, kTcRows, CU_TENSOR_MAP_SWIZZLE_NONE) != DQMK_OK)
    return cudaErrorInvalidValue;
  const int n_tiles = (a.n_rows + kTcRows - 1) / kTcRows;
  const int grid = std::min(n_tiles, sm_count());
  return launch(gemv_tc_kernel<QT>, dim3(grid), dim3(kTcThreads), TcLayout<QT>::smem(nbk), stream,
                pdl, mq, md, a);
}

cudaError_t tc_dispatch(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  return a.qtype == DQMK_Q80 ? tc_launch<DQMK_Q80>(a, stream, pdl)
                             : tc_launch<DQMK_Q40>(a, stream, pdl);
}

// ------------------------------------------------------ ring GEMV launches
// Every instantiation: X(quant type, rows per warp and tile, max consumer warps).
#define DQMK_RING_VARIANTS(X) \
  X(DQMK_Q40, 8, 16) X(DQMK_Q40, 8, 24) X(DQMK_Q80, 4, 16) X(DQMK_Q80, 4, 24)

struct RingPlan {
  RingDims dm{};
  int rw = 0, wmax = 0;
  size_t smem = 0;
  bool ok = false;
};

// Consumer warps: one per 32-block chunk, times as many row sets as fit in
// the target warp count, or one per chunk up to 24 chunks.  Stages:
// as many as fit 200 KB of shared memory, up to six.
RingPlan ring_plan(const GemvArgs& a, int rw, int wt) {
  RingPlan p;
  const int nbk = a.kp / 32, nch = (nbk + 31) / 32;
  const int rs = nch <= wt ? wt / nch : 1;
  const int W = rs * nch;
  if (W > 24) return p;
  const size_t row_bytes = (size_t)nbk * (a.qtype == DQMK_Q80 ? 32 : 16);
  const int TR = rs * rw;
  const size_t stage = (size_t)TR * row_bytes + align16((size_t)TR * nbk * 2);
  // partial row sums of a CTA's rows: at most ceil(tiles / grid) tiles each,
  // the grid being at least min(tiles, SM count)
  const int n_tiles = (a.n_rows + TR - 1) / TR;
  const int min_grid = std::min(n_tiles, sm_count());
  const int rows_cap = (n_tiles + min_grid - 1) / min_grid * TR;
  const size_t red = align16((size_t)nch * rows_cap * 4);
  const size_t budget = 200 * 1024;
  if (red + 2 * stage > budget) return p;
  int ns = (int)((budget - red) / stage);
  if (ns > kRingMaxStages) ns = kRingMaxStages;
  p.dm = RingDims{W, nch, TR, ns, rows_cap};
  p.rw = rw;
  p.wmax = W <= 16 ? 16 : 24;
  p.smem = red + (size_t)ns * stage;
  p.ok = true;
  return p;
}

// Rows per warp and tile, and consumer warps aimed at (16: enough warps per
// SM to hide the dp4a and shared-memory latencies of one CTA per SM), from a
// sweep of 8/16/24 warps and 4/8 rows at the Qwen2-7B shapes.
int ring_rw(const GemvArgs& a) { return a.qtype == DQMK_Q40 ? 8 : 4; }
int ring_wt(const GemvArgs&) { return 16; }

template <int QT, int RW, int WMAX, bool PEER>
cudaError_t ring_prepare(const RingPlan* p, int* resident_out) {
  static DeviceOnce once;
  cudaError_t e = once.run([] {
    return cudaFuncSetAttribute(gemv_ring_kernel<QT, RW, WMAX, PEER>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (e != cudaSuccess || !p) return e;
  static std::mutex mu;
  static size_t occ_key[kMaxDevices];
  static int occ[kMaxDevices];
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  const size_t key = p->smem * 64 + (size_t)p->dm.W;
  std::lock_guard<std::mutex> lock(mu);
  if (occ_key[dev] != key) {
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_ring_kernel<QT, RW, WMAX, PEER>,
                                                      (p->dm.W + 1) * 32, p->smem);
    if (e != cudaSuccess) return e;
    occ[dev] = n > 0 ? n : 1;
    occ_key[dev] = key;
  }
  *resident_out = occ[dev];
  return cudaSuccess;
}

template <int QT, int RW, int WMAX, bool PEER>
cudaError_t ring_launch(const GemvArgs& a, const RingPlan& p, cudaStream_t stream, bool pdl) {
  int resident = 1;
  cudaError_t e = ring_prepare<QT, RW, WMAX, PEER>(&p, &resident);
  if (e != cudaSuccess) return e;
  const int n_tiles = (a.n_rows + p.dm.TR - 1) / p.dm.TR;
  const int grid = std::min(n_tiles, sm_count() * resident);
  return launch(gemv_ring_kernel<QT, RW, WMAX, PEER>, dim3(grid), dim3((p.dm.W + 1) * 32),
                p.smem, stream, pdl, a, p.dm);
}

// Shapes the ring form takes, where it measured faster than the register and
// TMA forms (HBM-cold weights, back-to-back launches on a B200): Q4_0 with at
// least 65536 rows (a Qwen2-7B-class lm_head: 0.54 vs 0.41 of HBM) and Q8_0
// rows of at least 8192 values on fewer than 32768 rows (3584 x 18944: 0.55 vs
// 0.39).  The Qwen2-7B QKV / O / gate-up shapes stay with the register and
// TMA forms (ring 0.12 / 0.38 / 0.60 vs 0.24 / 0.38 / 0.67).  Further: whole
// 32-value blocks of x (k == kp), rows of at most 24576 values, 16-byte
// aligned x and RMSNorm weight, not the peer-memory epilogue.
bool ring_eligible(const GemvArgs& a) {
  if (a.epi == kEpiPeer) return false;
  const bool tall_q4 = a.qtype == DQMK_Q40 && a.n_rows >= 65536;
  const bool wide_q8 = a.qtype == DQMK_Q80 && a.kp >= 8192 && a.n_rows < 32768;
  if (!tall_q4 && !wide_q8) return false;
  if (a.kp < 2048 || a.kp > 24576 || a.k != a.kp) return false;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.norm_w)) & 15u)
    return false;
  return ring_plan(a, ring_rw(a), ring_wt(a)).ok;
}

cudaError_t ring_dispatch(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const RingPlan p = ring_plan(a, ring_rw(a), ring_wt(a));
  if (!p.ok) return cudaErrorInvalidValue;
#define DQMK_RING_CASE(QT, RW, WMAX)                 \
  if (a.qtype == QT && p.rw == RW && p.wmax == WMAX) \
    return ring_launch<QT, RW, WMAX, false>(a, p, stream, pdl);
  DQMK_RING_VARIANTS(DQMK_RING_CASE)
#undef DQMK_RING_CASE
  return cudaErrorInvalidValue;
}

// ------------------------------------------------ ggml-layout compatibility
// One warp per weight row, blocks read in place (34 / 18 / 20 bytes, 2-byte
// aligned), up to 8 input rows per pass.  Serves the drop-in entry points
// that receive raw ggml blocks (CudaQ80LinearDeviceInput and friends).
// Q4_1 (d * q + m): per block d * sum(q x) + m * sum(x).
template <int QT>
__global__ void linear_blocks_kernel(const float* __restrict__ x, int rows, int in_features,
                                     const uint8_t* __restrict__ blocks, int out_features,
                                     const float* __restrict__ bias, float* __restrict__ y) {
  constexpr int BYTES = QT == DQMK_Q80 ? 34 : (QT == DQMK_Q40 ? 18 : 20);
  constexpr int QS = QT == DQMK_Q41 ? 2 : 1;  // first 16-bit word of the quants
  const int lane = threadIdx.x & 31;
  const int nb = (in_features + 31) / 32;
  const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int o = warp; o < out_features; o += nwarps) {
    for (int r0 = 0; r0 < rows; r0 += 8) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
      for (int b = lane; b < nb; b += 32) {
        const uint8_t* p = blocks + ((size_t)o * nb + b) * BYTES;
        const uint16_t* p16 = reinterpret_cast<const uint16_t*>(p);
        const float d = h2f(__ldg(p16));
        const float mn = QT == DQMK_Q41 ? h2f(__ldg(p16 + 1)) : 0.0f;
        float w[32];
#pragma unroll
        for (int j = 0; j < (QT == DQMK_Q80 ? 16 : 8); ++j) {
          const uint16_t v = __ldg(p16 + QS + j);
          if constexpr (QT == DQMK_Q80) {
            w[2 * j] = (float)(int8_t)(v & 0xff);
            w[2 * j + 1] = (float)(int8_t)(v >> 8);
          } else {
            constexpr int off = QT == DQMK_Q40 ? 8 : 0;
            w[2 * j] = (float)((v & 0x0f) - off);
            w[2 * j + 16] = (float)(((v >> 4) & 0x0f) - off);
            w[2 * j + 1] = (float)(((v >> 8) & 0x0f) - off);
            w[2 * j + 17] = (float)((v >> 12) - off);
          }
        }
        const int valid = min(32, in_features - b * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (r0 + i < rows) {
            const float* xr = x + (size_t)(r0 + i) * in_features + b * 32;
            float s = 0.0f, sx = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < valid) {
                s = fmaf(w[j], xr[j], s);
                if constexpr (QT == DQMK_Q41) sx += xr[j];
              }
            acc[i] = fmaf(d, s, acc[i]);
            if constexpr (QT == DQMK_Q41) acc[i] = fmaf(mn, sx, acc[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = warp_sum(acc[i]);
        if (lane == 0 && r0 + i < rows)
          y[(size_t)(r0 + i) * out_features + o] = bias ? __fadd_rn(v, bias[o]) : v;
      }
    }
  }
}

// F32 weights (the reference's cuBLAS SGEMM path, src/cuda_matmul.cc:60-64,
// 181-216, which creates a cuBLAS handle per call): one warp per output row,
// the row streamed with 16-byte loads when in_features % 4 == 0 (otherwise
// scalar), up to 8 input rows per pass, warp-shuffle reduction.
__global__ void linear_f32_kernel(const float* __restrict__ x, int rows, int in_features,
                                  const float* __restrict__ w, int out_features,
                                  const float* __restrict__ bias, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const bool vec = (in_features & 3) == 0 && ((reinterpret_cast<uintptr_t>(w) |
                                               reinterpret_cast<uintptr_t>(x)) & 15u) == 0;
  for (int o = warp; o < out_features; o += nwarps) {
    const float* wr = w + (size_t)o * in_features;
    for (int r0 = 0; r0 < rows; r0 += 8) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
      if (vec) {
        const int k4 = in_features >> 2;
        for (int c = lane; c < k4; c += 32) {
          const float4 wv = ldg_f4_stream(wr + 4 * c);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (r0 + i < rows) {
              const float4 xv =
                  *reinterpret_cast<const float4*>(x + (size_t)(r0 + i) * in_features + 4 * c);
              acc[i] = fmaf(wv.x, xv.x, acc[i]);
              acc[i] = fmaf(wv.y, xv.y, acc[i]);
              acc[i] = fmaf(wv.z, xv.z, acc[i]);
              acc[i] = fmaf(wv.w, xv.w, acc[i]);
            }
          }
        }
      } else {
        for (int k = lane; k < in_features; k += 32) {
          const float wv = __ldg(wr + k);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (r0 + i < rows) acc[i] = fmaf(wv, x[(size_t)(r0 + i) * in_features + k], acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = warp_sum(acc[i]);
        if (lane == 0 && r0 + i < rows)
          y[(size_t)(r0 + i) * out_features + o] = bias ? __fadd_rn(v, bias[o]) : v;
      }
    }
  }
}

}  // namespace

cudaError_t gemv_prepare() {
  cudaError_t e = cudaSuccess;
#define DQMK_PREP(ID, QT, RPW, CPL, GW)                                  \
  if (e == cudaSuccess) e = prepare_t<QT, RPW, CPL, GW, false>(nullptr); \
  if (e == cudaSuccess) e = prepare_t<QT, RPW, CPL, GW, true>(nullptr);
  DQMK_GEMV_VARIANT_IDS(DQMK_PREP)
#undef DQMK_PREP
#define DQMK_TMA_PREP(QT, RPW) \
  if (e == cudaSuccess) e = tma_prepare<QT, RPW>();
  DQMK_TMA_VARIANTS(DQMK_TMA_PREP)
#undef DQMK_TMA_PREP
  if (e == cudaSuccess) e = tc_prepare<DQMK_Q80>();
  if (e == cudaSuccess) e = tc_prepare<DQMK_Q40>();
#define DQMK_RING_PREP(QT, RW, WMAX)                                              \
  if (e == cudaSuccess) e = ring_prepare<QT, RW, WMAX, false>(nullptr, nullptr);
  DQMK_RING_VARIANTS(DQMK_RING_PREP)
#undef DQMK_RING_PREP
  return e;
}

cudaError_t launch_gemv_tma_skip(const GemvArgs& a, cudaStream_t stream, int skip_tile) {
  return tma_dispatch(a, stream, false, skip_tile);
}

cudaError_t device_error_address(unsigned int** p) {
  return cudaGetSymbolAddress(reinterpret_cast<void**>(p), g_device_error);
}

cudaError_t read_device_error(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_device_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *flags) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned int));
  }
  return e;
}

// Shape -> variant, from a sweep of every variant over the decode shapes
// (Qwen2-0.5B Q8_0 / Q4_0, Qwen2-7B Q4_0 at TP 1/2/4) with HBM-cold weights.
// Q8_0 rows up to 64 chunks take a warp per row group; longer rows are split
// across the whole CTA.  Q4_0 rows (32 values per chunk) up to 32 chunks take
// a warp per pair of rows in one pass; up to 128 chunks a warp per group of 4
// rows walking the row in several passes; longer ones are split across the
// CTA.  Very tall weights take 4 rows per group to amortise the shared-memory
// reads of x.
int gemv_variant_id(const GemvArgs& a) {
  if (tma_eligible(a)) return -1;
  const bool wide = a.n_rows >= 32768 && a.epi != kEpiSwiGlu && a.epi != kEpiQkv;
  const int chunks = a.qtype == DQMK_Q80 ? a.kp / 16 : a.kp / 32;
  if (a.qtype == DQMK_Q80) {
    if (chunks <= 32) return 0;                   // <Q8_0, 2, 1, 1>
    if (chunks <= 64) return wide ? 2 : 1;        // <4, 2, 1> / <2, 2, 1>
    if (wide) return chunks <= 256 ? 6 : 7;       // <4, 2, 4> / <4, 4, 4>
    if (chunks <= 256) return 3;                  // <2, 2, 4>
    if (chunks <= 384) return 4;                  // <2, 3, 4>
    return 5;                                     // <2, 4, 4>
  }
  const bool tall = a.n_rows >= 8192;
  if (chunks <= 32) return wide ? 8 : 14;         // <Q4_0, 4, 1, 1> / <2, 1, 1>
  if (chunks <= 64) return tall ? 10 : 9;         // <4, 2, 1> / <2, 2, 1>
  if (chunks <= 128)
    return (a.n_rows >= 16384 && a.n_rows < 65536) ? 8 : 10;
  if (chunks <= 256) return 11;                   // <2, 2, 4>
  if (chunks <= 512 || chunks > 640) return 12;   // <2, 4, 4>
  return 13;                                      // <2, 5, 4>
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  if (tc_eligible(a)) return tc_dispatch(a, stream, pdl);
  if (ring_eligible(a)) return ring_dispatch(a, stream, pdl);
  switch (gemv_variant_id(a)) {
#define DQMK_LAUNCH_CASE(ID, QT, RPW, CPL, GW) \
  case ID:                                     \
    return launch_t<QT, RPW, CPL, GW>(a, stream, pdl);
    DQMK_GEMV_VARIANT_IDS(DQMK_LAUNCH_CASE)
#undef DQMK_LAUNCH_CASE
    default:
      return tma_dispatch(a, stream, pdl, -1);
  }
}

cudaError_t launch_linear_blocks(int qtype, const float* x, int rows, int in_features,
                                 const void* blocks, int out_features, const float* bias,
                                 float* y, cudaStream_t stream) {
  const int warps_per_cta = 4;
  int grid = (out_features + warps_per_cta - 1) / warps_per_cta;
  const int cap = sm_count() * 16;
  if (grid > cap) grid = cap;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  if (qtype == DQMK_Q80)
    linear_blocks_kernel<DQMK_Q80><<<grid, warps_per_cta * 32, 0, stream>>>(
        x, rows, in_features, b, out_features, bias, y);
  else if (qtype == DQMK_Q40)
    linear_blocks_kernel<DQMK_Q40><<<grid, warps_per_cta * 32, 0, stream>>>(
        x, rows, in_features, b, out_features, bias, y);
  else if (qtype == DQMK_Q41)
    linear_blocks_kernel<DQMK_Q41><<<grid, warps_per_cta * 32, 0, stream>>>(
        x, rows, in_features, b, out_features, bias, y);
  else
    linear_f32_kernel<<<grid, warps_per_cta * 32, 0, stream>>>(
        x, rows, in_features, static_cast<const float*>(blocks), out_features, bias, y);
  return cudaGetLastError();
}

}  // namespace dqmk

// ------------------------------------------------------------------ C ABI
using namespace dqmk;

namespace {

int linear_common(const char* api, int qtype, const float* x, int rows, int in_features,
                  const void* blocks, size_t block_count, int out_features, const float* bias,
                  float* y, void* stream) {
  if (rows <= 0 || in_features <= 0 || out_features <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape");
  const size_t expected = (size_t)out_features * (size_t)((in_features + 31) / 32);
  if (block_count != expected)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": block count mismatch: expected " +
                                      std::to_string(expected) + ", got " +
                                      std::to_string(block_count));
  if (!x || !blocks || !y) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  if (reinterpret_cast<uintptr_t>(blocks) & 1u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": blocks must be 2-byte aligned");
  DQMK_CUDA_RET(api, launch_linear_blocks(qtype, x, rows, in_features, blocks, out_features,
                                          bias, y, static_cast<cudaStream_t>(stream)));
  return DQMK_OK;
}

}  // namespace

extern "C" int dqmk_q80_linear(const float* x, int rows, int in_features, const void* blocks,
                               size_t block_count, int out_features, const float* bias,
                               float* y, void* stream) {
  return linear_common("CudaQ80Linear", DQMK_Q80, x, rows, in_features, blocks, block_count,
                       out_features, bias, y, stream);
}

extern "C" int dqmk_q40_linear(const float* x, int rows, int in_features, const void* blocks,
                               size_t block_count, int out_features, const float* bias,
                               float* y, void* stream) {
  return linear_common("CudaQ40Linear", DQMK_Q40, x, rows, in_features, blocks, block_count,
                       out_features, bias, y, stream);
}

extern "C" int dqmk_q41_linear(const float* x, int rows, int in_features, const void* blocks,
                               size_t block_count, int out_features, const float* bias,
                               float* y, void* stream) {
  return linear_common("CudaQ41Linear", DQMK_Q41, x, rows, in_features, blocks, block_count,
                       out_features, bias, y, stream);
}

extern "C" int dqmk_f32_linear(const float* x, int rows, int in_features, const float* w,
                               int out_features, const float* bias, float* y, void* stream) {
  const char* api = "CudaLinear";
  if (rows <= 0 || in_features <= 0 || out_features <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape");
  if (!x || !w || !y) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  DQMK_CUDA_RET(api, launch_linear_blocks(DQMK_F32, x, rows, in_features, w, out_features, bias,
                                          y, static_cast<cudaStream_t>(stream)));
  return DQMK_OK;
}

extern "C" int dqmk_gemv_packed(int qtype, const float* x, int in_features, const void* packed,
                                int out_features, const float* bias, const float* residual,
                                float* y, void* stream) {
  const char* api = qtype == DQMK_Q40 ? "CudaQ40Linear" : "CudaQ80Linear";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, "dqmk_gemv_packed: unsupported quant type");
  if (in_features <= 0 || out_features <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape");
  if (!x || !packed || !y) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  if (reinterpret_cast<uintptr_t>(packed) & 15u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": packed weight must be 16-byte aligned");
  const int kp = (in_features + 31) / 32 * 32;
  if (kp > 48 * 1024)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": in_features too large");
  GemvArgs a = {};
  a.qtype = qtype;
  a.qs = static_cast<const uint8_t*>(packed);
  const size_t qbytes = (size_t)out_features * (qtype == DQMK_Q80 ? kp : kp / 2);
  a.d = reinterpret_cast<const uint16_t*>(a.qs + qbytes);
  a.n_rows = out_features;
  a.k = in_features;
  a.kp = kp;
  a.x = x;
  a.epi = kEpiStore;
  a.bias = bias;
  a.residual = residual;
  a.y = y;
  DQMK_CUDA_RET(api, launch_gemv(a, static_cast<cudaStream_t>(stream), false));
  return DQMK_OK;
}

extern "C" int dqmk_gemv_packed_chained(int qtype, const float* x, int in_features,
                                        const void* packed, int out_features, const float* norm_w,
                                        float eps, int swiglu, float* y, void* stream) {
  const char* api = "dqmk_gemv_packed_chained";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": unsupported quant type");
  if (in_features <= 0 || out_features <= 0 || (swiglu && out_features % 2))
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape");
  if (!x || !packed || !y) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  if (reinterpret_cast<uintptr_t>(packed) & 15u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": packed weight must be 16-byte aligned");
  const int kp = (in_features + 31) / 32 * 32;
  if (kp > 48 * 1024)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": in_features too large");
  GemvArgs a = {};
  a.qtype = qtype;
  a.qs = static_cast<const uint8_t*>(packed);
  a.d = reinterpret_cast<const uint16_t*>(a.qs + (size_t)out_features *
                                                     (qtype == DQMK_Q80 ? kp : kp / 2));
  a.n_rows = out_features;
  a.k = in_features;
  a.kp = kp;
  a.x = x;
  a.norm_w = norm_w;
  a.eps = eps;
  a.epi = swiglu ? kEpiSwiGlu : kEpiStore;
  a.y = y;
  DQMK_CUDA_RET(api, launch_gemv(a, static_cast<cudaStream_t>(stream), use_pdl()));
  return DQMK_OK;
}

extern "C" int dqmk_device_error(int clear) {
  unsigned int flags = 0, prefill_flags = 0, tp_flags = 0, ops_flags = 0, batch_flags = 0;
  cudaError_t e = read_device_error(&flags, clear != 0);
  if (e == cudaSuccess) e = read_prefill_error(&prefill_flags, clear != 0);
  if (e == cudaSuccess) e = read_tp_error(&tp_flags, clear != 0);
  if (e == cudaSuccess) e = read_ops_error(&ops_flags, clear != 0);
  if (e == cudaSuccess) e = read_batch_error(&batch_flags, clear != 0);
  flags |= prefill_flags | tp_flags | ops_flags | batch_flags;
  if (e != cudaSuccess) {
    cuda_fail("dqmk_device_error", e);
    return -1;
  }
  return (int)flags;
}

extern "C" int dqmk_gemv_packed_withhold_tile(int qtype, const float* x, int in_features,
                                              const void* packed, int out_features, float* y,
                                              int tile, void* stream) {
  const char* api = "dqmk_gemv_packed_withhold_tile";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": unsupported quant type");
  if (in_features <= 0 || out_features <= 0 || !x || !packed || !y)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid argument");
  if (reinterpret_cast<uintptr_t>(packed) & 15u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": packed weight must be 16-byte aligned");
  const int kp = (in_features + 31) / 32 * 32;
  if (kp > 8192) return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": in_features too large");
  GemvArgs a = {};
  a.qtype = qtype;
  a.qs = static_cast<const uint8_t*>(packed);
  a.d = reinterpret_cast<const uint16_t*>(a.qs + (size_t)out_features * (qtype == DQMK_Q80 ? kp : kp / 2));
  a.n_rows = out_features;
  a.k = in_features;
  a.kp = kp;
  a.x = x;
  a.epi = kEpiStore;
  a.y = y;
  DQMK_CUDA_RET(api, launch_gemv_tma_skip(a, static_cast<cudaStream_t>(stream), tile));
  return DQMK_OK;
}

extern "C" int dqmk_lm_head_block_sums(int qtype, const float* x, int in_features,
                                       const void* packed, int out_features, int8_t* q_terms,
                                       float* scales, int32_t* sums, void* stream) {
  const char* api = "dqmk_lm_head_block_sums";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": unsupported quant type");
  if (in_features <= 0 || out_features <= 0 || !x || !packed || !q_terms || !scales || !sums)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid argument");
  if (reinterpret_cast<uintptr_t>(packed) & 15u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": packed weight must be 16-byte aligned");
  const int kp = (in_features + 31) / 32 * 32;
  if (kp > 8192) return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": in_features too large");
  const int nbk = kp / 32;
  const size_t smem = (size_t)kp * 4 + (size_t)3 * kp + (size_t)3 * nbk * 4 * 2;
  const uint8_t* qs = static_cast<const uint8_t*>(packed);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (qtype == DQMK_Q80) {
    DQMK_CUDA_RET(api, cudaFuncSetAttribute(block_sums_kernel<DQMK_Q80>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem));
    block_sums_kernel<DQMK_Q80><<<1, kTmaConsumers, smem, st>>>(
        x, in_features, kp, qs, out_features, q_terms, scales, sums);
  } else {
    DQMK_CUDA_RET(api, cudaFuncSetAttribute(block_sums_kernel<DQMK_Q40>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem));
    block_sums_kernel<DQMK_Q40><<<1, kTmaConsumers, smem, st>>>(
        x, in_features, kp, qs, out_features, q_terms, scales, sums);
  }
  DQMK_CUDA_RET(api, cudaGetLastError());
  return DQMK_OK;
}
