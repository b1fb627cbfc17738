// prefill.cu -- batched prefill on tcgen05 tensor cores (sm_100a).
//
// ForwardBatch in the reference runs ForwardToken once per prompt token
// (src/batch.cc:35-40), re-reading every weight per token.  Here a prompt of M
// tokens runs each projection as one GEMM, C[M,N] = X[M,K] W[N,K]^T, on the
// tensor cores, with results within fp32 summation-order differences of the
// F32 reference:
//
//   * weights: every dequantized weight d*q (fp16 scale times an integer of at
//     most 8 bits: at most 18 significant bits) is exact as the sum of two
//     fp16 values once its row is scaled by a power of two 2^-f (row maximum
//     in [2^14, 2^15)); the planes B_hi, B_lo and the row scales 2^f are
//     built once per weight;
//   * activations: each row (after its RMSNorm) is scaled by 2^-e the same way
//     and split into two fp16 planes, x 2^-e = A_hi + A_lo + r with
//     |r| <= 2^-22 |x 2^-e|;
//   * the GEMM: tcgen05.mma kind::f16 (M=128, N=128, K=16) accumulates
//     A_hi B_hi + A_hi B_lo + A_lo B_hi over the whole K dimension into an
//     fp32 tensor-memory (TMEM) accumulator (the dropped A_lo B_lo term is
//     below 2^-22 relative); the epilogue multiplies by 2^(e+f) (exact);
//   * persistent CTAs walk the output tiles; operand tiles arrive by TMA
//     (cp.async.bulk.tensor, 128-byte swizzle, no multicast) through a 3-stage
//     shared-memory ring; one warp issues TMA, one issues MMAs, four drain
//     the accumulators, with two TMEM accumulators so the epilogue of one
//     tile overlaps the main loop of the next; all hand-offs on mbarriers with
//     bounded waits;
//   * split-K: projections with few output tiles (N = dim) split K across
//     CTAs so all SMs work; a reduce kernel sums the partial products in a
//     fixed order (deterministic) and applies the epilogue.
// Epilogues mirror the decode GEMV's: residual add, SwiGLU of interleaved
// gate/up columns, QKV bias + RoPE + KV-cache store at each token's position.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "prefill.h"
#include "tc_dev.cuh"

namespace dqmk {
namespace {

constexpr int BM = 128, BN = 128;
constexpr int BKE = 64;                      // fp16 elements of K per stage
constexpr int kStages = 3;
constexpr int kTileBytes = BM * BKE * 2;     // 16 KB per operand tile
constexpr int kStageBytes = 4 * kTileBytes;  // A hi, A lo, B hi, B lo
constexpr int kAccBufs = 2;                  // TMEM accumulators (tile t, t+1)
constexpr uint32_t kTmemCols = kAccBufs * BN;
constexpr int kEpiWarps = 4;                 // one per TMEM lane quarter, 128 columns each
constexpr int kGemmThreads = (2 + kEpiWarps) * 32;

__device__ unsigned int g_prefill_error;  // kErrTimeout / kErrBadToken

using tc::bar_arrive;
using tc::bar_expect_tx;
using tc::bar_init;
using tc::mma_commit;
using tc::smem_desc;
using tc::su32;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tma_load_2d;
using tc::tmem_ld32;
using tc::tmem_wait_ld;

__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  return tc::bar_wait(b, parity, abort, &g_prefill_error);
}

// kind::f16, M = 128 (token rows), N = 128 (weight rows)
constexpr uint32_t kIdesc = tc::idesc_f16(BM, BN);
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
  tc::mma_f16(tmem_d, a, b, kIdesc, acc);
}

// QKV epilogue for the pair pp (head hh, pair index i) of token row m, bias
// already added: rotate (NeoX pairs (i, i + hd/2), Normal pairs (2i, 2i+1))
// with the position's (cos, sin) and store to q_out or the K / V cache.
__device__ __forceinline__ void epilogue_qkv(const PrefillGemm& p, int m, int pp, int q_pairs,
                                             int kv_pairs, int hh, int i, float x0, float x1,
                                             float2 cs) {
  const int pos = p.pos0 + m;
  float* dst;
  bool rotate = true;
  int nh;
  if (pp < q_pairs) {
    nh = p.n_heads;
    dst = p.q_out + (size_t)m * p.ldq;
  } else if (pp < q_pairs + kv_pairs) {
    nh = p.n_kv_heads;
    dst = p.k_cache + ((size_t)p.layer * p.max_seq + pos) * nh * p.head_dim;
  } else {
    nh = p.n_kv_heads;
    dst = p.v_cache + ((size_t)p.layer * p.max_seq + pos) * nh * p.head_dim;
    rotate = false;
  }
  const int half = p.head_dim / 2;
  int o0, o1;
  if (rotate && p.neox) {
    o0 = hh * p.head_dim + i;
    o1 = o0 + half;
  } else {
    o0 = hh * p.head_dim + 2 * i;
    o1 = o0 + 1;
  }
  if (rotate) {
    const float a = x0, b = x1;
    if (p.neox) {
      x0 = __fmaf_rn(a, cs.x, -__fmul_rn(b, cs.y));
      x1 = __fmaf_rn(a, cs.y, __fmul_rn(b, cs.x));
    } else {
      x0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
      x1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
    }
  }
  dst[o0] = x0;
  dst[o1] = x1;
}

// Output columns n, n+1 (n even) of token row m; column n+1 may lie past p.n.
__device__ __forceinline__ void epilogue_pair(const PrefillGemm& p, int m, int n, float v0,
                                              float v1) {
  if (p.epi == kEpiStore) {
    float* yr = p.y + (size_t)m * p.ldy;
    const float* rr = p.residual ? p.residual + (size_t)m * p.ldy : nullptr;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int nn = n + e;
      if (nn < p.n) {
        float v = e ? v1 : v0;
        if (p.bias) v = __fadd_rn(v, p.bias[nn]);
        if (rr) v = __fadd_rn(rr[nn], v);
        yr[nn] = v;
      }
    }
  } else if (p.epi == kEpiSwiGlu) {
    if (n + 1 < p.n) {
      const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v0)));
      p.y[(size_t)m * p.ldy + n / 2] = __fmul_rn(__fmul_rn(v0, sig), v1);
    }
  } else {  // kEpiQkv
    if (n + 1 >= p.n) return;
    const int half = p.head_dim / 2;
    const int q_pairs = p.n_heads * half, kv_pairs = p.n_kv_heads * half;
    const int pp = n / 2;
    const bool rotate = pp < q_pairs + kv_pairs;
    const int seg_pair = pp < q_pairs ? pp : (rotate ? pp - q_pairs : pp - q_pairs - kv_pairs);
    const int hh = seg_pair / half, i = seg_pair % half;
    const float2 cs =
        rotate ? p.rope_cs[(size_t)(p.pos0 + m) * half + i] : make_float2(1.0f, 0.0f);
    if (p.bias) {
      v0 = __fadd_rn(v0, p.bias[n]);
      v1 = __fadd_rn(v1, p.bias[n + 1]);
    }
    epilogue_qkv(p, m, pp, q_pairs, kv_pairs, hh, i, v0, v1, cs);
  }
}

// 32 rows (from m0) x 32 columns (from n0) of finished accumulators staged in
// shared memory [row][33]: scale by 2^(e+f), then the epilogue (or park the
// partial sums for split-K).  Lanes 0-15 take the column pairs of even rows,
// lanes 16-31 those of odd rows, so each store instruction covers whole row
// segments.  Every global load of the chunk (residual, RoPE table) is issued
// before the first store, so the loads overlap instead of serialising;
// rs_lane holds the row scale of row m0 + lane.
__device__ __forceinline__ void drain_chunk(const PrefillGemm& p, const float* stage, int m0,
                                            int n0, int z, int lane, float rs_lane) {
  constexpr int R = 16;  // rows per lane
  const int j = lane & 15, r0 = lane >> 4;
  const int n = n0 + 2 * j;
  const bool ok0 = n < p.n, ok1 = n + 1 < p.n;
  const float c0 = ok0 ? p.cs[n] : 0.0f, c1 = ok1 ? p.cs[n + 1] : 0.0f;
  float v0[R], v1[R];
#pragma unroll
  for (int it = 0; it < R; ++it) {
    const int rr = r0 + 2 * it;
    const float rs = __shfl_sync(0xffffffffu, rs_lane, rr);
    v0[it] = __fmul_rn(__fmul_rn(stage[rr * 33 + 2 * j], rs), c0);
    v1[it] = __fmul_rn(__fmul_rn(stage[rr * 33 + 2 * j + 1], rs), c1);
  }
  if (!ok0) return;
  const int rows = min(R, (p.m - m0 - r0 + 1) / 2);  // rows of this lane below p.m
  if (p.plan.splits > 1) {
#pragma unroll
    for (int it = 0; it < R; ++it) {
      if (it >= rows) break;
      float* dst = p.partial + ((size_t)z * p.m + m0 + r0 + 2 * it) * p.n + n;
      dst[0] = v0[it];
      if (ok1) dst[1] = v1[it];
    }
    return;
  }
  if (p.epi == kEpiStore) {
    const float b0 = p.bias ? p.bias[n] : 0.0f, b1 = p.bias && ok1 ? p.bias[n + 1] : 0.0f;
    float q0[R], q1[R];
#pragma unroll
    for (int it = 0; it < R; ++it) {
      q0[it] = 0.0f;
      q1[it] = 0.0f;
      if (p.residual && it < rows) {
        const float* rr = p.residual + (size_t)(m0 + r0 + 2 * it) * p.ldy + n;
        q0[it] = rr[0];
        if (ok1) q1[it] = rr[1];
      }
    }
#pragma unroll
    for (int it = 0; it < R; ++it) {
      if (it >= rows) break;
      float x0 = v0[it], x1 = v1[it];
      if (p.bias) {
        x0 = __fadd_rn(x0, b0);
        x1 = __fadd_rn(x1, b1);
      }
      if (p.residual) {
        x0 = __fadd_rn(q0[it], x0);
        x1 = __fadd_rn(q1[it], x1);
      }
      float* yr = p.y + (size_t)(m0 + r0 + 2 * it) * p.ldy + n;
      yr[0] = x0;
      if (ok1) yr[1] = x1;
    }
  } else if (p.epi == kEpiSwiGlu) {
    if (!ok1) return;
#pragma unroll
    for (int it = 0; it < R; ++it) {
      if (it >= rows) break;
      const float g = v0[it];
      const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
      p.y[(size_t)(m0 + r0 + 2 * it) * p.ldy + n / 2] = __fmul_rn(__fmul_rn(g, sig), v1[it]);
    }
  } else {  // kEpiQkv: the RoPE rotations of this lane's rows first
    if (!ok1) return;
    const int half = p.head_dim / 2;
    const int pp = n / 2;
    const int q_pairs = p.n_heads * half, kv_pairs = p.n_kv_heads * half;
    const bool rotate = pp < q_pairs + kv_pairs;
    const int seg_pair = pp < q_pairs ? pp : (rotate ? pp - q_pairs : pp - q_pairs - kv_pairs);
    const int hh = seg_pair / half, i = seg_pair % half;
    float2 rc[R];
#pragma unroll
    for (int it = 0; it < R; ++it)
      rc[it] = rotate && it < rows
                   ? p.rope_cs[(size_t)(p.pos0 + m0 + r0 + 2 * it) * half + i]
                   : make_float2(1.0f, 0.0f);
    const float bb0 = p.bias ? p.bias[n] : 0.0f, bb1 = p.bias ? p.bias[n + 1] : 0.0f;
#pragma unroll
    for (int it = 0; it < R; ++it) {
      if (it >= rows) break;
      epilogue_qkv(p, m0 + r0 + 2 * it, pp, q_pairs, kv_pairs, hh, i,
                   p.bias ? __fadd_rn(v0[it], bb0) : v0[it],
                   p.bias ? __fadd_rn(v1[it], bb1) : v1[it], rc[it]);
    }
  }
}

// Work item w of the persistent walk -> (row tile, column tile, K split).
// Consecutive items share a column tile, so a weight tile is fetched from HBM
// once and served to the other row tiles from L2.
struct Work {
  int m0, n0, z, kb0, kb1;
};
__device__ __forceinline__ Work decode_work(const PrefillGemm& p, int w, int m_tiles, int n_tiles) {
  Work r;
  const int mt = w % m_tiles;
  const int rest = w / m_tiles;
  const int nt = rest % n_tiles;
  r.z = rest / n_tiles;
  r.m0 = mt * BM;
  r.n0 = nt * BN;
  r.kb0 = r.z * p.plan.kb_per;
  r.kb1 = min(p.kp / 32, r.kb0 + p.plan.kb_per);
  return r;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap map_ahi,
                    const __grid_constant__ CUtensorMap map_alo,
                    const __grid_constant__ CUtensorMap map_bhi,
                    const __grid_constant__ CUtensorMap map_blo, const PrefillGemm p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], tfull[kAccBufs],
      tempty[kAccBufs];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (p.m + BM - 1) / BM, n_tiles = (p.n + BN - 1) / BN;
  const int total = m_tiles * n_tiles * p.plan.splits;
  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  float* epi_stage = reinterpret_cast<float*>(tiles + (size_t)kStages * kStageBytes);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      bar_init(&tfull[b], 1);
      bar_init(&tempty[b], kEpiWarps);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(&tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int it = 0;
      for (int w = blockIdx.x; w < total && !abort_flag; w += gridDim.x) {
        const Work t = decode_work(p, w, m_tiles, n_tiles);
        for (int ks = t.kb0 / 2; ks * 2 < t.kb1; ++ks, ++it) {
          const int st = it % kStages;
          if (it >= kStages &&
              !bar_wait(&empty[st], (uint32_t)((it / kStages - 1) & 1), &abort_flag))
            break;
          unsigned char* base = tiles + (size_t)st * kStageBytes;
          const int x = ks * BKE;
          bar_expect_tx(&full[st], kStageBytes);
          tma_load_2d(base, &map_ahi, x, t.m0, &full[st]);
          tma_load_2d(base + kTileBytes, &map_alo, x, t.m0, &full[st]);
          tma_load_2d(base + 2 * kTileBytes, &map_bhi, x, t.n0, &full[st]);
          tma_load_2d(base + 3 * kTileBytes, &map_blo, x, t.n0, &full[st]);
        }
      }
      // tail: every stage's last release (an MMA commit) has landed before
      // the CTA may exit
      for (int i = it > kStages ? it - kStages : 0; i < it && !abort_flag; ++i)
        if (!bar_wait(&empty[i % kStages], (uint32_t)((i / kStages) & 1), &abort_flag)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      int it = 0, tc = 0;
      for (int w = blockIdx.x; w < total && !abort_flag; w += gridDim.x, ++tc) {
        const Work t = decode_work(p, w, m_tiles, n_tiles);
        const int buf = tc % kAccBufs;
        if (tc >= kAccBufs &&
            !bar_wait(&tempty[buf], (uint32_t)((tc / kAccBufs - 1) & 1), &abort_flag))
          break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        uint32_t accumulate = 0u;
        bool ok = true;
        for (int ks = t.kb0 / 2; ks * 2 < t.kb1; ++ks, ++it) {
          const int st = it % kStages;
          if (!bar_wait(&full[st], (uint32_t)((it / kStages) & 1), &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ahi = su32(tiles + (size_t)st * kStageBytes);
          const uint32_t alo = ahi + kTileBytes, bhi = ahi + 2 * kTileBytes,
                         blo = ahi + 3 * kTileBytes;
#pragma unroll
          for (int k = 0; k < BKE / 16; ++k) {  // K=16 slices: 32 bytes apart
            const uint32_t off = (uint32_t)k * 32;
            const uint64_t dbhi = smem_desc(bhi + off);
            mma_f16(d, smem_desc(ahi + off), dbhi, accumulate);
            mma_f16(d, smem_desc(ahi + off), smem_desc(blo + off), 1u);
            mma_f16(d, smem_desc(alo + off), dbhi, 1u);
            accumulate = 1u;
          }
          mma_commit(&empty[st]);  // the stage is free once these MMAs finish
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);  // the accumulator is complete
      }
    }
  } else {  // ---------------- epilogue warps 2..5: TMEM lanes 32*(warp%4) ..
    const int quarter = warp & 3;  // tile rows 32*quarter + lane == TMEM lanes
    int tc = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++tc) {
      const Work t = decode_work(p, w, m_tiles, n_tiles);
      const int buf = tc % kAccBufs;
      // warp-uniform outcome: the TMEM loads below are .sync.aligned
      if (!__all_sync(0xffffffffu,
                      bar_wait(&tfull[buf], (uint32_t)((tc / kAccBufs) & 1), &abort_flag)))
        break;
      tc_fence_after();
      uint32_t r[BN];
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tmem_ld32(trow + (uint32_t)(c * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&tempty[buf]);  // the next-but-one tile may start
      // each 32 x 32 chunk (this warp's rows x 32 columns) goes through shared
      // memory so that the stores are row-contiguous across the warp
      float* stage = epi_stage + (size_t)(warp - 2) * 32 * 33;
      const int my_row = t.m0 + quarter * 32 + lane;
      const float rs_lane = my_row < p.m ? p.rs[my_row] : 0.0f;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
#pragma unroll
        for (int j = 0; j < 32; ++j) stage[lane * 33 + j] = __uint_as_float(r[c * 32 + j]);
        __syncwarp();
        drain_chunk(p, stage, t.m0 + quarter * 32, t.n0 + c * 32, t.z, lane, rs_lane);
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// Split-K: sum the partial products in split order, then the epilogue.
__global__ void splitk_epilogue_kernel(const PrefillGemm p) {
  const int m = blockIdx.x;
  const int n = 2 * (blockIdx.y * blockDim.x + threadIdx.x);
  if (n >= p.n) return;
  float v0 = 0.0f, v1 = 0.0f;
  for (int z = 0; z < p.plan.splits; ++z) {
    const float* src = p.partial + ((size_t)z * p.m + m) * p.n + n;
    v0 = __fadd_rn(v0, src[0]);
    if (n + 1 < p.n) v1 = __fadd_rn(v1, src[1]);
  }
  epilogue_pair(p, m, n, v0, v1);
}

// ----------------------------------------------------------- activations
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < 8; ++w) t = __fadd_rn(t, red[w]);
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < 8; ++w) t = fmaxf(t, red[w]);
  return t;
}

// One CTA per token row: optional RMSNorm (src/ops.cc:68-90), a power-of-two
// row scale 2^-e that brings the row's absmax into [2^14, 2^15), and the
// two-term fp16 split hi = fp16(v), lo = fp16(v - hi) of v = x 2^-e.  Writes
// hi/lo [row][kp] (zero past k) and rs[row] = 2^e.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int k,
                                                         int kp, int ldx,
                                                         const float* __restrict__ norm_w,
                                                         float eps, uint16_t* __restrict__ hi,
                                                         uint16_t* __restrict__ lo,
                                                         float* __restrict__ rs) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* xr = x + (size_t)row * ldx;
  float scale = 1.0f;
  if (norm_w) {
    float ss = 0.0f;
    for (int e = tid; e < k; e += 256) ss = __fadd_rn(ss, __fmul_rn(xr[e], xr[e]));
    const float t = block_sum(ss, red);
    scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)k), eps)));
  }
  auto val = [&](int col) -> float {
    const float v = xr[col];
    return norm_w ? __fmul_rn(__fmul_rn(v, scale), norm_w[col]) : v;
  };
  float mx = 0.0f;
  for (int e = tid; e < k; e += 256) mx = fmaxf(mx, fabsf(val(e)));
  mx = block_max(mx, red);
  int ex = 0;
  if (mx > 0.0f && mx <= 3.0e38f) {
    int fe;
    frexpf(mx, &fe);  // mx in [2^(fe-1), 2^fe)
    ex = min(max(fe - 15, -120), 120);
  }
  const float down = ldexpf(1.0f, -ex);
  if (tid == 0) rs[row] = ldexpf(1.0f, ex);
  uint16_t* hr = hi + (size_t)row * kp;
  uint16_t* lr = lo + (size_t)row * kp;
  for (int c = tid * 4; c < kp; c += 1024) {
    uint32_t h2[2], l2[2];
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      float v[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) v[t] = c + e + t < k ? __fmul_rn(val(c + e + t), down) : 0.0f;
      const __half ha = __float2half_rn(v[0]), hb = __float2half_rn(v[1]);
      const __half la = __float2half_rn(__fsub_rn(v[0], __half2float(ha)));
      const __half lb = __float2half_rn(__fsub_rn(v[1], __half2float(hb)));
      h2[e / 2] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
      l2[e / 2] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
    }
    *reinterpret_cast<uint2*>(hr + c) = make_uint2(h2[0], h2[1]);
    *reinterpret_cast<uint2*>(lr + c) = make_uint2(l2[0], l2[1]);
  }
}

// The same split with the row held in registers (J values per thread, element
// e = tid + 256 j, the order of the loops above): one load pass with every
// load in flight, instead of a round trip per pass; the sums, the maximum and
// every written value are those of split_rows_kernel bit for bit.  Launched
// with programmatic dependent launch in the decode chains: it waits for the
// producer of x before its first access, and reads x through L2 with
// ld.global.cg.  x is written by the previous kernel while this one may
// already be resident, so it is not read-only for this kernel's lifetime: a
// load the compiler turned into a read-only-path (.nc) load -- which a
// const __restrict__ pointer invites -- may be scheduled ahead of
// griddepcontrol.wait or hit a stale copy.  (Under tensor parallelism that
// corrupted the multi-sequence step's activations; the explicit .cg load,
// an asm volatile like griddepcontrol.wait, stays after it.)
template <int J>
__global__ void __launch_bounds__(256) split_rows_reg_kernel(const float* x, int k,
                                                             int kp, int ldx,
                                                             const float* __restrict__ norm_w,
                                                             float eps, uint16_t* __restrict__ hi,
                                                             uint16_t* __restrict__ lo,
                                                             float* __restrict__ rs) {
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* xr = x + (size_t)row * ldx;
  float v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = tid + 256 * j;
    v[j] = e < k ? __ldcg(xr + e) : 0.0f;
  }
  if (norm_w) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
      if (tid + 256 * j < k) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
    const float t = block_sum(ss, red);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)k), eps)));
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int e = tid + 256 * j;
      if (e < k) v[j] = __fmul_rn(__fmul_rn(v[j], scale), norm_w[e]);
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < J; ++j)
    if (tid + 256 * j < k) mx = fmaxf(mx, fabsf(v[j]));
  mx = block_max(mx, red);
  int ex = 0;
  if (mx > 0.0f && mx <= 3.0e38f) {
    int fe;
    frexpf(mx, &fe);  // mx in [2^(fe-1), 2^fe)
    ex = min(max(fe - 15, -120), 120);
  }
  const float down = ldexpf(1.0f, -ex);
  if (tid == 0) rs[row] = ldexpf(1.0f, ex);
  uint16_t* hr = hi + (size_t)row * kp;
  uint16_t* lr = lo + (size_t)row * kp;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = tid + 256 * j;
    if (e < kp) {
      const float t = e < k ? __fmul_rn(v[j], down) : 0.0f;
      const __half h = __float2half_rn(t);
      const __half l = __float2half_rn(__fsub_rn(t, __half2float(h)));
      hr[e] = __half_as_ushort(h);
      lr[e] = __half_as_ushort(l);
    }
  }
}

// Packed-row gather of M token embeddings (rows of the quantized token_embd).
// A token id outside [0, vocab) -- possible only when it comes from device
// state the host did not validate -- gathers nothing: the row is zeroed and
// kErrBadToken recorded.
__global__ void embed_rows_kernel(int qtype, const uint8_t* __restrict__ qs,
                                  const uint16_t* __restrict__ d, int dim, int kp, int vocab,
                                  const int* __restrict__ tokens, float* __restrict__ y) {
  const int row = blockIdx.x;
  const int token = tokens[row];
  if (token < 0 || token >= vocab) {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) y[(size_t)row * dim + i] = 0.0f;
    if (threadIdx.x == 0) atomicOr(&g_prefill_error, kErrBadToken);
    return;
  }
  const int nbk = kp / 32;
  const size_t row_bytes = qtype == DQMK_Q80 ? (size_t)kp : (size_t)kp / 2;
  const uint8_t* qr = qs + (size_t)token * row_bytes;
  const uint16_t* dr = d + (size_t)token * nbk;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float sc = h2f(dr[i / 32]);
    float v;
    if (qtype == DQMK_Q80) {
      v = (float)(int8_t)qr[i];
    } else {
      const int j = i % 32;
      const uint8_t byte = qr[(i / 32) * 16 + (j & 15)];
      v = (float)((j < 16 ? (byte & 0x0f) : (byte >> 4)) - 8);
    }
    y[(size_t)row * dim + i] = __fmul_rn(sc, v);
  }
}

// One CTA per weight row: the dequantized values w = d * q (Q8_0 int8 q;
// Q4_0 nibble - 8 with low nibbles as values 0..15 of a block and high
// nibbles as 16..31, src/quant.cc:148-175) are exact in fp32 (at most 19
// significant bits); scaled by 2^-f (row maximum in [2^14, 2^15)) each splits
// exactly into hi = fp16(w 2^-f) and lo = fp16(w 2^-f - hi).  Writes the two
// planes [row][kp] and cs[row] = 2^f.
__global__ void __launch_bounds__(256) weights_split_kernel(int qtype, const uint8_t* __restrict__ qs,
                                                            const uint16_t* __restrict__ d, int kp,
                                                            uint16_t* __restrict__ bhi,
                                                            uint16_t* __restrict__ blo,
                                                            float* __restrict__ cs) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  const int nbk = kp / 32;
  const uint16_t* dr = d + (size_t)row * nbk;
  const uint8_t* qr = qs + (size_t)row * (qtype == DQMK_Q80 ? kp : kp / 2);
  auto quant = [&](int e) -> int {
    if (qtype == DQMK_Q80) return (int)(int8_t)qr[e];
    const int j = e & 31;
    const uint8_t byte = qr[(e >> 5) * 16 + (j & 15)];
    return (int)(j < 16 ? (byte & 0x0f) : (byte >> 4)) - 8;
  };
  float mx = 0.0f;
  for (int e = tid; e < kp; e += 256) mx = fmaxf(mx, fabsf(__fmul_rn(h2f(dr[e >> 5]), (float)quant(e))));
  mx = block_max(mx, red);
  int ex = 0;
  if (mx > 0.0f && mx <= 3.0e38f) {
    int fe;
    frexpf(mx, &fe);
    ex = min(max(fe - 15, -120), 120);
  }
  const float down = ldexpf(1.0f, -ex);
  if (tid == 0) cs[row] = ldexpf(1.0f, ex);
  uint16_t* hr = bhi + (size_t)row * kp;
  uint16_t* lr = blo + (size_t)row * kp;
  for (int e = tid * 2; e < kp; e += 512) {
    uint32_t h2 = 0, l2 = 0;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float w = __fmul_rn(__fmul_rn(h2f(dr[(e + t) >> 5]), (float)quant(e + t)), down);
      const __half h = __float2half_rn(w);
      const __half l = __float2half_rn(__fsub_rn(w, __half2float(h)));
      h2 |= (uint32_t)__half_as_ushort(h) << (16 * t);
      l2 |= (uint32_t)__half_as_ushort(l) << (16 * t);
    }
    *reinterpret_cast<uint32_t*>(hr + e) = h2;
    *reinterpret_cast<uint32_t*>(lr + e) = l2;
  }
}

// Causal GQA attention for a block of 64 consecutive query positions of one
// head over cache positions 0 .. its last query (src/ops.cc attention per
// token: scores q.k / sqrt(head_dim), softmax, weighted sum of values), fp32
// throughout, flash-style online softmax over 64-key tiles.  Thread (ty, tx)
// of 256 owns queries ty + 16 i and keys tx + 16 j (i, j < 4) of each score
// tile and output dims tx*4 + 64 e of its queries: with 16-strided keys and
// rows padded to HD + 4 floats, the float4 shared-memory reads of a quarter
// warp hit distinct banks.
template <int HD>
__global__ void __launch_bounds__(256) attention_prefill_kernel(PrefillAttn a) {
  constexpr int BQ = 64, BKV = 64, LD = HD + 4, NV4 = HD / 64, LP = BKV + 1;
  extern __shared__ float4 smem4[];
  float* qs = reinterpret_cast<float*>(smem4);  // [BQ][LD]
  float* ks = qs + BQ * LD;                     // [BKV][LD]
  float* vs = ks + BKV * LD;                    // [BKV][HD]
  float* ps = vs + BKV * HD;                    // [BQ][LP]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int h = blockIdx.x, q0 = blockIdx.y * BQ;
  const int kvh = h / (a.n_heads / a.n_kv_heads);
  const size_t rstride = (size_t)a.n_kv_heads * HD;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * rstride + (size_t)kvh * HD;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * rstride + (size_t)kvh * HD;
  const int nq = min(BQ, a.m - q0);
  const int last = a.pos0 + q0 + nq - 1;  // the last key any query here sees
  for (int i = tid; i < BQ * HD / 4; i += 256) {
    const int r = i / (HD / 4), c4 = i % (HD / 4);
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (r < nq)
      v = *reinterpret_cast<const float4*>(a.q + (size_t)(q0 + r) * a.ldq + (size_t)h * HD + c4 * 4);
    *reinterpret_cast<float4*>(qs + r * LD + c4 * 4) = v;
  }
  const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
  float mrow[4], lrow[4], o[4][4 * NV4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.0f;
#pragma unroll
    for (int e = 0; e < 4 * NV4; ++e) o[i][e] = 0.0f;
  }
  for (int kt = 0; kt <= last; kt += BKV) {
    __syncthreads();  // the previous tile's K, V and P are consumed
    for (int i = tid; i < BKV * HD / 4; i += 256) {
      const int r = i / (HD / 4), c4 = i % (HD / 4);
      const int pos = kt + r;
      float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vv = kv;
      if (pos <= last) {
        kv = __ldcg(reinterpret_cast<const float4*>(kbase + (size_t)pos * rstride) + c4);
        vv = __ldcg(reinterpret_cast<const float4*>(vbase + (size_t)pos * rstride) + c4);
      }
      *reinterpret_cast<float4*>(ks + r * LD + c4 * 4) = kv;
      *reinterpret_cast<float4*>(vs + r * HD + c4 * 4) = vv;
    }
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(qs + (ty + 16 * i) * LD + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(ks + (tx + 16 * j) * LD + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc[i][j] = fmaf(qv[i].x, kv[j].x, sc[i][j]);
          sc[i][j] = fmaf(qv[i].y, kv[j].y, sc[i][j]);
          sc[i][j] = fmaf(qv[i].z, kv[j].z, sc[i][j]);
          sc[i][j] = fmaf(qv[i].w, kv[j].w, sc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ql = ty + 16 * i;
      const int qpos = a.pos0 + q0 + ql;
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool vis = ql < nq && kt + tx + 16 * j <= qpos;
        sc[i][j] = vis ? __fmul_rn(sc[i][j], scale) : -INFINITY;
        tmax = fmaxf(tmax, sc[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mnew = fmaxf(mrow[i], tmax);
      const float corr = mnew == -INFINITY ? 1.0f : expf(mrow[i] - mnew);
      float psum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = sc[i][j] == -INFINITY ? 0.0f : expf(sc[i][j] - mnew);
        ps[ql * LP + tx + 16 * j] = pv;
        psum += pv;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      lrow[i] = fmaf(lrow[i], corr, psum);
      mrow[i] = mnew;
#pragma unroll
      for (int e = 0; e < 4 * NV4; ++e) o[i][e] *= corr;
    }
    __syncwarp();  // a query row's P is written and read by the same 16 lanes
#pragma unroll 4
    for (int k = 0; k < BKV; ++k) {
      float pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pk[i] = ps[(ty + 16 * i) * LP + k];
#pragma unroll
      for (int e4 = 0; e4 < NV4; ++e4) {
        const float4 v = *reinterpret_cast<const float4*>(vs + k * HD + e4 * 64 + tx * 4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o[i][e4 * 4 + 0] = fmaf(pk[i], v.x, o[i][e4 * 4 + 0]);
          o[i][e4 * 4 + 1] = fmaf(pk[i], v.y, o[i][e4 * 4 + 1]);
          o[i][e4 * 4 + 2] = fmaf(pk[i], v.z, o[i][e4 * 4 + 2]);
          o[i][e4 * 4 + 3] = fmaf(pk[i], v.w, o[i][e4 * 4 + 3]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ql = ty + 16 * i;
    if (ql >= nq) continue;
    float* out = a.out + (size_t)(q0 + ql) * a.ldo + (size_t)h * HD;
#pragma unroll
    for (int e4 = 0; e4 < NV4; ++e4)
      *reinterpret_cast<float4*>(out + e4 * 64 + tx * 4) =
          make_float4(__fdiv_rn(o[i][e4 * 4 + 0], lrow[i]), __fdiv_rn(o[i][e4 * 4 + 1], lrow[i]),
                      __fdiv_rn(o[i][e4 * 4 + 2], lrow[i]), __fdiv_rn(o[i][e4 * 4 + 3], lrow[i]));
  }
}

template <int HD>
constexpr size_t attention_prefill_smem() {
  return sizeof(float) * (2 * 64 * (HD + 4) + 64 * HD + 64 * 65);
}

// ------------------------------------------- causal attention, tensor cores
// The same attention at head_dim 64 on tcgen05.  A CTA takes 128 query rows
// of one head (row r on TMEM lane r) and walks the cache in 64-position tiles
// with both contractions as kind::f16 MMAs over the two-term operands of the
// projections: each Q row, each K row (cache position) and each V column (one
// head dimension within a tile) is scaled by a power of two to a maximum in
// [2^14, 2^15) and split into fp16 hi + lo, and A_hi B_hi + A_hi B_lo +
// A_lo B_hi accumulate in fp32 tensor memory (about 2^-22 relative per
// product, as in the GEMMs):
//   S' = Q' K'^T   A = Q' (TMEM, once per CTA), B = K' tile [position][hd]
//   S  = S' 2^(eq + ek) / sqrt(64); masked online softmax in registers, in
//        the base-2 domain (scores times log2 e, exp2f)
//   O' = P V'      A = P in [0, 1], two-term (TMEM), B = V'^T tile [hd][position]
//   O  = O corr + O' 2^ev per tile in registers; O / l at the end.
// Eight warps: warps w and w + 4 read the same 32 TMEM lanes (rows) and take
// 32 of the 64 columns each, in the softmax and in the O update, exchanging
// row maxima through shared memory.  All 256 threads read the next tile's K
// and V from global memory (L2: the QKV epilogue just wrote them) and write
// it into the other shared-memory buffer while the score MMAs run.  Every
// wait is bounded and decided for the whole CTA (__syncthreads_and), so all
// threads leave the tile loop together.
namespace atc {
constexpr int kRows = 128, kKv = 64, kHd = 64, kThreads = 256;
constexpr int kPlane = kKv * 128;      // 64 rows of 64 fp16, 128-byte swizzle
constexpr int kBufBytes = 4 * kPlane;  // K hi, K lo, V^T hi, V^T lo
// two buffers + alignment, padded so that at most two CTAs (2 x 256 TMEM
// columns) share an SM
constexpr int kSmem = 80 * 1024;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColO = 64, kColQ = 128, kColP = 192;
constexpr uint32_t kIdesc = tc::idesc_f16(kRows, 64);
constexpr float kLog2e = 1.44269504088896341f;
static_assert(2 * kBufBytes + 1024 <= kSmem && 3 * kSmem > 227 * 1024, "smem plan");
// A query block's cache tiles split across at most kMaxSplits CTAs; each
// writes O (unnormalised), the running maximum m (base 2) and the sum l of
// its rows: kPartFloats per split.
constexpr int kMaxSplits = 8;
constexpr int kPartFloats = kRows * (kHd + 2);

// Tiles per split and number of splits of a query block with nt tiles, for
// a target of `target` tiles per split (0: no split); every split non-empty.
__host__ __device__ inline void split_plan(int nt, int target, int* per, int* splits) {
  if (target <= 0) {
    *per = nt;
    *splits = 1;
    return;
  }
  int sp = (nt + target - 1) / target;
  sp = sp < kMaxSplits ? sp : kMaxSplits;
  *per = (nt + sp - 1) / sp;
  *splits = (nt + *per - 1) / *per;
}

// Byte offset of 16-byte chunk c (8 fp16) of row r in a 128-byte-swizzled
// K-major operand tile (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}
// ex such that mx 2^-ex lies in [2^14, 2^15) for a normal mx > 0, read from
// the exponent field (mx in [2^(fe-1), 2^fe)); 0 for mx == 0; clamped to
// [-120, 120].
__device__ __forceinline__ int pow2_ex(float mx) {
  const int fe = ((__float_as_int(mx) >> 23) & 0xff) - 126;
  return mx > 0.0f ? min(max(fe - 15, -120), 120) : 0;
}
// 2^e for |e| <= 126, built from its exponent field.
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }
// Two values to packed fp16 pairs hi and lo with x = hi + lo + r,
// |r| <= 2^-22 |x| (element 0 in the low half).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 back = __half22float2(h);
  const __half2 l = __floats2half2_rn(__fsub_rn(x0, back.x), __fsub_rn(x1, back.y));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// One 64-position tile of K and V (positions kt.., zero past `last`) into a
// shared-memory buffer, with the per-position K scales 2^ek (sk) and the
// per-dimension V scales 2^ev (sv); 256 threads.
//   K: thread -> position j = tid / 4; its float4 i holds dimensions
//      16 i + 4 (tid % 4) .. +3 (a warp reads 8 rows x 64 contiguous bytes
//      per load), stored as 8-byte halves of the swizzled chunks;
//   V: thread -> dimensions 4 (tid / 16) .. +3 at positions kt + 4 (tid % 16)
//      .. +3, stored as 8-byte halves of its four B rows' chunks.
__device__ __forceinline__ void load_tile(const float* kbase, const float* vbase, size_t rstride,
                                          int kt, int last, unsigned char* buf, float* sk,
                                          float* sv, int tid) {
  {
    const int j = tid >> 2, p = tid & 3, pos = kt + j;
    float4 v[4];
    if (pos <= last) {
      const float4* src = reinterpret_cast<const float4*>(kbase + (size_t)pos * rstride) + p;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __ldcg(src + 4 * i);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const int ex = pow2_ex(mx);
    const float down = pow2f(-ex);
    if (p == 0) sk[j] = pow2f(ex);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint2 hi, lo;
      split2(__fmul_rn(v[i].x, down), __fmul_rn(v[i].y, down), hi.x, lo.x);
      split2(__fmul_rn(v[i].z, down), __fmul_rn(v[i].w, down), hi.y, lo.y);
      const uint32_t off = sw128(j, 2 * i + (p >> 1)) + (uint32_t)(p & 1) * 8;
      *reinterpret_cast<uint2*>(buf + off) = hi;
      *reinterpret_cast<uint2*>(buf + kPlane + off) = lo;
    }
  }
  {
    const int dg = tid >> 4, pg = tid & 15;
    float4 v[4];  // v[i] = V[kt + 4 pg + i][4 dg .. 4 dg + 3]
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pos = kt + 4 * pg + i;
      v[i] = pos <= last
                 ? __ldcg(reinterpret_cast<const float4*>(vbase + (size_t)pos * rstride + 4 * dg))
                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float mx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mx[0] = fmaxf(mx[0], fabsf(v[i].x));
      mx[1] = fmaxf(mx[1], fabsf(v[i].y));
      mx[2] = fmaxf(mx[2], fabsf(v[i].z));
      mx[3] = fmaxf(mx[3], fabsf(v[i].w));
    }
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int off = 1; off < 16; off <<= 1)
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], off));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ex = pow2_ex(mx[e]);
      const float down = pow2f(-ex);
      if (pg == 0) sv[4 * dg + e] = pow2f(ex);
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float val = e == 0 ? v[i].x : e == 1 ? v[i].y : e == 2 ? v[i].z : v[i].w;
        x[i] = __fmul_rn(val, down);
      }
      uint2 hi, lo;
      split2(x[0], x[1], hi.x, lo.x);
      split2(x[2], x[3], hi.y, lo.y);
      const uint32_t off = sw128(4 * dg + e, pg >> 1) + (uint32_t)(pg & 1) * 8;
      *reinterpret_cast<uint2*>(buf + 2 * kPlane + off) = hi;
      *reinterpret_cast<uint2*>(buf + 3 * kPlane + off) = lo;
    }
  }
}
}  // namespace atc

__global__ void __launch_bounds__(atc::kThreads, 2) attention_prefill_tc_kernel(PrefillAttn a) {
  using namespace atc;
  extern __shared__ unsigned char atc_raw[];
  __shared__ __align__(8) uint64_t bar_s, bar_o, bar_fin;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  // scales of three tiles: the one being read, the one being written, and the
  // one whose last readers may still be in their O update
  __shared__ float sk[3][kKv], sv[3][kHd];
  __shared__ float red[2][kRows];  // per row and column half: maxima, then partial sums
  __shared__ float qf[kRows];      // per row: 2^eq log2(e) / sqrt(64)
  unsigned char* bufs = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(atc_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;  // TMEM lanes 32 quarter.., columns 32 half..
  const int row = 32 * quarter + lane;
  const int h = blockIdx.x;
  const int qb = (int)(gridDim.y - 1 - blockIdx.y);  // longest blocks first
  const int q0 = qb * kRows;
  const int kvh = h / (a.n_heads / a.n_kv_heads);
  const size_t rstride = (size_t)a.n_kv_heads * kHd;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * rstride + (size_t)kvh * kHd;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * rstride + (size_t)kvh * kHd;
  const int nq = min(kRows, a.m - q0);
  const int qmin = a.pos0 + q0;           // the first query's position
  const int last = qmin + nq - 1;         // the last position any row here sees
  int per, splits;
  split_plan(last / kKv + 1, a.part ? a.tiles_per_split : 0, &per, &splits);
  const int split = blockIdx.z;
  if (split >= splits) return;  // this block needs fewer splits than the grid has
  const int t0 = split * per;
  const int nt = min(last / kKv + 1 - t0, per);  // tiles t0 .. t0 + nt - 1
  const bool valid = row < nq;
  const int qpos = qmin + row;

  if (tid == 0) {
    tc::bar_init(&bar_s, 1);
    tc::bar_init(&bar_o, 1);
    tc::bar_init(&bar_fin, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, atc::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;

  if (half == 0) {  // warps 0-3: this row of Q, scaled and split, into TMEM
    float4 v[16];
    const float4* src =
        reinterpret_cast<const float4*>(a.q + (size_t)(q0 + row) * a.ldq + (size_t)h * kHd);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = valid ? src[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    const int ex = pow2_ex(mx);
    const float down = pow2f(-ex);
    // 2^eq / sqrt(64) is exact; one rounding for log2(e)
    qf[row] = __fmul_rn(__fmul_rn(pow2f(ex), __fdiv_rn(1.0f, sqrtf((float)kHd))), kLog2e);
    uint32_t hi[32], lo[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      split2(__fmul_rn(v[i].x, down), __fmul_rn(v[i].y, down), hi[2 * i], lo[2 * i]);
      split2(__fmul_rn(v[i].z, down), __fmul_rn(v[i].w, down), hi[2 * i + 1], lo[2 * i + 1]);
    }
    tc::tmem_st32(tmem + lane_base + kColQ, hi);
    tc::tmem_st32(tmem + lane_base + kColQ + 32, lo);
    tc::tmem_wait_st();
  }
  load_tile(kbase, vbase, rstride, t0 * kKv, last, bufs, sk[0], sv[0], tid);
  tc::fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const float fq = qf[row];
  float o[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d] = 0.0f;
  float mrow = -INFINITY, lpart = 0.0f;
  bool ok = true;
  for (int t = 0; t < nt; ++t) {  // t: tile index within this split
    const int kt = (t0 + t) * kKv, set = t % 3;
    unsigned char* buf = bufs + (size_t)(t & 1) * kBufBytes;
    if (warp == 0) {  // S' = Q' K'^T
      if (tc::elect_one()) {
        const uint64_t khi = smem_desc(su32(buf)), klo = smem_desc(su32(buf + kPlane));
#pragma unroll
        for (int k = 0; k < kHd / 16; ++k) {
          // a K=16 slice: 8 TMEM columns of A, 32 bytes (+2) of the B descriptor
          const uint32_t qa = tmem + kColQ + 8u * k;
          tc::mma_f16_ts(tmem + kColS, qa, khi + 2u * k, atc::kIdesc, k > 0 ? 1u : 0u);
          tc::mma_f16_ts(tmem + kColS, qa, klo + 2u * k, atc::kIdesc, 1u);
          tc::mma_f16_ts(tmem + kColS, qa + 32, khi + 2u * k, atc::kIdesc, 1u);
        }
        mma_commit(&bar_s);
      }
      __syncwarp();
    }
    if (t + 1 < nt) {  // the next tile into the other buffer, under the MMAs
      load_tile(kbase, vbase, rstride, kt + kKv, last, bufs + (size_t)((t + 1) & 1) * kBufBytes,
                sk[(t + 1) % 3], sv[(t + 1) % 3], tid);
      tc::fence_proxy_async_smem();
    }
    ok = __syncthreads_and(bar_wait(&bar_s, (uint32_t)(t & 1), &abort_flag));
    if (!ok) break;
    tc_fence_after();

    uint32_t r[32];
    tmem_ld32(tmem + lane_base + kColS + 32u * half, r);
    tmem_wait_ld();
    const float* skp = sk[set] + 32 * half;
    float s[32];
    float tmax = -INFINITY;
    if (kt + kKv - 1 <= qmin) {  // every position of the tile is visible to every row
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        s[j] = __fmul_rn(__fmul_rn(__uint_as_float(r[j]), fq), skp[j]);
        tmax = fmaxf(tmax, s[j]);
      }
    } else {
      const int first = kt + 32 * half;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float v = __fmul_rn(__fmul_rn(__uint_as_float(r[j]), fq), skp[j]);
        s[j] = valid && first + j <= qpos ? v : -INFINITY;
        tmax = fmaxf(tmax, s[j]);
      }
    }
    red[half][row] = tmax;
    __syncthreads();
    const float mnew = fmaxf(mrow, fmaxf(red[0][row], red[1][row]));
    const float mref = mnew == -INFINITY ? 0.0f : mnew;  // rows with nothing visible yet
    const float corr = exp2f(mrow - mref);
    float psum = 0.0f;
    uint32_t ph[16], pl[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float p0 = exp2f(s[2 * j] - mref), p1 = exp2f(s[2 * j + 1] - mref);
      psum += p0;
      psum += p1;
      split2(p0, p1, ph[j], pl[j]);
    }
    lpart = fmaf(lpart, corr, psum);
    mrow = mnew;
    // P's columns are free: the previous tile's P V MMAs have completed
    tc::tmem_st16(tmem + lane_base + kColP + 16u * half, ph);
    tc::tmem_st16(tmem + lane_base + kColP + 32u + 16u * half, pl);
    tc::tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {  // O' = P V'
      if (tc::elect_one()) {
        const uint64_t vhi = smem_desc(su32(buf + 2 * kPlane)),
                       vlo = smem_desc(su32(buf + 3 * kPlane));
#pragma unroll
        for (int k = 0; k < kKv / 16; ++k) {
          const uint32_t pa = tmem + kColP + 8u * k;
          tc::mma_f16_ts(tmem + kColO, pa, vhi + 2u * k, atc::kIdesc, k > 0 ? 1u : 0u);
          tc::mma_f16_ts(tmem + kColO, pa, vlo + 2u * k, atc::kIdesc, 1u);
          tc::mma_f16_ts(tmem + kColO, pa + 32, vhi + 2u * k, atc::kIdesc, 1u);
        }
        mma_commit(&bar_o);
      }
      __syncwarp();
    }
    ok = __syncthreads_and(bar_wait(&bar_o, (uint32_t)(t & 1), &abort_flag));
    if (!ok) break;
    tc_fence_after();
    tmem_ld32(tmem + lane_base + kColO + 32u * half, r);
    tmem_wait_ld();
    const float* svp = sv[set] + 32 * half;
#pragma unroll
    for (int d = 0; d < 32; ++d)
      o[d] = __fmaf_rn(o[d], corr, __fmul_rn(__uint_as_float(r[d]), svp[d]));
    tc_fence_before();
  }

  // every MMA issued here has completed before TMEM is freed
  if (warp == 0) {
    if (tc::elect_one()) mma_commit(&bar_fin);
    __syncwarp();
  }
  {
    const unsigned long long t0 = tc::now_ns();
    while (!tc::bar_try(&bar_fin, 0u)) {
      if (tc::now_ns() - t0 > tc::kWaitNs) {
        atomicOr(&g_prefill_error, kErrTimeout);
        break;
      }
    }
  }
  red[half][row] = lpart;  // the last reads of red came before the tile loop's last barriers
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, atc::kTmemCols);
  const float l = red[0][row] + red[1][row];
  float4* out =
      reinterpret_cast<float4*>(a.out + (size_t)(q0 + row) * a.ldo + (size_t)h * kHd + 32 * half);
  if (splits == 1) {
    if (ok && valid) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        out[i] = make_float4(__fdiv_rn(o[4 * i], l), __fdiv_rn(o[4 * i + 1], l),
                             __fdiv_rn(o[4 * i + 2], l), __fdiv_rn(o[4 * i + 3], l));
    }
    return;
  }

  // Split block: this split's O, m and l to the scratch; the last of the
  // block's splits to arrive combines them in split order (deterministic)
  // and leaves the block's ticket at zero for the next launch.  Every split
  // takes its ticket, also after a timeout (the error flag is set then).
  const size_t blk = (size_t)h * gridDim.y + qb;
  float* part = a.part + blk * kMaxSplits * kPartFloats;
  if (valid) {
    float4* po = reinterpret_cast<float4*>(part + (size_t)split * kPartFloats + row * kHd + 32 * half);
#pragma unroll
    for (int i = 0; i < 8; ++i) po[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    if (half == 0) {
      part[(size_t)split * kPartFloats + kRows * kHd + row] = mrow;
      part[(size_t)split * kPartFloats + kRows * kHd + kRows + row] = l;
    }
  }
  __threadfence();
  __syncthreads();
  __shared__ unsigned int ticket;
  if (tid == 0) ticket = atomicAdd(&a.tickets[blk], 1u);
  __syncthreads();
  if (ticket != (unsigned int)(splits - 1)) return;
  __threadfence();
  if (tid == 0) a.tickets[blk] = 0u;
  if (!valid) return;
  // every valid row sees position 0 in split 0, so mx is finite
  float mx = -INFINITY;
  for (int sp = 0; sp < splits; ++sp)
    mx = fmaxf(mx, __ldcg(part + (size_t)sp * kPartFloats + kRows * kHd + row));
  float lt = 0.0f;
  float* acc = o;  // this split's O is in the scratch now
#pragma unroll
  for (int d = 0; d < 32; ++d) acc[d] = 0.0f;
  for (int sp = 0; sp < splits; ++sp) {
    const float* ps = part + (size_t)sp * kPartFloats;
    const float w = exp2f(__ldcg(ps + kRows * kHd + row) - mx);  // 0 for a split with nothing visible
    lt = fmaf(__ldcg(ps + kRows * kHd + kRows + row), w, lt);
    const float4* po = reinterpret_cast<const float4*>(ps + row * kHd + 32 * half);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = __ldcg(po + i);
      acc[4 * i] = fmaf(v.x, w, acc[4 * i]);
      acc[4 * i + 1] = fmaf(v.y, w, acc[4 * i + 1]);
      acc[4 * i + 2] = fmaf(v.z, w, acc[4 * i + 2]);
      acc[4 * i + 3] = fmaf(v.w, w, acc[4 * i + 3]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    out[i] = make_float4(__fdiv_rn(acc[4 * i], lt), __fdiv_rn(acc[4 * i + 1], lt),
                         __fdiv_rn(acc[4 * i + 2], lt), __fdiv_rn(acc[4 * i + 3], lt));
}


PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

size_t gemm_smem() {
  return (size_t)kStages * kStageBytes + (size_t)kEpiWarps * 32 * 33 * sizeof(float) + 1024;
}

}  // namespace

// 2D tiled tensor map over a row-major [outer][inner] array; the base, the
// row pitch and the box's inner extent must be 16-byte multiples.
int make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(DQMK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes % 16) != 0 ||
      ((uint64_t)box_inner * elem_bytes) % 16 != 0 || inner == 0 || outer == 0)
    return fail(DQMK_ERR_INVALID, "tensor map base, pitch or box not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DQMK_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return DQMK_OK;
}

// [rows][kp] fp16 plane, box_rows x 64-element (128-byte) boxes, 128-byte swizzle.
int make_f16_tile_map(CUtensorMap* map, const void* base, int rows, int kp, int box_rows) {
  if ((kp % 8) != 0 || rows <= 0)
    return fail(DQMK_ERR_INVALID, "ForwardBatch: tensor map base or stride not 16-byte aligned");
  return make_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, (uint64_t)kp, (uint64_t)rows,
                     (uint64_t)kp * 2, BKE, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Enough work items to cover the SMs, at least 8 scale blocks per split; an
// even block count per split keeps stages aligned to 64-element K steps.
GemmPlan plan_gemm(int m, int n, int kp) {
  const int nbk = kp / 32;
  const int tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  int splits = std::max(1, std::min(sm_count() / std::max(tiles, 1), nbk / 8));
  int kb_per = (nbk + splits - 1) / splits;
  kb_per = (kb_per + 1) / 2 * 2;
  splits = (nbk + kb_per - 1) / kb_per;
  return GemmPlan{splits, kb_per};
}

size_t partial_floats_bound(int m_max, int n, int kp) {
  size_t most = 0;
  for (int mt = 1; (mt - 1) * BM < m_max; ++mt) {
    const int m = std::min(mt * BM, m_max);
    const GemmPlan g = plan_gemm(m, n, kp);
    if (g.splits > 1) most = std::max(most, (size_t)g.splits * m * n);
  }
  return most;
}

cudaError_t prefill_prepare() {
  static DeviceOnce once;
  return once.run([] {
    cudaError_t e = cudaFuncSetAttribute(
        gemm_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_prefill_kernel<64>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)attention_prefill_smem<64>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_prefill_kernel<128>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)attention_prefill_smem<128>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_prefill_tc_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, atc::kSmem);
    return e;
  });
}

cudaError_t launch_prefill_gemm(const CUtensorMap& a_hi, const CUtensorMap& a_lo,
                                const CUtensorMap& b_hi, const CUtensorMap& b_lo,
                                const PrefillGemm& p, cudaStream_t s) {
  const int nbk = p.kp / 32;
  const GemmPlan& g = p.plan;
  if (p.m <= 0 || p.n <= 0 || p.kp <= 0 || p.kp % 32 != 0 || !p.rs || !p.cs || g.splits < 1 ||
      g.kb_per < 2 || g.kb_per % 2 != 0 || (g.splits - 1) * g.kb_per >= nbk ||
      g.splits * g.kb_per < nbk || (g.splits > 1 && !p.partial))
    return cudaErrorInvalidValue;
  cudaError_t e = prefill_prepare();
  if (e != cudaSuccess) return e;
  const long long total =
      (long long)((p.m + BM - 1) / BM) * ((p.n + BN - 1) / BN) * g.splits;
  if (total > (1ll << 30)) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>(total, sm_count());
  gemm_f16_kernel<<<grid, kGemmThreads, gemm_smem(), s>>>(a_hi, a_lo, b_hi, b_lo, p);
  e = cudaGetLastError();
  if (e != cudaSuccess || g.splits == 1) return e;
  const int pairs = (p.n + 1) / 2;
  splitk_epilogue_kernel<<<dim3(p.m, (pairs + 127) / 128), 128, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_split_rows(const float* x, int m, int k, int kp, int ldx, const float* norm_w,
                              float eps, uint16_t* hi, uint16_t* lo, float* rs, cudaStream_t st,
                              bool pdl) {
  const dim3 grid(m), block(256);
  if (kp <= 16 * 256)
    return launch(split_rows_reg_kernel<16>, grid, block, 0, st, pdl, x, k, kp, ldx, norm_w, eps,
                  hi, lo, rs);
  if (kp <= 32 * 256)
    return launch(split_rows_reg_kernel<32>, grid, block, 0, st, pdl, x, k, kp, ldx, norm_w, eps,
                  hi, lo, rs);
  if (kp <= 80 * 256)
    return launch(split_rows_reg_kernel<80>, grid, block, 0, st, pdl, x, k, kp, ldx, norm_w, eps,
                  hi, lo, rs);
  split_rows_kernel<<<m, 256, 0, st>>>(x, k, kp, ldx, norm_w, eps, hi, lo, rs);
  return cudaGetLastError();
}

cudaError_t launch_embed_rows(int qtype, const uint8_t* qs, const uint16_t* d, int dim, int kp,
                              int vocab, const int* tokens, int m, float* y, cudaStream_t st) {
  embed_rows_kernel<<<m, 256, 0, st>>>(qtype, qs, d, dim, kp, vocab, tokens, y);
  return cudaGetLastError();
}

size_t prefill_attn_part_floats(int m_max, int n_heads) {
  return (size_t)n_heads * ((m_max + atc::kRows - 1) / atc::kRows) * atc::kMaxSplits *
         atc::kPartFloats;
}
size_t prefill_attn_tickets(int m_max, int n_heads) {
  return (size_t)n_heads * ((m_max + atc::kRows - 1) / atc::kRows);
}

cudaError_t launch_attention_prefill(const PrefillAttn& a, cudaStream_t st) {
  cudaError_t e = prefill_prepare();
  if (e != cudaSuccess) return e;
  if (a.m <= 0 || a.n_kv_heads <= 0 || a.n_heads % a.n_kv_heads != 0 || a.ldq % 4 != 0 ||
      a.ldo % 4 != 0)
    return cudaErrorInvalidValue;
  // head_dim 64 on the tensor cores unless DQMK_PREFILL_ATTN=fma asks for the
  // fp32 kernel (kept for head_dim 128 and for comparisons)
  const char* mode = std::getenv("DQMK_PREFILL_ATTN");
  if (a.head_dim == 64 && !(mode && std::string(mode) == "fma")) {
    // Split the query blocks' cache ranges for about one CTA per SM, with at
    // least four 64-position tiles per CTA: at 602 and 2048 tokens this beat
    // two CTAs per SM with two tiles each (per-CTA set-up is a large share).
    const int nqb = (a.m + atc::kRows - 1) / atc::kRows;
    auto tiles_of = [&](int b) {
      const int nq = std::min(atc::kRows, a.m - b * atc::kRows);
      return (a.pos0 + b * atc::kRows + nq - 1) / atc::kKv + 1;
    };
    PrefillAttn t = a;
    int zmax = 1;
    t.tiles_per_split = 0;
    if (a.part && a.tickets) {
      long long total = 0;
      for (int b = 0; b < nqb; ++b) total += tiles_of(b);
      total *= a.n_heads;
      const long long slots = sm_count();
      t.tiles_per_split = (int)std::max(4ll, (total + slots - 1) / slots);
      for (int b = 0; b < nqb; ++b) {
        int per, splits;
        atc::split_plan(tiles_of(b), t.tiles_per_split, &per, &splits);
        zmax = std::max(zmax, splits);
      }
    }
    const dim3 tgrid(a.n_heads, nqb, zmax);
    attention_prefill_tc_kernel<<<tgrid, atc::kThreads, atc::kSmem, st>>>(t);
    return cudaGetLastError();
  }
  dim3 grid(a.n_heads, (a.m + 63) / 64);
  if (a.head_dim == 64) {
    attention_prefill_kernel<64><<<grid, 256, attention_prefill_smem<64>(), st>>>(a);
  } else if (a.head_dim == 128) {
    attention_prefill_kernel<128><<<grid, 256, attention_prefill_smem<128>(), st>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_weights_split(int qtype, const uint8_t* qs, const uint16_t* d, int rows, int kp,
                                 uint16_t* bhi, uint16_t* blo, float* cs, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  weights_split_kernel<<<rows, 256, 0, st>>>(qtype, qs, d, kp, bhi, blo, cs);
  return cudaGetLastError();
}

cudaError_t read_prefill_error(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_prefill_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *flags) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_prefill_error, &zero, sizeof(unsigned int));
  }
  return e;
}

}  // namespace dqmk

// ------------------------------------------------------------------ C ABI
using namespace dqmk;

extern "C" int dqmk_linear_batch_packed(int qtype, const float* x, int m, int in_features,
                                        const void* packed, int out_features, const float* bias,
                                        const float* residual, float* y, void* stream) {
  const char* api = qtype == DQMK_Q40 ? "CudaQ40Linear" : "CudaQ80Linear";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, "dqmk_linear_batch_packed: unsupported quant type");
  if (m <= 0 || in_features <= 0 || out_features <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape");
  if (!x || !packed || !y) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  if (reinterpret_cast<uintptr_t>(packed) & 15u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": packed weight must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int kp = (in_features + 31) / 32 * 32;
  const uint8_t* qs = static_cast<const uint8_t*>(packed);
  const size_t qbytes = (size_t)out_features * (qtype == DQMK_Q80 ? kp : kp / 2);
  const uint16_t* d = reinterpret_cast<const uint16_t*>(qs + qbytes);
  const GemmPlan plan = plan_gemm(m, out_features, kp);
  // stream-ordered scratch: fp16 activation planes and row scales, the fp16
  // weight planes and column scales, split-K partial sums
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t b_act = up((size_t)m * kp * 2), b_rs = up((size_t)m * 4);
  const size_t b_w = up((size_t)out_features * kp * 2), b_cs = up((size_t)out_features * 4);
  const size_t b_part = plan.splits > 1 ? up((size_t)plan.splits * m * out_features * 4) : 0;
  unsigned char* scratch = nullptr;
  DQMK_CUDA_RET(api, cudaMallocAsync(reinterpret_cast<void**>(&scratch),
                                     2 * b_act + b_rs + 2 * b_w + b_cs + b_part + 256, st));
  unsigned char* cur = scratch;
  auto take = [&](size_t b) {
    unsigned char* r = cur;
    cur += b;
    return r;
  };
  uint16_t* ahi = reinterpret_cast<uint16_t*>(take(b_act));
  uint16_t* alo = reinterpret_cast<uint16_t*>(take(b_act));
  float* rs = reinterpret_cast<float*>(take(b_rs));
  uint16_t* bhi = reinterpret_cast<uint16_t*>(take(b_w));
  uint16_t* blo = reinterpret_cast<uint16_t*>(take(b_w));
  float* cs = reinterpret_cast<float*>(take(b_cs));
  float* part = reinterpret_cast<float*>(take(b_part));
  int rc = DQMK_OK;
  cudaError_t e = cudaSuccess;
  CUtensorMap mahi, malo, mbhi, mblo;
  do {
    if ((rc = make_f16_tile_map(&mahi, ahi, m, kp))) break;
    if ((rc = make_f16_tile_map(&malo, alo, m, kp))) break;
    if ((rc = make_f16_tile_map(&mbhi, bhi, out_features, kp))) break;
    if ((rc = make_f16_tile_map(&mblo, blo, out_features, kp))) break;
    if ((e = launch_weights_split(qtype, qs, d, out_features, kp, bhi, blo, cs, st)) !=
        cudaSuccess)
      break;
    if ((e = launch_split_rows(x, m, in_features, kp, in_features, nullptr, 0.0f, ahi, alo, rs,
                               st)) != cudaSuccess)
      break;
    PrefillGemm g = {};
    g.m = m;
    g.n = out_features;
    g.kp = kp;
    g.rs = rs;
    g.cs = cs;
    g.plan = plan;
    g.partial = part;
    g.epi = kEpiStore;
    g.bias = bias;
    g.residual = residual;
    g.y = y;
    g.ldy = out_features;
    e = launch_prefill_gemm(mahi, malo, mbhi, mblo, g, st);
  } while (false);
  cudaError_t ef = cudaFreeAsync(scratch, st);
  if (rc) return rc;
  if (e == cudaSuccess) e = ef;
  if (e != cudaSuccess) return cuda_fail(api, e);
  return DQMK_OK;
}
