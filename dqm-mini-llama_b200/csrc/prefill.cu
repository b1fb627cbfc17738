// prefill.cu -- batched prefill on tcgen05 int8 tensor cores (sm_100a).
//
// ForwardBatch in the reference runs ForwardToken once per prompt token
// (src/batch.cc:35-40), re-reading every weight per token.  Here a prompt of M
// tokens runs each projection as one GEMM, C[M,N] = X[M,K] W[N,K]^T, with the
// Q8_0 / Q4_0 weights kept as int8 on the tensor cores:
//
//   * activations: each 32-value block of a row of X (after its RMSNorm) is
//     split into two int8 terms, x ~= s1 q1 + s2 q2 (s2 = s1/254; the
//     residual is below 1.6e-5 of the block's absmax), by quantize_rows;
//   * the GEMM: per 32-wide K block kb and term t one tcgen05.mma kind::i8
//     (M=128, N=128, K=32) computes the exact int32 block sums
//     P[m,n] = sum_j q_t[m,j] qW[n,j] into tensor memory (TMEM);
//   * per-block scale epilogue: four epilogue warps read each block's two
//     accumulators back (tcgen05.ld) and fold
//     acc[m,n] += dW[n,kb] (s1[m,kb] P1 + s2[m,kb] P2) into fp32 registers.
//     The weight scales differ per block, so int32 sums cannot run across
//     blocks; TMEM is double-buffered so the tensor core works on block kb+1
//     while block kb drains.
//   * operand tiles arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle,
//     no multicast) through a 3-stage shared-memory ring; one warp issues
//     TMA, one issues MMAs, four run the epilogue (warp specialisation), all
//     hand-offs on mbarriers with bounded waits.
// Epilogues mirror the decode GEMV's: residual add, SwiGLU of interleaved
// gate/up columns, QKV bias + RoPE + KV-cache store at each token's position.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "prefill.h"

namespace dqmk {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;  // BK in int8 elements (4 scale blocks)
constexpr int kStages = 3;
constexpr int kTileBytes = BM * BK;          // 16 KB per operand tile
constexpr int kStageBytes = 3 * kTileBytes;  // A term 0, A term 1, B
constexpr int kEpiWarps = 8;                 // two per TMEM lane quarter, 64 columns each
constexpr int kEpiCols = BN / 2;
constexpr int kGemmThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;          // 2 buffers x 2 terms x 128 columns
constexpr unsigned long long kWaitNs = 1000000000ull;

__device__ unsigned int g_prefill_error;  // bit 0: a bounded wait timed out

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; also gives up early once another role has aborted.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  if (bar_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  while (true) {
    if (bar_try(b, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > kWaitNs) {
      *abort = 1;
      atomicOr(&g_prefill_error, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

// K-major operand in a 128-byte-swizzled tile: rows of 128 bytes, 8-row atoms
// 1024 bytes apart (stride byte offset), version 1 (sm_100), layout
// SWIZZLE_128B.  The start address moves by 32 bytes per K=32 slice.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;            // leading byte offset (unused when swizzled)
  d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;            // descriptor version
  d |= (uint64_t)2u << 61;            // SWIZZLE_128B
  return d;
}

// kind::i8 instruction descriptor: s32 accumulate, signed int8 A and B, both
// K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a, uint64_t b) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(kIdesc), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   su32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// int32 in (-2^22, 2^22) -> float, exact, without the int->float unit
__device__ __forceinline__ float i2f_exact(uint32_t v) {
  return __int_as_float((int)v + 0x4B400000) - 12582912.0f;
}

__device__ __forceinline__ void prefill_epilogue(const PrefillGemm& p, int m, int n0,
                                                 const float (&acc)[kEpiCols]) {
  if (p.epi == kEpiStore) {
    float* yr = p.y + (size_t)m * p.ldy;
    const float* rr = p.residual ? p.residual + (size_t)m * p.ldy : nullptr;
#pragma unroll
    for (int c = 0; c < kEpiCols; ++c) {
      const int n = n0 + c;
      if (n < p.n) {
        float v = acc[c];
        if (p.bias) v = __fadd_rn(v, p.bias[n]);
        if (rr) v = __fadd_rn(rr[n], v);
        yr[n] = v;
      }
    }
  } else if (p.epi == kEpiSwiGlu) {
    float* yr = p.y + (size_t)m * p.ldy;
#pragma unroll
    for (int c = 0; c < kEpiCols; c += 2) {
      const int n = n0 + c;
      if (n + 1 < p.n) {
        const float g = acc[c], u = acc[c + 1];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
        yr[n / 2] = __fmul_rn(__fmul_rn(g, sig), u);
      }
    }
  } else {  // kEpiQkv
    const int pos = p.pos0 + m;
    const int half = p.head_dim / 2;
    const int q_pairs = p.n_heads * half;
    const int kv_pairs = p.n_kv_heads * half;
#pragma unroll
    for (int c = 0; c < kEpiCols; c += 2) {
      const int n = n0 + c;
      if (n + 1 >= p.n) continue;
      const int pp = n / 2;
      float x0 = acc[c], x1 = acc[c + 1];
      if (p.bias) {
        x0 = __fadd_rn(x0, p.bias[n]);
        x1 = __fadd_rn(x1, p.bias[n + 1]);
      }
      int seg_pair, nh;
      float* dst;
      bool rotate = true;
      if (pp < q_pairs) {
        seg_pair = pp;
        nh = p.n_heads;
        dst = p.q_out + (size_t)m * p.ldq;
      } else if (pp < q_pairs + kv_pairs) {
        seg_pair = pp - q_pairs;
        nh = p.n_kv_heads;
        dst = p.k_cache + ((size_t)p.layer * p.max_seq + pos) * nh * p.head_dim;
      } else {
        seg_pair = pp - q_pairs - kv_pairs;
        nh = p.n_kv_heads;
        dst = p.v_cache + ((size_t)p.layer * p.max_seq + pos) * nh * p.head_dim;
        rotate = false;
      }
      const int h = seg_pair / half, i = seg_pair % half;
      int o0, o1;
      if (rotate && p.neox) {
        o0 = h * p.head_dim + i;
        o1 = o0 + half;
      } else {
        o0 = h * p.head_dim + 2 * i;
        o1 = o0 + 1;
      }
      if (rotate) {
        const float2 cs = p.rope_cs[(size_t)pos * half + i];
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
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap map_a0,
                   const __grid_constant__ CUtensorMap map_a1,
                   const __grid_constant__ CUtensorMap map_b, const PrefillGemm p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], tfull[2], tempty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int nbk = p.kp / 32;
  const int ksteps = (nbk + 3) / 4;
  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
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
      for (int s = 0; s < ksteps; ++s) {
        const int st = s % kStages;
        if (s >= kStages && !bar_wait(&empty[st], (uint32_t)((s / kStages - 1) & 1), &abort_flag))
          break;
        unsigned char* base = tiles + (size_t)st * kStageBytes;
        bar_expect_tx(&full[st], kStageBytes);
        tma_load_2d(base, &map_a0, s * BK, m0, &full[st]);
        tma_load_2d(base + kTileBytes, &map_a1, s * BK, m0, &full[st]);
        tma_load_2d(base + 2 * kTileBytes, &map_b, s * BK, n0, &full[st]);
      }
      // tail: every stage's last release (an MMA commit) has landed before
      // the CTA may exit
      for (int s = ksteps > kStages ? ksteps - kStages : 0; s < ksteps && !abort_flag; ++s)
        if (!bar_wait(&empty[s % kStages], (uint32_t)((s / kStages) & 1), &abort_flag)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      int g = 0;
      for (int s = 0; s < ksteps && !abort_flag; ++s) {
        const int st = s % kStages;
        if (!bar_wait(&full[st], (uint32_t)((s / kStages) & 1), &abort_flag)) break;
        tc_fence_after();
        const uint32_t base = su32(tiles + (size_t)st * kStageBytes);
        for (int j = 0; j < 4; ++j) {
          const int kb = s * 4 + j;
          if (kb >= nbk) break;
          const int buf = g & 1;
          if (g >= 2 && !bar_wait(&tempty[buf], (uint32_t)((g / 2 - 1) & 1), &abort_flag)) break;
          tc_fence_after();
          const uint64_t bdesc = smem_desc(base + 2 * kTileBytes + j * 32);
          mma_i8(tmem + buf * 256 + 0, smem_desc(base + j * 32), bdesc);
          mma_i8(tmem + buf * 256 + 128, smem_desc(base + kTileBytes + j * 32), bdesc);
          mma_commit(&tfull[buf]);
          ++g;
        }
        mma_commit(&empty[st]);  // the stage is free once these MMAs finish
      }
    }
  } else {  // ---------------- epilogue warps 2..9: TMEM lanes 32*(warp%4) ..
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;    // which 64 columns of the tile
    const int ml = quarter * 32 + lane;  // tile row == TMEM lane
    const int m = m0 + ml;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + half * kEpiCols;
    float acc[kEpiCols];
#pragma unroll
    for (int c = 0; c < kEpiCols; ++c) acc[c] = 0.0f;
    const float* sx0 = p.sx + (size_t)m * nbk;
    const float* sx1 = p.sx + (size_t)(p.m_pad + m) * nbk;
    for (int kb = 0; kb < nbk; ++kb) {
      const int buf = kb & 1;
      // warp-uniform outcome: the TMEM loads below are .sync.aligned
      if (!__all_sync(0xffffffffu, bar_wait(&tfull[buf], (uint32_t)((kb >> 1) & 1), &abort_flag)))
        break;
      tc_fence_after();
      const float s0 = __ldg(sx0 + kb), s1 = __ldg(sx1 + kb);
      const float4* dw = reinterpret_cast<const float4*>(p.dwt + (size_t)kb * p.n + n0 + half * kEpiCols);
#pragma unroll
      for (int q = 0; q < kEpiCols / 16; ++q) {
        uint32_t r0[16], r1[16];
        tmem_ld16(trow + buf * 256 + q * 16, r0);
        tmem_ld16(trow + buf * 256 + 128 + q * 16, r1);
        tmem_wait_ld();
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const float4 w = __ldg(dw + q * 4 + j4);
          const float wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j4 * 4 + e;
            const float u = __fmaf_rn(i2f_exact(r1[j]), s1, __fmul_rn(i2f_exact(r0[j]), s0));
            acc[q * 16 + j] = __fmaf_rn(u, wv[e], acc[q * 16 + j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&tempty[buf]);
    }
    if (m < p.m && !abort_flag) prefill_epilogue(p, m, n0 + half * kEpiCols, acc);
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

// ----------------------------------------------------------- activations
// One CTA per token row: optional RMSNorm (src/ops.cc:68-90), then each
// 32-value block split into two int8 terms (see the file comment).  Writes
// q[t][row][kp] (zero past k) and s[t][row][nbk].
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ x, int k,
                                                            int kp, int ldx,
                                                            const float* __restrict__ norm_w,
                                                            float eps, int m_pad,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ s) {
  __shared__ float red[8];
  __shared__ float scale_s;
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* xr = x + (size_t)row * ldx;
  const int nbk = kp / 32;
  float scale = 1.0f;
  if (norm_w) {
    float ss = 0.0f;
    for (int e = tid; e < k; e += 256) ss = __fadd_rn(ss, __fmul_rn(xr[e], xr[e]));
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < 8; ++w) t += red[w];
      scale_s = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)k), eps)));
    }
    __syncthreads();
    scale = scale_s;
  }
  const int sub = tid & 7;
  for (int base = 0; base < nbk * 8; base += 256) {
    const int b = (base + tid) >> 3;
    const bool valid = b < nbk;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = b * 32 + sub * 4 + e;
      float val = (valid && col < k) ? xr[col] : 0.0f;
      if (norm_w && valid && col < k) val = __fmul_rn(__fmul_rn(val, scale), norm_w[col]);
      v[e] = val;
    }
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float inv = sc > 0.0f ? __frcp_rn(sc) : 0.0f;
      uint32_t packed = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int qq = __float2int_rn(__fmul_rn(v[e], inv));
        qq = qq > 127 ? 127 : (qq < -127 ? -127 : qq);
        v[e] = __fmaf_rn(-sc, (float)qq, v[e]);
        packed |= ((uint32_t)qq & 0xffu) << (8 * e);
      }
      if (valid) {
        reinterpret_cast<uint32_t*>(q + ((size_t)t * m_pad + row) * kp)[b * 8 + sub] = packed;
        if (sub == 0) s[((size_t)t * m_pad + row) * nbk + b] = sc;
      }
      sc = __fmul_rn(sc, 1.0f / 254.0f);
    }
  }
}

// Packed-row gather of M token embeddings (rows of the quantized token_embd).
__global__ void embed_rows_kernel(int qtype, const uint8_t* __restrict__ qs,
                                  const uint16_t* __restrict__ d, int dim, int kp,
                                  const int* __restrict__ tokens, float* __restrict__ y) {
  const int row = blockIdx.x;
  const int token = tokens[row];
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

// Causal GQA attention for a block of BQ consecutive query positions of one
// head, over cache positions 0 .. pos0 + m (flash-style online softmax).
template <int HD>
__global__ void __launch_bounds__(256) attention_prefill_kernel(PrefillAttn a) {
  constexpr int BQ = 32, BKV = 64, PAD = HD + 1;
  constexpr int DPT = HD / 8;  // output dims per thread
  extern __shared__ float sm[];
  float* sq = sm;                    // [BQ][PAD]
  float* sk = sq + BQ * PAD;         // [BKV][PAD]
  float* sv = sk + BKV * PAD;        // [BKV][HD]
  float* sp = sv + BKV * HD;         // [BQ][BKV]
  const int tid = threadIdx.x;
  const int h = blockIdx.x;
  const int q0 = blockIdx.y * BQ;
  const int G = a.n_heads / a.n_kv_heads;
  const int kvh = h / G;
  const size_t row_stride = (size_t)a.n_kv_heads * HD;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD;
  const int nq = min(BQ, a.m - q0);
  for (int i = tid; i < BQ * HD; i += 256) {
    const int r = i / HD, d = i % HD;
    sq[r * PAD + d] = r < nq ? a.q[(size_t)(q0 + r) * a.ldq + (size_t)h * HD + d] : 0.0f;
  }
  const int qi = tid >> 3;       // query row of this thread
  const int sub = tid & 7;       // score columns sub*8 .. +7 / output dims sub*DPT ..
  const int qpos = a.pos0 + q0 + qi;
  const int last = a.pos0 + q0 + nq - 1;
  const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
  float mrow = -INFINITY, lrow = 0.0f;
  float o[DPT];
#pragma unroll
  for (int e = 0; e < DPT; ++e) o[e] = 0.0f;
  for (int kt = 0; kt <= last; kt += BKV) {
    __syncthreads();
    for (int i = tid; i < BKV * HD; i += 256) {
      const int r = i / HD, d = i % HD;
      const int pos = kt + r;
      const bool ok = pos <= last;
      sk[r * PAD + d] = ok ? __ldcg(kbase + (size_t)pos * row_stride + d) : 0.0f;
      sv[r * HD + d] = ok ? __ldcg(vbase + (size_t)pos * row_stride + d) : 0.0f;
    }
    __syncthreads();
    float s[8];
    float tmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int j = sub * 8 + c;
      float dot = 0.0f;
#pragma unroll 16
      for (int d = 0; d < HD; ++d) dot = fmaf(sq[qi * PAD + d], sk[j * PAD + d], dot);
      const bool visible = qi < nq && kt + j <= qpos;
      s[c] = visible ? __fmul_rn(dot, scale) : -INFINITY;
      tmax = fmaxf(tmax, s[c]);
    }
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
    const float mnew = fmaxf(mrow, tmax);
    const float corr = mnew == -INFINITY ? 1.0f : expf(mrow - mnew);
    float psum = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float pv = s[c] == -INFINITY ? 0.0f : expf(s[c] - mnew);
      sp[qi * BKV + sub * 8 + c] = pv;
      psum += pv;
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    psum += __shfl_xor_sync(0xffffffffu, psum, 4);
    lrow = fmaf(lrow, corr, psum);
    mrow = mnew;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] *= corr;
    for (int j = 0; j < BKV; ++j) {
      const float pv = sp[qi * BKV + j];
#pragma unroll
      for (int e = 0; e < DPT; ++e) o[e] = fmaf(pv, sv[j * HD + sub * DPT + e], o[e]);
    }
  }
  if (qi < nq) {
    float* out = a.out + (size_t)(q0 + qi) * a.ldo + (size_t)h * HD + sub * DPT;
#pragma unroll
    for (int e = 0; e < DPT; ++e) out[e] = __fdiv_rn(o[e], lrow);
  }
}

// [N][nbk] fp16 scales -> [nbk][N] fp32 (the epilogue's per-block row of dW)
__global__ void transpose_scales_kernel(const uint16_t* __restrict__ d, int n, int nbk,
                                        float* __restrict__ out) {
  const size_t total = (size_t)n * nbk;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / nbk, kb = i % nbk;
    out[kb * n + row] = h2f(d[i]);
  }
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

}  // namespace

// [rows][kp] int8 matrix, 128 x 128-byte boxes, 128-byte swizzle.
int make_i8_tile_map(CUtensorMap* map, const void* base, int rows, int kp) {
  auto fn = encode_fn();
  if (!fn) return fail(DQMK_ERR_CUDA, "ForwardBatch: cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (kp % 16) != 0)
    return fail(DQMK_ERR_INVALID, "ForwardBatch: tensor map base or stride not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kp};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DQMK_ERR_CUDA, "ForwardBatch: cuTensorMapEncodeTiled failed (" +
                                   std::to_string((int)r) + ")");
  return DQMK_OK;
}

size_t prefill_gemm_smem() { return (size_t)kStages * kStageBytes + 1024; }

cudaError_t prefill_prepare() {
  static bool done = false;
  if (done) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)prefill_gemm_smem());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_prefill_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_prefill_kernel<128>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  if (e == cudaSuccess) done = true;
  return e;
}

cudaError_t launch_prefill_gemm(const CUtensorMap& a0, const CUtensorMap& a1,
                                const CUtensorMap& b, const PrefillGemm& p, cudaStream_t s) {
  cudaError_t e = prefill_prepare();
  if (e != cudaSuccess) return e;
  if (p.m <= 0 || p.m > p.m_pad || p.m_pad % BM != 0 || p.n % BN != 0 || p.kp % 32 != 0)
    return cudaErrorInvalidValue;
  dim3 grid(p.n / BN, (p.m + BM - 1) / BM);
  gemm_i8_kernel<<<grid, kGemmThreads, prefill_gemm_smem(), s>>>(a0, a1, b, p);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float* x, int m, int k, int kp, int ldx,
                                 const float* norm_w, float eps, int m_pad, int8_t* q, float* s,
                                 cudaStream_t st) {
  quantize_rows_kernel<<<m, 256, 0, st>>>(x, k, kp, ldx, norm_w, eps, m_pad, q, s);
  return cudaGetLastError();
}

cudaError_t launch_embed_rows(int qtype, const uint8_t* qs, const uint16_t* d, int dim, int kp,
                              const int* tokens, int m, float* y, cudaStream_t st) {
  embed_rows_kernel<<<m, 256, 0, st>>>(qtype, qs, d, dim, kp, tokens, y);
  return cudaGetLastError();
}

cudaError_t launch_attention_prefill(const PrefillAttn& a, cudaStream_t st) {
  cudaError_t e = prefill_prepare();
  if (e != cudaSuccess) return e;
  dim3 grid(a.n_heads, (a.m + 31) / 32);
  if (a.head_dim == 64) {
    const size_t smem = sizeof(float) * (32 * 65 + 64 * 65 + 64 * 64 + 32 * 64);
    attention_prefill_kernel<64><<<grid, 256, smem, st>>>(a);
  } else if (a.head_dim == 128) {
    const size_t smem = sizeof(float) * (32 * 129 + 64 * 129 + 64 * 128 + 32 * 64);
    attention_prefill_kernel<128><<<grid, 256, smem, st>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_transpose_scales(const uint16_t* d, int n, int nbk, float* out,
                                    cudaStream_t st) {
  transpose_scales_kernel<<<sm_count() * 4, 256, 0, st>>>(d, n, nbk, out);
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
