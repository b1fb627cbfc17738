// batch.cu -- decode of many sequences at once on tcgen05 tensor cores (sm_100a).
//
// The reference decodes one sequence at a time (ForwardToken,
// src/forward.cc:667-754), so every weight byte is read once per token.  With
// C sequences decoded together each weight is read once per step and used C
// times, and the projection becomes a skinny GEMM Y[c][row] = sum_k W[row][k]
// X[c][k] that belongs on the tensor cores.  Results stay within fp32
// summation-order differences of the F32 reference:
//
//   * weights stay in HBM as the packed Q8_0 / Q4_0 blocks of the decode GEMV
//     (the step streams the same bytes a batch-1 step would; the block scales
//     are read from a copy padded to 16-byte rows).  TMA brings a 256-row x
//     64-value tile of quants and its scales into a raw ring in shared memory;
//     eight dequant warps turn it into the exact two-term fp16 operand of the
//     prefill GEMM: with the row scaled by 2^-f (row maximum in
//     [2^14, 2^15)) every value d * q * 2^-f is exactly hi + lo,
//     hi = fp16(d' q), lo = fma(d', q, -hi) with d' = fp16(d * 2^-f) (exact),
//     computed in packed half arithmetic and stored straight into tensor
//     memory (tcgen05.st), where the MMA takes it as its A operand -- shared
//     memory carries only the raw tiles and the activation tiles;
//   * activations: each column (after its RMSNorm) is split into two fp16
//     planes by the prefill's split kernel and arrives by TMA;
//   * tcgen05.mma kind::f16, M = 128 weight rows (two per 256-row tile), N =
//     the columns rounded up to 16, K = 16: W_hi X_hi + W_hi X_lo + W_lo X_hi
//     accumulate in TMEM (fp32) over the tile's K range;
//   * split-K where row tiles are few: each split parks its raw sums and a
//     reduce kernel over the whole grid adds them in split order
//     (deterministic) and runs the epilogue;
//   * epilogues: residual add, SwiGLU of interleaved gate/up rows, QKV bias +
//     RoPE + KV-cache store at each column's (slot, position), logits with a
//     per-column argmax key (value, first index) combined by atomicMax.
// Warp roles: 0 TMA, 1 MMA issue, 2-5 epilogue (one TMEM lane quarter each),
// 6-13 dequant (one weight row each).  TMEM: two accumulators (256 columns)
// and two weight-operand stages (256 columns).  Every hand-off is an mbarrier with a
// bounded wait; a wait that runs out sets a device flag and the CTA unwinds
// (its own copies in flight land first, TMEM is freed).  Under programmatic
// dependent launch the weight copies and their dequantization start before the
// previous kernel has finished; only activation loads and the epilogue wait.
#include <cuda_fp16.h>

#include <algorithm>
#include <string>

#include "attention_dev.cuh"
#include "batch.h"
#include "common.cuh"
#include "dqmk.h"
#include "internal.h"
#include "tc_dev.cuh"

namespace dqmk {
namespace {

constexpr int kTileRows = 256;                             // weight rows per work item
constexpr int kHalfRows = 128;                             // rows per MMA (M)
constexpr int kChunkK = 64;                                // K values per stage
#ifndef DQMK_BATCH_RAW_STAGES
#define DQMK_BATCH_RAW_STAGES 4
#endif
#ifndef DQMK_BATCH_A_STAGES
#define DQMK_BATCH_A_STAGES 2
#endif
#ifndef DQMK_BATCH_ACC_BUFS
#define DQMK_BATCH_ACC_BUFS 2
#endif
#ifndef DQMK_BATCH_EPI_SLEEP
#define DQMK_BATCH_EPI_SLEEP 128
#endif
constexpr int kRawStages = DQMK_BATCH_RAW_STAGES;          // quant tiles (shared memory)
constexpr int kXStages = 8;                                // activation tiles (shared memory)
constexpr int kAStages = DQMK_BATCH_A_STAGES;              // weight operand tiles (TMEM)
constexpr int kXPlaneBytes = kBatchMaxCols * kChunkK * 2;  // 8 KB
constexpr int kXStageBytes = 2 * kXPlaneBytes;             // hi + lo
constexpr int kEpiWarps = 4, kDeqWarps = 8;
constexpr int kFirstEpiWarp = 2, kFirstDeqWarp = kFirstEpiWarp + kEpiWarps;
constexpr int kThreads = (kFirstDeqWarp + kDeqWarps) * 32;
constexpr int kAccBufs = DQMK_BATCH_ACC_BUFS;
// TMEM columns: accumulators [buffer][half][64 columns], then the weight
// operand stages [stage][half][hi 32 | lo 32] (two fp16 per column)
constexpr uint32_t kAccCols = 2 * kBatchMaxCols;
constexpr uint32_t kACol0 = kAccBufs * kAccCols;           // 256
constexpr uint32_t kAStageCols = 2 * 2 * (kChunkK / 2);    // 128
constexpr uint32_t kTmemNeed = kACol0 + kAStages * kAStageCols;  // 512
constexpr uint32_t kTmemCols = kTmemNeed <= 256 ? 256 : 512;
static_assert(kTmemNeed <= 512, "at most the whole tensor memory of the SM");
static_assert(kDeqWarps * 32 == kTileRows, "one dequant thread per tile row");

__device__ unsigned int g_batch_error;  // kErrTimeout / kErrNoToken

template <int QT>
constexpr int raw_row_bytes() {
  return QT == DQMK_Q80 ? kChunkK : kChunkK / 2;
}
// A raw stage: the quants of 256 rows x 64 values, then each row's group of
// 8 block scales (16 bytes) that holds the stage's two blocks.
template <int QT>
constexpr int raw_scale_off() {
  return kTileRows * raw_row_bytes<QT>();
}
template <int QT>
constexpr int raw_stage_bytes() {
  return kTileRows * (raw_row_bytes<QT>() + 16);
}
template <int QT>
constexpr size_t gemm_smem() {
  return 1024 + (size_t)kXStages * kXStageBytes + (size_t)kRawStages * raw_stage_bytes<QT>();
}

__device__ __forceinline__ bool wait(uint64_t* b, uint32_t parity, volatile int* abort,
                                     unsigned sleep_ns = 0) {
  return tc::bar_wait(b, parity, abort, &g_batch_error, sleep_ns);
}
// Bounded wait that ignores the abort flag: a CTA lets its own copies land
// before it exits.
__device__ __forceinline__ void wait_landed(uint64_t* b, uint32_t parity) {
  volatile int never = 0;
  tc::bar_wait(b, parity, &never, &g_batch_error);
}

// Work item w -> (row tile, K split, chunk range).  The splits of one tile
// are consecutive items, so they run at the same time.
struct Item {
  int tile, z, c0, c1;
};
__device__ __forceinline__ Item item_of(const BatchGemm& p, int w) {
  Item t;
  t.tile = w / p.plan.splits;
  t.z = w % p.plan.splits;
  const int nb = p.kp / 32;
  const int kb0 = t.z * p.plan.kb_per;
  const int kb1 = min(nb, kb0 + p.plan.kb_per);
  t.c0 = kb0 / 2;
  t.c1 = (kb1 + 1) / 2;
  return t;
}

// The CTA's chunks in order (items blockIdx.x, + gridDim.x, ...).
struct Walk {
  int w, c, total;
  Item t;
  bool valid;
  __device__ __forceinline__ void begin(const BatchGemm& p, int n_items) {
    total = n_items;
    w = blockIdx.x;
    valid = w < total;
    if (valid) {
      t = item_of(p, w);
      c = t.c0;
    }
  }
  __device__ __forceinline__ void next(const BatchGemm& p) {
    if (++c < t.c1) return;
    w += gridDim.x;
    valid = w < total;
    if (valid) {
      t = item_of(p, w);
      c = t.c0;
    }
  }
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Two exact fp16 terms of t * s (t a small integer held exactly in fp16, s
// an fp16 power-of-two-scaled block scale): hi rounded, lo the exact rest.
__device__ __forceinline__ void two_term(__half2 t, __half2 s, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __hmul2_rn(t, s);
  const __half2 l = __hfma2(t, s, __hneg2(h));
  hi = h2u(h);
  lo = h2u(l);
}

// Q4_0 block (16 bytes: byte i holds value i in its low nibble and value
// i + 16 in its high nibble, src/quant.cc:160-175) -> its 32 values as 16
// hi / lo pairs in K order (h[m] = values 2m, 2m+1).
__device__ __forceinline__ void dequant_q4_block(uint4 q, __half2 s, uint32_t* h, uint32_t* l) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  const __half2 off = __half2half2(__ushort_as_half(0x6408));  // 1032 = 1024 + 8
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo4 = w[i] & 0x0F0F0F0Fu, hi4 = (w[i] >> 4) & 0x0F0F0F0Fu;
    // values 4i, 4i+1 | 4i+2, 4i+3 (low nibbles) and 16+4i .. 16+4i+3 (high)
    two_term(__hsub2(u2h(prmt(lo4, 0x64646464u, 0x4140u)), off), s, h[2 * i], l[2 * i]);
    two_term(__hsub2(u2h(prmt(lo4, 0x64646464u, 0x4342u)), off), s, h[2 * i + 1], l[2 * i + 1]);
    two_term(__hsub2(u2h(prmt(hi4, 0x64646464u, 0x4140u)), off), s, h[8 + 2 * i], l[8 + 2 * i]);
    two_term(__hsub2(u2h(prmt(hi4, 0x64646464u, 0x4342u)), off), s, h[9 + 2 * i], l[9 + 2 * i]);
  }
}

// 16 Q8_0 values (int8, in order) -> 8 hi / lo pairs in K order.
__device__ __forceinline__ void dequant_q8_16(uint4 q, __half2 s, uint32_t* h, uint32_t* l) {
  const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                         q.w ^ 0x80808080u};
  const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152 = 1024 + 128
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    two_term(__hsub2(u2h(prmt(w[i], 0x64646464u, 0x4140u)), off), s, h[2 * i], l[2 * i]);
    two_term(__hsub2(u2h(prmt(w[i], 0x64646464u, 0x4342u)), off), s, h[2 * i + 1], l[2 * i + 1]);
  }
}

// fp16 block scale d times the row's 2^-f, as a broadcast half2 (exact: a
// power-of-two multiple of an fp16 value, at most 2^15 / |q|max).
__device__ __forceinline__ __half2 block_scale(uint32_t d_bits, float inv_cs) {
  const float v = __fmul_rn(__half2float(__ushort_as_half((unsigned short)d_bits)), inv_cs);
  return __half2half2(__float2half_rn(v));
}

// ------------------------------------------------------------------ epilogue
// Per-column data of the step, staged once per CTA.
struct ColInfo {
  float rs[kBatchMaxCols];
  int pos[kBatchMaxCols];
  int slot[kBatchMaxCols];
};

// Row `row` (this thread's TMEM lane) and columns cb .. cb+NC-1 of finished
// sums v (raw accumulator values): scale by rs[c] * cs[row] (exact powers of
// two), then the epilogue.  Every lane of the warp calls this together with
// consecutive rows on consecutive lanes (the paired epilogues exchange values
// with the neighbouring lane).
template <int NC>
__device__ __forceinline__ void finish(const BatchGemm& p, const ColInfo& ci, int row, int cb,
                                       float (&v)[NC]) {
  constexpr int G = NC < 8 ? NC : 8;  // columns per load batch
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const bool ok = row < p.n;
  const float c = ok ? __ldg(p.cs + row) : 0.0f;
#pragma unroll
  for (int j = 0; j < NC; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], ci.rs[(cb + j) & 63]), c);
  const int ncol = min(NC, p.cols - cb);  // valid columns of this group
  if (p.epi == kEpiStore) {
    if (!ok) return;
    const float b = p.bias ? __ldg(p.bias + row) : 0.0f;
#pragma unroll
    for (int g = 0; g < NC / G; ++g) {  // loads of a batch first, then its stores
      float r[G];
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int j = G * g + u;
        // the residual is the previous kernel's output: read through L2
        r[u] = (p.residual && j < ncol) ? __ldcg(p.residual + (size_t)(cb + j) * p.ldy + row) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int j = G * g + u;
        if (j < ncol) {
          float x = p.bias ? __fadd_rn(v[j], b) : v[j];
          if (p.residual) x = __fadd_rn(r[u], x);
          p.y[(size_t)(cb + j) * p.ldy + row] = x;
        }
      }
    }
  } else if (p.epi == kEpiSwiGlu) {
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      const float u = __shfl_down_sync(full, v[j], 1);
      if (ok && !(lane & 1) && j < ncol) {
        const float g = v[j];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
        p.y[(size_t)(cb + j) * p.ldy + row / 2] = __fmul_rn(__fmul_rn(g, sig), u);
      }
    }
  } else if (p.epi == kEpiQkv) {
    const float b = (ok && p.bias) ? __ldg(p.bias + row) : 0.0f;
    const int half = p.head_dim / 2;
    const int q_pairs = p.n_heads * half, kv_pairs = p.n_kv_heads * half;
    const int pp = row / 2;
    const bool is_q = pp < q_pairs, is_k = !is_q && pp < q_pairs + kv_pairs;
    const bool rotate = is_q || is_k;
    const int seg = is_q ? pp : (is_k ? pp - q_pairs : pp - q_pairs - kv_pairs);
    const int hh = seg / half, i = seg % half;
    int o0, o1;
    if (rotate && p.neox) {
      o0 = hh * p.head_dim + i;
      o1 = o0 + half;
    } else {
      o0 = hh * p.head_dim + 2 * i;
      o1 = o0 + 1;
    }
    const int kvd = p.n_kv_heads * p.head_dim;
    const bool writer = ok && !(lane & 1);
#pragma unroll
    for (int g = 0; g < NC / G; ++g) {
      float a[G], bb[G];
      float2 rc[G];
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int j = G * g + u;
        a[u] = p.bias ? __fadd_rn(v[j], b) : v[j];
        bb[u] = __shfl_down_sync(full, a[u], 1);
        rc[u] = (writer && rotate && j < ncol)
                    ? __ldg(p.rope_cs + (size_t)ci.pos[cb + j] * half + i)
                    : make_float2(1.0f, 0.0f);
      }
      if (!writer) continue;
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int j = G * g + u;
        if (j >= ncol) continue;
        float x0 = a[u], x1 = bb[u];
        if (rotate) {
          const float2 cs = rc[u];
          if (p.neox) {
            x0 = __fmaf_rn(a[u], cs.x, -__fmul_rn(bb[u], cs.y));
            x1 = __fmaf_rn(a[u], cs.y, __fmul_rn(bb[u], cs.x));
          } else {
            x0 = __fsub_rn(__fmul_rn(a[u], cs.x), __fmul_rn(bb[u], cs.y));
            x1 = __fadd_rn(__fmul_rn(a[u], cs.y), __fmul_rn(bb[u], cs.x));
          }
        }
        const int col = cb + j;
        float* dst;
        if (is_q) {
          dst = p.q_out + (size_t)col * p.ldq;
        } else {
          float* cache = is_k ? p.k_cache : p.v_cache;
          dst = cache + (size_t)ci.slot[col] * p.slot_stride +
                ((size_t)p.layer * p.max_seq + ci.pos[col]) * kvd;
        }
        dst[o0] = x0;
        dst[o1] = x1;
      }
    }
  } else {  // kEpiLogits
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      if (ok && p.y && j < ncol) p.y[(size_t)(cb + j) * p.ldy + row] = v[j];
      unsigned long long k = ok ? argmax_key(v[j], (uint32_t)(row + p.row_offset)) : 0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(full, k, o);
        k = other > k ? other : k;
      }
      if (lane == 0 && j < ncol) atomicMax(p.keys + cb + j, k);
    }
  }
}

__device__ __forceinline__ void stage_cols(const BatchGemm& p, ColInfo& ci, int tid, int nthreads) {
  for (int c = tid; c < kBatchMaxCols; c += nthreads) {
    const bool v = c < p.cols;
    ci.rs[c] = v ? p.rs[c] : 0.0f;
    ci.pos[c] = v && p.col_pos ? p.col_pos[c] : 0;
    ci.slot[c] = v && p.col_slot ? p.col_slot[c] : 0;
  }
}

// Split-K: sum of the splits' raw sums (partial[z][column][row]) in split
// order, then the epilogue.  Thread (row = 32 * blockIdx.x + lane, columns
// 4 * (8 * blockIdx.y + warp) .. + 3): all splits' loads of a batch of 8 are in
// flight at once, lanes read consecutive rows (coalesced).
constexpr int kReduceCols = 4;
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const BatchGemm p) {
  __shared__ ColInfo ci;
  pdl_trigger();
  pdl_wait();
  stage_cols(p, ci, threadIdx.x, blockDim.x);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 32 + lane;
  const int c0 = (blockIdx.y * 8 + warp) * kReduceCols;
  if (c0 >= p.cols) return;  // warp-uniform
  const int rowc = row < p.n ? row : p.n - 1;
  float v[kReduceCols];
#pragma unroll
  for (int j = 0; j < kReduceCols; ++j) v[j] = 0.0f;
  for (int z0 = 0; z0 < p.plan.splits; z0 += 8) {
    float t[8][kReduceCols];
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int j = 0; j < kReduceCols; ++j)
        t[u][j] = z0 + u < p.plan.splits
                      ? __ldcg(p.partial + ((size_t)(z0 + u) * kBatchMaxCols + c0 + j) * p.n + rowc)
                      : 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (z0 + u < p.plan.splits)
#pragma unroll
        for (int j = 0; j < kReduceCols; ++j) v[j] = __fadd_rn(v[j], t[u][j]);
  }
  finish<kReduceCols>(p, ci, row, c0, v);
}

// ------------------------------------------------------------------- kernel
template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    batch_gemm_kernel(const __grid_constant__ CUtensorMap map_w,
                      const __grid_constant__ CUtensorMap map_d,
                      const __grid_constant__ CUtensorMap map_xhi,
                      const __grid_constant__ CUtensorMap map_xlo, const BatchGemm p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  __shared__ __align__(8) uint64_t x_full[kXStages], x_empty[kXStages];
  __shared__ __align__(8) uint64_t a_full[kAStages], a_empty[kAStages];
  __shared__ __align__(8) uint64_t acc_full[kAccBufs], acc_empty[kAccBufs], mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ ColInfo ci;

  constexpr int RB = raw_row_bytes<QT>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (p.n + kTileRows - 1) / kTileRows;
  const int n_items = n_tiles * p.plan.splits;
  const int n_mma = (p.cols + 15) / 16 * 16;
  unsigned char* xs = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  unsigned char* raws = xs + (size_t)kXStages * kXStageBytes;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      tc::bar_init(&raw_full[s], 1);
      tc::bar_init(&raw_empty[s], kDeqWarps);
    }
    for (int s = 0; s < kXStages; ++s) {
      tc::bar_init(&x_full[s], 1);
      tc::bar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) {
      tc::bar_init(&a_full[s], kDeqWarps);
      tc::bar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      tc::bar_init(&acc_full[b], 1);
      tc::bar_init(&acc_empty[b], kEpiWarps);
    }
    tc::bar_init(&mma_done, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::tma_prefetch_desc(&map_w);
    tc::tma_prefetch_desc(&map_d);
    tc::tma_prefetch_desc(&map_xhi);
    tc::tma_prefetch_desc(&map_xlo);
  }
  if (warp == 1) tc::tmem_alloc(&tmem_slot, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------- TMA producer
      Walk rw, xw;
      rw.begin(p, n_items);
      xw.begin(p, n_items);
      int gr = 0, gx = 0;
      auto issue_raw = [&]() {
        const int st = gr % kRawStages;
        unsigned char* dst = raws + (size_t)st * raw_stage_bytes<QT>();
        tc::bar_expect_tx(&raw_full[st], (uint32_t)raw_stage_bytes<QT>());
        tc::tma_load_2d(dst, &map_w, rw.c * RB, rw.t.tile * kTileRows, &raw_full[st]);
        tc::tma_load_2d(dst + raw_scale_off<QT>(), &map_d, (2 * rw.c) & ~7, rw.t.tile * kTileRows,
                        &raw_full[st]);
        rw.next(p);
        ++gr;
      };
      // weight tiles do not depend on the previous kernel: start them first
      while (rw.valid && gr < kRawStages) issue_raw();
      pdl_wait();
      // Both rings are kept as full as their consumers allow, independently:
      // the activation tiles (the same for every CTA, so slow to arrive from
      // L2) run up to kXStages chunks ahead of the MMA, the quant tiles
      // kRawStages ahead of the dequant warps.  Non-blocking polls; no
      // progress for about a second records the timeout and unwinds.
      unsigned long long idle_since = 0;
      while ((rw.valid || xw.valid) && !abort_flag) {
        bool progressed = false;
        if (rw.valid && tc::bar_try(&raw_empty[gr % kRawStages],
                                    (uint32_t)((gr / kRawStages - 1) & 1))) {
          issue_raw();
          progressed = true;
        }
        if (xw.valid && (gx < kXStages || tc::bar_try(&x_empty[gx % kXStages],
                                                      (uint32_t)((gx / kXStages - 1) & 1)))) {
          const int xs_ = gx % kXStages;
          unsigned char* st = xs + (size_t)xs_ * kXStageBytes;
          tc::bar_expect_tx(&x_full[xs_], (uint32_t)kXStageBytes);
          tc::tma_load_2d(st, &map_xhi, xw.c * kChunkK, 0, &x_full[xs_]);
          tc::tma_load_2d(st + kXPlaneBytes, &map_xlo, xw.c * kChunkK, 0, &x_full[xs_]);
          xw.next(p);
          ++gx;
          progressed = true;
        }
        if (progressed) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = tc::now_ns();
        } else if (tc::now_ns() - idle_since > tc::kWaitNs) {
          abort_flag = 1;
          atomicOr(&g_batch_error, 1u);
        }
      }
      if (abort_flag) {  // let this thread's copies in flight land before exit
        for (int g = gr - kRawStages < 0 ? 0 : gr - kRawStages; g < gr; ++g)
          wait_landed(&raw_full[g % kRawStages], (uint32_t)((g / kRawStages) & 1));
        for (int g = gx - kXStages < 0 ? 0 : gx - kXStages; g < gx; ++g)
          wait_landed(&x_full[g % kXStages], (uint32_t)((g / kXStages) & 1));
      }
    }
  } else if (warp == 1) {  // ------------------------------------------ MMA issue
    // The whole warp runs the loop (operands stay warp-uniform); one elected
    // lane issues the tcgen05 instructions; every wait decision is voted so
    // the warp stays converged.
    const uint32_t idesc = tc::idesc_f16(kHalfRows, n_mma);
    int g = 0, tcnt = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++tcnt) {
      const Item it = item_of(p, w);
      const int buf = tcnt % kAccBufs;
      if (tcnt >= kAccBufs)
        ok = __all_sync(0xffffffffu,
                        wait(&acc_empty[buf], (uint32_t)((tcnt / kAccBufs - 1) & 1), &abort_flag));
      if (!ok) break;
      tc::tc_fence_after();
      const uint32_t dacc = tmem + (uint32_t)(buf * kAccCols);
      for (int c = it.c0; c < it.c1; ++c, ++g) {
        const int as = g % kAStages, xs_ = g % kXStages;
        ok = __all_sync(0xffffffffu,
                        wait(&a_full[as], (uint32_t)((g / kAStages) & 1), &abort_flag) &&
                            wait(&x_full[xs_], (uint32_t)((g / kXStages) & 1), &abort_flag));
        if (!ok) break;
        tc::tc_fence_after();
        const uint64_t bhi0 = tc::smem_desc(tc::su32(xs + (size_t)xs_ * kXStageBytes));
        const uint64_t blo0 = tc::smem_desc(tc::su32(xs + (size_t)xs_ * kXStageBytes + kXPlaneBytes));
        const uint32_t acol = tmem + kACol0 + (uint32_t)as * kAStageCols;
        const uint32_t first = c > it.c0 ? 1u : 0u;
        if (tc::elect_one()) {
#pragma unroll
          for (int k = 0; k < kChunkK / 16; ++k) {
            // a K=16 slice is 32 bytes further: +2 in the descriptor's address field
            const uint64_t bhi = bhi0 + 2u * k, blo = blo0 + 2u * k;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t d = dacc + (uint32_t)(h * kBatchMaxCols);
              const uint32_t ahi = acol + (uint32_t)(h * 64 + 8 * k);
              tc::mma_f16_ts(d, ahi, bhi, idesc, k > 0 ? 1u : first);
              tc::mma_f16_ts(d, ahi, blo, idesc, 1u);
              tc::mma_f16_ts(d, ahi + 32, bhi, idesc, 1u);
            }
          }
          // the operand stages are free once these MMAs finish
          tc::mma_commit(&a_empty[as]);
          tc::mma_commit(&x_empty[xs_]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (tc::elect_one()) tc::mma_commit(&acc_full[buf]);
      __syncwarp();
    }
    // every MMA this warp issued has finished before TMEM is freed
    if (tc::elect_one()) tc::mma_commit(&mma_done);
    __syncwarp();
    wait_landed(&mma_done, 0u);
  } else if (warp >= kFirstDeqWarp) {  // ------------------------------- dequant
    // one weight row per thread: half (0: warps 6-9, 1: warps 10-13), TMEM
    // lane quarter warp % 4
    const int half = (warp - kFirstDeqWarp) / 4, quarter = warp & 3;
    const int t = half * kHalfRows + 32 * quarter + lane;  // tile row
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
    int g = 0;
    for (int w = blockIdx.x; w < n_items && !abort_flag; w += gridDim.x) {
      const Item it = item_of(p, w);
      const int row = it.tile * kTileRows + t;
      const bool ok = row < p.n;
      const float inv = ok ? __frcp_rn(__ldg(p.cs + row)) : 0.0f;
      bool okw = true;
      for (int c = it.c0; c < it.c1; ++c, ++g) {
        const int rs_ = g % kRawStages, as = g % kAStages;
        // waits are voted: the tcgen05 stores below are warp-wide
        if (!__all_sync(0xffffffffu,
                        wait(&raw_full[rs_], (uint32_t)((g / kRawStages) & 1), &abort_flag))) {
          okw = false;
          break;
        }
        const unsigned char* stage = raws + (size_t)rs_ * raw_stage_bytes<QT>();
        const uint4* q = reinterpret_cast<const uint4*>(stage + (size_t)t * RB);
        const uint16_t* sr = reinterpret_cast<const uint16_t*>(stage + raw_scale_off<QT>() + t * 16);
        uint4 qv[RB / 16];
#pragma unroll
        for (int i = 0; i < RB / 16; ++i) qv[i] = q[i];
        const __half2 s_a = block_scale(sr[(2 * c) & 7], inv),
                      s_b = block_scale(sr[(2 * c + 1) & 7], inv);
        uint32_t hv[32], lv[32];
        if constexpr (QT == DQMK_Q80) {
          dequant_q8_16(qv[0], s_a, hv, lv);
          dequant_q8_16(qv[1], s_a, hv + 8, lv + 8);
          dequant_q8_16(qv[2], s_b, hv + 16, lv + 16);
          dequant_q8_16(qv[3], s_b, hv + 24, lv + 24);
        } else {
          dequant_q4_block(qv[0], s_a, hv, lv);
          dequant_q4_block(qv[1], s_b, hv + 16, lv + 16);
        }
        // The raw stage is released only once every lane's reads of it have
        // returned (the values above depend on them) and are ordered before
        // the next TMA write into it: a thread read followed by an async-proxy
        // write of the same shared memory.
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::bar_arrive(&raw_empty[rs_]);
        if (g >= kAStages &&
            !__all_sync(0xffffffffu,
                        wait(&a_empty[as], (uint32_t)((g / kAStages - 1) & 1), &abort_flag))) {
          okw = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t col = tmem + lane_base + kACol0 + (uint32_t)as * kAStageCols +
                             (uint32_t)(half * 64);
        tc::tmem_st32(col, hv);
        tc::tmem_st32(col + 32, lv);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::bar_arrive(&a_full[as]);
      }
      if (!okw) break;
    }
  } else {  // ---------------------------------------- epilogue warps 2..5
    const int et = threadIdx.x - kFirstEpiWarp * 32;
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter ..
    pdl_wait();
    stage_cols(p, ci, et, kEpiWarps * 32);
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
    int tcnt = 0;
    for (int w = blockIdx.x; w < n_items && !abort_flag; w += gridDim.x, ++tcnt) {
      const Item it = item_of(p, w);
      const int buf = tcnt % kAccBufs;
      // voted: the tensor-memory loads below are warp-wide
      if (!__all_sync(0xffffffffu, wait(&acc_full[buf], (uint32_t)((tcnt / kAccBufs) & 1),
                                        &abort_flag, DQMK_BATCH_EPI_SLEEP)))
        break;
      tc::tc_fence_after();
      const bool split = p.plan.splits > 1;
      for (int h = 0; h < 2; ++h) {
        const int row = it.tile * kTileRows + h * kHalfRows + 32 * quarter + lane;
        for (int cb = 0; cb < n_mma; cb += 32) {
          uint32_t r[32];
          tc::tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) +
                            (uint32_t)(buf * kAccCols + h * kBatchMaxCols + cb),
                        r);
          tc::tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (split) {  // raw sums, column-major [z][column][row]
            if (row < p.n) {
              float* dst = p.partial + ((size_t)it.z * kBatchMaxCols + cb) * p.n + row;
#pragma unroll
              for (int j = 0; j < 32; ++j) __stcg(dst + (size_t)j * p.n, v[j]);
            }
          } else {
            finish<32>(p, ci, row, cb, v);
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::bar_arrive(&acc_empty[buf]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) tc::tmem_free(tmem, kTmemCols);
}

// ------------------------------------------------------------- side kernels
// One CTA per weight row: cs[row] = 2^f with the row's max |d q| 2^-f in
// [2^14, 2^15) -- the scaling of the prefill's two-term weight planes.
__global__ void __launch_bounds__(256) row_scales_kernel(int qtype, const uint8_t* __restrict__ qs,
                                                         const uint16_t* __restrict__ d, int kp,
                                                         float* __restrict__ cs) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  const int nb = kp / 32;
  const uint16_t* dr = d + (size_t)row * nb;
  const uint8_t* qr = qs + (size_t)row * (qtype == DQMK_Q80 ? kp : kp / 2);
  float mx = 0.0f;
  for (int e = tid; e < kp; e += 256) {
    int q;
    if (qtype == DQMK_Q80) {
      q = (int)(int8_t)qr[e];
    } else {
      const int j = e & 31;
      const uint8_t byte = qr[(e >> 5) * 16 + (j & 15)];
      q = (int)(j < 16 ? (byte & 0x0f) : (byte >> 4)) - 8;
    }
    mx = fmaxf(mx, fabsf(__fmul_rn(h2f(dr[e >> 5]), (float)q)));
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    int ex = 0;
    if (m > 0.0f && m <= 3.0e38f) {
      int fe;
      frexpf(m, &fe);  // m in [2^(fe-1), 2^fe)
      ex = min(max(fe - 15, -120), 120);
    }
    cs[row] = ldexpf(1.0f, ex);
  }
}

// Decode attention of column blockIdx.z: the single-sequence body over the
// column's slot cache and position.
template <int HD>
__global__ void __launch_bounds__(256) attention_cols_kernel(const BatchAttn b, int chunk_cap) {
  extern __shared__ float sm[];
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.z;
  const size_t so = (size_t)__ldg(b.col_slot + c) * b.slot_stride;
  AttnArgs a = {};
  a.q = b.q + (size_t)c * b.ldq;
  a.out = b.out + (size_t)c * b.ldq;
  a.keys = b.keys + so;
  a.values = b.values + so;
  a.max_seq = b.max_seq;
  a.n_kv_heads = b.n_kv_heads;
  a.head_dim = HD;
  a.layer = b.layer;
  a.n_heads = b.n_heads;
  a.pos_dev = b.col_pos + c;
  a.partials = b.partials + (size_t)c * b.n_heads * b.max_splits * at::part_stride(HD);
  a.tickets = b.tickets + (size_t)c * b.n_kv_heads;
  a.max_splits = b.max_splits;
  at::attention_hd_body<HD, 256>(a, chunk_cap, blockIdx.x, blockIdx.y, gridDim.y, sm);
}

// Decode attention of one (column, KV head, split), head_dim 128 and G query
// heads per KV head, in one pass over the split's positions.  Four warps take
// 4-position steps in turn (warp w: steps w, w + 4, ...); lane l owns dims
// 4l..4l+3 of every K / V row.  Each lane streams its own 16-byte slices of
// the rows into a private ring in shared memory with cp.async (kStreamDepth
// steps ahead, zero-filled past the split's end), so a warp keeps 16 KB of
// the cache in flight without holding it in registers.  Per step: the 4 x 8
// partial dots are summed by a transposed butterfly that leaves lane l with
// the score of position l / 8, head l % 8; an online softmax per head
// (running max and sum, the accumulators rescaled when the max moves); p and
// the rescale factors go through shared memory to every lane for P.V.  The
// warps' states are merged in the CTA, then across splits by the same
// last-CTA combine as the other decode attention kernels.
constexpr int kStreamWarps = 4, kStreamDepth = 4, kStreamPos = 4;
constexpr size_t kStreamRingBytes =
    (size_t)kStreamWarps * kStreamDepth * 2 * kStreamPos * 32 * sizeof(float4);  // 64 KB
constexpr size_t kStreamPBytes = (size_t)kStreamWarps * 48 * sizeof(float);

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ unsigned long long fmul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <int G>
__global__ void __launch_bounds__(kStreamWarps * 32, 3)
    attention_cols_stream_kernel(const BatchAttn b) {
  constexpr int HD = 128, NW = kStreamWarps, D = kStreamDepth, P = kStreamPos;
  constexpr int PS = at::part_stride(HD);
  static_assert(G >= 1 && G <= at::kMaxGroup, "query heads per KV head");
  extern __shared__ __align__(16) unsigned char smem_s[];
  float4* ring = reinterpret_cast<float4*>(smem_s);                       // [NW][D][2][P][32]
  float* pbuf = reinterpret_cast<float*>(smem_s + kStreamRingBytes);      // [NW][48]
  __shared__ int is_last;
  pdl_trigger();
  pdl_wait();

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int c = blockIdx.z, kvh = blockIdx.x, split = blockIdx.y;
  const size_t so = (size_t)__ldg(b.col_slot + c) * b.slot_stride;
  AttnArgs a = {};
  a.q = b.q + (size_t)c * b.ldq;
  a.out = b.out + (size_t)c * b.ldq;
  a.keys = b.keys + so;
  a.values = b.values + so;
  a.max_seq = b.max_seq;
  a.n_kv_heads = b.n_kv_heads;
  a.head_dim = HD;
  a.layer = b.layer;
  a.n_heads = b.n_heads;
  a.pos_dev = b.col_pos + c;
  a.partials = b.partials + (size_t)c * b.n_heads * b.max_splits * PS;
  a.tickets = b.tickets + (size_t)c * b.n_kv_heads;
  a.max_splits = b.max_splits;
  const int pos = __ldcg(a.pos_dev);
  const at::Split sp = at::split_of(a, split, pos);

  if (split < sp.n_active) {
    const size_t row_stride = (size_t)a.n_kv_heads * HD;
    const size_t lbase = (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD + 4 * lane;
    const float* kb = a.keys + lbase;
    const float* vb = a.values + lbase;
    const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
    unsigned long long q2[G][2];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float4 qv =
          __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)(kvh * G + h) * HD) + lane);
      q2[h][0] = f2_pack(qv.x, qv.y);
      q2[h][1] = f2_pack(qv.z, qv.w);
    }
    const int n_steps = (sp.n + P - 1) / P;
    const int count = n_steps > w ? (n_steps - w + NW - 1) / NW : 0;
    const uint32_t ring_u32 = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
    auto slot_addr = [&](int stage, int kind, int i) -> uint32_t {
      return ring_u32 + (uint32_t)((((w * D + stage) * 2 + kind) * P + i) * 32 + lane) *
                            (uint32_t)sizeof(float4);
    };
    auto issue = [&](int k, int stage) {
      const int j = w + k * NW;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const int t = j * P + i;
        const bool valid = t < sp.n;
        const size_t row = (size_t)(sp.t0 + (valid ? t : 0)) * row_stride;
        cp_async16(slot_addr(stage, 0, i), kb + row, valid ? 16u : 0u);
        cp_async16(slot_addr(stage, 1, i), vb + row, valid ? 16u : 0u);
      }
    };
#pragma unroll
    for (int k = 0; k < D; ++k) {
      if (k < count) issue(k, k);
      cp_async_commit();
    }
    float m_run = -INFINITY, l_run = 0.0f;
    unsigned long long acc[G][2];
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h][0] = acc[h][1] = 0ull;
    float* pb = pbuf + w * 48;
    const int hs = lane & 7, is = lane >> 3;  // this lane's (head, position) after the butterfly
    for (int k = 0; k < count; ++k) {
      const int stage = k % D;
      cp_async_wait<D - 1>();
      float4 kr[P], vr[P];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        kr[i] = ring[(((w * D + stage) * 2 + 0) * P + i) * 32 + lane];
        vr[i] = ring[(((w * D + stage) * 2 + 1) * P + i) * 32 + lane];
      }
      float v[32];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const unsigned long long k01 = f2_pack(kr[i].x, kr[i].y), k23 = f2_pack(kr[i].z, kr[i].w);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          if (h < G) {
            const unsigned long long d2 = ffma2(q2[h][1], k23, fmul2(q2[h][0], k01));
            v[i * 8 + h] = f2_lo(d2) + f2_hi(d2);
          } else {
            v[i * 8 + h] = 0.0f;
          }
        }
      }
#pragma unroll
      for (int m = 16, n = 32; m >= 1; m >>= 1, n >>= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int u = 0; u < n / 2; ++u) {
          const float send = upper ? v[u] : v[u + n / 2];
          const float keep = upper ? v[u + n / 2] : v[u];
          v[u] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
      }
      const int t = (w + k * NW) * P + is;
      const bool valid = t < sp.n && hs < G;
      const float s = valid ? __fmul_rn(v[0], scale) : -INFINITY;
      float mx = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m_run, mx);
      const float p = valid ? expf(s - m_new) : 0.0f;
      const float corr = m_new == -INFINITY ? 1.0f : expf(m_run - m_new);
      float ps = p + __shfl_xor_sync(0xffffffffu, p, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l_run = fmaf(l_run, corr, ps);
      m_run = m_new;
      pb[lane] = p;
      if (lane < 8) pb[32 + lane] = corr;
      __syncwarp();
      float pr[P][8], cr[8];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const float4 lo = reinterpret_cast<const float4*>(pb)[2 * i];
        const float4 hi = reinterpret_cast<const float4*>(pb)[2 * i + 1];
        pr[i][0] = lo.x; pr[i][1] = lo.y; pr[i][2] = lo.z; pr[i][3] = lo.w;
        pr[i][4] = hi.x; pr[i][5] = hi.y; pr[i][6] = hi.z; pr[i][7] = hi.w;
      }
      {
        const float4 lo = reinterpret_cast<const float4*>(pb)[8];
        const float4 hi = reinterpret_cast<const float4*>(pb)[9];
        cr[0] = lo.x; cr[1] = lo.y; cr[2] = lo.z; cr[3] = lo.w;
        cr[4] = hi.x; cr[5] = hi.y; cr[6] = hi.z; cr[7] = hi.w;
      }
      __syncwarp();
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const unsigned long long c2 = f2_pack(cr[h], cr[h]);
        unsigned long long a0 = fmul2(acc[h][0], c2), a1 = fmul2(acc[h][1], c2);
#pragma unroll
        for (int i = 0; i < P; ++i) {
          const unsigned long long p2 = f2_pack(pr[i][h], pr[i][h]);
          a0 = ffma2(p2, f2_pack(vr[i].x, vr[i].y), a0);
          a1 = ffma2(p2, f2_pack(vr[i].z, vr[i].w), a1);
        }
        acc[h][0] = a0;
        acc[h][1] = a1;
      }
      if (k + D < count) issue(k + D, stage);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();  // every warp is done with the ring: reuse it for the merge
    float* mst = reinterpret_cast<float*>(smem_s);  // [NW][8]
    float* lst = mst + NW * 8;                      // [NW][8]
    float* accb = lst + NW * 8;                     // [NW][G][HD]
    if (lane < 8) {
      mst[w * 8 + lane] = m_run;
      lst[w * 8 + lane] = l_run;
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
      reinterpret_cast<float4*>(accb + (size_t)(w * G + h) * HD)[lane] =
          make_float4(f2_lo(acc[h][0]), f2_hi(acc[h][0]), f2_lo(acc[h][1]), f2_hi(acc[h][1]));
    __syncthreads();
    const bool direct = sp.n_active == 1;
    const int d = tid;  // one output dim per thread
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float M = -INFINITY;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) M = fmaxf(M, mst[ww * 8 + h]);
      float L = 0.0f, O = 0.0f;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) {
        const float mw = mst[ww * 8 + h];
        const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
        L = fmaf(f, lst[ww * 8 + h], L);
        O = fmaf(f, accb[(size_t)(ww * G + h) * HD + d], O);
      }
      if (direct) {
        a.out[(size_t)(kvh * G + h) * HD + d] = __fdiv_rn(O, L);
      } else {
        float* pp = a.partials + ((size_t)(kvh * G + h) * a.max_splits + split) * PS;
        pp[d] = O;
        if (d == 0) *reinterpret_cast<float2*>(pp + HD) = make_float2(M, L);
      }
    }
    __syncthreads();  // the merge buffers are free again (the combine reuses them)
  }
  if (sp.n_active > 1)
    at::split_combine_hd<kStreamWarps * 32, HD>(a, kvh, G, sp.n_active, gridDim.y,
                                                 reinterpret_cast<float*>(smem_s), &is_last);
}

// Without a valid key for a column (an lm_head wait ran out) that column
// keeps its token and position, and kErrNoToken is recorded.
__global__ void cols_advance_kernel(unsigned long long* __restrict__ keys, int cols,
                                    const int* __restrict__ col_slot, int* __restrict__ col_token,
                                    int* __restrict__ col_pos, int* __restrict__ history,
                                    int max_seq, int vocab) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const unsigned long long key = keys[c];
  keys[c] = 0ull;
  int idx = 0;
  if (!argmax_token(key, vocab, &idx)) {
    atomicOr(&g_batch_error, kErrNoToken);
    return;
  }
  const int p = col_pos[c];
  if (history && p >= 0 && p < max_seq) history[(size_t)col_slot[c] * max_seq + p] = idx;
  col_token[c] = idx;
  col_pos[c] = p + 1;
}

}  // namespace

// --------------------------------------------------------------------- host
int batch_row_tiles(int n) { return (n + kTileRows - 1) / kTileRows; }

// K splits so that row tiles x splits covers the SMs, at least 4 scale
// blocks (two stages) per split, an even block count per split.
GemmPlan plan_batch_gemm(int n, int kp) {
  const int nb = kp / 32, tiles = batch_row_tiles(n), sms = sm_count();
  int splits = 1;
  if (tiles < sms) splits = std::max(1, std::min(sms / std::max(tiles, 1), nb / 4));
  int kb_per = (nb + splits - 1) / splits;
  kb_per = (kb_per + 1) / 2 * 2;
  splits = (nb + kb_per - 1) / kb_per;
  return GemmPlan{splits, kb_per};
}

size_t batch_partial_floats(int n, int kp) {
  const GemmPlan pl = plan_batch_gemm(n, kp);
  return pl.splits > 1 ? (size_t)pl.splits * n * kBatchMaxCols : 0;
}

int make_quant_map(CUtensorMap* map, int qtype, const uint8_t* qs, int rows, int kp) {
  const uint64_t rb = qtype == DQMK_Q80 ? (uint64_t)kp : (uint64_t)kp / 2;
  const uint32_t box = qtype == DQMK_Q80 ? kChunkK : kChunkK / 2;
  return make_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qs, rb, (uint64_t)rows, rb, box,
                     kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int make_cols_map(CUtensorMap* map, const uint16_t* plane, int kp) {
  return make_f16_tile_map(map, plane, kBatchMaxCols, kp, kBatchMaxCols);
}

cudaError_t batch_prepare_device();

cudaError_t batch_prepare() {
  static DeviceOnce once;
  return once.run(batch_prepare_device);
}

cudaError_t batch_prepare_device() {
  cudaError_t e = cudaFuncSetAttribute(batch_gemm_kernel<DQMK_Q80>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gemm_smem<DQMK_Q80>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(batch_gemm_kernel<DQMK_Q40>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)gemm_smem<DQMK_Q40>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_cols_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_cols_kernel<128>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  // the attention CTAs are small: let as many share an SM as registers allow
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_cols_kernel<64>,
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_cols_kernel<128>,
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_cols_stream_kernel<7>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(kStreamRingBytes + kStreamPBytes));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_cols_stream_kernel<7>,
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  return e;
}

cudaError_t launch_batch_gemm(const CUtensorMap& wq, const CUtensorMap& wd,
                              const CUtensorMap& xhi, const CUtensorMap& xlo, const BatchGemm& p,
                              cudaStream_t s, bool pdl) {
  if (p.cols < 1 || p.cols > kBatchMaxCols || p.n < 1 || p.kp < 32 || p.kp % 32 != 0 ||
      p.plan.splits < 1 || p.plan.kb_per < 2 || p.plan.kb_per % 2 != 0 || !p.rs || !p.cs ||
      !p.d || (p.plan.splits > 1 && !p.partial))
    return cudaErrorInvalidValue;
  if ((p.epi == kEpiSwiGlu || p.epi == kEpiQkv) && (p.n % 2 != 0)) return cudaErrorInvalidValue;
  if (p.epi == kEpiLogits && !p.keys) return cudaErrorInvalidValue;
  if (p.epi != kEpiLogits && !p.y && p.epi != kEpiQkv) return cudaErrorInvalidValue;
  cudaError_t e = batch_prepare();
  if (e != cudaSuccess) return e;
  const int items = batch_row_tiles(p.n) * p.plan.splits;
  const dim3 grid(std::min(items, sm_count()));
  if (p.qtype == DQMK_Q80)
    e = launch(batch_gemm_kernel<DQMK_Q80>, grid, dim3(kThreads), gemm_smem<DQMK_Q80>(), s, pdl,
               wq, wd, xhi, xlo, p);
  else if (p.qtype == DQMK_Q40)
    e = launch(batch_gemm_kernel<DQMK_Q40>, grid, dim3(kThreads), gemm_smem<DQMK_Q40>(), s, pdl,
               wq, wd, xhi, xlo, p);
  else
    return cudaErrorInvalidValue;
  if (e != cudaSuccess || p.plan.splits == 1) return e;
  const dim3 rgrid((p.n + 31) / 32, (p.cols + 8 * kReduceCols - 1) / (8 * kReduceCols));
  return launch(splitk_reduce_kernel, rgrid, dim3(256), 0, s, pdl, p);
}

int scale_pitch(int kp) { return ((kp / 32) + 7) / 8 * 8; }

int make_scale_map(CUtensorMap* map, const uint16_t* d_pad, int rows, int kp) {
  const uint64_t nbp = (uint64_t)scale_pitch(kp);
  return make_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, d_pad, nbp, (uint64_t)rows, nbp * 2,
                     8, kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

cudaError_t copy_scales_padded(const uint16_t* d, int rows, int kp, uint16_t* d_pad,
                               cudaStream_t s) {
  const size_t nb = (size_t)kp / 32, nbp = (size_t)scale_pitch(kp);
  cudaError_t e = cudaMemsetAsync(d_pad, 0, (size_t)rows * nbp * 2, s);
  if (e != cudaSuccess) return e;
  return cudaMemcpy2DAsync(d_pad, nbp * 2, d, nb * 2, nb * 2, rows, cudaMemcpyDeviceToDevice, s);
}

cudaError_t launch_weight_row_scales(int qtype, const uint8_t* qs, const uint16_t* d, int rows,
                                     int kp, float* cs, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  row_scales_kernel<<<rows, 256, 0, s>>>(qtype, qs, d, kp, cs);
  return cudaGetLastError();
}

// Splits per (column, KV head): at least two CTAs per SM over all pairs and
// at most about 256 positions per split (many short CTAs balance across the
// SMs; a few long ones leave a ragged last wave), each split at least
// kMinChunk positions long.
int batch_attention_splits(int cols, int n_kv_heads, int max_seq) {
  const int pairs = std::max(1, cols * n_kv_heads);
  int sp = std::max((2 * sm_count() + pairs - 1) / pairs, (max_seq + 255) / 256);
  const int by_len = (max_seq + at::kMinChunk - 1) / at::kMinChunk;
  sp = std::min(sp, by_len);
  return std::max(1, sp);
}

size_t batch_attention_partials_floats(int cols, int n_heads, int head_dim, int max_splits) {
  return (size_t)cols * n_heads * max_splits * at::part_stride(head_dim);
}

cudaError_t launch_attention_cols(const BatchAttn& a, cudaStream_t s, bool pdl) {
  if (a.cols < 1 || a.n_kv_heads <= 0 || a.n_heads % a.n_kv_heads != 0 ||
      a.n_heads / a.n_kv_heads > at::kMaxGroup || a.ldq % 4 != 0 ||
      ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.out)) & 15u))
    return cudaErrorInvalidValue;
  cudaError_t e = batch_prepare();
  if (e != cudaSuccess) return e;
  const dim3 grid(a.n_kv_heads, a.max_splits, a.cols);
  // head_dim 128 with 7 query heads per KV head (Qwen2-7B): the one-pass
  // streaming kernel; its merge and split-combine buffers reuse the ring
  if (a.head_dim == 128 && a.n_heads / a.n_kv_heads == 7 &&
      (size_t)(2 * a.max_splits + 1) * at::kMaxGroup * sizeof(float) <= kStreamRingBytes)
    return launch(attention_cols_stream_kernel<7>, grid, dim3(kStreamWarps * 32),
                  kStreamRingBytes + kStreamPBytes, s, pdl, a);
  const int cap = attention_chunk_cap(a.max_seq, a.max_splits);
  const size_t smem = at::smem_bytes_hd(a.head_dim, cap, a.max_splits, 256);
  if (a.head_dim == 64)
    return launch(attention_cols_kernel<64>, grid, dim3(256), smem, s, pdl, a, cap);
  if (a.head_dim == 128)
    return launch(attention_cols_kernel<128>, grid, dim3(256), smem, s, pdl, a, cap);
  return cudaErrorInvalidValue;
}

cudaError_t launch_cols_advance(unsigned long long* keys, int cols, const int* col_slot,
                                int* col_token, int* col_pos, int* history, int max_seq, int vocab,
                                cudaStream_t s, bool pdl) {
  return launch(cols_advance_kernel, dim3(1), dim3(kBatchMaxCols), 0, s, pdl, keys, cols, col_slot,
                col_token, col_pos, history, max_seq, vocab);
}

cudaError_t read_batch_error(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_batch_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *flags) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_batch_error, &zero, sizeof(unsigned int));
  }
  return e;
}

}  // namespace dqmk

// ------------------------------------------------------------------ C ABI
using namespace dqmk;

extern "C" int dqmk_linear_cols_packed(int qtype, const float* x, int cols, int in_features,
                                       const void* packed, int out_features, const float* bias,
                                       const float* residual, float* y, void* stream) {
  const char* api = qtype == DQMK_Q40 ? "CudaQ40Linear" : "CudaQ80Linear";
  if (qtype != DQMK_Q80 && qtype != DQMK_Q40)
    return fail(DQMK_ERR_UNSUPPORTED, "dqmk_linear_cols_packed: unsupported quant type");
  if (cols < 1 || cols > kBatchMaxCols || in_features <= 0 || out_features <= 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid shape (1 to 64 columns)");
  if (!x || !packed || !y) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  if (reinterpret_cast<uintptr_t>(packed) & 15u)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": packed weight must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int kp = (in_features + 31) / 32 * 32;
  const uint8_t* qs = static_cast<const uint8_t*>(packed);
  const size_t qbytes = (size_t)out_features * (qtype == DQMK_Q80 ? kp : kp / 2);
  const uint16_t* d = reinterpret_cast<const uint16_t*>(qs + qbytes);
  const GemmPlan plan = plan_batch_gemm(out_features, kp);
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t b_act = up((size_t)kBatchMaxCols * kp * 2), b_rs = up(kBatchMaxCols * 4);
  const size_t b_cs = up((size_t)out_features * 4);
  const size_t b_part = up(batch_partial_floats(out_features, kp) * 4);
  const size_t b_dp = up((size_t)out_features * scale_pitch(kp) * 2);
  unsigned char* scratch = nullptr;
  const size_t total = 2 * b_act + b_rs + b_cs + b_part + b_dp + 256;
  DQMK_CUDA_RET(api, cudaMallocAsync(reinterpret_cast<void**>(&scratch), total, st));
  unsigned char* cur = scratch;
  auto take = [&](size_t b) {
    unsigned char* r = cur;
    cur += b;
    return r;
  };
  uint16_t* hi = reinterpret_cast<uint16_t*>(take(b_act));
  uint16_t* lo = reinterpret_cast<uint16_t*>(take(b_act));
  float* rs = reinterpret_cast<float*>(take(b_rs));
  float* cs = reinterpret_cast<float*>(take(b_cs));
  float* part = reinterpret_cast<float*>(take(b_part));
  uint16_t* d_pad = reinterpret_cast<uint16_t*>(take(b_dp));
  int rc = DQMK_OK;
  cudaError_t e = cudaSuccess;
  CUtensorMap mw, md, mhi, mlo;
  do {
    if ((rc = make_quant_map(&mw, qtype, qs, out_features, kp))) break;
    if ((rc = make_scale_map(&md, d_pad, out_features, kp))) break;
    if ((rc = make_cols_map(&mhi, hi, kp))) break;
    if ((rc = make_cols_map(&mlo, lo, kp))) break;
    // unused columns of the planes stay finite (zero)
    if ((e = cudaMemsetAsync(scratch, 0, 2 * b_act + b_rs, st)) != cudaSuccess) break;
    if ((e = copy_scales_padded(d, out_features, kp, d_pad, st)) != cudaSuccess) break;
    if ((e = launch_weight_row_scales(qtype, qs, d, out_features, kp, cs, st)) != cudaSuccess)
      break;
    if ((e = launch_split_rows(x, cols, in_features, kp, in_features, nullptr, 0.0f, hi, lo, rs,
                               st)) != cudaSuccess)
      break;
    BatchGemm g = {};
    g.qtype = qtype;
    g.d = d;
    g.n = out_features;
    g.kp = kp;
    g.cols = cols;
    g.rs = rs;
    g.cs = cs;
    g.plan = plan;
    g.partial = part;
    g.epi = kEpiStore;
    g.bias = bias;
    g.residual = residual;
    g.y = y;
    g.ldy = out_features;
    e = launch_batch_gemm(mw, md, mhi, mlo, g, st, false);
  } while (false);
  cudaError_t ef = cudaFreeAsync(scratch, st);
  if (rc) return rc;
  if (e == cudaSuccess) e = ef;
  if (e != cudaSuccess) return cuda_fail(api, e);
  return DQMK_OK;
}
