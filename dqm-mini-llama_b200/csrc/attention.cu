// attention.cu -- GQA decode attention over the device-resident f32 KV cache.
//
// Reference math (src/forward.cc:461-506, the CPU branch the GPU must match):
// for each query head h with KV head h / (n_heads / n_kv_heads):
//   s_t = (q_h . K_t) / sqrt(head_dim), p = softmax(s_0..s_pos),
//   out_h = sum_t p_t V_t.
//
// B200 form: grid (n_kv_heads, splits).  Each CTA takes one KV head and one
// slice of positions, so the K/V rows of a head are read once for all of its
// (n_heads / n_kv_heads) query heads.  It computes its slice's scores, a
// local max m and sum l of exp(s - m), and o = sum exp(s - m) V; then bumps a
// per-KV-head ticket.  The CTA that takes the last ticket merges the slices
// (rescaling by exp(m_i - M)) and resets the ticket, so the whole op is one
// launch and replays inside a CUDA graph.  Positions come from device memory
// so a captured graph serves every decode step.
#include <mutex>

#include "attention_dev.cuh"
#include "common.cuh"
#include "internal.h"

namespace dqmk {
namespace {

using namespace at;


// Completion ticket per KV head; the CTA that takes the last one merges the
// splits: out = sum_i e^(m_i - M) o_i / sum_i e^(m_i - M) l_i.  Split
// statistics are staged in shared memory in one pass, then every output
// issues its partial-vector loads together.
template <int NT>
__device__ __forceinline__ void split_combine(const AttnArgs& a, int kvh, int G, int hd,
                                              int n_active, float* stats, int* is_last) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int done = atomicAdd(&a.tickets[kvh], 1u);
    *is_last = done == gridDim.y - 1;
  }
  __syncthreads();
  if (!*is_last) return;
  __threadfence();
  float* w = stats;                                  // [n_active][8] weights
  float* inv_den = stats + (size_t)a.max_splits * kMaxGroup;  // [8]
  for (int i = threadIdx.x; i < n_active * G; i += NT) {
    const int sp = i / G, h = i % G;
    const float* ps = a.partials + ((size_t)(kvh * G + h) * a.max_splits + sp) * part_stride(hd);
    w[sp * kMaxGroup + h] = __ldcg(ps + hd);
    w[(a.max_splits + 1) * kMaxGroup + sp * kMaxGroup + h] = __ldcg(ps + hd + 1);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < n_active; ++sp) M = fmaxf(M, w[sp * kMaxGroup + h]);
    float den = 0.0f;
    for (int sp = 0; sp < n_active; ++sp) {
      const float e = expf(w[sp * kMaxGroup + h] - M);
      w[sp * kMaxGroup + h] = e;
      den = fmaf(e, w[(a.max_splits + 1) * kMaxGroup + sp * kMaxGroup + h], den);
    }
    inv_den[h] = den;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * hd; i += NT) {
    const int h = i / hd, dcol = i % hd;
    const float* part = a.partials + (size_t)(kvh * G + h) * a.max_splits * part_stride(hd) + dcol;
    float num = 0.0f;
    int sp = 0;
    for (; sp + 8 <= n_active; sp += 8) {
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = __ldcg(part + (size_t)(sp + u) * part_stride(hd));
#pragma unroll
      for (int u = 0; u < 8; ++u) num = fmaf(w[(sp + u) * kMaxGroup + h], o[u], num);
    }
    for (; sp < n_active; ++sp) num = fmaf(w[sp * kMaxGroup + h], __ldcg(part + (size_t)sp * part_stride(hd)), num);
    a.out[(size_t)(kvh * G + h) * hd + dcol] = __fdiv_rn(num, inv_den[h]);
  }
  if (threadIdx.x == 0) a.tickets[kvh] = 0u;
}

// Rows t0..min(t0 + n, pos) - 1 of this KV head's K and V in the split: those
// earlier steps wrote, requested into L2 before the dependency wait so the
// body's loads after it hit L2 (128-byte lines, every thread of the CTA).
template <int HD>
__device__ __forceinline__ void prefetch_split_l2(const AttnArgs& a, int kvh, int split, int pos) {
  const Split sp = split_of(a, split, pos);
  const int n = min(sp.n, pos - sp.t0);
  if (n <= 0) return;
  constexpr int LPR = HD * 4 / 128;  // 128-byte lines per row
  const size_t row_stride = (size_t)a.n_kv_heads * HD;
  const size_t base = (size_t)a.layer * a.max_seq * row_stride + (size_t)sp.t0 * row_stride +
                      (size_t)kvh * HD;
  for (int i = threadIdx.x; i < 2 * n * LPR; i += blockDim.x) {
    const int kv = i / (n * LPR), r = (i / LPR) % n, l = i % LPR;
    const float* p = (kv ? a.values : a.keys) + base + (size_t)r * row_stride + l * 32;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
  }
}

template <int HD>
__global__ void __launch_bounds__(256) attention_hd_kernel(const AttnArgs a, int chunk_cap) {
  extern __shared__ float sm[];
  // the position is advanced only between steps: stable across this one
  prefetch_split_l2<HD>(a, blockIdx.x, blockIdx.y, a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg);
  pdl_trigger();
  pdl_wait();
  attention_hd_body<HD, 256>(a, chunk_cap, blockIdx.x, blockIdx.y, gridDim.y, sm);
}

// When the whole context is one split (max_seq <= 128 positions) the grouped
// kernel would run one CTA per KV head doing all G query heads in turn.
// Here blockIdx.z picks one query head and the CTA runs the same body as a
// group of one: K / V rows are read G times, from L2, and each head's
// arithmetic is exactly that of the grouped kernel (heads are independent in
// it), so outputs are bit-identical with a G times shorter critical path.
template <int HD>
__global__ void __launch_bounds__(256) attention_hd_head_kernel(const AttnArgs a, int chunk_cap) {
  extern __shared__ float sm[];
  prefetch_split_l2<HD>(a, blockIdx.x, 0, a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg);
  pdl_trigger();
  pdl_wait();
  const int kvh = blockIdx.x, g = blockIdx.z;
  const int G = a.n_heads / a.n_kv_heads;
  AttnArgs b = a;
  b.n_heads = a.n_kv_heads;  // one query head per KV head
  b.max_splits = 1;
  // the body addresses query head kvh of b: shift q / out onto head kvh * G + g
  const size_t shift = (size_t)(kvh * (G - 1) + g) * HD;
  b.q = a.q + shift;
  b.out = a.out + shift;
  attention_hd_body<HD, 256>(b, chunk_cap, kvh, 0, 1, sm);
}

// Short caches (max_seq <= kShortMax, the whole cache one split): one CTA
// per query head, every global load issued at once right after the
// dependency wait -- the thread's 16 dims of q, the K rows of its score
// positions and the V rows of its P.V positions -- so the kernel pays one L2
// round trip instead of three (q, then K, then V).  Scores: HD/16 threads
// per position; softmax statistics computed redundantly by every warp from
// the scores in shared memory (no extra barrier); P.V: thread (d4, group)
// owns 4 dims and every NG-th position; the NG group sums are added in
// shared memory.  Same arithmetic per term as attention_hd_body (fp32,
// expf(s - m), divide by l), different summation order.
constexpr int kShortMax = 128;

// One query head over a cache of at most kShortMax positions, by a CTA of
// 256 threads.  Rows 0..pos-1 of the cache were written by earlier steps, so
// they are loaded before the dependency wait (under programmatic dependent
// launch they arrive while the QKV GEMV that this kernel waits on still
// runs); after the wait only q and row pos (written by that GEMV) are read.
// Then scores to shared memory, softmax statistics per warp, P.V in position
// groups, and the head's output.
template <int HD>
struct ShortShape {
  static constexpr int NT = 256;
  static constexpr int TPP = HD / 16;          // threads per score position (16 dims each)
  static constexpr int PPASS = NT / TPP;       // positions per score pass
  static constexpr int NPASS = kShortMax / PPASS;
  static constexpr int D4 = HD / 4;            // float4 columns of a row
  static constexpr int NG = NT / D4;           // position groups in P.V
  static constexpr int NPV = kShortMax / NG;   // positions per thread in P.V
};

template <int HD>
__global__ void __launch_bounds__(256) attention_short_kernel(const AttnArgs a) {
  using SS = ShortShape<HD>;
  constexpr int TPP = SS::TPP, PPASS = SS::PPASS, NPASS = SS::NPASS, D4 = SS::D4, NG = SS::NG,
                NPV = SS::NPV;
  __shared__ float ss[kShortMax];
  __shared__ float4 red[NG][D4];
  const int kvh = blockIdx.x, G = a.n_heads / a.n_kv_heads;
  const int head = kvh * G + blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31;
  // the position is advanced only between steps: stable across this one
  const int pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
  const int T = pos + 1;
  const size_t row_stride = (size_t)a.n_kv_heads * HD;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD;
  const int part = tid % TPP, p0 = tid / TPP;
  const int d4 = tid % D4, grp = tid / D4;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  // ---- before the dependency: the rows earlier steps wrote (t < pos)
  float4 qv[4], kr[NPASS][4], vr[NPV];
#pragma unroll
  for (int u = 0; u < NPASS; ++u) {
    const int t = p0 + u * PPASS;
    const float4* kp = reinterpret_cast<const float4*>(kbase + (size_t)t * row_stride) + part * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) kr[u][i] = t < pos ? __ldcg(kp + i) : zero;
  }
#pragma unroll
  for (int j = 0; j < NPV; ++j) {
    const int t = grp + j * NG;
    vr[j] = t < pos ? __ldcg(reinterpret_cast<const float4*>(vbase + (size_t)t * row_stride) + d4)
                    : zero;
  }
  pdl_trigger();
  pdl_wait();
  // ---- after it: q and row pos
  const float4* q4 = reinterpret_cast<const float4*>(a.q + (size_t)head * HD) + part * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) qv[i] = __ldcg(q4 + i);
#pragma unroll
  for (int u = 0; u < NPASS; ++u) {
    if (p0 + u * PPASS == pos) {
      const float4* kp =
          reinterpret_cast<const float4*>(kbase + (size_t)pos * row_stride) + part * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) kr[u][i] = __ldcg(kp + i);
    }
  }
#pragma unroll
  for (int j = 0; j < NPV; ++j)
    if (grp + j * NG == pos)
      vr[j] = __ldcg(reinterpret_cast<const float4*>(vbase + (size_t)pos * row_stride) + d4);
  // ---- scores
  const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
#pragma unroll
  for (int u = 0; u < NPASS; ++u) {
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      d = fmaf(qv[i].x, kr[u][i].x, d);
      d = fmaf(qv[i].y, kr[u][i].y, d);
      d = fmaf(qv[i].z, kr[u][i].z, d);
      d = fmaf(qv[i].w, kr[u][i].w, d);
    }
#pragma unroll
    for (int o = TPP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    const int t = p0 + u * PPASS;
    if (part == 0 && t < T) ss[t] = __fmul_rn(d, scale);
  }
  __syncthreads();
  // ---- softmax statistics (every warp alike)
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kShortMax / 32; ++k) {
    const int t = lane + 32 * k;
    if (t < T) m = fmaxf(m, ss[t]);
  }
  m = warp_max(m);
  float l = 0.0f;
#pragma unroll
  for (int k = 0; k < kShortMax / 32; ++k) {
    const int t = lane + 32 * k;
    if (t < T) l += expf(ss[t] - m);
  }
  l = warp_sum(l);
  // ---- P.V over this thread's positions
  float4 acc = zero;
#pragma unroll
  for (int j = 0; j < NPV; ++j) {
    const int t = grp + j * NG;
    if (t < T) {
      const float pr = expf(ss[t] - m);
      acc.x = fmaf(pr, vr[j].x, acc.x);
      acc.y = fmaf(pr, vr[j].y, acc.y);
      acc.z = fmaf(pr, vr[j].z, acc.z);
      acc.w = fmaf(pr, vr[j].w, acc.w);
    }
  }
  red[grp][d4] = acc;
  __syncthreads();
  if (tid < D4) {
    float4 o = red[0][tid];
#pragma unroll
    for (int g2 = 1; g2 < NG; ++g2) {
      const float4 x = red[g2][tid];
      o.x += x.x;
      o.y += x.y;
      o.z += x.z;
      o.w += x.w;
    }
    reinterpret_cast<float4*>(a.out + (size_t)head * HD)[tid] =
        make_float4(__fdiv_rn(o.x, l), __fdiv_rn(o.y, l), __fdiv_rn(o.z, l), __fdiv_rn(o.w, l));
  }
}

// Any head_dim that is a multiple of 4 up to 256: one thread per position.
__global__ void __launch_bounds__(kThreads) attention_kernel(const AttnArgs a, int chunk_cap) {
  extern __shared__ float sm[];
  __shared__ float head_m[kMaxGroup], head_l[kMaxGroup];
  __shared__ int is_last;

  pdl_trigger();
  pdl_wait();

  const int kvh = blockIdx.x, split = blockIdx.y;
  const int hd = a.head_dim;
  const int G = a.n_heads / a.n_kv_heads;
  const int pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
  const Split sp = split_of(a, split, pos);
  const int t0 = sp.t0, n = sp.n;
  const size_t row_stride = (size_t)a.n_kv_heads * hd;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * hd;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * hd;

  float* sq = sm;
  float* ss = sq + kMaxGroup * hd;
  float* sacc = ss + kMaxGroup * chunk_cap;

  if (split < sp.n_active) {
    for (int i = threadIdx.x; i < G * hd; i += kThreads)
      sq[i] = __ldcg(a.q + (size_t)(kvh * G) * hd + i);
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    for (int t = threadIdx.x; t < n; t += kThreads) {
      const float4* kr = reinterpret_cast<const float4*>(kbase + (size_t)(t0 + t) * row_stride);
      float dot[kMaxGroup];
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) dot[h] = 0.0f;
      for (int i = 0; i < hd / 4; ++i) {
        const float4 k4 = __ldcg(kr + i);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
          if (h < G) {
            const float4 q4 = reinterpret_cast<const float4*>(sq + h * hd)[i];
            float d = dot[h];
            d = fmaf(q4.x, k4.x, d);
            d = fmaf(q4.y, k4.y, d);
            d = fmaf(q4.z, k4.z, d);
            d = fmaf(q4.w, k4.w, d);
            dot[h] = d;
          }
        }
      }
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h)
        if (h < G) ss[h * chunk_cap + t] = __fmul_rn(dot[h], scale);
    }
    __syncthreads();
    split_softmax<kThreads>(ss, chunk_cap, G, n, head_m, head_l);
    __syncthreads();

    const int groups = kThreads / hd > 0 ? kThreads / hd : 1;
    const int d = threadIdx.x % hd;
    const int gi = threadIdx.x / hd;
    if (gi < groups && threadIdx.x < groups * hd) {
      float acc[kMaxGroup];
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
      for (int t = gi; t < n; t += groups) {
        const float v = __ldcg(vbase + (size_t)(t0 + t) * row_stride + d);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
          if (h < G) acc[h] = fmaf(ss[h * chunk_cap + t], v, acc[h]);
      }
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h)
        if (h < G) sacc[(gi * kMaxGroup + h) * hd + d] = acc[h];
    }
    for (int dd = kThreads; dd < hd; dd += kThreads) {
      const int d2 = dd + threadIdx.x;
      if (d2 < hd) {
        float acc[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
        for (int t = 0; t < n; ++t) {
          const float v = __ldcg(vbase + (size_t)(t0 + t) * row_stride + d2);
#pragma unroll
          for (int h = 0; h < kMaxGroup; ++h)
            if (h < G) acc[h] = fmaf(ss[h * chunk_cap + t], v, acc[h]);
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
          if (h < G) sacc[h * hd + d2] = acc[h];
      }
    }
    __syncthreads();

    for (int i = threadIdx.x; i < G * hd; i += kThreads) {
      const int h = i / hd, dcol = i % hd;
      float o = 0.0f;
      const int ng = hd <= kThreads ? groups : 1;
      for (int g2 = 0; g2 < ng; ++g2) o += sacc[(g2 * kMaxGroup + h) * hd + dcol];
      if (sp.n_active == 1) {
        a.out[(size_t)(kvh * G + h) * hd + dcol] = __fdiv_rn(o, head_l[h]);
        continue;
      }
      float* part = a.partials + ((size_t)(kvh * G + h) * a.max_splits + split) * part_stride(hd);
      part[dcol] = o;
      if (dcol == 0) {
        part[hd] = head_m[h];
        part[hd + 1] = head_l[h];
      }
    }
  }
  if (sp.n_active > 1)
    split_combine<kThreads>(a, kvh, G, hd, sp.n_active, sacc + kMaxGroup * hd * (kThreads / hd > 0 ? kThreads / hd : 1), &is_last);
}

}  // namespace

int attention_chunk_cap(int max_seq, int max_splits) {
  int c = (max_seq + max_splits - 1) / max_splits;
  c = (c + 31) & ~31;
  return c < kMinChunk ? kMinChunk : c;
}

namespace {

int chunk_cap_for(int max_seq, int max_splits, int min_chunk) {
  int c = (max_seq + max_splits - 1) / max_splits;
  c = (c + 31) & ~31;
  const int mc = min_chunk > 0 ? min_chunk : kMinChunk;
  return c < mc ? mc : c;
}

size_t smem_bytes(int threads, int head_dim, int chunk_cap, int max_splits) {
  const int groups = threads / head_dim > 0 ? threads / head_dim : 1;
  return sizeof(float) * ((size_t)kMaxGroup * head_dim + (size_t)kMaxGroup * chunk_cap +
                          (size_t)groups * kMaxGroup * head_dim +
                          (size_t)(2 * max_splits + 3) * kMaxGroup);
}

}  // namespace

int decode_min_chunk(int head_dim) { return head_dim >= 128 ? 64 : kMinChunk; }

int attention_splits(int max_seq, int n_kv_heads, int min_chunk) {
  const int mc = min_chunk > 0 ? min_chunk : kMinChunk;
  int s = (max_seq + mc - 1) / mc;
  int cap = sm_count() / (n_kv_heads > 0 ? n_kv_heads : 1);
  if (cap < 1) cap = 1;
  if (s > cap) s = cap;
  return s < 1 ? 1 : s;
}

size_t attention_partials_floats(int n_heads, int head_dim, int max_splits) {
  return (size_t)n_heads * max_splits * part_stride(head_dim);
}

cudaError_t attention_prepare() {
  static DeviceOnce once;
  return once.run([] {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_hd_kernel<64>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_hd_kernel<128>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_hd_head_kernel<64>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_hd_head_kernel<128>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    return e;
  });
}

// Any head configuration the fast kernels do not take (head_dim not a
// multiple of 4 or above 256, more than 8 query heads per KV head): one CTA
// per query head, plain float loads.  Pass 1 keeps a running (max, sum) of
// the scaled scores per thread and merges them across the CTA; pass 2 turns
// 1024 positions at a time into probabilities in shared memory and
// accumulates P.V with one thread per output dimension.  Drop-in entry
// points only (the decode step's shapes all have a fast kernel).
constexpr int kAnyThreads = 256;
constexpr int kAnyChunk = 1024;

__global__ void __launch_bounds__(kAnyThreads) attention_any_kernel(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float w[kAnyChunk];
  __shared__ float red_m[kAnyThreads / 32], red_l[kAnyThreads / 32];
  __shared__ float stat[2];
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int hd = a.head_dim;
  const int G = a.n_heads / a.n_kv_heads;
  const int kvh = h / G;
  const int pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
  const size_t row_stride = (size_t)a.n_kv_heads * hd;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * hd;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * hd;
  const float* qh = a.q + (size_t)h * hd;
  const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
  auto score = [&](int t) {
    const float* kr = kbase + (size_t)t * row_stride;
    float d = 0.0f;
    for (int i = 0; i < hd; ++i) d = fmaf(__ldcg(qh + i), __ldcg(kr + i), d);
    return __fmul_rn(d, scale);
  };
  float m = -INFINITY, l = 0.0f;
  for (int t = tid; t <= pos; t += kAnyThreads) {
    const float sc = score(t);
    const float nm = fmaxf(m, sc);
    l = l * expf(m - nm) + expf(sc - nm);
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float ol = __shfl_xor_sync(0xffffffffu, l, o);
    const float nm = fmaxf(m, om);
    l = (m == -INFINITY ? 0.0f : l * expf(m - nm)) + (om == -INFINITY ? 0.0f : ol * expf(om - nm));
    m = nm;
  }
  if (lane == 0) {
    red_m[wid] = m;
    red_l[wid] = l;
  }
  __syncthreads();
  if (tid == 0) {
    float M = -INFINITY, L = 0.0f;
    for (int i = 0; i < kAnyThreads / 32; ++i) {
      const float nm = fmaxf(M, red_m[i]);
      L = (M == -INFINITY ? 0.0f : L * expf(M - nm)) +
          (red_m[i] == -INFINITY ? 0.0f : red_l[i] * expf(red_m[i] - nm));
      M = nm;
    }
    stat[0] = M;
    stat[1] = L;
  }
  __syncthreads();
  const float M = stat[0], L = stat[1];
  for (int d0 = 0; d0 < hd; d0 += kAnyThreads) {
    const int d = d0 + tid;
    float acc = 0.0f;
    for (int c0 = 0; c0 <= pos; c0 += kAnyChunk) {
      const int n = min(kAnyChunk, pos + 1 - c0);
      __syncthreads();
      for (int t = tid; t < n; t += kAnyThreads) w[t] = expf(score(c0 + t) - M);
      __syncthreads();
      if (d < hd)
        for (int t = 0; t < n; ++t)
          acc = fmaf(w[t], __ldcg(vbase + (size_t)(c0 + t) * row_stride + d), acc);
    }
    if (d < hd) a.out[(size_t)h * hd + d] = __fdiv_rn(acc, L);
  }
}

bool attention_fast_shape(int head_dim, int n_heads, int n_kv_heads) {
  return head_dim % 4 == 0 && head_dim <= 256 && n_heads / n_kv_heads <= kMaxGroup;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t stream, bool pdl) {
  if (!attention_fast_shape(a.head_dim, a.n_heads, a.n_kv_heads))
    return launch(attention_any_kernel, dim3(a.n_heads), dim3(kAnyThreads), 0, stream, pdl, a);
  const int cap = chunk_cap_for(a.max_seq, a.max_splits, a.min_chunk);
  // the templated kernel reads q and writes out with 16-byte vectors
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.out) |
        reinterpret_cast<uintptr_t>(a.partials)) & 15u) == 0;
  const bool hd_kernel = (a.head_dim == 64 || a.head_dim == 128) && aligned;
  const size_t smem = hd_kernel ? smem_bytes_hd(a.head_dim, cap, a.max_splits, 256)
                                : smem_bytes(kThreads, a.head_dim, cap, a.max_splits);
  cudaError_t e = attention_prepare();
  if (e != cudaSuccess) return e;
  const dim3 grid(a.n_kv_heads, a.max_splits);
  const int G = a.n_kv_heads > 0 ? a.n_heads / a.n_kv_heads : 1;
  if (hd_kernel && a.max_splits == 1 && a.max_seq <= kShortMax) {
    const dim3 hgrid(a.n_kv_heads, 1, G);
    if (a.head_dim == 64)
      return launch(attention_short_kernel<64>, hgrid, dim3(256), 0, stream, pdl, a);
    return launch(attention_short_kernel<128>, hgrid, dim3(256), 0, stream, pdl, a);
  }
  if (hd_kernel && a.max_splits == 1 && G > 1) {
    const dim3 hgrid(a.n_kv_heads, 1, G);
    if (a.head_dim == 64)
      return launch(attention_hd_head_kernel<64>, hgrid, dim3(256), smem, stream, pdl, a, cap);
    return launch(attention_hd_head_kernel<128>, hgrid, dim3(256), smem, stream, pdl, a, cap);
  }
  if (hd_kernel && a.head_dim == 64)
    return launch(attention_hd_kernel<64>, grid, dim3(256), smem, stream, pdl, a, cap);
  if (hd_kernel && a.head_dim == 128)
    return launch(attention_hd_kernel<128>, grid, dim3(256), smem, stream, pdl, a, cap);
  return launch(attention_kernel, grid, dim3(kThreads), smem, stream, pdl, a, cap);
}

}  // namespace dqmk

// ------------------------------------------------------------------ C ABI
using namespace dqmk;

extern "C" int dqmk_attention_decode(const float* q, const float* keys, const float* values,
                                     int n_layers, int max_seq, int n_kv_heads, int head_dim,
                                     int layer, int pos, int n_heads, float* out,
                                     void* stream) {
  const char* api = "CudaAttentionDecode";
  if (layer < 0 || layer >= n_layers) return fail(DQMK_ERR_RANGE, std::string(api) + ": layer out of range");
  if (pos < 0 || pos >= max_seq) return fail(DQMK_ERR_RANGE, std::string(api) + ": pos out of range");
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || n_heads % n_kv_heads != 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid head configuration");
  if (!q || !keys || !values || !out) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  // the fast kernels read the cache with 16-byte vectors; other shapes take
  // the general kernel
  if (attention_fast_shape(head_dim, n_heads, n_kv_heads) &&
      ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values)) & 15u))
    return fail(DQMK_ERR_INVALID, std::string(api) + ": KV cache must be 16-byte aligned");
  const int splits = attention_splits(max_seq, n_kv_heads);
  const size_t tickets_bytes = 256;
  const size_t part_bytes = attention_partials_floats(n_heads, head_dim, splits) * sizeof(float);
  void* scratch = nullptr;
  DQMK_CUDA_RET(api, device_scratch(4096 + tickets_bytes + part_bytes, &scratch));
  AttnArgs a = {};
  a.q = q;
  a.keys = keys;
  a.values = values;
  a.max_seq = max_seq;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer;
  a.n_heads = n_heads;
  a.pos_dev = nullptr;
  a.pos_arg = pos;
  a.out = out;
  // scratch layout: [0,4096) argmax slot, then tickets, then partials
  a.tickets = reinterpret_cast<unsigned int*>(static_cast<char*>(scratch) + 4096);
  a.partials = reinterpret_cast<float*>(static_cast<char*>(scratch) + 4096 + tickets_bytes);
  a.max_splits = splits;
  if (n_kv_heads * sizeof(unsigned int) > tickets_bytes)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": too many KV heads");
  DQMK_CUDA_RET(api, launch_attention(a, static_cast<cudaStream_t>(stream), false));
  return DQMK_OK;
}

// ------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory when they run attention: an
// engine that reserves its whole device budget at start-up and treats any
// later cudaMalloc as a failure, or a host that embeds this library and
// forbids allocations outside its own allocator.  For them the split
// partials and completion tickets live in this fixed, file-scope buffer
// instead of the library's growable scratch.  Every GPU that loads the
// library holds these 2 MiB until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
constexpr size_t kNoAllocTicketBytes = 256;               // zeroed before every call
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attention_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};  // device address of the buffer, per device

// Host code sees the array's name only as a stand-in symbol; the device
// address comes from cudaGetSymbolAddress with that device current.
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attention_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int dqmk_attention_decode_noalloc(const float* q, const float* keys,
                                             const float* values, int n_layers, int max_seq,
                                             int n_kv_heads, int head_dim, int layer, int pos,
                                             int n_heads, float* out, void* stream) {
  const char* api = "CudaAttentionDecodeNoAlloc";
  if (layer < 0 || layer >= n_layers) return fail(DQMK_ERR_RANGE, std::string(api) + ": layer out of range");
  if (pos < 0 || pos >= max_seq) return fail(DQMK_ERR_RANGE, std::string(api) + ": pos out of range");
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || n_heads % n_kv_heads != 0)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid head configuration");
  if (!q || !keys || !values || !out) return fail(DQMK_ERR_INVALID, std::string(api) + ": null pointer");
  // the fast kernels read the cache with 16-byte vectors; other shapes take
  // the general kernel
  if (attention_fast_shape(head_dim, n_heads, n_kv_heads) &&
      ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values)) & 15u))
    return fail(DQMK_ERR_INVALID, std::string(api) + ": KV cache must be 16-byte aligned");
  if (n_kv_heads * sizeof(unsigned int) > kNoAllocTicketBytes)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": too many KV heads");
  const int splits = attention_splits(max_seq, n_kv_heads);
  const size_t need =
      kNoAllocTicketBytes + attention_partials_floats(n_heads, head_dim, splits) * sizeof(float);
  if (need > kNoAllocScratchBytes)
    return fail(DQMK_ERR_UNSUPPORTED,
                std::string(api) + ": needs " + std::to_string(need) +
                    " bytes of scratch, the static buffer holds " +
                    std::to_string(kNoAllocScratchBytes) + " (fewer heads, a smaller head_dim or "
                    "a shorter max_seq fit)");
  void* scratch = nullptr;
  DQMK_CUDA_RET(api, noalloc_scratch(&scratch));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the buffer keeps the previous call's contents: tickets must start at zero
  DQMK_CUDA_RET(api, cudaMemsetAsync(scratch, 0, kNoAllocTicketBytes, s));
  AttnArgs a = {};
  a.q = q;
  a.keys = keys;
  a.values = values;
  a.max_seq = max_seq;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer;
  a.n_heads = n_heads;
  a.pos_dev = nullptr;
  a.pos_arg = pos;
  a.out = out;
  a.tickets = static_cast<unsigned int*>(scratch);
  a.partials = reinterpret_cast<float*>(static_cast<char*>(scratch) + kNoAllocTicketBytes);
  a.max_splits = splits;
  DQMK_CUDA_RET(api, launch_attention(a, s, false));
  return DQMK_OK;
}
