// attention_dev.cuh -- device code of GQA decode attention shared by the
// batch-1 kernels (attention.cu) and the multi-sequence kernels (batch.cu).
// See attention.cu for the design.
#pragma once

#include "common.cuh"
#include "internal.h"

namespace dqmk {
namespace at {

constexpr int kThreads = 128;
constexpr int kMaxGroup = 8;  // query heads per KV head
constexpr int kMinChunk = 128;

// Floats per split partial: the head_dim sums, then m and l, padded so every
// row starts 16-byte aligned (float4 reads in the combine).
__host__ __device__ constexpr int part_stride(int hd) { return hd + 4; }

__device__ __forceinline__ int round_up32(int v) { return (v + 31) & ~31; }

// Split bookkeeping shared by both kernel forms.
struct Split {
  int T, chunk, n_active, t0, n;
};

__device__ __forceinline__ Split split_of(const AttnArgs& a, int split, int pos) {
  Split s;
  s.T = pos + 1;
  s.chunk = round_up32((s.T + a.max_splits - 1) / a.max_splits);
  const int mc = a.min_chunk > 0 ? a.min_chunk : kMinChunk;
  if (s.chunk < mc) s.chunk = mc;
  s.n_active = (s.T + s.chunk - 1) / s.chunk;
  s.t0 = split * s.chunk;
  s.n = max(0, min(s.T, s.t0 + s.chunk) - s.t0);
  return s;
}

// Softmax statistics of one split's scores (one warp per head); scores are
// replaced by exp(s - m).
template <int NT>
__device__ __forceinline__ void split_softmax(float* ss, int chunk_cap, int G, int n,
                                              float* head_m, float* head_l) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int h = wid; h < G; h += NT / 32) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, ss[h * chunk_cap + t]);
    m = warp_max(m);
    float l = 0.0f;
    for (int t = lane; t < n; t += 32) {
      const float p = expf(ss[h * chunk_cap + t] - m);
      ss[h * chunk_cap + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      head_m[h] = m;
      head_l[h] = l;
    }
  }
}

// Last-CTA merge for the head_dim-templated kernel: the same arithmetic as
// split_combine, with each thread producing 4 consecutive output dims from
// float4 partial reads, all of its splits' loads issued in groups of 16.
template <int NT, int HD>
__device__ __forceinline__ void split_combine_hd(const AttnArgs& a, int kvh, int G, int n_active,
                                                 int n_splits, float* stats, int* is_last) {
  constexpr int PS = part_stride(HD);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int done = atomicAdd(&a.tickets[kvh], 1u);
    *is_last = done == (unsigned int)n_splits - 1;
  }
  __syncthreads();
  if (!*is_last) return;
  __threadfence();
  float* w = stats;                                              // [n_active][8] weights
  float* lsum = stats + (size_t)a.max_splits * kMaxGroup;        // [n_active][8] l
  float* inv_den = lsum + (size_t)a.max_splits * kMaxGroup;      // [8]
  for (int i = threadIdx.x; i < n_active * G; i += NT) {
    const int sp = i / G, h = i % G;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(
        a.partials + ((size_t)(kvh * G + h) * a.max_splits + sp) * PS + HD));
    w[sp * kMaxGroup + h] = ml.x;
    lsum[sp * kMaxGroup + h] = ml.y;
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
      den = fmaf(e, lsum[sp * kMaxGroup + h], den);
    }
    inv_den[h] = den;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * (HD / 4); i += NT) {
    const int h = i / (HD / 4), d4 = i % (HD / 4);
    const float4* part = reinterpret_cast<const float4*>(
                             a.partials + (size_t)(kvh * G + h) * a.max_splits * PS) + d4;
    float4 num = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int sp0 = 0; sp0 < n_active; sp0 += 16) {
      float4 o[16];
#pragma unroll
      for (int u = 0; u < 16; ++u)
        o[u] = sp0 + u < n_active ? __ldcg(part + (size_t)(sp0 + u) * (PS / 4))
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        if (sp0 + u < n_active) {
          const float wt = w[(sp0 + u) * kMaxGroup + h];
          num.x = fmaf(wt, o[u].x, num.x);
          num.y = fmaf(wt, o[u].y, num.y);
          num.z = fmaf(wt, o[u].z, num.z);
          num.w = fmaf(wt, o[u].w, num.w);
        }
      }
    }
    const float den = inv_den[h];
    *reinterpret_cast<float4*>(a.out + (size_t)(kvh * G + h) * HD + d4 * 4) =
        make_float4(__fdiv_rn(num.x, den), __fdiv_rn(num.y, den), __fdiv_rn(num.z, den),
                    __fdiv_rn(num.w, den));
  }
  if (threadIdx.x == 0) a.tickets[kvh] = 0u;
}

// head_dim known at compile time (64 / 128), 256 threads.  Scores: HD/16
// threads per position, each holding 16 dims of the K row (4 x 16-byte loads),
// two position passes' loads issued together, partial dots folded with
// shuffles.  P.V: thread (d4, group) owns 4 consecutive dims and every
// GROUPS-th position, with 8 float4 V loads in flight.  A single active split
// writes its output directly.
template <int HD, int NT>
constexpr int hd_groups() {
  return NT / (HD / 4);
}

// One (KV head, split) work item of the grid: kvh, split of n_splits.
template <int HD, int NT>
__device__ __forceinline__ void attention_hd_body(const AttnArgs& a, int chunk_cap, int kvh,
                                                  int split, int n_splits, float* sm) {
  constexpr int TPT = HD / 16;          // threads per position (scores)
  constexpr int TOK = NT / TPT;         // positions per score pass
  constexpr int D4 = HD / 4;            // float4 columns
  constexpr int GROUPS = hd_groups<HD, NT>();  // position groups in P.V
  constexpr int PV = 8;                 // float4 V loads in flight per thread
  constexpr int PS = part_stride(HD);
  __shared__ float head_m[kMaxGroup], head_l[kMaxGroup];
  __shared__ int is_last;

  const int tid = threadIdx.x;
  const int G = a.n_heads / a.n_kv_heads;
  const int pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
  const Split sp = split_of(a, split, pos);
  const size_t row_stride = (size_t)a.n_kv_heads * HD;
  const float* kbase = a.keys + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD;
  const float* vbase = a.values + (size_t)a.layer * a.max_seq * row_stride + (size_t)kvh * HD;
  float* sq = sm;                            // [8][HD]
  float* ss = sq + kMaxGroup * HD;           // [8][chunk_cap]
  float* sacc = ss + kMaxGroup * chunk_cap;  // [GROUPS][8][HD]
  float* stats = sacc + GROUPS * kMaxGroup * HD;

  if (split < sp.n_active) {
    const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
    if constexpr (HD == 128) {
      // Scores with one K row per warp load: lane l holds dims 4l..4l+3 of
      // the row and of every query head (registers); a warp takes 4
      // consecutive positions per step, and the 4 x 8 partial dots are
      // summed across the lanes by a transposed butterfly (31 shuffles) that
      // leaves lane l with the score of position l / 8, head l % 8.
      const int lane = tid & 31, wid = tid >> 5;
      float4 qv[kMaxGroup];
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h)
        qv[h] = h < G ? __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)(kvh * G + h) * HD) +
                               lane)
                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int t0 = 4 * wid; t0 < sp.n; t0 += 4 * (NT / 32)) {
        float4 kr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          kr[i] = t0 + i < sp.n ? __ldcg(reinterpret_cast<const float4*>(
                                      kbase + (size_t)(sp.t0 + t0 + i) * row_stride) + lane)
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float v[32];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int h = 0; h < kMaxGroup; ++h) {
            float d = __fmul_rn(qv[h].x, kr[i].x);
            d = fmaf(qv[h].y, kr[i].y, d);
            d = fmaf(qv[h].z, kr[i].z, d);
            d = fmaf(qv[h].w, kr[i].w, d);
            v[i * kMaxGroup + h] = d;
          }
#pragma unroll
        for (int m = 16, n = 32; m >= 1; m >>= 1, n >>= 1) {
          const bool upper = (lane & m) != 0;
#pragma unroll
          for (int k = 0; k < n / 2; ++k) {
            const float send = upper ? v[k] : v[k + n / 2];
            const float keep = upper ? v[k + n / 2] : v[k];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, m);
          }
        }
        const int t = t0 + (lane >> 3), h = lane & 7;
        if (h < G && t < sp.n) ss[h * chunk_cap + t] = __fmul_rn(v[0], scale);
      }
    } else {
    for (int i = tid; i < G * D4; i += NT)
      reinterpret_cast<float4*>(sq)[i] =
          __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)(kvh * G) * HD) + i);
    __syncthreads();
    const int part = tid % TPT;
    for (int base = 0; base < sp.n; base += 2 * TOK) {
      float4 k4[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = base + u * TOK + tid / TPT;
        const float4* kr =
            reinterpret_cast<const float4*>(kbase + (size_t)(sp.t0 + t) * row_stride) + part * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          k4[u][i] = t < sp.n ? __ldcg(kr + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = base + u * TOK + tid / TPT;
        float dot[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
          float d = 0.0f;
          if (h < G) {
            const float4* q4 = reinterpret_cast<const float4*>(sq + h * HD) + part * 4;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 qq = q4[i];
              d = fmaf(qq.x, k4[u][i].x, d);
              d = fmaf(qq.y, k4[u][i].y, d);
              d = fmaf(qq.z, k4[u][i].z, d);
              d = fmaf(qq.w, k4[u][i].w, d);
            }
          }
          dot[h] = d;
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
#pragma unroll
          for (int o = TPT / 2; o > 0; o >>= 1) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], o);
        }
        if (t < sp.n && part == 0) {
#pragma unroll
          for (int h = 0; h < kMaxGroup; ++h)
            if (h < G) ss[h * chunk_cap + t] = __fmul_rn(dot[h], scale);
        }
      }
    }
    }
    __syncthreads();
    split_softmax<NT>(ss, chunk_cap, G, sp.n, head_m, head_l);
    __syncthreads();

    const int d4 = tid % D4, gi = tid / D4;
    float4 acc[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) acc[h] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int t = gi; t < sp.n; t += PV * GROUPS) {
      float4 v[PV];
#pragma unroll
      for (int u = 0; u < PV; ++u) {
        const int tt = t + u * GROUPS;
        v[u] = tt < sp.n ? __ldcg(reinterpret_cast<const float4*>(
                               vbase + (size_t)(sp.t0 + tt) * row_stride) + d4)
                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < PV; ++u) {
        const int tt = t + u * GROUPS;
        if (tt < sp.n) {
#pragma unroll
          for (int h = 0; h < kMaxGroup; ++h) {
            if (h < G) {
              const float pr = ss[h * chunk_cap + tt];
              acc[h].x = fmaf(pr, v[u].x, acc[h].x);
              acc[h].y = fmaf(pr, v[u].y, acc[h].y);
              acc[h].z = fmaf(pr, v[u].z, acc[h].z);
              acc[h].w = fmaf(pr, v[u].w, acc[h].w);
            }
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < G) reinterpret_cast<float4*>(sacc + (gi * kMaxGroup + h) * HD)[d4] = acc[h];
    __syncthreads();

    const bool direct = sp.n_active == 1;
    for (int i = tid; i < G * D4; i += NT) {
      const int h = i / D4, c4 = i % D4;
      float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int g2 = 0; g2 < GROUPS; ++g2) {
        const float4 x = reinterpret_cast<const float4*>(sacc + (g2 * kMaxGroup + h) * HD)[c4];
        o.x += x.x;
        o.y += x.y;
        o.z += x.z;
        o.w += x.w;
      }
      if (direct) {
        const float l = head_l[h];
        *reinterpret_cast<float4*>(a.out + (size_t)(kvh * G + h) * HD + c4 * 4) =
            make_float4(__fdiv_rn(o.x, l), __fdiv_rn(o.y, l), __fdiv_rn(o.z, l),
                        __fdiv_rn(o.w, l));
      } else {
        float* pp = a.partials + ((size_t)(kvh * G + h) * a.max_splits + split) * PS;
        reinterpret_cast<float4*>(pp)[c4] = o;
        if (c4 == 0) *reinterpret_cast<float2*>(pp + HD) = make_float2(head_m[h], head_l[h]);
      }
    }
  }
  if (sp.n_active > 1) split_combine_hd<NT, HD>(a, kvh, G, sp.n_active, n_splits, stats, &is_last);
}


// Dynamic shared memory of attention_hd_body<HD, NT>.
inline size_t smem_bytes_hd(int head_dim, int chunk_cap, int max_splits, int nt) {
  const int groups = nt / (head_dim / 4);
  return sizeof(float) * ((size_t)kMaxGroup * head_dim + (size_t)kMaxGroup * chunk_cap +
                          (size_t)groups * kMaxGroup * head_dim +
                          (size_t)(2 * max_splits + 1) * kMaxGroup);
}

}  // namespace at
}  // namespace dqmk
