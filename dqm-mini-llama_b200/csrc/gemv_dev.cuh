// gemv_dev.cuh -- device code of the batch-1 decode GEMV over Q8_0 / Q4_0
// weights, instantiated by the kernels of gemv.cu.  See gemv.cu for the
// design.
#pragma once

#include "common.cuh"
#include "internal.h"

// Every register-GEMV instantiation the dispatcher (gemv.cu, gemv_variant_id)
// can pick, with its id: X(id, quant type, rows per group, chunks per lane,
// warps per row group).
#define DQMK_GEMV_VARIANT_IDS_Q80(X)                                                        \
  X(0, DQMK_Q80, 2, 1, 1) X(1, DQMK_Q80, 2, 2, 1) X(2, DQMK_Q80, 4, 2, 1)                  \
  X(3, DQMK_Q80, 2, 2, 4) X(4, DQMK_Q80, 2, 3, 4) X(5, DQMK_Q80, 2, 4, 4)
#define DQMK_GEMV_VARIANT_IDS_WIDE(X) X(6, DQMK_Q80, 4, 2, 4) X(7, DQMK_Q80, 4, 4, 4)
#define DQMK_GEMV_VARIANT_IDS_Q40(X)                                                        \
  X(8, DQMK_Q40, 4, 1, 1) X(9, DQMK_Q40, 2, 2, 1) X(10, DQMK_Q40, 4, 2, 1)                 \
  X(11, DQMK_Q40, 2, 2, 4) X(12, DQMK_Q40, 2, 4, 4) X(13, DQMK_Q40, 2, 5, 4)                 \
  X(14, DQMK_Q40, 2, 1, 1)
#define DQMK_GEMV_VARIANT_IDS(X) \
  DQMK_GEMV_VARIANT_IDS_Q80(X) DQMK_GEMV_VARIANT_IDS_WIDE(X) DQMK_GEMV_VARIANT_IDS_Q40(X)

namespace dqmk {
namespace gv {

constexpr float kMagicQ8 = -8388736.0f;  // -(2^23 + 128): biased byte -> int8 value
constexpr float kMagicQ4 = -8388616.0f;  // -(2^23 + 8):   nibble -> value - 8
constexpr int kWarps = 4;                // warps per CTA

template <int QT>
struct Fmt;
template <>
struct Fmt<DQMK_Q80> {
  static constexpr int kElems = 16;  // values per 16-byte chunk
  static constexpr int kSlots = 4;   // float4 slots of x per chunk
};
template <>
struct Fmt<DQMK_Q40> {
  static constexpr int kElems = 32;
  static constexpr int kSlots = 8;
};

// Shared-memory float4 index of slot s of chunk c.  The XOR swizzle makes the
// 8 lanes of one LDS.128 phase (consecutive chunks) hit 8 distinct 16-byte
// bank groups.
template <int QT>
__device__ __forceinline__ int xslot(int c, int s) {
  if constexpr (QT == DQMK_Q80) {
    return c * 4 + (s ^ ((c >> 1) & 3));
  } else {
    return c * 8 + (s ^ (c & 7));
  }
}

template <int QT>
__device__ __forceinline__ int xphys(int e) {
  constexpr int E = Fmt<QT>::kElems;
  const int c = e / E;
  const int s = (e % E) >> 2;
  return xslot<QT>(c, s) * 4 + (e & 3);
}

// 16 int8 weights . 16 floats
__device__ __forceinline__ float dot_q8(const uint4 w, const float4 (&xv)[8]) {
  const unsigned long long M = f2_pack(kMagicQ8, kMagicQ8);
  unsigned long long a0 = 0ull, a1 = 0ull;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t wb = ws[i] ^ 0x80808080u;
    const unsigned long long q01 = fadd2(f2_pack(magic_byte(wb, 0), magic_byte(wb, 1)), M);
    const unsigned long long q23 = fadd2(f2_pack(magic_byte(wb, 2), magic_byte(wb, 3)), M);
    a0 = ffma2(q01, f2_pack(xv[i].x, xv[i].y), a0);
    a1 = ffma2(q23, f2_pack(xv[i].z, xv[i].w), a1);
  }
  const unsigned long long s = fadd2(a0, a1);
  return f2_lo(s) + f2_hi(s);
}

// one Q4_0 block (32 nibbles) . 32 floats; word i holds values 4i..4i+3 in
// its low nibbles and 16+4i..16+4i+3 in its high nibbles.
__device__ __forceinline__ float dot_q4(const uint4 w, const float4 (&xv)[8]) {
  const unsigned long long M = f2_pack(kMagicQ4, kMagicQ4);
  unsigned long long a0 = 0ull, a1 = 0ull;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = ws[i] & 0x0f0f0f0fu;
    const uint32_t hi = (ws[i] >> 4) & 0x0f0f0f0fu;
    const unsigned long long l01 = fadd2(f2_pack(magic_byte(lo, 0), magic_byte(lo, 1)), M);
    const unsigned long long l23 = fadd2(f2_pack(magic_byte(lo, 2), magic_byte(lo, 3)), M);
    const unsigned long long h01 = fadd2(f2_pack(magic_byte(hi, 0), magic_byte(hi, 1)), M);
    const unsigned long long h23 = fadd2(f2_pack(magic_byte(hi, 2), magic_byte(hi, 3)), M);
    a0 = ffma2(l01, f2_pack(xv[i].x, xv[i].y), a0);
    a1 = ffma2(l23, f2_pack(xv[i].z, xv[i].w), a1);
    a0 = ffma2(h01, f2_pack(xv[4 + i].x, xv[4 + i].y), a0);
    a1 = ffma2(h23, f2_pack(xv[4 + i].z, xv[4 + i].w), a1);
  }
  const unsigned long long s = fadd2(a0, a1);
  return f2_lo(s) + f2_hi(s);
}

template <int QT, int RPW, int CPL>
struct Tile {
  uint4 w[RPW][CPL];
  uint16_t d[RPW][CPL];
};

// Row groups are RPW rows; GT threads (one warp, or the whole CTA) share a
// group and stride over its 16-byte chunks.
struct Geo {
  int chunks, row_bytes, nbk, seg_chunks, nseg, gw, nw;
};

template <int QT, int RPW, int CPL, int GT>
__device__ __forceinline__ void load_step(Tile<QT, RPW, CPL>& t, const GemvArgs& a,
                                          const Geo& g, int step, int gt) {
  const int gi = step / g.nseg;
  const int seg = step - gi * g.nseg;
  const int grp = g.gw + gi * g.nw;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int row = grp * RPW + r;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = seg * g.seg_chunks + j * GT + gt;
      if (row < a.n_rows && c < g.chunks) {
        t.w[r][j] = ldg_stream(a.qs + (size_t)row * g.row_bytes + (size_t)c * 16);
        t.d[r][j] = __ldg(a.d + (size_t)row * g.nbk + (QT == DQMK_Q80 ? (c >> 1) : c));
      } else {
        t.w[r][j] = make_uint4(0u, 0u, 0u, 0u);
        t.d[r][j] = 0;
      }
    }
  }
}

template <int QT, int RPW, int CPL, int GT>
__device__ __forceinline__ void compute_step(const Tile<QT, RPW, CPL>& t, const Geo& g,
                                             int step, int gt, const float4* xs,
                                             float (&acc)[RPW]) {
  const int seg = step % g.nseg;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = seg * g.seg_chunks + j * GT + gt;
    if (c < g.chunks) {
      float4 xv[8];
#pragma unroll
      for (int s = 0; s < Fmt<QT>::kSlots; ++s) xv[s] = xs[xslot<QT>(c, s)];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const float part = QT == DQMK_Q80 ? dot_q8(t.w[r][j], xv) : dot_q4(t.w[r][j], xv);
        acc[r] = fmaf(h2f(t.d[r][j]), part, acc[r]);
      }
    }
  }
}

// RoPE rotation of one (x0, x1) pair with the reference's rounding pattern:
// NeoX pairs fuse the left product (src/ops.cc:46-49 as built), Normal pairs
// round every product (src/ops.cc:24-27 as built).
__device__ __forceinline__ void rope_pair(float& x0, float& x1, float c, float s, int neox) {
  const float a = x0, b = x1;
  if (neox) {
    x0 = __fmaf_rn(a, c, -__fmul_rn(b, s));
    x1 = __fmaf_rn(a, s, __fmul_rn(b, c));
  } else {
    x0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    x1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  }
}

// Epilogue operands of one row group fetched ahead of the arithmetic: the
// bias and the RoPE (cos, sin) of the QKV rows do not depend on the previous
// kernel (the position is advanced only between steps), so they are loaded
// before the dependency wait; the residual is loaded right after it, beside
// the staging of x, instead of after the dot products.  Lane r holds what
// the epilogue's writer of row r (kEpiStore) or of pair r (kEpiQkv) needs.
struct EpiPre {
  int grp = -1;  // row group these belong to (-1: none)
  float b0 = 0.0f, b1 = 0.0f, res = 0.0f;
  float2 cs = make_float2(1.0f, 0.0f);
};

// Position of a QKV pair's rotation in the RoPE table, and whether it rotates.
__device__ __forceinline__ bool qkv_pair_rope(const GemvArgs& a, int pp, int* i) {
  const int half = a.head_dim / 2;
  const int q_pairs = a.n_heads * half, kv_pairs = a.n_kv_heads * half;
  const int seg_pair = pp < q_pairs ? pp : (pp < q_pairs + kv_pairs ? pp - q_pairs : pp - q_pairs - kv_pairs);
  *i = seg_pair % half;
  return pp < q_pairs + kv_pairs;
}

template <int RPW>
__device__ __forceinline__ void epi_prefetch_const(const GemvArgs& a, int grp, int lane, int pos,
                                                   EpiPre& e) {
  if (a.epi == kEpiStore) {
    const int row = grp * RPW + lane;
    if (lane < RPW && row < a.n_rows && a.bias) e.b0 = __ldg(a.bias + row);
    e.grp = grp;
  } else if (a.epi == kEpiQkv) {
    const int pp = (grp * RPW) / 2 + lane;
    if (lane < RPW / 2 && 2 * pp + 1 < a.n_rows) {
      if (a.bias) {
        e.b0 = __ldg(a.bias + 2 * pp);
        e.b1 = __ldg(a.bias + 2 * pp + 1);
      }
      int i = 0;
      if (qkv_pair_rope(a, pp, &i)) e.cs = __ldg(a.rope_cs + (size_t)pos * (a.head_dim / 2) + i);
    }
    e.grp = grp;
  }
}

template <int RPW>
__device__ __forceinline__ void epi_prefetch_res(const GemvArgs& a, int lane, EpiPre& e) {
  if (a.epi == kEpiStore && a.residual && e.grp >= 0) {
    const int row = e.grp * RPW + lane;
    if (lane < RPW && row < a.n_rows) e.res = __ldcg(a.residual + row);
  }
}

template <int RPW, bool PEER>
__device__ __forceinline__ void epilogue(const GemvArgs& a, int grp, int lane,
                                         const float (&acc)[RPW], int pos,
                                         unsigned long long& best, const EpiPre* pre = nullptr) {
  const bool have = pre && pre->grp == grp;
  if constexpr (PEER) {
    // row-parallel partial sum (kEpiPeer): to slot [parity][own rank] of every
    // rank.  A separate instantiation, so the other kernels' code is untouched.
    const unsigned int s = a.peer.seq[0] + 1;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int row = grp * RPW + r;
      if (lane == r && row < a.n_rows) {
        for (int w = 0; w < a.peer.world; ++w)
          reinterpret_cast<float*>(a.peer.base[w] + tp_vec_off((int)(s & 1u), a.peer.rank,
                                                               a.peer.world, a.peer.dim))[row] =
              acc[r];
      }
    }
    return;
  }
  if (a.epi == kEpiStore) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int row = grp * RPW + r;
      if (lane == r && row < a.n_rows) {
        float v = acc[r];
        if (a.bias) v = __fadd_rn(v, have ? pre->b0 : a.bias[row]);
        if (a.residual) v = __fadd_rn(have ? pre->res : __ldcg(a.residual + row), v);
        a.y[row] = v;
      }
    }
  } else if (a.epi == kEpiLogits) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int row = grp * RPW + r;
      if (lane == r && row < a.n_rows) {
        a.y[row] = acc[r];
        const unsigned long long key = argmax_key(acc[r], (uint32_t)(row + a.row_offset));
        best = key > best ? key : best;
      }
    }
  } else if (a.epi == kEpiSwiGlu) {
    // packed rows (2p, 2p+1) = (gate_o, up_o); src/ops.cc:140-151
#pragma unroll
    for (int p = 0; p < RPW / 2; ++p) {
      const int o = (grp * RPW) / 2 + p;
      if (lane == p && 2 * o + 1 < a.n_rows) {
        const float gt = acc[2 * p], up = acc[2 * p + 1];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt)));
        a.y[o] = __fmul_rn(__fmul_rn(gt, sig), up);
      }
    }
  } else {  // kEpiQkv
    const int half = a.head_dim / 2;
    const int q_pairs = a.n_heads * half;
    const int kv_pairs = a.n_kv_heads * half;
#pragma unroll
    for (int p = 0; p < RPW / 2; ++p) {
      const int pp = (grp * RPW) / 2 + p;  // packed pair index
      if (lane == p && 2 * pp + 1 < a.n_rows) {
        float x0 = acc[2 * p], x1 = acc[2 * p + 1];
        if (a.bias) {
          x0 = __fadd_rn(x0, have ? pre->b0 : a.bias[2 * pp]);
          x1 = __fadd_rn(x1, have ? pre->b1 : a.bias[2 * pp + 1]);
        }
        int seg_pair, nh;
        float* dst;
        bool rotate = true;
        if (pp < q_pairs) {
          seg_pair = pp;
          nh = a.n_heads;
          dst = a.q_out;
        } else if (pp < q_pairs + kv_pairs) {
          seg_pair = pp - q_pairs;
          nh = a.n_kv_heads;
          dst = a.k_cache + ((size_t)a.layer * a.max_seq + pos) * nh * a.head_dim;
        } else {
          seg_pair = pp - q_pairs - kv_pairs;
          nh = a.n_kv_heads;
          dst = a.v_cache + ((size_t)a.layer * a.max_seq + pos) * nh * a.head_dim;
          rotate = false;
        }
        const int h = seg_pair / half, i = seg_pair % half;
        int o0, o1;
        if (rotate && a.neox) {
          o0 = h * a.head_dim + i;
          o1 = o0 + half;
        } else {
          o0 = h * a.head_dim + 2 * i;
          o1 = o0 + 1;
        }
        if (rotate) {
          const float2 cs = have ? pre->cs : a.rope_cs[(size_t)pos * half + i];
          rope_pair(x0, x1, cs.x, cs.y, a.neox);
        }
        dst[o0] = x0;
        dst[o1] = x1;
      }
    }
  }
}

constexpr int kNormRegs = 8;  // float4 of RMSNorm weight prefetched per thread

// 16-byte global -> shared copy that does not go through registers.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src)
               : "memory");
}

// Stage x (k floats, zero-padded to kp) into swizzled shared memory, RMS-
// normalised when norm_w is set.  One global round trip: every thread issues
// all of its loads before using any.  Activations come from the previous
// kernel of the chain, so they are read through L2 (ld.global.cg).
// nws: the RMSNorm weight, copied into shared memory by the prefetch phase
// (each thread reads back exactly the float4s it copied).
template <int QT, int NWARPS, int NR>
__device__ __forceinline__ void stage_x(const GemvArgs& a, float4* xs, const float4* nws,
                                        bool norm_pref, float* red, float* bcast) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int NT = NWARPS * 32;
  float* xsf = reinterpret_cast<float*>(xs);
  const int nf4 = a.kp >> 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) && ((a.k & 3) == 0);
  float ss = 0.0f;
  if (vec) {
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
          const int e = i4 * 4;
          xs[xslot<QT>(e / Fmt<QT>::kElems, (e % Fmt<QT>::kElems) >> 2)] = v[u];
        }
      }
    }
  } else {
    for (int e = tid; e < a.kp; e += NT) {
      const float v = e < a.k ? __ldcg(a.x + e) : 0.0f;
      xsf[xphys<QT>(e)] = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  }
  if (a.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) red[wid] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < NWARPS; ++w) t += red[w];
      const float mean = __fdiv_rn(t, (float)a.k);
      *bcast = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, a.eps)));
    }
    __syncthreads();
    const float scale = *bcast;
    // the prefetch phase's copies of the norm weight (none in flight when it
    // issued none) land before any use and before the kernel can exit
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (vec && norm_pref) {
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        const int i4 = u * NT + tid;
        if (i4 < (a.k >> 2)) {
          const int e = i4 * 4;
          float4* p = &xs[xslot<QT>(e / Fmt<QT>::kElems, (e % Fmt<QT>::kElems) >> 2)];
          float4 v = *p;
          const float4 nw = nws[i4];
          v.x = __fmul_rn(__fmul_rn(v.x, scale), nw.x);
          v.y = __fmul_rn(__fmul_rn(v.y, scale), nw.y);
          v.z = __fmul_rn(__fmul_rn(v.z, scale), nw.z);
          v.w = __fmul_rn(__fmul_rn(v.w, scale), nw.w);
          *p = v;
        }
      }
    } else {
      // every element is rescaled by the thread that wrote it
      if (vec) {
        for (int i4 = tid; i4 < (a.k >> 2); i4 += NT) {
          const int e = i4 * 4;
          float4* p = &xs[xslot<QT>(e / Fmt<QT>::kElems, (e % Fmt<QT>::kElems) >> 2)];
          const float4 w4 = __ldg(reinterpret_cast<const float4*>(a.norm_w) + i4);
          float4 v = *p;
          v.x = __fmul_rn(__fmul_rn(v.x, scale), w4.x);
          v.y = __fmul_rn(__fmul_rn(v.y, scale), w4.y);
          v.z = __fmul_rn(__fmul_rn(v.z, scale), w4.z);
          v.w = __fmul_rn(__fmul_rn(v.w, scale), w4.w);
          *p = v;
        }
      } else {
        for (int e = tid; e < a.k; e += NT) {
          const int p = xphys<QT>(e);
          xsf[p] = __fmul_rn(__fmul_rn(xsf[p], scale), a.norm_w[e]);
        }
      }
    }
  }
  __syncthreads();
}

// Thread 0 of each CTA with the CTA's best (value, index) key: fold it into
// the device argmax; the last CTA then advances the greedy state (token,
// position, history) unless ticket is null (tensor parallel: the ranks' keys
// are combined by a later kernel).  Without a valid key (a CTA's bounded wait
// ran out before its rows were scored) the state is kept and kErrNoToken
// recorded in *err.
__device__ __forceinline__ void logits_finish(const GemvArgs& a, unsigned long long b,
                                              int n_ctas, unsigned int* err) {
  if (!a.argmax_slot) return;
  atomicMax(a.argmax_slot, b);
  if (!a.ticket) return;
  __threadfence();
  const unsigned int done = atomicAdd(a.ticket, 1u);
  if (done != (unsigned int)n_ctas - 1) return;
  __threadfence();
  const unsigned long long key = atomicAdd(a.argmax_slot, 0ull);
  *a.ticket = 0u;
  int idx = 0;
  if (!argmax_token(key, a.row_offset + a.n_rows, &idx)) {
    atomicOr(err, kErrNoToken);
    return;
  }
  const int p = *a.pos_slot;
  if (a.history && p >= 0 && p < a.history_cap) a.history[p] = idx;
  *a.token_slot = idx;
  *a.pos_slot = p + 1;
}

// One GEMV on one CTA of a grid of n_ctas, in two parts: prefetch() computes
// the CTA's share of row groups and loads its first two weight tiles into
// registers and the RMSNorm weight into shared memory -- none of it depends
// on the previous step of
// the chain, so callers issue it before griddepcontrol.wait; run() stages x
// and does the math and the epilogue.
template <int QT, int RPW, int CPL, int GW>
struct GemvPhase {
  static_assert(GW == 1 || GW == kWarps, "a row group is one warp or the whole CTA");
  static constexpr int GT = GW * 32;       // threads per row group
  static constexpr int GPC = kWarps / GW;  // row groups per CTA
  Geo g;
  int total, gt, pos;
  Tile<QT, RPW, CPL> ta, tb;
  bool norm_pref;
  EpiPre pre;

  // nws: shared memory for the RMSNorm weight (kp floats, after x's).
  __device__ __forceinline__ void prefetch(const GemvArgs& a, int cta, int n_ctas, float4* nws) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    gt = (wid % GW) * 32 + lane;
    g.chunks = a.kp / Fmt<QT>::kElems;
    g.row_bytes = QT == DQMK_Q80 ? a.kp : a.kp / 2;
    g.nbk = a.kp / 32;
    g.seg_chunks = GT * CPL;
    g.nseg = (g.chunks + g.seg_chunks - 1) / g.seg_chunks;
    g.gw = cta * GPC + wid / GW;
    g.nw = n_ctas * GPC;
    const int n_groups = (a.n_rows + RPW - 1) / RPW;
    const int my_groups = g.gw < n_groups ? (n_groups - g.gw + g.nw - 1) / g.nw : 0;
    total = my_groups * g.nseg;
    // the warp's first two tiles: both are in flight before the dependency
    // resolves (the tile registers exist for the two-stage pipeline anyway)
    if (total > 0) load_step<QT, RPW, CPL, GT>(ta, a, g, 0, gt);
    if (total > 1) load_step<QT, RPW, CPL, GT>(tb, a, g, 1, gt);
    // the position is advanced only between steps: stable across this one
    pos = 0;
    if (a.epi == kEpiQkv) pos = a.pos_dev ? __ldcg(a.pos_dev) : a.pos_arg;
    if (total > 0) epi_prefetch_const<RPW>(a, g.gw, lane, pos, pre);
    norm_pref = a.norm_w && (a.kp >> 2) <= kNormRegs * kWarps * 32 && ((a.k & 3) == 0) &&
                ((reinterpret_cast<uintptr_t>(a.norm_w) & 15u) == 0);
    if (norm_pref) {
#pragma unroll
      for (int u = 0; u < kNormRegs; ++u) {
        const int i4 = u * kWarps * 32 + tid;
        if (i4 < (a.k >> 2)) cp_async16(nws + i4, reinterpret_cast<const float4*>(a.norm_w) + i4);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
};

template <int QT, int RPW, int CPL, int GW, bool PEER>
__device__ __forceinline__ void gemv_run(GemvPhase<QT, RPW, CPL, GW>& ph, const GemvArgs& a,
                                         float4* xs, int n_ctas, unsigned int* err) {
  constexpr int GT = GW * 32;
  __shared__ float red[kWarps];
  __shared__ float red_rows[kWarps][RPW];
  __shared__ float bcast;
  __shared__ unsigned long long best_w[kWarps];

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int gt = ph.gt;
  const Geo& g = ph.g;
  const int total = ph.total;
  Tile<QT, RPW, CPL>& ta = ph.ta;
  Tile<QT, RPW, CPL>& tb = ph.tb;

  epi_prefetch_res<RPW>(a, lane, ph.pre);
  stage_x<QT, kWarps, kNormRegs>(a, xs, xs + (a.kp >> 2), ph.norm_pref, red, &bcast);

  const int pos = ph.pos;
  unsigned long long best = 0ull;
  float acc[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = 0.0f;

  auto finish = [&](int step) {
    if ((step % g.nseg) != g.nseg - 1) return;
    const int grp = g.gw + (step / g.nseg) * g.nw;
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = warp_sum(acc[r]);
    if constexpr (GW > 1) {
      // the CTA's warps hold partial sums of the same rows
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) red_rows[wid][r] = acc[r];
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) t += red_rows[w][r];
        acc[r] = t;
      }
      __syncthreads();
      if (wid == 0) epilogue<RPW, PEER>(a, grp, lane, acc, pos, best, &ph.pre);
    } else {
      epilogue<RPW, PEER>(a, grp, lane, acc, pos, best, &ph.pre);
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = 0.0f;
  };

  // two-stage register pipeline: load step s+1 while step s computes
  for (int s = 0; s < total; s += 2) {
    if (s + 1 < total && s > 0) load_step<QT, RPW, CPL, GT>(tb, a, g, s + 1, gt);
    compute_step<QT, RPW, CPL, GT>(ta, g, s, gt, xs, acc);
    finish(s);
    if (s + 1 < total) {
      if (s + 2 < total) load_step<QT, RPW, CPL, GT>(ta, a, g, s + 2, gt);
      compute_step<QT, RPW, CPL, GT>(tb, g, s + 1, gt, xs, acc);
      finish(s + 1);
    }
  }

  if (a.epi == kEpiLogits) {
    // CTA max -> one atomic per CTA; the last CTA to finish advances the
    // greedy decode state (token, position, history).
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) best_w[wid] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kWarps; ++w) b = best_w[w] > b ? best_w[w] : b;
      logits_finish(a, b, n_ctas, err);
    }
  }
  if constexpr (PEER) peer_signal(a.peer, 0, a.peer.seq[0] + 1, n_ctas);
}

}  // namespace gv
}  // namespace dqmk
