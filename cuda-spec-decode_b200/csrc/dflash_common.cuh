// DFlash per-row streaming state and its merges (shared by the ring kernels
// and the 128-bit-load kernels).
//
// For a row pair (xl = draft logits, xt = verifier logits) the state keeps,
// relative to the running maxima mq (draft) and mp (verifier):
//   sq = sum e^(xl - mq),  sp = sum e^(xt - mp),  t = sum e^(xt - mp) (xt - xl)
// (KL), or for CE the first-index argmax of xt (bx, bi) and the draft logit
// at that index (bl). Merges are exact rescalings, applied in a fixed order.
#pragma once

#include <climits>
#include <cstdint>
#include <type_traits>

#include "bulk_copy.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

struct DfState {
  float mq, sq;      // draft log-sum-exp state (running max, sum of e^(x - max))
  float mp, sp, t;   // verifier log-sum-exp state and the p-weighted (xt - xl) sum (KL)
  float bx, bl;       // CE: best verifier logit, draft logit at that index
  int bi;             // CE: index of the best verifier logit (first occurrence)
};

__device__ __forceinline__ void df_init(DfState& st) {
  st.mq = kNegSeed;
  st.sq = 0.f;
  st.mp = kNegSeed;
  st.sp = 0.f;
  st.t = 0.f;
  st.bx = -INFINITY;
  st.bl = 0.f;
  st.bi = INT_MAX;
}

template <int KIND>
__device__ __forceinline__ void df_merge(DfState& x, const DfState& o) {
  lse_merge(x.mq, x.sq, o.mq, o.sq);
  if (KIND == kKindKL) {
    const float M = fmaxf(x.mp, o.mp);
    const float fa = exp_shift(x.mp, M), fb = exp_shift(o.mp, M);
    x.sp = x.sp * fa + o.sp * fb;
    x.t = x.t * fa + o.t * fb;
    x.mp = M;
  } else {
    if (o.bx > x.bx || (o.bx == x.bx && o.bi < x.bi)) {
      x.bx = o.bx;
      x.bi = o.bi;
      x.bl = o.bl;
    }
  }
}

template <int KIND>
__device__ __forceinline__ DfState df_shfl(const DfState& s, int o) {
  DfState r;
  r.mq = __shfl_xor_sync(kFullMask, s.mq, o);
  r.sq = __shfl_xor_sync(kFullMask, s.sq, o);
  if (KIND == kKindKL) {
    r.mp = __shfl_xor_sync(kFullMask, s.mp, o);
    r.sp = __shfl_xor_sync(kFullMask, s.sp, o);
    r.t = __shfl_xor_sync(kFullMask, s.t, o);
  } else {
    r.bx = __shfl_xor_sync(kFullMask, s.bx, o);
    r.bl = __shfl_xor_sync(kFullMask, s.bl, o);
    r.bi = __shfl_xor_sync(kFullMask, s.bi, o);
  }
  return r;
}

// Merges the 32 lanes' states into the warp's, valid in every lane: each
// log-sum-exp state is rescaled to the warp maximum (skipped when every lane
// already holds it -- a factor of e^0 = 1 exactly, the same bits) and summed
// over a fixed butterfly; the CE argmax is the largest verifier logit, ties
// to the smallest index.
template <int KIND>
__device__ __forceinline__ void df_warp_merge(DfState& s) {
  const float Mq = warp_max(s.mq);
  if (__any_sync(kFullMask, s.mq != Mq)) s.sq *= exp_shift(s.mq, Mq);
  s.mq = Mq;
  if (KIND == kKindKL) {
    const float Mp = warp_max(s.mp);
    if (__any_sync(kFullMask, s.mp != Mp)) {
      const float f = exp_shift(s.mp, Mp);
      s.sp *= f;
      s.t *= f;
    }
    s.mp = Mp;
  } else {
    const float Mx = warp_max(s.bx);
    // first index among the lanes that hold the maximum (INT_MAX: none)
    const unsigned cand = s.bx == Mx ? (unsigned)s.bi : (unsigned)INT_MAX;
    const unsigned bi = __reduce_min_sync(kFullMask, cand);
    const unsigned who = __ballot_sync(kFullMask, s.bx == Mx && (unsigned)s.bi == bi);
    s.bl = __shfl_sync(kFullMask, s.bl, who ? __ffs(who) - 1 : 0);
    s.bx = Mx;
    s.bi = (int)bi;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s.sq += __shfl_xor_sync(kFullMask, s.sq, o);
    if (KIND == kKindKL) {
      s.sp += __shfl_xor_sync(kFullMask, s.sp, o);
      s.t += __shfl_xor_sync(kFullMask, s.t, o);
    }
  }
}

// One element (scalar path); idx is the index within the row.
template <int KIND>
__device__ __forceinline__ void df_push(DfState& s, float a, float b, int idx) {
  lse_push(s.mq, s.sq, a);
  if (KIND == kKindKL) {
    if (b > s.mp) {
      const float f = exp_shift(s.mp, b);
      s.sp *= f;
      s.t *= f;
      s.mp = b;
    }
    const float e = exp_shift(b, s.mp);
    s.sp += e;
    s.t = fmaf(e, b - a, s.t);
  } else {
    if (b > s.bx || (b == s.bx && idx < s.bi)) {
      s.bx = b;
      s.bi = idx;
      s.bl = a;
    }
  }
}

template <int KIND, int U>
__device__ __forceinline__ void df_group(DfState& s, const float4 (&a)[U], const float4 (&b)[U],
                                         int base_idx, int stride_idx, uint64_t* empty = nullptr) {
  float cma = max4(a[0]);
#pragma unroll
  for (int u = 1; u < U; ++u) cma = fmaxf(cma, max4(a[u]));
  float cmb = max4(b[0]);
#pragma unroll
  for (int u = 1; u < U; ++u) cmb = fmaxf(cmb, max4(b[u]));
  if (empty) {  // a full stage, the whole warp here
    release_stage(empty, fmaxf(cma, cmb));  // both streams are in registers
    // one running maximum per stream for the whole warp: the piece's close needs no rescale
    cma = warp_max(cma);
    if (KIND == kKindKL) cmb = warp_max(cmb);
  }
  if (cma > s.mq) {
    s.sq *= exp_shift(s.mq, cma);
    s.mq = cma;
  }
  const float mq = s.mq;
  float accq = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    accq += exp_shift(a[u].x, mq) + exp_shift(a[u].y, mq) + exp_shift(a[u].z, mq) +
            exp_shift(a[u].w, mq);
  }
  s.sq += accq;
  if (KIND == kKindKL) {
    if (cmb > s.mp) {
      const float f = exp_shift(s.mp, cmb);
      s.sp *= f;
      s.t *= f;
      s.mp = cmb;
    }
    const float mp = s.mp;
    float accp = 0.f, acct = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float ex = exp_shift(b[u].x, mp);
      const float ey = exp_shift(b[u].y, mp);
      const float ez = exp_shift(b[u].z, mp);
      const float ew = exp_shift(b[u].w, mp);
      accp += (ex + ey) + (ez + ew);
      acct = fmaf(ex, b[u].x - a[u].x, acct);
      acct = fmaf(ey, b[u].y - a[u].y, acct);
      acct = fmaf(ez, b[u].z - a[u].z, acct);
      acct = fmaf(ew, b[u].w - a[u].w, acct);
    }
    s.sp += accp;
    s.t += acct;
  } else {
    if (cmb > s.bx) {
      // first element of the group equal to its max, in index order
#pragma unroll
      for (int u = U - 1; u >= 0; --u) {
        const int k = base_idx + u * stride_idx;
        if (b[u].w == cmb) { s.bi = k + 3; s.bl = a[u].w; }
        if (b[u].z == cmb) { s.bi = k + 2; s.bl = a[u].z; }
        if (b[u].y == cmb) { s.bi = k + 1; s.bl = a[u].y; }
        if (b[u].x == cmb) { s.bi = k + 0; s.bl = a[u].x; }
      }
      s.bx = cmb;
    }
  }
}

// bf16 vectors: lane element k of vector u is row index base_idx +
// u * stride_idx + k (k = 0..7, the low half of word k/2 first). Maxima are
// taken on the packed words; each element is widened once.
template <int KIND, int U>
__device__ __forceinline__ void df_group(DfState& s, const uint4 (&a)[U], const uint4 (&b)[U], int base_idx,
                                         int stride_idx, uint64_t* empty = nullptr) {
  uint32_t pa = bmax8(a[0]);
#pragma unroll
  for (int u = 1; u < U; ++u) pa = bmax2(pa, bmax8(a[u]));
  float cma = fmaxf(bf16_lo(pa), bf16_hi(pa));
  uint32_t pb = bmax8(b[0]);
#pragma unroll
  for (int u = 1; u < U; ++u) pb = bmax2(pb, bmax8(b[u]));
  float cmb = fmaxf(bf16_lo(pb), bf16_hi(pb));
  if (empty) {  // a full stage, the whole warp here
    release_stage(empty, fmaxf(cma, cmb));  // both streams are in registers
    cma = warp_max(cma);
    if (KIND == kKindKL) cmb = warp_max(cmb);
  }
  if (cma > s.mq) {
    s.sq *= exp_shift(s.mq, cma);
    s.mq = cma;
  }
  const float mq = s.mq;
  float2 accq = make_float2(0.f, 0.f);
#pragma unroll
  for (int u = 0; u < U; ++u) accq = fadd2(accq, vec8_expsum2(a[u], mq));
  s.sq += accq.x + accq.y;
  if (KIND == kKindKL) {
    if (cmb > s.mp) {
      const float f = exp_shift(s.mp, cmb);
      s.sp *= f;
      s.t *= f;
      s.mp = cmb;
    }
    const float mp = s.mp;
    float2 accp = make_float2(0.f, 0.f), acct = make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t wa[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
      const uint32_t wb[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 xl = bf16x2_f32(wa[h]), xt = bf16x2_f32(wb[h]);
        const float2 e = exp_shift2(xt, mp);
        accp = fadd2(accp, e);
        acct = ffma2(e, fsub2(xt, xl), acct);
      }
    }
    s.sp += accp.x + accp.y;
    s.t += acct.x + acct.y;
  } else {
    if (cmb > s.bx) {
      // first element of the group equal to its max, in index order
#pragma unroll
      for (int u = U - 1; u >= 0; --u) {
        const int k = base_idx + u * stride_idx;
        const uint32_t wa[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
        const uint32_t wb[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
        for (int h = 3; h >= 0; --h) {
          if (bf16_hi(wb[h]) == cmb) { s.bi = k + 2 * h + 1; s.bl = bf16_hi(wa[h]); }
          if (bf16_lo(wb[h]) == cmb) { s.bi = k + 2 * h; s.bl = bf16_lo(wa[h]); }
        }
      }
      s.bx = cmb;
    }
  }
}

// A stage range [a, b) of both streams (a stage cut by a row edge):
// element k of the stage is row index row_off + k. Scalar head and tail to
// 16-byte boundaries, then 16-byte vectors, four per lane per round.
template <int KIND, class T>
__device__ __forceinline__ void df_range(DfState& st, const T* sl, const T* sx, int a, int b, int row_off) {
  using Vec = typename std::conditional<sizeof(T) == 4, float4, uint4>::type;
  constexpr int kVec = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int av = (a + kVec - 1) & ~(kVec - 1), bv = b & ~(kVec - 1);
  if (av >= bv) {
    for (int k = a + lane; k < b; k += 32) df_push<KIND>(st, to_f32(sl[k]), to_f32(sx[k]), row_off + k);
    return;
  }
  if (lane < av - a) df_push<KIND>(st, to_f32(sl[a + lane]), to_f32(sx[a + lane]), row_off + a + lane);
  if (lane < b - bv) df_push<KIND>(st, to_f32(sl[bv + lane]), to_f32(sx[bv + lane]), row_off + bv + lane);
  const Vec* ql = reinterpret_cast<const Vec*>(sl);
  const Vec* qx = reinterpret_cast<const Vec*>(sx);
  int k = av / kVec + lane;
  const int kend = bv / kVec;
  for (; k + 96 < kend; k += 128) {
    const Vec va[4] = {ql[k], ql[k + 32], ql[k + 64], ql[k + 96]};
    const Vec vb[4] = {qx[k], qx[k + 32], qx[k + 64], qx[k + 96]};
    df_group<KIND, 4>(st, va, vb, row_off + k * kVec, 32 * kVec);
  }
  for (; k < kend; k += 32) {
    const Vec va[1] = {ql[k]};
    const Vec vb[1] = {qx[k]};
    df_group<KIND, 1>(st, va, vb, row_off + k * kVec, 32 * kVec);
  }
}

}  // namespace specdec
