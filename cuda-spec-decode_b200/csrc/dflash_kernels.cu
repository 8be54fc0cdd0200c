// DFlash objective (KL or CE against verifier logits, slot decay), forward and
// backward, for sm_100a.
//
// Reference behaviour (harvestingmoon/cuda-spec-decode):
//   models/dflash/loss.py:31-126   dflash_loss_fwd  (two passes: maxima, then A, B, C, D sums)
//   models/dflash/loss.py:128-166  dflash_loss_bwd  (s * (softmax(draft) - softmax(target) | onehot))
//   models/dflash/tests/test_loss.py:21-49  speculators oracle whose numbers this file reproduces
//     (decay index j % block_size as in test_loss.py:62; raw float mask in the
//      numerator and the denominator as in test_loss.py:46-49)
//
// Forward, one launch, ONE read of each row pair. With xl = draft logits,
// xt = verifier logits, p = softmax(xt), q = softmax(xl):
//   KL(p || q) = sum_v p_v (xt_v - xl_v) - logZp + logZq
// Each piece keeps, relative to the running maxima mq (draft) and mp (verifier),
//   sq = sum e^(xl - mq),  sp = sum e^(xt - mp),  t = sum e^(xt - mp) * (xt - xl),
// (t rescales with the verifier max only), or for CE the first-index argmax
// of xt with the draft logit at that index. The CTA landing last on a row
// merges the pieces in slot order and writes the row's loss, scale and
// log-normalisers; a global counter elects the CTA that sums the row losses
// in index order into the scalar loss. Rows whose weight mask*decay is 0 are
// never read.
#include "dflash_common.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

#include <climits>

namespace specdec {

namespace {

// Streams one piece [lo, hi) of a row pair. `vec` selects 128-bit loads (both
// rows share the same 16-byte phase).
template <int KIND, int NT, int U>
__device__ __forceinline__ void df_stream(DfState& s, const float* __restrict__ xl,
                                          const float* __restrict__ xt, int64_t lo, int64_t hi) {
  const int tid = threadIdx.x;
  const float* pl = xl + lo;
  const float* pt = xt + lo;
  const int64_t n = hi - lo;
  const bool vec = ((reinterpret_cast<uintptr_t>(pl) ^ reinterpret_cast<uintptr_t>(pt)) & 15) == 0;
  int64_t head = vec ? (((16 - (reinterpret_cast<uintptr_t>(pl) & 15)) & 15) >> 2) : n;
  if (head > n) head = n;
  const int64_t body = (n - head) >> 2;
  const int64_t tail0 = head + (body << 2);
  // index order per thread: head, body, tail (the CE argmax keeps the first max)
  for (int64_t i = tid; i < head; i += NT) df_push<KIND>(s, pl[i], pt[i], (int)(lo + i));
  const float4* ql = reinterpret_cast<const float4*>(pl + head);
  const float4* qt = reinterpret_cast<const float4*>(pt + head);
  const int base = (int)(lo + head);
  int64_t i = tid;
  for (; i + (U - 1) * NT < body; i += U * NT) {
    float4 a[U], b[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      a[u] = ld_stream(ql + i + u * NT);
      b[u] = ld_stream(qt + i + u * NT);
    }
    df_group<KIND, U>(s, a, b, base + 4 * (int)i, 4 * NT);
  }
  for (; i < body; i += NT) {
    float4 a[1], b[1];
    a[0] = ld_stream(ql + i);
    b[0] = ld_stream(qt + i);
    df_group<KIND, 1>(s, a, b, base + 4 * (int)i, 0);
  }
  for (int64_t i2 = tail0 + tid; i2 < n; i2 += NT) df_push<KIND>(s, pl[i2], pt[i2], (int)(lo + i2));
}

// Row weight w = mask * decay(pos) / (sum_j mask + 1e-5), pos = j % block_size.
// Follows models/dflash/tests/test_loss.py:23-27,43-49 (raw float mask).
__device__ __forceinline__ float df_decay(const DflashFwdArgs& a, int j) {
  const int pos = j % a.block_size;
  if (a.sfa) return expf(__fdiv_rn(-(float)pos, a.gamma));
  if (pos == 0) return 0.f;
  return expf(__fdiv_rn(-(float)(pos - 1), a.gamma));
}

__device__ __forceinline__ float df_mask(const DflashFwdArgs& a, int64_t r) {
  return a.mask ? a.mask[r] : 1.f;
}

// Numerator of the weight only (mask * decay): zero exactly when the row's
// weight is zero, so the row can be skipped.
__device__ __forceinline__ float df_numer(const DflashFwdArgs& a, int64_t r) {
  return __fmul_rn(df_mask(a, r), df_decay(a, (int)(r % a.B)));
}

template <int KIND>
__device__ void df_finalize_row(const DflashFwdArgs& a, int64_t r, int* sh_last) {
  const int lane = threadIdx.x & 31;
  __threadfence();
  const int64_t n = r / a.B;
  // denominator: sum of the sequence's raw mask values + 1e-5
  float m = 0.f;
  for (int i = lane; i < a.B; i += 32) m += df_mask(a, n * a.B + i);
  const float denom = warp_sum(m) + 1e-5f;
  const float numer = df_numer(a, r);
  const float w = __fdiv_rn(numer, denom);
  float el = 0.f, lzq = 0.f, lzp = 0.f;
  int64_t tgt = 0;
  if (numer != 0.f) {
    DfState s;
    df_init(s);
    const int k = a.pt.pieces(r);
    const DfPiece* part = a.part + r * a.pt.pmax;
    for (int q = lane; q < k; q += 32) {
      DfState o;
      const float4 lo4 = __ldcg(reinterpret_cast<const float4*>(part + q));
      const float4 hi4 = __ldcg(reinterpret_cast<const float4*>(part + q) + 1);
      o.mq = lo4.x; o.sq = lo4.y; o.mp = lo4.z; o.sp = lo4.w;
      o.t = hi4.x; o.bx = hi4.y; o.bl = hi4.z; o.bi = __float_as_int(hi4.w);
      df_merge<KIND>(s, o);
    }
    df_warp_merge<KIND>(s);
    lzq = s.mq + logf(s.sq);
    if (KIND == kKindKL) {
      lzp = s.mp + logf(s.sp);
      // KL = sum p (xt - xl) - logZp + logZq; the normaliser difference is
      // (mq - mp) + log(sq / sp): one log of a ratio, no cancellation of two
      // large log-normalisers
      el = s.t / s.sp + ((s.mq - s.mp) + logf(s.sq / s.sp));
    } else {
      int bi = s.bi;
      float bl = s.bl;
      if (bi == INT_MAX) {  // no finite maximum (all -inf): argmax is index 0
        bi = 0;
        bl = static_cast<const float*>(a.logits)[r * a.V];
      }
      tgt = bi;
      el = lzq - bl;
    }
  }
  if (lane == 0) {
    const float lr = numer != 0.f ? __fmul_rn(w, el) : 0.f;
    if (a.loss_rows) a.loss_rows[r] = lr;
    a.row_loss[r] = lr;
    a.scale[r] = __fdiv_rn(w, (float)a.n_global);
    a.logzq[r] = lzq;
    a.logzp[r] = lzp;
    if (a.target_id) a.target_id[r] = tgt;
    a.row_cnt[r] = 0u;
    __threadfence();
    const unsigned prev = atomicAdd(a.done_cnt, 1u);
    *sh_last = (prev + 1 == (unsigned)(a.N * a.B));
  }
  __syncwarp();
}

template <int KIND, int NT, int U>
__global__ void __launch_bounds__(NT) dflash_fwd_kernel(const __grid_constant__ DflashFwdArgs a) {
  constexpr int NW = NT / 32;
  __shared__ __align__(16) DfState sh_red[NW];
  __shared__ int sh_flag, sh_last;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int64_t c = blockIdx.x;
  const Partition& pt = a.pt;
  const int64_t e_begin = c * pt.chunk;
  const int64_t e_end = min(e_begin + pt.chunk, pt.E);
  int64_t r = e_begin / pt.V;
  for (int64_t e = e_begin; e < e_end; ++r) {
    const int64_t row0 = r * pt.V;
    const int64_t lo = e - row0;
    const int64_t hi = min(e_end, row0 + pt.V) - row0;
    e = row0 + hi;
    const bool live = df_numer(a, r) != 0.f;
    if (live) {
      DfState s;
      df_init(s);
      df_stream<KIND, NT, U>(s, static_cast<const float*>(a.logits) + row0,
                             static_cast<const float*>(a.target_logits) + row0, lo, hi);
      df_warp_merge<KIND>(s);
      if (lane == 0) sh_red[w] = s;
      __syncthreads();
      if (w == 0) {
        if (lane < NW) s = sh_red[lane];
        else df_init(s);
        df_warp_merge<KIND>(s);
        if (lane == 0) {
          float4* dst = reinterpret_cast<float4*>(a.part + r * pt.pmax + (c - pt.first_cta(r)));
          dst[0] = make_float4(s.mq, s.sq, s.mp, s.sp);
          dst[1] = make_float4(s.t, s.bx, s.bl, __int_as_float(s.bi));
        }
      }
    }
    if (tid == 0) {
      int last = 1;
      if (pt.pieces(r) > 1) {
        __threadfence();
        const unsigned prev = atomicAdd(a.row_cnt + r, 1u);
        last = (prev + 1 == (unsigned)pt.pieces(r));
      }
      sh_flag = last;
    }
    __syncthreads();
    if (sh_flag && w == 0) df_finalize_row<KIND>(a, r, &sh_last);
    __syncthreads();
    if (sh_flag && sh_last && w == 0) {
      __threadfence();
      const float total = warp_sum_l2(a.row_loss, a.N * a.B);
      if (lane == 0) {
        a.loss[0] = total / (float)a.n_global;
        *a.done_cnt = 0u;
      }
    }
    __syncthreads();
  }
}

template <int KIND, int NT, int U>
__global__ void __launch_bounds__(NT) dflash_bwd_kernel(const __grid_constant__ DflashBwdArgs a) {
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const Partition& pt = a.pt;
  const int64_t e_begin = c * pt.chunk;
  const int64_t e_end = min(e_begin + pt.chunk, pt.E);
  const float g = a.dloss ? __ldg(a.dloss) : 1.f;
  const uint64_t pol = policy_evict_first();
  int64_t r = e_begin / pt.V;
  for (int64_t e = e_begin; e < e_end; ++r) {
    const int64_t row0 = r * pt.V;
    const int64_t lo = e - row0;
    const int64_t hi = min(e_end, row0 + pt.V) - row0;
    e = row0 + hi;
    const int64_t n = hi - lo;
    const float sc = __fmul_rn(a.scale[r], g);
    const float* pl = static_cast<const float*>(a.logits) + row0 + lo;
    const float* px = static_cast<const float*>(a.target_logits) + row0 + lo;
    float* dst = static_cast<float*>(a.dlogits) + row0 + lo;
    const uintptr_t al = reinterpret_cast<uintptr_t>(pl), ad = reinterpret_cast<uintptr_t>(dst);
    const uintptr_t ax = KIND == kKindKL ? reinterpret_cast<uintptr_t>(px) : al;
    const bool vec = (((al ^ ad) | (al ^ ax)) & 15) == 0;
    int64_t head = vec ? (((16 - (al & 15)) & 15) >> 2) : n;
    if (head > n) head = n;
    const int64_t body = (n - head) >> 2;
    const int64_t tail0 = head + (body << 2);
    if (sc == 0.f) {
      for (int64_t i = tid; i < head; i += NT) dst[i] = 0.f;
      for (int64_t i = tail0 + tid; i < n; i += NT) dst[i] = 0.f;
      float4* q = reinterpret_cast<float4*>(dst + head);
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t i = tid; i < body; i += NT) st_stream(q + i, z);
      continue;
    }
    const float lq = a.logzq[r];
    const float lp = a.logzp[r];
    const int64_t t = (KIND == kKindCE ? a.target_id[r] : -1) - lo;
    auto elem = [&](float xl, float xt, int64_t i) -> float {
      const float q = exp_shift(xl, lq);
      const float p = KIND == kKindKL ? exp_shift(xt, lp) : (i == t ? 1.f : 0.f);
      return sc * (q - p);
    };
    for (int64_t i = tid; i < head; i += NT) dst[i] = elem(pl[i], KIND == kKindKL ? px[i] : 0.f, i);
    for (int64_t i = tail0 + tid; i < n; i += NT)
      dst[i] = elem(pl[i], KIND == kKindKL ? px[i] : 0.f, i);
    const float4* ql = reinterpret_cast<const float4*>(pl + head);
    const float4* qx = reinterpret_cast<const float4*>(px + head);
    float4* qd = reinterpret_cast<float4*>(dst + head);
    const int64_t tb = t - head;
    int64_t i = tid;
    for (; i + (U - 1) * NT < body; i += U * NT) {
      float4 va[U], vb[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        va[u] = ld_last(ql + i + u * NT, pol);
        if (KIND == kKindKL) vb[u] = ld_last(qx + i + u * NT, pol);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t k = i + u * NT;
        float4 y;
        y.x = exp_shift(va[u].x, lq);
        y.y = exp_shift(va[u].y, lq);
        y.z = exp_shift(va[u].z, lq);
        y.w = exp_shift(va[u].w, lq);
        if (KIND == kKindKL) {
          y.x -= exp_shift(vb[u].x, lp);
          y.y -= exp_shift(vb[u].y, lp);
          y.z -= exp_shift(vb[u].z, lp);
          y.w -= exp_shift(vb[u].w, lp);
        } else {
          const uint64_t d = (uint64_t)(tb - 4 * k);
          if (d < 4) {
            if (d == 0) y.x -= 1.f;
            else if (d == 1) y.y -= 1.f;
            else if (d == 2) y.z -= 1.f;
            else y.w -= 1.f;
          }
        }
        y.x *= sc;
        y.y *= sc;
        y.z *= sc;
        y.w *= sc;
        st_stream(qd + k, y);
      }
    }
    for (; i < body; i += NT) {
      const float4 va = ld_last(ql + i, pol);
      float4 y;
      y.x = exp_shift(va.x, lq);
      y.y = exp_shift(va.y, lq);
      y.z = exp_shift(va.z, lq);
      y.w = exp_shift(va.w, lq);
      if (KIND == kKindKL) {
        const float4 vb = ld_last(qx + i, pol);
        y.x -= exp_shift(vb.x, lp);
        y.y -= exp_shift(vb.y, lp);
        y.z -= exp_shift(vb.z, lp);
        y.w -= exp_shift(vb.w, lp);
      } else {
        const uint64_t d = (uint64_t)(tb - 4 * i);
        if (d < 4) {
          if (d == 0) y.x -= 1.f;
          else if (d == 1) y.y -= 1.f;
          else if (d == 2) y.z -= 1.f;
          else y.w -= 1.f;
        }
      }
      y.x *= sc;
      y.y *= sc;
      y.z *= sc;
      y.w *= sc;
      st_stream(qd + i, y);
    }
  }
}

template <class K>
int occupancy_ctas(K kernel, int nt, int device, int cap_per_sm) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, nt, 0) != cudaSuccess) return 0;
  if (cap_per_sm > 0 && per_sm > cap_per_sm) per_sm = cap_per_sm;
  if (per_sm < 1) per_sm = 1;
  return sms * per_sm;
}

template <int KIND, int NT, int U>
struct DflashVariant {
  static int fwd_ctas(int device, int cap) {
    return occupancy_ctas(dflash_fwd_kernel<KIND, NT, U>, NT, device, cap);
  }
  static int bwd_ctas(int device, int cap) {
    return occupancy_ctas(dflash_bwd_kernel<KIND, NT, U>, NT, device, cap);
  }
  static cudaError_t fwd(const DflashFwdArgs& a, cudaStream_t st) {
    dflash_fwd_kernel<KIND, NT, U><<<(unsigned)a.pt.grid, NT, 0, st>>>(a);
    return cudaGetLastError();
  }
  static cudaError_t bwd(const DflashBwdArgs& a, cudaStream_t st) {
    dflash_bwd_kernel<KIND, NT, U><<<(unsigned)a.pt.grid, NT, 0, st>>>(a);
    return cudaGetLastError();
  }
};

template <int KIND>
int fwd_ctas_k(int shape, int device, int cap) {
  switch (shape) {
    case 1: return DflashVariant<KIND, 256, 4>::fwd_ctas(device, cap);
    case 4: return DflashVariant<KIND, 512, 2>::fwd_ctas(device, cap);
    default: return DflashVariant<KIND, 256, 2>::fwd_ctas(device, cap);
  }
}
template <int KIND>
int bwd_ctas_k(int shape, int device, int cap) {
  switch (shape) {
    case 1: return DflashVariant<KIND, 256, 4>::bwd_ctas(device, cap);
    case 4: return DflashVariant<KIND, 512, 2>::bwd_ctas(device, cap);
    default: return DflashVariant<KIND, 512, 4>::bwd_ctas(device, cap);
  }
}
template <int KIND>
cudaError_t fwd_launch_k(int shape, const DflashFwdArgs& a, cudaStream_t st) {
  switch (shape) {
    case 1: return DflashVariant<KIND, 256, 4>::fwd(a, st);
    case 4: return DflashVariant<KIND, 512, 2>::fwd(a, st);
    default: return DflashVariant<KIND, 256, 2>::fwd(a, st);
  }
}
template <int KIND>
cudaError_t bwd_launch_k(int shape, const DflashBwdArgs& a, cudaStream_t st) {
  switch (shape) {
    case 1: return DflashVariant<KIND, 256, 4>::bwd(a, st);
    case 4: return DflashVariant<KIND, 512, 2>::bwd(a, st);
    default: return DflashVariant<KIND, 512, 4>::bwd(a, st);
  }
}

}  // namespace

int dflash_fwd_ctas(int kind, int shape, int device, int cap) {
  return kind == kKindKL ? fwd_ctas_k<kKindKL>(shape, device, cap) : fwd_ctas_k<kKindCE>(shape, device, cap);
}
int dflash_bwd_ctas(int kind, int shape, int device, int cap) {
  return kind == kKindKL ? bwd_ctas_k<kKindKL>(shape, device, cap) : bwd_ctas_k<kKindCE>(shape, device, cap);
}
cudaError_t dflash_fwd_launch(int shape, const DflashFwdArgs& a, cudaStream_t st) {
  return a.kind == kKindKL ? fwd_launch_k<kKindKL>(shape, a, st) : fwd_launch_k<kKindCE>(shape, a, st);
}
cudaError_t dflash_bwd_launch(int shape, const DflashBwdArgs& a, cudaStream_t st) {
  return a.kind == kKindKL ? bwd_launch_k<kKindKL>(shape, a, st) : bwd_launch_k<kKindCE>(shape, a, st);
}

}  // namespace specdec
