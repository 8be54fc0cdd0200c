// DFlash objective, forward and backward, on the warp-specialized CTA ring
// (ring.cuh), two input streams (draft and verifier logits) per stage.
//
// Same arithmetic and outputs as dflash_kernels.cu (the 128-bit-load kernels,
// kept for inputs whose base addresses are not 16-byte aligned).
//
// Forward = two launches on the stream:
//   1. dflash_fwd_ring_kernel streams each (draft, verifier) row pair once:
//      every consumer warp keeps the DfState of the row it is in (KL: draft
//      and verifier log-sum-exp plus t = sum e^(xt - mp) (xt - xl); CE: draft
//      log-sum-exp plus the first-index argmax of xt and the draft logit
//      there) and stores it per (row, block) piece at
//      part[(r * pmax + block_in_row) * NC + warp]. Plain stores only.
//   2. dflash_finalize_kernel (programmatic dependent launch): one CTA per
//      sequence, warp j <-> row j merges the row's pieces in slot order,
//      forms KL = t/sp + (mq - mp) + log(sq/sp) or CE = logZq - xl[argmax],
//      the weight mask * decay(j % block_size) / (sum mask + 1e-5), writes the
//      per-row outputs; the last CTA (done counter) sums the per-sequence
//      losses in index order.
// Backward = one launch: dflash_bwd_ring_kernel streams the draft (and for KL
// the verifier) and writes s * (softmax(draft) - softmax(verifier) | onehot).
// Rows whose weight mask * decay is 0 are never copied.
//
// Element type T: float, or bf16_t (bfloat16 bit patterns) for both streams
// and the gradient; elements are widened exactly to float, the bf16 gradient
// is rounded to nearest even.
//
// Reference behaviour: models/dflash/loss.py:31-126 (forward), :128-166
// (backward); numbers follow models/dflash/tests/test_loss.py:21-49.
#include <climits>
#include <type_traits>

#include "dflash_common.cuh"
#include "ring.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

// Weight numerator mask * decay(pos), pos = j % block_size (test_loss.py:23-27).
__device__ __forceinline__ float dr_numer(const DflashFwdArgs& a, int64_t r) {
  const int pos = (int)(r % a.B) % a.block_size;
  float decay;
  if (a.sfa) decay = expf(__fdiv_rn(-(float)pos, a.gamma));
  else decay = pos == 0 ? 0.f : expf(__fdiv_rn(-(float)(pos - 1), a.gamma));
  return __fmul_rn(a.mask ? a.mask[r] : 1.f, decay);
}

template <class T, int KIND, int NC, int S, int SE, int BS>
__global__ void __launch_bounds__((NC + 1) * 32, (ring_min_ctas<NC, 2, S, SE, T>())) dflash_fwd_ring_kernel(const __grid_constant__ DflashFwdArgs a) {
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int kSub = SE / NC;
  constexpr int U = kSub / (32 * kVec);  // 16-byte vectors per lane per stream in a full sub-range
  constexpr int64_t BL = (int64_t)BS * SE;
  constexpr int kLogBL = __builtin_ctzll(BL);
  static_assert(kSub % (32 * kVec) == 0, "sub-range must be whole 16-byte rounds of a warp");
  static_assert((BL & (BL - 1)) == 0, "block length must be a power of two");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<RingSmem<2, S, SE, T>*>(smem_raw);
  const T* XL = static_cast<const T*>(a.logits);
  const T* XT = static_cast<const T*>(a.target_logits);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t E = a.pt.E, V = a.pt.V, R = E / V;
  const int pmax = a.pt.pmax;

  BlockQueue q;
  q.ctr = a.q_ctr;
  q.retired = a.q_retired;
  q.nblocks = (unsigned)((E + BL - 1) / BL);
  q.dynamic = a.q_dynamic;
  // the producer's first block is its own index; with SPECDEC_EARLY_FIRST_STAGE
  // the producer lane initialises the ring and posts that block's first stage
  // before the liveness table is built
  const unsigned first = q.first();
  const bool withhold = a.withhold_stage && blockIdx.x == 0;
#if SPECDEC_EARLY_FIRST_STAGE
  ring_init(sm, NC, NC * 32);
  bool posted = false;
  if (warp == NC && lane == 0) {
    const T* src0[2] = {XL, XT};
    posted = ring_post_first<2, S, SE>(src0, make_block_map(E, BL, SE, -1), V, q, sm.ring, sm.full, sm.sf0,
                                       sm.srow, first, withhold, static_cast<RingTrack<S>*>(nullptr));
  }
#else
  ring_init(sm, NC);
  const bool posted = false;
#endif
  const RowBits rb = build_row_bits(sm.bits, R, NC + 1, [&](int64_t r) { return dr_numer(a, r) != 0.f; });
  __syncthreads();

  if (warp == NC) {  // producer
    if (lane == 0) {
      const T* src[2] = {XL, XT};
      if (!ring_produce<2, S, SE>(src, make_block_map(E, BL, SE, -1), V, rb, q, sm.ring, sm.full, sm.empty,
                                  sm.sf0, sm.srow, first, withhold, static_cast<RingTrack<S>*>(nullptr), posted))
        atomicOr(a.flag, 2);
      q.retire();
    }
    pdl_trigger();
    return;
  }

  const T* ringl = sm.ring;
  const T* ringt = sm.ring + (size_t)S * SE;
  DfState st;
  df_init(st);
  int64_t r = 0, blk = -1;
  bool live = false;
  auto enter_row = [&](int64_t row) {
    live = row < R && (rb.valid ? rb.live(row) : dr_numer(a, row) != 0.f);
  };
  auto close_piece = [&]() {
    if (live) {
      df_warp_merge<KIND>(st);
      if (lane == 0) {
        const int64_t slot = blk - (r * V) / BL;
        float4* dst = reinterpret_cast<float4*>(a.part + (r * pmax + slot) * NC + warp);
        dst[0] = make_float4(st.mq, st.sq, st.mp, st.sp);
        dst[1] = make_float4(st.t, st.bx, st.bl, __int_as_float(st.bi));
      }
    }
    df_init(st);
  };
  for (int64_t it = 0;; ++it) {
    const int slot = (int)(it % S);
    if (!__all_sync(kFullMask, mbar_wait(sm.full + slot, (uint32_t)((it / S) & 1)))) {
      if (lane == 0) atomicOr(a.flag, 2);
      ring_drain<S>(sm.full, it + 1);
      break;
    }
    const int64_t f0 = sm.sf0[slot];
    if (f0 < 0) break;
    const int64_t b = f0 >> kLogBL;
    const int64_t blk_end = min((b + 1) * BL, E);
    const int64_t f1 = min(f0 + SE, blk_end);
    if (b != blk) {
      blk = b;
      r = sm.srow[slot];
      enter_row(r);
    }
    const T* sl = ringl + (size_t)slot * SE;
    const T* sx = ringt + (size_t)slot * SE;
    if (f1 - f0 == SE && (r + 1) * V >= f1) {
      // fast path: a full stage inside one row
      if (live) {
        using Vec = typename std::conditional<sizeof(T) == 4, float4, uint4>::type;
        const Vec* ql = reinterpret_cast<const Vec*>(sl + warp * kSub) + lane;
        const Vec* qx = reinterpret_cast<const Vec*>(sx + warp * kSub) + lane;
        Vec va[U], vb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          va[u] = ql[32 * u];
          vb[u] = qx[32 * u];
        }
        const int base = (int)(f0 - r * V) + warp * kSub + kVec * lane;
        // the slot is released inside, once both streams are in registers
        df_group<KIND, U>(st, va, vb, base, 32 * kVec, sm.empty + slot);
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.empty + slot);
      }
      if ((r + 1) * V == f1) {
        close_piece();
        ++r;
        enter_row(r);
      } else if (f1 == blk_end) {
        close_piece();
      }
      continue;
    }
    const int64_t fv = copied_end<T>(f0, f1);  // end of the copied part
    const int64_t w0 = f0 + (int64_t)warp * kSub, w1 = min(w0 + kSub, f1);
    int64_t f = f0;
    while (f < f1) {
      const int64_t rend = (r + 1) * V;
      const int64_t g = min(f1, rend);
      if (live) {
        const int64_t lo = max(f, w0), hi = min(g, w1);
        const int64_t hv = min(hi, fv);
        if (hv > lo) df_range<KIND>(st, sl, sx, (int)(lo - f0), (int)(hv - f0), (int)(f0 - r * V));
        for (int64_t x = max(lo, fv) + lane; x < hi; x += 32)  // past the copied part: global memory
          df_push<KIND>(st, ldg_f32(XL + x), ldg_f32(XT + x), (int)(x - r * V));
      }
      f = g;
      if (g == rend) {
        close_piece();
        ++r;
        enter_row(r);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.empty + slot);
    if (f1 == blk_end && r * V < blk_end) close_piece();
  }
  pdl_trigger();
}

// One CTA per sequence n with min(B, 32) warps; warp w finalizes rows
// j = w, w + 32, ... of the sequence (for B <= 32: warp j <-> row j).
template <class T, int KIND>
__global__ void __launch_bounds__(1024) dflash_finalize_kernel(const __grid_constant__ DflashFwdArgs a) {
  __shared__ float sh_loss[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int B = a.B;
  const int64_t n = blockIdx.x, V = a.pt.V, BL = a.pt.chunk;
  const int NC = a.nc;
  // denominator: sum of the sequence's raw mask values + 1e-5 (the mask is
  // not written by the streaming grid: read it while that grid drains)
  float mv = 0.f;
  for (int i = lane; i < B; i += 32) mv += a.mask ? a.mask[n * B + i] : 1.f;
  const float denom = warp_sum(mv) + 1e-5f;
  // the first row's numerator depends on the mask only: read it before the wait too
  const float numer0 = warp < B ? dr_numer(a, n * B + warp) : 0.f;
  pdl_wait();  // the streaming grid has completed and its stores are visible
  // a wait of the streaming grid expired: pieces may be missing, so every
  // per-row output is NaN (a backward from them gives a NaN gradient)
  const bool timed_out = (*reinterpret_cast<volatile int*>(a.flag) & 2) != 0;
  float acc = 0.f;  // this warp's rows, in row order
  for (int j = warp; j < B; j += nwarps) {
    const int64_t r = n * B + j;
    const float numer = j == warp ? numer0 : dr_numer(a, r);
    const float w = __fdiv_rn(numer, denom);
    float el = 0.f, lzq = 0.f, lzp = 0.f;
    int64_t tgt = 0;
    if (numer != 0.f) {
      const int k = blocks_in_row(r, V, BL) * NC;
      const DfPiece* part = a.part + r * a.pt.pmax * NC;
      DfState s;
      df_init(s);
      for (int qd = lane; qd < k; qd += 32) {  // slot-major, warp-minor: fixed order
        const float4 lo4 = reinterpret_cast<const float4*>(part + qd)[0];
        const float4 hi4 = reinterpret_cast<const float4*>(part + qd)[1];
        DfState o;
        o.mq = lo4.x; o.sq = lo4.y; o.mp = lo4.z; o.sp = lo4.w;
        o.t = hi4.x; o.bx = hi4.y; o.bl = hi4.z; o.bi = __float_as_int(hi4.w);
        df_merge<KIND>(s, o);
      }
      df_warp_merge<KIND>(s);
      lzq = s.mq + logf(s.sq);
      if (KIND == kKindKL) {
        lzp = s.mp + logf(s.sp);
        // KL = sum p (xt - xl) - logZp + logZq, the normaliser difference as one log of a ratio
        el = s.t / s.sp + ((s.mq - s.mp) + logf(s.sq / s.sp));
      } else {
        int bi = s.bi;
        float bl = s.bl;
        if (bi == INT_MAX) {  // no finite maximum (all -inf): argmax is index 0
          bi = 0;
          bl = to_f32(static_cast<const T*>(a.logits)[r * V]);
        }
        tgt = bi;
        el = lzq - bl;
      }
    }
    const float lr = numer != 0.f ? __fmul_rn(w, el) : 0.f;
    if (lane == 0) {
      const float nan = __int_as_float(0x7fc00000);
      if (a.loss_rows) a.loss_rows[r] = lr;
      a.scale[r] = timed_out ? nan : __fdiv_rn(w, (float)a.n_global);
      a.logzq[r] = timed_out ? nan : lzq;
      a.logzp[r] = timed_out ? nan : lzp;
      if (a.target_id) a.target_id[r] = tgt;
    }
    acc += lr;
  }
  if (lane == 0) sh_loss[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    const float seq = warp_sum(lane < nwarps ? sh_loss[lane] : 0.f);
    unsigned last = 0;
    if (lane == 0) {
      a.seq_loss[n] = seq;
      __threadfence();
      last = (atomicAdd(a.done_cnt, 1u) + 1 == (unsigned)a.N);
    }
    last = __shfl_sync(kFullMask, last, 0);
    if (last) {
      __threadfence();
      // the flag exchange and the loss loads are independent: both in flight at once
      int f = 0;
      if (lane == 0) f = atomicExch(a.flag, 0);
      const float total = warp_sum_l2(a.seq_loss, a.N);
      if (lane == 0) {
        // a timed-out copy wait left partials unwritten: the loss is NaN, not a wrong number
        a.loss[0] = (f & 2) ? __int_as_float(0x7fc00000) : total / (float)a.n_global;
        *a.done_cnt = 0u;
      }
    }
  }
}

template <class T, int KIND, int NC, int S, int SE, int BS>
__global__ void __launch_bounds__((NC + 1) * 32, (ring_min_ctas<NC, (KIND == kKindKL ? 2 : 1), S, SE, T>())) dflash_bwd_ring_kernel(const __grid_constant__ DflashBwdArgs a) {
  constexpr int NIN = KIND == kKindKL ? 2 : 1;
  constexpr int kVec = 16 / sizeof(T);
  constexpr int kSub = SE / NC;
  constexpr int64_t BL = (int64_t)BS * SE;
  constexpr int kLogBL = __builtin_ctzll(BL);
  static_assert(kSub % kVec == 0, "sub-range must be whole 16-byte vectors");
  static_assert((BL & (BL - 1)) == 0, "block length must be a power of two");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<RingSmem<NIN, S, SE, T>*>(smem_raw);
  const T* XL = static_cast<const T*>(a.logits);
  const T* XT = static_cast<const T*>(a.target_logits);
  T* dst = static_cast<T*>(a.dlogits);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t E = a.pt.E, V = a.pt.V, R = E / V;
  const float g = a.dloss ? __ldg(a.dloss) : 1.f;
  BlockQueue q;
  q.ctr = a.q_ctr;
  q.retired = a.q_retired;
  q.nblocks = (unsigned)((E + BL - 1) / BL);
  q.dynamic = a.q_dynamic;
  // the producer's first block: its own index (no atomic)
  const unsigned first = (warp == NC && lane == 0) ? q.first() : 0u;
  ring_init(sm, NC);
  const RowBits rb = build_row_bits(sm.bits, R, NC + 1, [&](int64_t r) { return __fmul_rn(a.scale[r], g) != 0.f; });
  __syncthreads();

  if (warp == NC) {
    if (lane == 0) {
      const T* src[2] = {XL, XT};
      if (!ring_produce<NIN, S, SE>(src, make_block_map(E, BL, SE, -1), V, rb, q, sm.ring, sm.full, sm.empty,
                                    sm.sf0, sm.srow, first, a.withhold_stage && blockIdx.x == 0, &sm.trk))
        sm.trk.timeout = 1;
    }
  } else {
    const T* ringl = sm.ring;
    const T* ringt = sm.ring + (size_t)S * SE;  // KL only
    int64_t r = 0, blk = -1, tf = -1;
    float sc = 0.f, lq = 0.f, lp = 0.f;
    auto load_row = [&](int64_t row) {
      sc = __fmul_rn(a.scale[row], g);
      lq = a.logzq[row];
      lp = a.logzp[row];
      tf = KIND == kKindCE ? row * V + a.target_id[row] : -1;
    };
    int64_t it = 0;
    for (;; ++it) {
      const int slot = (int)(it % S);
      if (!__all_sync(kFullMask, mbar_wait(sm.full + slot, (uint32_t)((it / S) & 1)))) {
        if (lane == 0) sm.trk.timeout = 1;
        ring_drain<S>(sm.full, it + 1);
        break;
      }
      const int64_t f0 = sm.sf0[slot];
      if (f0 < 0) break;
      const int64_t b = f0 >> kLogBL;
      const int64_t blk_end = min((b + 1) * BL, E);
      const int64_t f1 = min(f0 + SE, blk_end);
      if (b != blk) {
        blk = b;
        r = sm.srow[slot];
        load_row(r);
      }
      const int64_t fv = copied_end<T>(f0, f1);
      const int64_t w0 = f0 + (int64_t)warp * kSub, w1 = min(w0 + kSub, f1);
      const T* sl = ringl + (size_t)slot * SE;
      const T* sx = ringt + (size_t)slot * SE;
      int64_t f = f0;
      while (f < f1) {
        const int64_t rend = (r + 1) * V;
        const int64_t ge = min(f1, rend);
        const int64_t lo = max(f, w0), hi = min(ge, w1);
        if (lo < hi) {
          const bool zero = sc == 0.f || !rb.live(r);
          const int64_t lov = (lo + kVec - 1) & ~int64_t(kVec - 1), hiv = min(hi, fv) & ~int64_t(kVec - 1);
          auto scalar = [&](int64_t x) {
            if (zero) {
              store_elem(dst + x, 0.f);
            } else {
              const float vl = x < fv ? to_f32(sl[x - f0]) : ldg_f32(XL + x);
              const float qv = exp_shift(vl, lq);
              float pv;
              if (KIND == kKindKL) pv = exp_shift(x < fv ? to_f32(sx[x - f0]) : ldg_f32(XT + x), lp);
              else pv = x == tf ? 1.f : 0.f;
              store_elem(dst + x, sc * (qv - pv));
            }
          };
          if (lov < hiv) {
            for (int64_t x = lo + lane; x < lov; x += 32) scalar(x);
            for (int64_t x = hiv + lane; x < hi; x += 32) scalar(x);
            const int nv = (int)((hiv - lov) / kVec);
            if (zero) {
              const uint4 z = make_uint4(0u, 0u, 0u, 0u);
              uint4* d4 = reinterpret_cast<uint4*>(dst + lov);
              for (int k = lane; k < nv; k += 32) st_stream_u4(d4 + k, z);
            } else if constexpr (sizeof(T) == 4) {
              float4* d4 = reinterpret_cast<float4*>(dst + lov);
              const float4* s4 = reinterpret_cast<const float4*>(sl + (lov - f0));
              const float4* t4 = reinterpret_cast<const float4*>(sx + (lov - f0));
              const int64_t tq = tf - lov;
              for (int k = lane; k < nv; k += 32) {
                const float4 v = s4[k];
                float4 y;
                y.x = exp_shift(v.x, lq);
                y.y = exp_shift(v.y, lq);
                y.z = exp_shift(v.z, lq);
                y.w = exp_shift(v.w, lq);
                if (KIND == kKindKL) {
                  const float4 u = t4[k];
                  y.x -= exp_shift(u.x, lp);
                  y.y -= exp_shift(u.y, lp);
                  y.z -= exp_shift(u.z, lp);
                  y.w -= exp_shift(u.w, lp);
                } else {
                  const uint64_t d = (uint64_t)(tq - 4 * (int64_t)k);
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
                st_stream(d4 + k, y);
              }
            } else {
              uint4* d4 = reinterpret_cast<uint4*>(dst + lov);
              const uint4* s4 = reinterpret_cast<const uint4*>(sl + (lov - f0));
              const uint4* t4 = reinterpret_cast<const uint4*>(sx + (lov - f0));
              const int64_t tq = tf - lov;
              const float2 sc2 = make_float2(sc, sc);
              for (int k = lane; k < nv; k += 32) {
                const uint4 v = s4[k];
                const uint32_t wl[4] = {v.x, v.y, v.z, v.w};
                float2 q[4], y[4];
  #pragma unroll
                for (int h = 0; h < 4; ++h) q[h] = exp_shift2(bf16x2_f32(wl[h]), lq);
                if (KIND == kKindKL) {
                  const uint4 u = t4[k];
                  const uint32_t wt[4] = {u.x, u.y, u.z, u.w};
  #pragma unroll
                  for (int h = 0; h < 4; ++h) y[h] = fmul2(fsub2(q[h], exp_shift2(bf16x2_f32(wt[h]), lp)), sc2);
                } else {
  #pragma unroll
                  for (int h = 0; h < 4; ++h) y[h] = fmul2(q[h], sc2);
                  const uint64_t d = (uint64_t)(tq - 8 * (int64_t)k);
                  if (d < 8) {  // the argmax target: sc * (q - 1), as the float kernel
  #pragma unroll
                    for (int h = 0; h < 4; ++h) {
                      if (d == (uint64_t)(2 * h)) y[h].x = sc * (q[h].x - 1.f);
                      if (d == (uint64_t)(2 * h + 1)) y[h].y = sc * (q[h].y - 1.f);
                    }
                  }
                }
                st_stream_u4(d4 + k, make_uint4(pack_bf16x2(y[0].x, y[0].y), pack_bf16x2(y[1].x, y[1].y),
                                                pack_bf16x2(y[2].x, y[2].y), pack_bf16x2(y[3].x, y[3].y)));
              }
            }
          } else {
            for (int64_t x = lo + lane; x < hi; x += 32) scalar(x);
          }
        }
        f = ge;
        if (ge == rend && ge < E) {
          ++r;
          load_row(r);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(sm.empty + slot);
    }
    if (lane == 0) sm.trk.done[warp] = it;
  }
  __syncthreads();
  if (sm.trk.timeout) ring_poison<T, S>(dst, E, BL, q.nblocks, sm.trk, NC, q.dynamic ? 0u : gridDim.x);
  if (warp == 0) bwd_finish(q, a, sm.trk.timeout != 0);
}

// Stages per queue block of the backward kernels: small blocks (the backward
// has no per-block partials), so that no CTA holds more than a little
// unstarted work when the queue runs dry.
#ifndef SPECDEC_DFBWD_BLOCK_STAGES
#define SPECDEC_DFBWD_BLOCK_STAGES 2
#endif
constexpr int kDfBwdBlockStages = SPECDEC_DFBWD_BLOCK_STAGES;

template <class T, int NC, int S, int SE, int BS>
struct DfRing {
  template <int KIND>
  static constexpr size_t fsmem() { return sizeof(RingSmem<2, S, SE, T>); }
  template <int KIND>
  static constexpr size_t bsmem() { return sizeof(RingSmem<KIND == kKindKL ? 2 : 1, S, SE, T>); }
  template <int KIND>
  static int fwd_ctas(int device, int cap) {
    return ring_occupancy_ctas(dflash_fwd_ring_kernel<T, KIND, NC, S, SE, BS>, (NC + 1) * 32, fsmem<KIND>(),
                               device, cap);
  }
  template <int KIND>
  static int bwd_ctas(int device, int cap) {
    return ring_occupancy_ctas(dflash_bwd_ring_kernel<T, KIND, NC, S, SE, kDfBwdBlockStages>, (NC + 1) * 32, bsmem<KIND>(),
                               device, cap);
  }
  template <int KIND>
  static cudaError_t fwd(DflashFwdArgs a, int ctas, cudaStream_t st) {
    cudaError_t e = ensure_smem_limit<dflash_fwd_ring_kernel<T, KIND, NC, S, SE, BS>>(fsmem<KIND>());
    if (e != cudaSuccess) return e;
    a.nc = NC;
    // plain launch for the streaming kernel (its predecessor is the caller's),
    // PDL only for the finalize that always follows it
    dflash_fwd_ring_kernel<T, KIND, NC, S, SE, BS><<<ctas, (NC + 1) * 32, fsmem<KIND>(), st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_pdl(dflash_finalize_kernel<T, KIND>, dim3((unsigned)a.N), dim3(32 * (a.B < 32 ? a.B : 32)), 0,
                      st, a);
  }
  template <int KIND>
  static cudaError_t bwd(const DflashBwdArgs& a, int ctas, cudaStream_t st) {
    const cudaError_t e = ensure_smem_limit<dflash_bwd_ring_kernel<T, KIND, NC, S, SE, kDfBwdBlockStages>>(bsmem<KIND>());
    if (e != cudaSuccess) return e;
    dflash_bwd_ring_kernel<T, KIND, NC, S, SE, kDfBwdBlockStages><<<ctas, (NC + 1) * 32, bsmem<KIND>(), st>>>(a);
    return cudaGetLastError();
  }
};

// Ring shapes (consumer warps x stages x stage elements per stream x stages
// per block), float elements; the forward ring holds both streams:
// 0 = 4 x 4 x 2048 x 8 (64 KB ring, 64 KB blocks per stream, 3 CTAs/SM);
// 1 = 4 x 4 x 4096 x 4 (128 KB ring, 1 CTA/SM); 2 = 4 x 6 x 2048 x 8 (96 KB
// ring, 2 CTAs/SM); 3 = 2 x 4 x 2048 x 8 (64 KB ring, 3 CTAs/SM);
// 4 = 8 x 3 x 4096 x 4 (96 KB ring, 2 CTAs/SM); 5 = 8 x 4 x 2048 x 8 (64 KB
// ring, 8 consumer warps); 6 = 4 x 2 x 2048 x 8 (32 KB ring, 4 CTAs/SM). bf16
// shapes have the same bytes (twice the elements).
template <class T>
struct DfShapes {
  static constexpr int k = 4 / sizeof(T);
  using D0 = DfRing<T, 4, 4, 2048 * k, 8>;
  using D1 = DfRing<T, 4, 4, 4096 * k, 4>;
  using D2 = DfRing<T, 4, 6, 2048 * k, 8>;
  using D3 = DfRing<T, 2, 4, 2048 * k, 8>;
  using D4 = DfRing<T, 8, 3, 4096 * k, 4>;
  using D5 = DfRing<T, 8, 4, 2048 * k, 8>;
  using D6 = DfRing<T, 4, 2, 2048 * k, 8>;

  static int block_elems(int shape) {
    switch (shape) {
      case 1: return 4096 * 4 * k;
      case 4: return 4096 * 4 * k;
      default: return 2048 * 8 * k;
    }
  }
  template <int KIND>
  static int fwd_ctas(int shape, int device, int cap) {
    switch (shape) {
      case 1: return D1::template fwd_ctas<KIND>(device, cap);
      case 2: return D2::template fwd_ctas<KIND>(device, cap);
      case 3: return D3::template fwd_ctas<KIND>(device, cap);
      case 4: return D4::template fwd_ctas<KIND>(device, cap);
      case 5: return D5::template fwd_ctas<KIND>(device, cap);
      case 6: return D6::template fwd_ctas<KIND>(device, cap);
      default: return D0::template fwd_ctas<KIND>(device, cap);
    }
  }
  template <int KIND>
  static int bwd_ctas(int shape, int device, int cap) {
    switch (shape) {
      case 1: return D1::template bwd_ctas<KIND>(device, cap);
      case 2: return D2::template bwd_ctas<KIND>(device, cap);
      case 3: return D3::template bwd_ctas<KIND>(device, cap);
      case 4: return D4::template bwd_ctas<KIND>(device, cap);
      case 5: return D5::template bwd_ctas<KIND>(device, cap);
      case 6: return D6::template bwd_ctas<KIND>(device, cap);
      default: return D0::template bwd_ctas<KIND>(device, cap);
    }
  }
  template <int KIND>
  static cudaError_t fwd(int shape, const DflashFwdArgs& a, int ctas, cudaStream_t st) {
    switch (shape) {
      case 1: return D1::template fwd<KIND>(a, ctas, st);
      case 2: return D2::template fwd<KIND>(a, ctas, st);
      case 3: return D3::template fwd<KIND>(a, ctas, st);
      case 4: return D4::template fwd<KIND>(a, ctas, st);
      case 5: return D5::template fwd<KIND>(a, ctas, st);
      case 6: return D6::template fwd<KIND>(a, ctas, st);
      default: return D0::template fwd<KIND>(a, ctas, st);
    }
  }
  template <int KIND>
  static cudaError_t bwd(int shape, const DflashBwdArgs& a, int ctas, cudaStream_t st) {
    switch (shape) {
      case 1: return D1::template bwd<KIND>(a, ctas, st);
      case 2: return D2::template bwd<KIND>(a, ctas, st);
      case 3: return D3::template bwd<KIND>(a, ctas, st);
      case 4: return D4::template bwd<KIND>(a, ctas, st);
      case 5: return D5::template bwd<KIND>(a, ctas, st);
      case 6: return D6::template bwd<KIND>(a, ctas, st);
      default: return D0::template bwd<KIND>(a, ctas, st);
    }
  }
  static int fwd_ctas_kind(int kind, int shape, int device, int cap) {
    return kind == kKindKL ? fwd_ctas<kKindKL>(shape, device, cap) : fwd_ctas<kKindCE>(shape, device, cap);
  }
  static int bwd_ctas_kind(int kind, int shape, int device, int cap) {
    return kind == kKindKL ? bwd_ctas<kKindKL>(shape, device, cap) : bwd_ctas<kKindCE>(shape, device, cap);
  }
  static cudaError_t fwd_kind(int shape, const DflashFwdArgs& a, int ctas, cudaStream_t st) {
    return a.kind == kKindKL ? fwd<kKindKL>(shape, a, ctas, st) : fwd<kKindCE>(shape, a, ctas, st);
  }
  static cudaError_t bwd_kind(int shape, const DflashBwdArgs& a, int ctas, cudaStream_t st) {
    return a.kind == kKindKL ? bwd<kKindKL>(shape, a, ctas, st) : bwd<kKindCE>(shape, a, ctas, st);
  }
};

}  // namespace

int dflash_ring_block_elems(int dtype, int shape) {
  return dtype == kDtypeBF16 ? DfShapes<bf16_t>::block_elems(shape) : DfShapes<float>::block_elems(shape);
}

int dflash_ring_consumers(int shape) {
  switch (shape) {
    case 3: return 2;
    case 4: return 8;
    case 5: return 8;
    default: return 4;
  }
}

int dflash_fwd_ring_ctas(int dtype, int kind, int shape, int device, int cap) {
  return dtype == kDtypeBF16 ? DfShapes<bf16_t>::fwd_ctas_kind(kind, shape, device, cap)
                             : DfShapes<float>::fwd_ctas_kind(kind, shape, device, cap);
}
int dflash_bwd_ring_ctas(int dtype, int kind, int shape, int device, int cap) {
  return dtype == kDtypeBF16 ? DfShapes<bf16_t>::bwd_ctas_kind(kind, shape, device, cap)
                             : DfShapes<float>::bwd_ctas_kind(kind, shape, device, cap);
}
cudaError_t dflash_fwd_ring_launch(int dtype, int shape, const DflashFwdArgs& a, int ctas, cudaStream_t st) {
  return dtype == kDtypeBF16 ? DfShapes<bf16_t>::fwd_kind(shape, a, ctas, st)
                             : DfShapes<float>::fwd_kind(shape, a, ctas, st);
}
cudaError_t dflash_bwd_ring_launch(int dtype, int shape, const DflashBwdArgs& a, int ctas, cudaStream_t st) {
  return dtype == kDtypeBF16 ? DfShapes<bf16_t>::bwd_kind(shape, a, ctas, st)
                             : DfShapes<float>::bwd_kind(shape, a, ctas, st);
}

}  // namespace specdec
