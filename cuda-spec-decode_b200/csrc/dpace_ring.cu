// D-PACE forward and backward on the warp-specialized CTA ring (ring.cuh).
//
// Same arithmetic and outputs as dpace_kernels.cu (the 128-bit-load kernels,
// kept for inputs whose base address is not 16-byte aligned).
//
// Forward = two launches on the stream:
//   1. dpace_fwd_ring_kernel streams the logits once, in queue blocks of
//      BS stages and, over the last SPECDEC_FWD_TAIL_BLOCKS blocks' worth of
//      elements, of one stage (BlockMap). Each consumer warp keeps an online
//      (max, sum of e^(x - max)) for the row it is in and, whenever a
//      (row, block) piece ends, stores it to part[(block + r) * NC + warp]
//      (row r's slots start at index(r V) + r). Plain stores only, no
//      counters, no global loads in the consumers.
//   2. dpace_finalize_kernel (chained with programmatic dependent launch): one
//      CTA per sequence, warp j <-> row j merges the row's partials in slot
//      order -> lse_j, reads x[target_j], ce_j = lse_j - x[target_j]; warp 0 runs the B-scan
//      (q, smoothing, prefix product, suffix sum, weights), writes scale and
//      loss_n; the last CTA (done counter) sums loss_n in index order.
// Backward = one launch: dpace_bwd_ring_kernel streams logits through the ring
// and writes (w_j / N) * dloss * (softmax - onehot) with streaming stores.
// Rows with position mask 0 are never copied (forward); rows with scale 0 are
// never copied and written as zeros (backward).
//
// Element type T: float, or bf16_t (bfloat16 bit patterns). bf16 stages hold
// twice the elements in the same bytes; every element is widened exactly to
// float and all arithmetic is float; the bf16 backward rounds each gradient
// element to nearest even.
//
// Reference behaviour: losses/dpace.py:15-118 (forward), :120-145 (backward);
// numbers follow losses/dpace_ref.py:8-51.
#include <cfloat>

#include "ring.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

template <class T, int NC, int S, int SE, int BS>
__global__ void __launch_bounds__((NC + 1) * 32, (ring_min_ctas<NC, 1, S, SE, T>())) dpace_fwd_ring_kernel(const __grid_constant__ DpaceFwdArgs a) {
  constexpr int kSub = SE / NC;
  constexpr int64_t BL = (int64_t)BS * SE;
  static_assert(kSub % (32 * (16 / sizeof(T))) == 0, "sub-range must be whole 16-byte rounds of a warp");
  static_assert((BL & (BL - 1)) == 0, "block length must be a power of two");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<RingSmem<1, S, SE, T>*>(smem_raw);
  const T* X = static_cast<const T*>(a.logits);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t E = a.pt.E, V = a.pt.V, R = E / V;
  // blocks of BL elements, then one-stage blocks from a.pt.split on
  const BlockMap bm = make_block_map(E, BL, SE, a.pt.split);

  BlockQueue q;
  q.ctr = a.q_ctr;
  q.retired = a.q_retired;
  q.nblocks = bm.nblocks;
  q.dynamic = a.q_dynamic;
  // the producer's first block is its own index; with SPECDEC_EARLY_FIRST_STAGE
  // the producer lane initialises the ring and posts that block's first stage
  // before the liveness table is built, so the copy's latency overlaps the
  // table's loads
  const unsigned first = q.first();
  const bool withhold = a.withhold_stage && blockIdx.x == 0;
#if SPECDEC_EARLY_FIRST_STAGE
  ring_init(sm, NC, NC * 32);
  bool posted = false;
  if (warp == NC && lane == 0) {
    const T* src0[1] = {X};
    posted = ring_post_first<1, S, SE>(src0, bm, V, q, sm.ring, sm.full, sm.sf0, sm.srow, first, withhold,
                                       static_cast<RingTrack<S>*>(nullptr));
  }
#else
  ring_init(sm, NC);
  const bool posted = false;
#endif
  const RowBits rb = build_row_bits(sm.bits, R, NC + 1, [&](int64_t r) {
    return a.mask == nullptr || a.mask[r] > 0.f;
  });
  __syncthreads();

  if (warp == NC) {  // producer
    if (lane == 0) {
      const T* src[1] = {X};
      if (!ring_produce<1, S, SE>(src, bm, V, rb, q, sm.ring, sm.full, sm.empty, sm.sf0, sm.srow, first,
                                  withhold, static_cast<RingTrack<S>*>(nullptr), posted)) {
        atomicOr(a.flag, 2);
        if (a.status) a.status[0] = kStatusTimeout;
      }
      q.retire();
    }
    pdl_trigger();
    return;
  }

  // consumer warp `warp`
  float m = kNegSeed, s = 0.f;
  int64_t r = 0, blk = -1;
  bool live = false;
  auto enter_row = [&](int64_t row) {
    live = row < R && (rb.valid ? rb.live(row) : (a.mask == nullptr || a.mask[row] > 0.f));
  };
  auto close_piece = [&]() {  // the (r, blk) piece of this warp is complete
    if (live) {
      warp_lse(m, s);
      if (lane == 0) {
        a.part[(blk + r) * NC + warp] = make_float2(m, s);  // row r's slot blk - index(r V)
      }
    }
    m = kNegSeed;
    s = 0.f;
  };
  for (int64_t it = 0;; ++it) {
    const int slot = (int)(it % S);
    if (!__all_sync(kFullMask, mbar_wait(sm.full + slot, (uint32_t)((it / S) & 1)))) {
      if (lane == 0) {
        atomicOr(a.flag, 2);
        if (a.status) a.status[0] = kStatusTimeout;
      }
      ring_drain<S>(sm.full, it + 1);
      break;
    }
    const int64_t f0 = sm.sf0[slot];
    if (f0 < 0) break;
    const int64_t b = bm.index(f0);
    const int64_t blk_end = bm.end((unsigned)b);
    const int64_t f1 = min(f0 + SE, blk_end);
    if (b != blk) {  // first stage of a new block
      blk = b;
      r = sm.srow[slot];
      enter_row(r);
    }
    const T* sb = sm.ring + (size_t)slot * SE;
    if (f1 - f0 == SE && (r + 1) * V >= f1) {
      // fast path: a full stage inside one row; the slot is released as soon
      // as the warp's values are in registers
      if (live) {
        warp_lse_full<kSub>(sb + warp * kSub, m, s, sm.empty + slot);
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.empty + slot);
      }
      if ((r + 1) * V == f1) {
        close_piece();
        ++r;
        enter_row(r);
      } else if (f1 == blk_end) {
        close_piece();  // the block ends inside row r
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
        if (hv > lo) warp_lse_smem(sb, (int)(lo - f0), (int)(hv - f0), m, s);
        for (int64_t x = max(lo, fv) + lane; x < hi; x += 32) lse_push(m, s, ldg_f32(X + x));
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
    if (f1 == blk_end && r * V < blk_end) close_piece();  // the block ends inside row r
  }
  pdl_trigger();
}

// One CTA per sequence n, warp j <-> row j (B <= 32 warps).
template <class T>
__global__ void __launch_bounds__(1024) dpace_finalize_kernel(const __grid_constant__ DpaceFwdArgs a) {
  __shared__ float sh_ce[32];
  __shared__ int sh_live[32];
  // a backward chained behind this kernel (specdec_dpace_forward_backward)
  // may become resident now: it streams logits and waits for lse / scale
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = a.B;
  const int64_t n = blockIdx.x, V = a.pt.V;
  const int NC = a.nc;
  const BlockMap bm = make_block_map(a.pt.E, a.pt.chunk, a.pt.stage, a.pt.split);
  bool timed_out;
  {
    const int64_t r = n * B + warp;
    // inputs the streaming grid does not write: read them while it drains
    const float mk = a.mask ? a.mask[r] : 1.f;
    const int64_t t = a.targets[r];
    const bool tvalid = t >= 0 && t < V;
    const float xt = tvalid ? ldg_f32(static_cast<const T*>(a.logits) + r * V + t) : 0.f;  // x[target]
    pdl_wait();  // the streaming grid has completed and its stores are visible
    // a wait of the streaming grid expired: partials may be missing, so every
    // per-row output is NaN (a backward from them gives a NaN gradient)
    timed_out = (*reinterpret_cast<volatile int*>(a.flag) & 2) != 0;
    const int k = bm.pieces(r, V) * NC;
    const float2* part = a.part + (bm.index(r * V) + r) * NC;
    // up to 8 partials per lane are loaded before the first merge (rows in
    // the one-stage blocks at the end have up to ceil(V / stage) + 1 slots);
    // merging an absent one (kNegSeed, 0) leaves (m, s) bit for bit unchanged
    constexpr int kPre = 8;
    float2 pv[kPre];
#pragma unroll
    for (int i = 0; i < kPre; ++i) pv[i] = lane + 32 * i < k ? part[lane + 32 * i] : make_float2(kNegSeed, 0.f);
    const bool live = mk > 0.f;
    float lse = 0.f, ce = 0.f;
    if (live) {
      float m = pv[0].x, s = pv[0].y;  // slot-major, warp-minor, then a fixed butterfly
#pragma unroll
      for (int i = 1; i < kPre; ++i) lse_merge(m, s, pv[i].x, pv[i].y);
      for (int qd = lane + 32 * kPre; qd < k; qd += 32) {
        const float2 v = part[qd];
        lse_merge(m, s, v.x, v.y);
      }
      warp_lse(m, s);
      lse = __fadd_rn(m, logf(s));  // no contraction into logf: the same bits in every kernel
      if (tvalid) ce = lse - xt;
    }
    if (!tvalid && lane == 0) atomicOr(a.flag, 1);
    if (lane == 0) {
      a.lse[r] = timed_out ? __int_as_float(0x7fc00000) : lse;
      sh_ce[warp] = ce;
      sh_live[warp] = live;
    }
  }
  __syncthreads();
  if (warp == 0) {
    const int j = lane;
    const bool in = j < B;
    const int64_t r = n * B + (in ? j : 0);
    const bool live = in && sh_live[j];
    const float ce = in ? sh_ce[j] : 0.f;
    const float mk = live ? 1.f : 0.f;
    const float sm = live ? __fadd_rn(__fmul_rn(a.one_minus_alpha, expf(-ce)), a.alpha) : 1.f;
    // prefix product and suffix sum in double, in sequence order (torch CPU
    // cumprod / cumsum accumulate in double); every lane runs the serial scan
    // on factors gathered first, so the dependent chain is arithmetic only
    float f[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __shfl_sync(kFullMask, sm, i);
    double run = 1.0;
    float P = 1.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < B) run *= (double)f[i];
      if (i == j) P = (float)run;
    }
    const float pm = __fmul_rn(P, mk);
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __shfl_sync(kFullMask, pm, i);
    double acc = 0.0;
    float S = 0.f;
#pragma unroll
    for (int i = 31; i >= 0; --i) {
      if (i < B) acc += (double)f[i];
      if (i == j) S = (float)acc;
    }
    float w = a.loss_type == 1 ? P : (a.loss_type == 2 ? __fdiv_rn(S, fmaxf(P, FLT_MIN)) : S);
    w = __fmul_rn(w, mk);
    const float contrib = live ? __fmul_rn(ce, w) : 0.f;
    if (in) a.scale[r] = timed_out ? __int_as_float(0x7fc00000) : __fmul_rn(w, a.inv_n);
    const float loss_n = warp_sum(contrib);
    unsigned last = 0;
    if (lane == 0) {
      if (a.loss_n) a.loss_n[n] = loss_n;
      a.seq_loss[n] = loss_n;
      if (!a.defer_loss) {  // deferred: the chained backward sums seq_loss when it retires
        __threadfence();
        last = (atomicAdd(a.done_cnt, 1u) + 1 == (unsigned)a.N);
      }
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
        if (a.status) a.status[0] = (f & 2) ? kStatusTimeout : ((f & 1) ? kStatusTargetRange : kStatusOk);
        *a.done_cnt = 0u;
      }
    }
  }
}

template <class T, int NC, int S, int SE, int BS>
__global__ void __launch_bounds__((NC + 1) * 32, (ring_min_ctas<NC, 1, S, SE, T>())) dpace_bwd_ring_kernel(const __grid_constant__ DpaceBwdArgs a) {
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int kSub = SE / NC;
  constexpr int64_t BL = (int64_t)BS * SE;
  static_assert(kSub % kVec == 0, "sub-range must be whole 16-byte vectors");
  static_assert((BL & (BL - 1)) == 0, "block length must be a power of two");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<RingSmem<1, S, SE, T>*>(smem_raw);
  const T* X = static_cast<const T*>(a.logits);
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
  // Rows to read: those with a nonzero scale * dloss -- or, when chained
  // behind the finalize that writes scale, those with a scored mask, which is
  // known at once (a row with mask 0 has scale 0; a scored row whose scale is
  // 0 is read and written as zeros). Everything before the consumers' wait
  // touches only inputs the finalize does not write.
  if (!a.mask_liveness) pdl_wait();
  const RowBits rb = build_row_bits(sm.bits, R, NC + 1, [&](int64_t r) {
    return a.mask_liveness ? (a.live_mask == nullptr || a.live_mask[r] > 0.f) : __fmul_rn(a.scale[r], g) != 0.f;
  });
  __syncthreads();

  if (warp == NC) {
    if (lane == 0) {
      const T* src[1] = {X};
      if (!ring_produce<1, S, SE>(src, make_block_map(E, BL, SE, -1), V, rb, q, sm.ring, sm.full, sm.empty,
                                  sm.sf0, sm.srow, first, a.withhold_stage && blockIdx.x == 0, &sm.trk))
        sm.trk.timeout = 1;
    }
  } else {
    pdl_wait();  // lse and scale (chained: written by the finalize)
    int64_t r = 0, blk = -1, tf = -1;
    float sc = 0.f, l = 0.f;
    auto load_row = [&](int64_t row) {
      sc = __fmul_rn(a.scale[row], g);
      l = a.lse[row];
      tf = row * V + a.targets[row];
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
      const int64_t b = f0 / BL;
      const int64_t blk_end = min((b + 1) * BL, E);
      const int64_t f1 = min(f0 + SE, blk_end);
      if (b != blk) {
        blk = b;
        r = sm.srow[slot];
        load_row(r);
      }
      const int64_t fv = copied_end<T>(f0, f1);
      const int64_t w0 = f0 + (int64_t)warp * kSub, w1 = min(w0 + kSub, f1);
      const T* sb = sm.ring + (size_t)slot * SE;
      int64_t f = f0;
      while (f < f1) {
        const int64_t rend = (r + 1) * V;
        const int64_t ge = min(f1, rend);
        const int64_t lo = max(f, w0), hi = min(ge, w1);
        if (lo < hi) {
          const bool zero = sc == 0.f || !rb.live(r);
          // [lo, hi): scalar head to a vector boundary, 16-byte body, scalar tail
          const int64_t lov = (lo + kVec - 1) & ~int64_t(kVec - 1), hiv = min(hi, fv) & ~int64_t(kVec - 1);
          auto scalar = [&](int64_t x) {
            if (zero) {
              store_elem(dst + x, 0.f);
            } else {
              const float v = x < fv ? to_f32(sb[x - f0]) : ldg_f32(X + x);
              store_elem(dst + x, sc * (exp_shift(v, l) - (x == tf ? 1.f : 0.f)));
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
              const float4* s4 = reinterpret_cast<const float4*>(sb + (lov - f0));
              const int64_t tq = tf - lov;
              for (int k = lane; k < nv; k += 32) {
                const float4 v = s4[k];
                float4 y;
                y.x = exp_shift(v.x, l);
                y.y = exp_shift(v.y, l);
                y.z = exp_shift(v.z, l);
                y.w = exp_shift(v.w, l);
                const uint64_t d = (uint64_t)(tq - 4 * (int64_t)k);
                if (d < 4) {
                  if (d == 0) y.x -= 1.f;
                  else if (d == 1) y.y -= 1.f;
                  else if (d == 2) y.z -= 1.f;
                  else y.w -= 1.f;
                }
                y.x *= sc;
                y.y *= sc;
                y.z *= sc;
                y.w *= sc;
                st_stream(d4 + k, y);
              }
            } else {
              uint4* d4 = reinterpret_cast<uint4*>(dst + lov);
              const uint4* s4 = reinterpret_cast<const uint4*>(sb + (lov - f0));
              const int64_t tq = tf - lov;
              const float2 sc2 = make_float2(sc, sc);
              for (int k = lane; k < nv; k += 32) {
                const uint4 v = s4[k];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                float2 e[4], y[4];
  #pragma unroll
                for (int h = 0; h < 4; ++h) {
                  e[h] = exp_shift2(bf16x2_f32(w[h]), l);
                  y[h] = fmul2(e[h], sc2);
                }
                const uint64_t d = (uint64_t)(tq - 8 * (int64_t)k);
                if (d < 8) {  // the target: sc * (p - 1), as the float kernel
  #pragma unroll
                  for (int h = 0; h < 4; ++h) {
                    if (d == (uint64_t)(2 * h)) y[h].x = sc * (e[h].x - 1.f);
                    if (d == (uint64_t)(2 * h + 1)) y[h].y = sc * (e[h].y - 1.f);
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

// Stages per queue block of the backward kernels. The backward has no
// per-block partials (the forward's slot layout depends on its block length),
// so its blocks can be small: a CTA never holds more than one unstarted
// stage when the queue runs dry, which keeps the end of the launch tight.
#ifndef SPECDEC_BWD_BLOCK_STAGES
#define SPECDEC_BWD_BLOCK_STAGES 1
#endif
constexpr int kBwdBlockStages = SPECDEC_BWD_BLOCK_STAGES;
// Stages per forward block of shapes 0, 6 and 8 (8 is the forward's default). A
// smaller block shortens the end of the launch (the last blocks finish closer
// together) at the cost of more piece closes and more partials per row for
// the finalize to merge.
#ifndef SPECDEC_FWD_BLOCK_STAGES
#define SPECDEC_FWD_BLOCK_STAGES 4
#endif
constexpr int kFwdBlockStages = SPECDEC_FWD_BLOCK_STAGES;
// The D-PACE forward's last SPECDEC_FWD_TAIL_BLOCKS blocks' worth of elements
// are queued as one-stage blocks (BlockMap), so the launch's CTAs finish within
// about a stage of one another; 0: every block is kFwdBlockStages long. A
// constant, not a multiple of the grid: the block boundaries, and so the
// results, do not depend on the CTA count.
#ifndef SPECDEC_FWD_TAIL_BLOCKS
#define SPECDEC_FWD_TAIL_BLOCKS 512
#endif
constexpr int64_t kFwdTailBlocks = SPECDEC_FWD_TAIL_BLOCKS;

template <class T, int NC, int S, int SE, int BS>
struct RingVariant {
  static constexpr size_t smem() { return sizeof(RingSmem<1, S, SE, T>); }
  static int fwd_ctas(int device, int cap) {
    return ring_occupancy_ctas(dpace_fwd_ring_kernel<T, NC, S, SE, BS>, (NC + 1) * 32, smem(), device, cap);
  }
  static int bwd_ctas(int device, int cap) {
    return ring_occupancy_ctas(dpace_bwd_ring_kernel<T, NC, S, SE, kBwdBlockStages>, (NC + 1) * 32, smem(), device, cap);
  }
  static cudaError_t fwd(DpaceFwdArgs a, int ctas, cudaStream_t st) {
    // the attribute must be set on the launching device before the launch
    cudaError_t e = ensure_smem_limit<dpace_fwd_ring_kernel<T, NC, S, SE, BS>>(smem());
    if (e != cudaSuccess) return e;
    a.nc = NC;
    // the streaming kernel follows whatever the caller enqueued (possibly a
    // wait on another stream): a plain launch. Only the finalize, whose
    // predecessor is always this streaming kernel, is chained with PDL.
    dpace_fwd_ring_kernel<T, NC, S, SE, BS><<<ctas, (NC + 1) * 32, smem(), st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_pdl(dpace_finalize_kernel<T>, dim3((unsigned)a.N), dim3(32 * a.B), 0, st, a);
  }
  static cudaError_t bwd(const DpaceBwdArgs& a, int ctas, cudaStream_t st) {
    const cudaError_t e = ensure_smem_limit<dpace_bwd_ring_kernel<T, NC, S, SE, kBwdBlockStages>>(smem());
    if (e != cudaSuccess) return e;
    // chained only behind this library's own finalize (forward_backward)
    if (a.chained)
      return launch_pdl(dpace_bwd_ring_kernel<T, NC, S, SE, kBwdBlockStages>, dim3(ctas), dim3((NC + 1) * 32), smem(), st, a);
    dpace_bwd_ring_kernel<T, NC, S, SE, kBwdBlockStages><<<ctas, (NC + 1) * 32, smem(), st>>>(a);
    return cudaGetLastError();
  }
};

// Ring shapes (consumer warps x stages x stage elements x stages per block),
// float elements: 0 = 4 x 4 x 4096 x 4 (64 KB ring, 64 KB blocks, 3 CTAs/SM:
// the fastest measured on the [64, 16, 128256] workload); 1 = 8 x 4 x 8192 x 2
// (128 KB ring, 1 CTA/SM); 2 = 4 x 6 x 4096 x 4 (96 KB ring, 2 CTAs/SM); 3 =
// 4 x 8 x 4096 x 8 (128 KB ring, 128 KB blocks); 4 = 2 x 6 x 2048 x 8 (48 KB
// ring, 4 CTAs/SM); 5 = 8 x 4 x 4096 x 4 (64 KB ring, 8 consumer warps); 6 =
// 4 x 3 x 4096 x 4 (48 KB ring, 4 CTAs/SM); 7 = 4 x 6 x 2048 x 8 (48 KB ring
// in 8 KB stages, 4 CTAs/SM); 8 = 4 x 2 x 4096 x 4 (32 KB ring, 4 CTAs/SM for
// fp32, 5 for bf16: the D-PACE forward's default). bf16 shapes have the same
// bytes (twice the elements).
template <class T>
struct Shapes {
  static constexpr int k = 4 / sizeof(T);  // elements per float's bytes
  using R0 = RingVariant<T, 4, 4, 4096 * k, kFwdBlockStages>;
  using R1 = RingVariant<T, 8, 4, 8192 * k, 2>;
  using R2 = RingVariant<T, 4, 6, 4096 * k, 4>;
  using R3 = RingVariant<T, 4, 8, 4096 * k, 8>;
  using R4 = RingVariant<T, 2, 6, 2048 * k, 8>;
  using R5 = RingVariant<T, 8, 4, 4096 * k, 4>;
  using R6 = RingVariant<T, 4, 3, 4096 * k, kFwdBlockStages>;
  using R7 = RingVariant<T, 4, 6, 2048 * k, 8>;
  using R8 = RingVariant<T, 4, 2, 4096 * k, kFwdBlockStages>;

  static int block_elems(int shape) {
    switch (shape) {
      case 1: return 8192 * 2 * k;
      case 2: return 4096 * 4 * k;
      case 3: return 4096 * 8 * k;
      case 4: return 2048 * 8 * k;
      case 5: return 4096 * 4 * k;
      case 6: return 4096 * kFwdBlockStages * k;
      case 7: return 2048 * 8 * k;
      case 8: return 4096 * kFwdBlockStages * k;
      default: return 4096 * kFwdBlockStages * k;
    }
  }
  static int stage_elems(int shape) {
    switch (shape) {
      case 1: return 8192 * k;
      case 4: return 2048 * k;
      case 7: return 2048 * k;
      default: return 4096 * k;
    }
  }
  static int fwd_ctas(int shape, int device, int cap) {
    switch (shape) {
      case 1: return R1::fwd_ctas(device, cap);
      case 2: return R2::fwd_ctas(device, cap);
      case 3: return R3::fwd_ctas(device, cap);
      case 4: return R4::fwd_ctas(device, cap);
      case 5: return R5::fwd_ctas(device, cap);
      case 6: return R6::fwd_ctas(device, cap);
      case 7: return R7::fwd_ctas(device, cap);
      case 8: return R8::fwd_ctas(device, cap);
      default: return R0::fwd_ctas(device, cap);
    }
  }
  static int bwd_ctas(int shape, int device, int cap) {
    switch (shape) {
      case 1: return R1::bwd_ctas(device, cap);
      case 2: return R2::bwd_ctas(device, cap);
      case 3: return R3::bwd_ctas(device, cap);
      case 4: return R4::bwd_ctas(device, cap);
      case 5: return R5::bwd_ctas(device, cap);
      case 6: return R6::bwd_ctas(device, cap);
      case 7: return R7::bwd_ctas(device, cap);
      case 8: return R8::bwd_ctas(device, cap);
      default: return R0::bwd_ctas(device, cap);
    }
  }
  static cudaError_t fwd(int shape, const DpaceFwdArgs& a, int ctas, cudaStream_t st) {
    switch (shape) {
      case 1: return R1::fwd(a, ctas, st);
      case 2: return R2::fwd(a, ctas, st);
      case 3: return R3::fwd(a, ctas, st);
      case 4: return R4::fwd(a, ctas, st);
      case 5: return R5::fwd(a, ctas, st);
      case 6: return R6::fwd(a, ctas, st);
      case 7: return R7::fwd(a, ctas, st);
      case 8: return R8::fwd(a, ctas, st);
      default: return R0::fwd(a, ctas, st);
    }
  }
  static cudaError_t bwd(int shape, const DpaceBwdArgs& a, int ctas, cudaStream_t st) {
    switch (shape) {
      case 1: return R1::bwd(a, ctas, st);
      case 2: return R2::bwd(a, ctas, st);
      case 3: return R3::bwd(a, ctas, st);
      case 4: return R4::bwd(a, ctas, st);
      case 5: return R5::bwd(a, ctas, st);
      case 6: return R6::bwd(a, ctas, st);
      case 7: return R7::bwd(a, ctas, st);
      case 8: return R8::bwd(a, ctas, st);
      default: return R0::bwd(a, ctas, st);
    }
  }
};

}  // namespace

int dpace_ring_block_elems(int dtype, int shape) {
  return dtype == kDtypeBF16 ? Shapes<bf16_t>::block_elems(shape) : Shapes<float>::block_elems(shape);
}

int dpace_ring_stage_elems(int dtype, int shape) {
  return dtype == kDtypeBF16 ? Shapes<bf16_t>::stage_elems(shape) : Shapes<float>::stage_elems(shape);
}

int64_t dpace_fwd_split(int64_t E, int64_t BL) {
  if (kFwdTailBlocks <= 0 || E <= 0) return -1;
  const int64_t nb = (E + BL - 1) / BL;
  return (nb > kFwdTailBlocks ? nb - kFwdTailBlocks : 0) * BL;
}

int dpace_ring_consumers(int shape) {
  switch (shape) {
    case 1: return 8;
    case 4: return 2;
    case 5: return 8;
    default: return 4;
  }
}

int dpace_fwd_ring_ctas(int dtype, int shape, int device, int cap) {
  return dtype == kDtypeBF16 ? Shapes<bf16_t>::fwd_ctas(shape, device, cap)
                             : Shapes<float>::fwd_ctas(shape, device, cap);
}

int dpace_bwd_ring_ctas(int dtype, int shape, int device, int cap) {
  return dtype == kDtypeBF16 ? Shapes<bf16_t>::bwd_ctas(shape, device, cap)
                             : Shapes<float>::bwd_ctas(shape, device, cap);
}

cudaError_t dpace_fwd_ring_launch(int dtype, int shape, const DpaceFwdArgs& a, int ctas, cudaStream_t st) {
  return dtype == kDtypeBF16 ? Shapes<bf16_t>::fwd(shape, a, ctas, st) : Shapes<float>::fwd(shape, a, ctas, st);
}

cudaError_t dpace_bwd_ring_launch(int dtype, int shape, const DpaceBwdArgs& a, int ctas, cudaStream_t st) {
  return dtype == kDtypeBF16 ? Shapes<bf16_t>::bwd(shape, a, ctas, st) : Shapes<float>::bwd(shape, a, ctas, st);
}

}  // namespace specdec
