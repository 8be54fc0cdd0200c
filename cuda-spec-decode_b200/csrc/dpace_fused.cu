// D-PACE forward and backward in one persistent kernel that reads the logits
// from HBM once: the backward pass re-reads them from L2.
//
// The separate forward / backward kernels (dpace_ring.cu) read every live
// logit twice from HBM (forward, then backward) and write the gradient once.
// Here one grid works through a single queue of 64 KB blocks in which each
// forward (F) block b is followed, about D blocks later, by the backward (B)
// block b over the same elements:
//   F: stream the logits (bulk copies with an L2 evict_last policy), keep the
//      per-piece (max, sum of e^(x - max)) partials as the forward kernel
//      does. When a CTA finishes an F block it counts it for every sequence
//      the block overlaps; the CTA that completes a sequence's count
//      finalizes that sequence in place (merge partials -> lse, ce, the
//      B-scan, scale, loss_n) and publishes a per-sequence ready flag
//      (release store).
//   B: stream the same logits again -- within about D x 64 KB of their F
//      read, so from L2 (loads marked evict_first, the last use) -- wait
//      (acquire load, bounded) for the row's sequence to be ready, and write
//      scale * (softmax - onehot) with streaming stores.
// HBM traffic per call: one read of the live logits and one write of the
// gradient, instead of two reads and one write.
//
// Coordination is per warp, with no CTA barrier in the loop (a barrier has
// no timeout): each consumer warp counts its own share of a finished F block,
// and the warp whose count completes a sequence finalizes it alone.
// Deadlock freedom: the grid is exactly the resident capacity (persistent
// CTAs); F work never waits on other warps; the lag D is at least one
// sequence's worth of blocks, so every F block a B block depends on is handed
// out before it, and a CTA processes its blocks in hand-out order -- a wait
// can never close a cycle. Every wait is still bounded (1 s): an expired one
// sets the flag and the call reports status 5 with a NaN loss.
//
// Results equal the separate kernels' bit for bit (same partial layout and
// merge order, same finalize arithmetic, same gradient expression).
//
// Reference behaviour: losses/dpace.py:15-145; numbers follow
// losses/dpace_ref.py:8-51.
#include <cfloat>

#include "ring.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

// Work item w -> (phase, block): F blocks 0..D-1 first, then B block k and
// F block D+k alternate; when the F blocks run out, the rest are B blocks.
__device__ __forceinline__ void fused_map(int64_t w, int64_t nb, int64_t D, int& phase, int64_t& b) {
  if (w < D) {
    phase = 0;
    b = w;
  } else if (w < 2 * nb - D) {
    const int64_t k = w - D;
    phase = (k & 1) ? 0 : 1;
    b = (k & 1) ? D + (k >> 1) : (k >> 1);
  } else {
    phase = 1;
    b = w - nb;
  }
}

template <int S, int SE, class T>
struct FusedSmem {
  RingSmem<1, S, SE, T> ring;
  int sph[S];  // phase of the stage in each slot
};

// Bounded wait until the sequence's ready flag is set (every lane loads it
// with acquire semantics, so each lane's later loads see the finalize's
// stores). False on timeout.
__device__ __forceinline__ bool wait_ready(const unsigned* ready) {
  if (ld_acquire(ready)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!ld_acquire(ready)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// Finalize sequence n with one warp (lane j <-> row j, B <= 32): the
// arithmetic of dpace_finalize_kernel. The partial loads of all rows are
// issued before any merge.
template <class T, int NC>
__device__ void fused_finalize(const DpaceFusedArgs& a, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int B = a.f.B;
  const int64_t V = a.f.pt.V, BL = a.f.pt.chunk;
  const int pmax = a.f.pt.pmax;
  const int j = lane;
  const bool in = j < B;
  const int64_t rj = n * B + (in ? j : 0);
  const float mkj = in ? (a.f.mask ? a.f.mask[rj] : 1.f) : 0.f;
  const int64_t tj = in ? a.f.targets[rj] : 0;
  const bool tvalid = tj >= 0 && tj < V;
  const float xt = in && tvalid && mkj > 0.f ? ldg_f32(static_cast<const T*>(a.f.logits) + rj * V + tj) : 0.f;
  const unsigned livebits = __ballot_sync(kFullMask, in && mkj > 0.f);
  float lse_j = 0.f;
  constexpr int kRows = 8;  // rows whose partial loads are in flight together
  for (int i0 = 0; i0 < B; i0 += kRows) {
    float2 p0[kRows], p1[kRows];
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      const int i = i0 + u;
      p0[u] = p1[u] = make_float2(kNegSeed, 0.f);
      if (i < B && ((livebits >> i) & 1u)) {
        const int64_t r = n * B + i;
        const int k = blocks_in_row(r, V, BL) * NC;
        const float2* part = a.f.part + r * pmax * NC;
        if (lane < k) p0[u] = __ldcg(part + lane);
        if (lane + 32 < k) p1[u] = __ldcg(part + lane + 32);
      }
    }
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      const int i = i0 + u;
      if (i >= B || !((livebits >> i) & 1u)) continue;
      const int64_t r = n * B + i;
      const int k = blocks_in_row(r, V, BL) * NC;
      const float2* part = a.f.part + r * pmax * NC;
      float m = p0[u].x, s = p0[u].y;  // slot-major, warp-minor, then a fixed butterfly
      lse_merge(m, s, p1[u].x, p1[u].y);
      for (int qd = lane + 64; qd < k; qd += 32) {
        const float2 v = __ldcg(part + qd);
        lse_merge(m, s, v.x, v.y);
      }
      warp_lse(m, s);
      // the butterfly leaves the lanes' (m, s) up to an ulp apart (a merge
      // rounds its two operands asymmetrically): lane 0's value is the
      // result, as in dpace_finalize_kernel
      const float lse = __shfl_sync(kFullMask, __fadd_rn(m, logf(s)), 0);
      if (lane == i) lse_j = lse;
    }
  }
  const bool live = in && mkj > 0.f;
  const float ce = live && tvalid ? lse_j - xt : 0.f;
  if (in && !tvalid) atomicOr(a.f.flag, 1);
  if (in) a.f.lse[rj] = live ? lse_j : 0.f;
  const float mk = live ? 1.f : 0.f;
  const float sm = live ? __fadd_rn(__fmul_rn(a.f.one_minus_alpha, expf(-ce)), a.f.alpha) : 1.f;
  // prefix product and suffix sum in double, in sequence order
  double run = 1.0;
  float P = 1.f;
  for (int i = 0; i < B; ++i) {
    run *= (double)__shfl_sync(kFullMask, sm, i);
    if (i == j) P = (float)run;
  }
  const float pm = __fmul_rn(P, mk);
  double acc = 0.0;
  float Sx = 0.f;
  for (int i = B - 1; i >= 0; --i) {
    acc += (double)__shfl_sync(kFullMask, pm, i);
    if (i == j) Sx = (float)acc;
  }
  float w = a.f.loss_type == 1 ? P : (a.f.loss_type == 2 ? __fdiv_rn(Sx, fmaxf(P, FLT_MIN)) : Sx);
  w = __fmul_rn(w, mk);
  const float contrib = live ? __fmul_rn(ce, w) : 0.f;
  if (in) a.f.scale[rj] = __fmul_rn(w, a.f.inv_n);
  const float loss_n = warp_sum(contrib);
  if (lane == 0) {
    if (a.f.loss_n) a.f.loss_n[n] = loss_n;
    a.f.seq_loss[n] = loss_n;
  }
  __syncwarp();
  __threadfence();  // scale / lse / seq_loss before the flag
  unsigned last = 0;
  if (lane == 0) {
    st_release(a.ready + n, 1u);
    last = atomicAdd(a.f.done_cnt, 1u) + 1 == (unsigned)a.f.N;
  }
  last = __shfl_sync(kFullMask, last, 0);
  if (last) {
    __threadfence();
    const float total = warp_sum_l2(a.f.seq_loss, a.f.N);
    if (lane == 0) a.f.loss[0] = total / (float)a.f.n_global;
  }
}

// Compiled for 3 resident CTAs per SM (the ring's occupancy) in both types.
template <class T, int NC, int S, int SE, int BS>
__global__ void __launch_bounds__((NC + 1) * 32, 3) dpace_fused_ring_kernel(const __grid_constant__ DpaceFusedArgs a) {
  constexpr int kVec = 16 / sizeof(T);
  constexpr int kSub = SE / NC;
  constexpr int64_t BL = (int64_t)BS * SE;
  constexpr int kLogBL = __builtin_ctzll(BL);
  static_assert(kSub % (32 * kVec) == 0, "sub-range must be whole 16-byte rounds of a warp");
  static_assert((BL & (BL - 1)) == 0, "block length must be a power of two");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<FusedSmem<S, SE, T>*>(smem_raw);
  const T* X = static_cast<const T*>(a.f.logits);
  T* dst = static_cast<T*>(a.dlogits);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t E = a.f.pt.E, V = a.f.pt.V, R = E / V;
  const int B = a.f.B;
  const int64_t seq_len = (int64_t)B * V;
  const int pmax = a.f.pt.pmax;
  const int64_t nb = (E + BL - 1) / BL;
  const int64_t D = a.lag < 1 ? 1 : (a.lag > nb ? nb : a.lag);
  const unsigned total = (unsigned)(2 * nb);

  ring_init(sm.ring, NC);
  const RowBits rb = build_row_bits(sm.ring.bits, R, NC + 1, [&](int64_t r) {
    return a.f.mask == nullptr || a.f.mask[r] > 0.f;
  });
  __syncthreads();

  if (warp == NC) {  // producer (lane 0)
    if (lane == 0) {
      const uint64_t keep = policy_evict_last(), last_use = policy_evict_first();
      unsigned w = atomicAdd(a.f.q_ctr, 1u);
      unsigned wn = w < total ? atomicAdd(a.f.q_ctr, 1u) : total;
      int phase = 0;
      int64_t b = 0, blk_end = 0, r_issue = 0;
      int k = 0;
      if (w < total) {
        fused_map(w, nb, D, phase, b);
        blk_end = min((b + 1) * BL, E);
        r_issue = (b * BL) / V;
      }
      for (int64_t it = 0;; ++it) {
        const int slot = (int)(it % S);
        if (!mbar_wait(sm.ring.empty + slot, (uint32_t)(((it / S) & 1) ^ 1))) {
          atomicOr(a.f.flag, 2);
          break;
        }
        if (a.withhold_stage && blockIdx.x == 0 && it == 0) continue;  // failure-detection tests
        if (w >= total) {
          sm.ring.sf0[slot] = -1;
          mbar_arrive(sm.ring.full + slot);
          break;
        }
        const int64_t f0 = b * BL + (int64_t)k * SE;
        const int64_t f1 = min(f0 + SE, blk_end);
        while ((r_issue + 1) * V <= f0) ++r_issue;
        sm.ring.sf0[slot] = f0;
        sm.ring.srow[slot] = r_issue;
        sm.sph[slot] = phase;
        bool live = !rb.valid;
        for (int64_t r = r_issue; !live && r * V < f1; ++r) live = rb.live(r);
        const uint32_t vbytes = (uint32_t)(((f1 - f0) * (int64_t)sizeof(T)) & ~int64_t(15));
        if (live && vbytes) {
          mbar_arrive_expect_tx(sm.ring.full + slot, vbytes);
          bulk_g2s_hint(sm.ring.ring + (size_t)slot * SE, X + f0, vbytes, sm.ring.full + slot,
                        phase == 0 ? keep : last_use);
        } else {
          mbar_arrive(sm.ring.full + slot);
        }
        if (f1 == blk_end) {
          w = wn;
          k = 0;
          if (w < total) {
            wn = atomicAdd(a.f.q_ctr, 1u);
            fused_map(w, nb, D, phase, b);
            blk_end = min((b + 1) * BL, E);
            r_issue = (b * BL) / V;
          }
        } else {
          ++k;
        }
      }
    }
    return;
  }

  // ---- consumer warps ----------------------------------------------------
  // F state (as the forward kernel)
  float m = kNegSeed, s = 0.f;
  // B state (as the backward kernel)
  float sc = 0.f, l = 0.f;
  int64_t tf = -1, ready_seq = -1;
  bool zero = true, timed_out = false;
  int64_t r = 0, blk = -1;
  int phase = 0;
  bool live = false;
  auto enter_row = [&](int64_t row) {
    live = row < R && (rb.valid ? rb.live(row) : (a.f.mask == nullptr || a.f.mask[row] > 0.f));
    if (phase == 1) {
      zero = true;
      if (live && !timed_out) {
        const int64_t n = row / B;
        if (n != ready_seq) {
          if (!wait_ready(a.ready + n)) {
            // the call reports the timeout; this warp writes zeros for the
            // rest of its work instead of waiting again
            timed_out = true;
            if (lane == 0) atomicOr(a.f.flag, 2);
            return;
          }
          ready_seq = n;
        }
        sc = __ldcg(a.f.scale + row);
        l = __ldcg(a.f.lse + row);
        tf = row * V + a.f.targets[row];
        zero = sc == 0.f;
      }
    }
  };
  auto close_piece = [&]() {  // F: the (r, blk) piece of this warp is complete
    if (live) {
      warp_lse(m, s);
      if (lane == 0) {
        const int64_t slot = blk - (r * V) / BL;
        a.f.part[(r * pmax + slot) * NC + warp] = make_float2(m, s);
      }
    }
    m = kNegSeed;
    s = 0.f;
  };
  // F block done (this warp's share): count it for every sequence the block
  // overlaps; the warp whose count completes a sequence finalizes it.
  auto f_block_done = [&](int64_t bb, int64_t bend) {
    __syncwarp();
    __threadfence();  // this warp's partials before its count
    const int64_t n0 = (bb * BL) / seq_len, n1 = (bend - 1) / seq_len;
    for (int64_t n = n0; n <= n1; ++n) {
      unsigned complete = 0;
      if (lane == 0) {
        const int64_t first = (n * seq_len) / BL, lastb = ((n + 1) * seq_len - 1) / BL;
        const unsigned expected = (unsigned)((lastb - first + 1) * NC);
        complete = atomicAdd(a.seq_done + n, 1u) + 1 == expected;
      }
      if (__shfl_sync(kFullMask, complete, 0)) {
        __threadfence();  // the other warps' partials, published before their counts
        fused_finalize<T, NC>(a, n);
      }
    }
  };

  for (int64_t it = 0;; ++it) {
    const int slot = (int)(it % S);
    if (!__all_sync(kFullMask, mbar_wait(sm.ring.full + slot, (uint32_t)((it / S) & 1)))) {
      if (lane == 0) atomicOr(a.f.flag, 2);
      ring_drain<S>(sm.ring.full, it + 1);
      break;
    }
    const int64_t f0 = sm.ring.sf0[slot];
    if (f0 < 0) break;
    const int64_t b = f0 >> kLogBL;
    const int64_t blk_end = min((b + 1) * BL, E);
    const int64_t f1 = min(f0 + SE, blk_end);
    if ((f0 & (BL - 1)) == 0) {  // first stage of a block (a block may follow itself: F b, then B b)
      blk = b;
      phase = sm.sph[slot];
      r = sm.ring.srow[slot];
      m = kNegSeed;
      s = 0.f;
      enter_row(r);
    }
    const T* sb = sm.ring.ring + (size_t)slot * SE;
    const int64_t fv = copied_end<T>(f0, f1);
    if (phase == 0) {
      if (f1 - f0 == SE && (r + 1) * V >= f1) {  // a full stage inside one row
        if (live) warp_lse_full<kSub>(sb + warp * kSub, m, s);
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.ring.empty + slot);
        if ((r + 1) * V == f1) {
          close_piece();
          ++r;
          enter_row(r);
        } else if (f1 == blk_end) {
          close_piece();
        }
      } else {
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
        if (lane == 0) mbar_arrive(sm.ring.empty + slot);
        if (f1 == blk_end && r * V < blk_end) close_piece();
      }
      if (f1 == blk_end) f_block_done(b, blk_end);
      continue;
    }
    // phase B: the backward kernel's body
    const int64_t w0 = f0 + (int64_t)warp * kSub, w1 = min(w0 + kSub, f1);
    int64_t f = f0;
    while (f < f1) {
      const int64_t rend = (r + 1) * V;
      const int64_t ge = min(f1, rend);
      const int64_t lo = max(f, w0), hi = min(ge, w1);
      if (lo < hi) {
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
            for (int kk = lane; kk < nv; kk += 32) st_stream_u4(d4 + kk, z);
          } else if constexpr (sizeof(T) == 4) {
            float4* d4 = reinterpret_cast<float4*>(dst + lov);
            const float4* s4 = reinterpret_cast<const float4*>(sb + (lov - f0));
            const int64_t tq = tf - lov;
            for (int kk = lane; kk < nv; kk += 32) {
              const float4 v = s4[kk];
              float4 y;
              y.x = exp_shift(v.x, l);
              y.y = exp_shift(v.y, l);
              y.z = exp_shift(v.z, l);
              y.w = exp_shift(v.w, l);
              const uint64_t d = (uint64_t)(tq - 4 * (int64_t)kk);
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
              st_stream(d4 + kk, y);
            }
          } else {
            uint4* d4 = reinterpret_cast<uint4*>(dst + lov);
            const uint4* s4 = reinterpret_cast<const uint4*>(sb + (lov - f0));
            const int64_t tq = tf - lov;
            const float2 sc2 = make_float2(sc, sc);
            for (int kk = lane; kk < nv; kk += 32) {
              const uint4 v = s4[kk];
              const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
              float2 e[4], y[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                e[h] = exp_shift2(bf16x2_f32(wv[h]), l);
                y[h] = fmul2(e[h], sc2);
              }
              const uint64_t d = (uint64_t)(tq - 8 * (int64_t)kk);
              if (d < 8) {
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  if (d == (uint64_t)(2 * h)) y[h].x = sc * (e[h].x - 1.f);
                  if (d == (uint64_t)(2 * h + 1)) y[h].y = sc * (e[h].y - 1.f);
                }
              }
              st_stream_u4(d4 + kk, make_uint4(pack_bf16x2(y[0].x, y[0].y), pack_bf16x2(y[1].x, y[1].y),
                                               pack_bf16x2(y[2].x, y[2].y), pack_bf16x2(y[3].x, y[3].y)));
            }
          }
        } else {
          for (int64_t x = lo + lane; x < hi; x += 32) scalar(x);
        }
      }
      f = ge;
      if (ge == rend) {
        ++r;
        // enter (and wait for) the next row only if it starts inside this
        // block; a row of a later block is entered at that block's start
        if (ge < blk_end) enter_row(r);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.ring.empty + slot);
  }

  // ---- exit: the last consumer warp of the grid reports and resets ---------
  __syncwarp();
  __threadfence();
  unsigned last = 0;
  if (lane == 0) last = atomicAdd(a.done_warps, 1u) + 1 == gridDim.x * (unsigned)NC;
  if (__shfl_sync(kFullMask, last, 0)) {
    __threadfence();
    const int64_t N = a.f.N;
    for (int64_t i = lane; i < N; i += 32) {
      a.seq_done[i] = 0u;
      a.ready[i] = 0u;
    }
    if (lane == 0) {
      const int fl = atomicExch(a.f.flag, 0);
      if (fl & 2) a.f.loss[0] = __int_as_float(0x7fc00000);  // a wait expired: no result
      if (a.f.status) a.f.status[0] = (fl & 2) ? kStatusTimeout : ((fl & 1) ? kStatusTargetRange : kStatusOk);
      *a.f.q_ctr = 0u;
      *a.f.done_cnt = 0u;
      *a.done_warps = 0u;
    }
  }
}

template <class T>
struct FusedVariant {
  static constexpr int k = 4 / sizeof(T);
  static constexpr int NC = 4, S = 4, SE = 4096 * k, BS = 4;
  static constexpr size_t smem() { return sizeof(FusedSmem<S, SE, T>); }
  static int ctas(int device, int cap) {
    return ring_occupancy_ctas(dpace_fused_ring_kernel<T, NC, S, SE, BS>, (NC + 1) * 32, smem(), device, cap);
  }
  static cudaError_t launch(DpaceFusedArgs a, int ctas, cudaStream_t st) {
    cudaError_t e = ensure_smem_limit<dpace_fused_ring_kernel<T, NC, S, SE, BS>>(smem());
    if (e != cudaSuccess) return e;
    a.f.nc = NC;
    dpace_fused_ring_kernel<T, NC, S, SE, BS><<<ctas, (NC + 1) * 32, smem(), st>>>(a);
    return cudaGetLastError();
  }
};

// x *= *factor in place, 16-byte vectors; returns at once when the factor is
// exactly 1 (the usual upstream gradient of a loss), so that case costs no
// pass over x.
template <class T>
__global__ void __launch_bounds__(256) scale_inplace_kernel(T* x, int64_t n, const float* factor) {
  const float fct = __ldg(factor);
  if (fct == 1.0f) return;
  constexpr int kVec = 16 / sizeof(T);
  const int64_t nv = n / kVec;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if constexpr (sizeof(T) == 4) {
    float4* x4 = reinterpret_cast<float4*>(x);
    for (int64_t i = i0; i < nv; i += stride) {
      float4 v = x4[i];
      v.x *= fct;
      v.y *= fct;
      v.z *= fct;
      v.w *= fct;
      x4[i] = v;
    }
  } else {
    uint4* x4 = reinterpret_cast<uint4*>(x);
    const float2 f2 = make_float2(fct, fct);
    for (int64_t i = i0; i < nv; i += stride) {
      const uint4 v = x4[i];
      const float2 a0 = fmul2(bf16x2_f32(v.x), f2), a1 = fmul2(bf16x2_f32(v.y), f2);
      const float2 a2 = fmul2(bf16x2_f32(v.z), f2), a3 = fmul2(bf16x2_f32(v.w), f2);
      x4[i] = make_uint4(pack_bf16x2(a0.x, a0.y), pack_bf16x2(a1.x, a1.y), pack_bf16x2(a2.x, a2.y),
                         pack_bf16x2(a3.x, a3.y));
    }
  }
  for (int64_t i = nv * kVec + i0; i < n; i += stride) store_elem(x + i, to_f32(x[i]) * fct);
}

}  // namespace

cudaError_t scale_inplace_launch(int dtype, void* x, int64_t n, const float* factor, int ctas, cudaStream_t st) {
  if (dtype == kDtypeBF16)
    scale_inplace_kernel<bf16_t><<<ctas, 256, 0, st>>>(static_cast<bf16_t*>(x), n, factor);
  else
    scale_inplace_kernel<float><<<ctas, 256, 0, st>>>(static_cast<float*>(x), n, factor);
  return cudaGetLastError();
}

int dpace_fused_block_elems(int dtype) { return 4096 * 4 * (dtype == kDtypeBF16 ? 2 : 1); }
int dpace_fused_consumers() { return 4; }

int dpace_fused_ctas(int dtype, int device, int cap) {
  return dtype == kDtypeBF16 ? FusedVariant<bf16_t>::ctas(device, cap) : FusedVariant<float>::ctas(device, cap);
}

cudaError_t dpace_fused_launch(int dtype, const DpaceFusedArgs& a, int ctas, cudaStream_t st) {
  return dtype == kDtypeBF16 ? FusedVariant<bf16_t>::launch(a, ctas, st) : FusedVariant<float>::launch(a, ctas, st);
}

}  // namespace specdec
