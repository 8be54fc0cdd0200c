// D-PACE forward and backward in one persistent kernel that reads the logits
// from HBM once: the backward pass re-reads them from L2.
//
// The separate forward / backward kernels (dpace_ring.cu) read every live
// logit twice from HBM (forward, then backward) and write the gradient once.
// Here one grid works through two queues of blocks (BL elements, 64 KB):
//   F: stream the logits (bulk copies with an L2 evict_last policy), keep the
//      per-piece (max, sum of e^(x - max)) partials as the forward kernel
//      does. When a warp finishes its share of an F block it counts it for
//      every sequence the block overlaps; the warp that completes a
//      sequence's count finalizes that sequence in place (merge partials ->
//      lse, ce, the B-scan, scale, loss_n) and publishes a per-sequence ready
//      flag (release store).
//   B: stream the same logits again, soon after their F read, so from L2
//      (loads marked evict_first, the last use), and write
//      scale * (softmax - onehot) with streaming stores.
// HBM traffic per call: one read of the live logits and one write of the
// gradient, instead of two reads and one write.
//
// Scheduling is done by each CTA's producer lane, so consumer warps never
// wait on another CTA. F blocks come from one grid-wide queue; each CTA keeps
// the F blocks it read in a FIFO and re-reads them itself (its B pass) --
// L2 is split between the two dies and a partition caches the lines of its
// own SMs' accesses, so the re-read must come from the SM that made the
// first read. The producer issues the oldest B block as soon as the
// sequences it overlaps are ready (acquire loads); until then it claims and
// issues F blocks, as long as the F front is less than `ahead` sequences past
// the number of finalized sequences -- that cap bounds how far the F reads
// run ahead of their B re-reads (the L2 window).
// Deadlock freedom: a producer waits only when its oldest B block is not
// ready and no F block can be claimed. If the cap is closed, every F block
// before the front has been claimed and issued by a running CTA (F work
// depends on nothing), so the sequences before the front get finalized and
// the cap opens. If its FIFO is full, the newest entry lies past the last
// block of the oldest entry's sequences (the FIFO holds more than a
// sequence's blocks + 2), so those sequences are claimed in full and get
// finalized. Every wait is still bounded (1 s): an expired one sets the flag
// and the call reports status 5 with a NaN loss. Blocks must overlap at most
// two sequences (B * V >= BL); the host runs the separate kernels otherwise.
//
// Results equal the separate kernels' bit for bit (same partial layout and
// merge tree, same finalize arithmetic, same gradient expression).
//
// Reference behaviour: losses/dpace.py:15-145; numbers follow
// losses/dpace_ref.py:8-51.
#include <cfloat>

#include "ring.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

// F blocks a CTA has read and not yet re-read (its B queue). The host keeps
// one sequence's blocks + 2 within it (dpace_fused_max_seq_blocks).
constexpr int kFifo = 1024;

template <int S, int SE, class T>
struct FusedSmem {
  RingSmem<1, S, SE, T> ring;
  int sph[S];         // phase of the stage in each slot
  int fifo[kFifo];    // producer only
};

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Finalize sequence n with one warp (B <= 32): the arithmetic of
// dpace_finalize_kernel, with the lse merges spread over all 32 lanes.
//
// dpace_finalize_kernel gives row r one warp: lane l folds partials l, l+32,
// l+64, ... into a leaf, then the xor butterfly (offsets 16, 8, 4, 2, 1)
// merges the leaves and lane 0's value is kept. Lane 0's value is the left-
// to-right pairwise tree over the leaves taken in bit-reversed lane order
// p -> l = rev5(p): the round with offset o merges lane i (left) with lane
// i ^ o, so offset 16 pairs neighbours in p order, offset 8 pairs of pairs,
// and so on. Here each row gets G = 32 / B' lanes (B' = B rounded up to a
// power of two); lane q of the group evaluates the subtree of leaves
// p in [q * B', (q + 1) * B') with a stack (a binary counter over the leaf
// index), then the group combines with xor shuffles 1, 2, ..., G / 2, the
// lower lane on the left: the same merges in the same order, so the same
// bits, with B' + log2(G) dependent merges per lane instead of B * 36.
template <class T, int NC>
__device__ __noinline__ void fused_finalize(const DpaceFusedArgs& a, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int B = a.f.B;
  const int64_t V = a.f.pt.V, BL = a.f.pt.chunk;
  const int pmax = a.f.pt.pmax;
  // lane j <-> row j for the inputs and the scan
  const int j = lane;
  const bool in = j < B;
  const int64_t rj = n * B + (in ? j : 0);
  const float mkj = in ? (a.f.mask ? a.f.mask[rj] : 1.f) : 0.f;
  const int64_t tj = in ? a.f.targets[rj] : 0;
  const bool tvalid = tj >= 0 && tj < V;
  const float xt = in && tvalid && mkj > 0.f ? ldg_f32(static_cast<const T*>(a.f.logits) + rj * V + tj) : 0.f;
  // lane group of the row for the merges
  int lgB = 0;
  while ((1 << lgB) < B) ++lgB;
  const int lgG = 5 - lgB, nleaf = 1 << lgB;
  const int row = lane >> lgG, q = lane & ((1 << lgG) - 1);
  const bool rlive = __shfl_sync(kFullMask, in && mkj > 0.f, row);  // row < 32
  const int64_t r = n * B + row;
  const int k = rlive ? blocks_in_row(r, V, BL) * NC : 0;
  const float2* part = a.f.part + r * pmax * NC;
  const float2 seed = make_float2(kNegSeed, 0.f);
  const int p0 = q * nleaf;
  constexpr int KB = 8;  // leaves whose partial loads are in flight together
  float2 c0[KB], c1[KB], n0[KB], n1[KB];
#pragma unroll
  for (int u = 0; u < KB; ++u) n0[u] = n1[u] = seed;
  auto load_leaves = [&](int i0, float2* x0, float2* x1) {
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const int i = i0 + u;
      const int l = (int)(__brev((unsigned)(p0 + i)) >> 27);
      x0[u] = i < nleaf && l < k ? __ldcg(part + l) : seed;
      x1[u] = i < nleaf && l + 32 < k ? __ldcg(part + l + 32) : seed;
    }
  };
  float sm_[5], ss_[5];
  float m = kNegSeed, s = 0.f;
  load_leaves(0, c0, c1);
  for (int i0 = 0; i0 < nleaf; i0 += KB) {
    if (i0 + KB < nleaf) load_leaves(i0 + KB, n0, n1);
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const int i = i0 + u;
      if (i >= nleaf) break;
      const int l = (int)(__brev((unsigned)(p0 + i)) >> 27);
      m = c0[u].x;
      s = c0[u].y;
      lse_merge(m, s, c1[u].x, c1[u].y);
      for (int qd = l + 64; qd < k; qd += 32) {
        const float2 v = __ldcg(part + qd);
        lse_merge(m, s, v.x, v.y);
      }
      // push leaf i: merge with the pending left subtrees of equal size
#pragma unroll
      for (int L = 0; L < 5; ++L) {
        if ((i >> L) & 1) {
          lse_merge(sm_[L], ss_[L], m, s);
          m = sm_[L];
          s = ss_[L];
        } else {
          sm_[L] = m;
          ss_[L] = s;
          break;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      c0[u] = n0[u];
      c1[u] = n1[u];
    }
  }
  for (int o = 1; o < (1 << lgG); o <<= 1) {
    const float om = __shfl_xor_sync(kFullMask, m, o);
    const float os = __shfl_xor_sync(kFullMask, s, o);
    lse_merge(m, s, om, os);
  }
  const float lse_row = __fadd_rn(m, logf(s));  // valid in lane q == 0 of a live row
  float lse_j = __shfl_sync(kFullMask, lse_row, in ? (j << lgG) : 0);
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

  ring_init(sm.ring, NC);
  const RowBits rb = build_row_bits(sm.ring.bits, R, NC + 1, [&](int64_t r) {
    return a.f.mask == nullptr || a.f.mask[r] > 0.f;
  });
  __syncthreads();

  if (warp == NC) {  // producer (lane 0)
    if (lane == 0) {
      const uint64_t keep = policy_evict_last(), last_use = policy_evict_first();
      int64_t it = 0;  // stages posted (ring position)
      bool withhold = a.withhold_stage && blockIdx.x == 0;  // failure-detection tests
      // Posts the stages of block b (phase 0 = F, 1 = B); false if a wait for
      // a free slot expired.
      auto issue_block = [&](int64_t b, int phase) -> bool {
        const int64_t blk_end = min((b + 1) * BL, E);
        int64_t r_issue = (b * BL) / V;
        for (int64_t f0 = b * BL; f0 < blk_end;) {
          const int slot = (int)(it % S);
          if (!mbar_wait(sm.ring.empty + slot, (uint32_t)(((it / S) & 1) ^ 1))) return false;
          ++it;
          if (withhold) {  // slot left empty: its consumers' wait expires
            withhold = false;
            continue;
          }
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
          f0 = f1;
        }
        return true;
      };
      // the sequences a block overlaps (at most two: seq_len >= BL)
      auto b_ready = [&](int64_t b) -> bool {
        const int64_t s0 = (b * BL) / seq_len, s1 = (min((b + 1) * BL, E) - 1) / seq_len;
        return ld_acquire(a.ready + s0) != 0u && (s1 == s0 || ld_acquire(a.ready + s1) != 0u);
      };
      bool ok = true;
      int head = 0, tail = 0;  // this CTA's F blocks awaiting their B pass: fifo[head..tail)
      int64_t f_seen = 0;      // lower bound of the F queue's head
      bool f_out = false;      // the F queue is empty
      uint64_t idle_since = 0;
      while (ok) {
        if (head != tail && b_ready(sm.fifo[head % kFifo])) {
          ok = issue_block(sm.fifo[head % kFifo], 1);
          ++head;
          idle_since = 0;
          continue;
        }
        if (!f_out && tail - head < kFifo &&
            (f_seen * BL) / seq_len < (int64_t)ld_relaxed(a.f.done_cnt) + a.ahead) {
          const int64_t fb = (int64_t)atomicAdd(a.f.q_ctr, 1u);
          if (fb < nb) {
            f_seen = fb + 1;
            sm.fifo[tail % kFifo] = (int)fb;
            ++tail;
            ok = issue_block(fb, 0);
            idle_since = 0;
            continue;
          }
          f_out = true;
        }
        if (f_out && head == tail) break;
        // nothing can be posted yet: the oldest B block waits for a finalize,
        // or the F front waits for the cap to open
        const uint64_t now = globaltimer_ns();
        if (idle_since == 0) {
          idle_since = now;
        } else if (now - idle_since > kWaitLimitNs) {
          ok = false;
          break;
        }
        __nanosleep(256);
      }
      if (!ok) atomicOr(a.f.flag, 2);
      // end marker for the consumers
      const int slot = (int)(it % S);
      if (mbar_wait(sm.ring.empty + slot, (uint32_t)(((it / S) & 1) ^ 1))) {
        sm.ring.sf0[slot] = -1;
        mbar_arrive(sm.ring.full + slot);
      } else {
        atomicOr(a.f.flag, 2);
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
  bool zero = true;
  int64_t r = 0, blk = -1;
  int phase = 0;
  bool live = false;
  auto enter_row = [&](int64_t row) {
    live = row < R && (rb.valid ? rb.live(row) : (a.f.mask == nullptr || a.f.mask[row] > 0.f));
    if (phase == 1) {
      zero = true;
      if (live) {
        const int64_t n = row / B;
        if (n != ready_seq) {
          // the producer posted this block after seeing the flag; each lane's
          // own acquire orders its loads below after the finalize's stores
          if (!ld_acquire(a.ready + n)) {
            if (lane == 0) atomicOr(a.f.flag, 2);  // not reached: reported, zeros written
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
int dpace_fused_max_seq_blocks() { return kFifo - 2; }

int dpace_fused_ctas(int dtype, int device, int cap) {
  return dtype == kDtypeBF16 ? FusedVariant<bf16_t>::ctas(device, cap) : FusedVariant<float>::ctas(device, cap);
}

cudaError_t dpace_fused_launch(int dtype, const DpaceFusedArgs& a, int ctas, cudaStream_t st) {
  return dtype == kDtypeBF16 ? FusedVariant<bf16_t>::launch(a, ctas, st) : FusedVariant<float>::launch(a, ctas, st);
}

}  // namespace specdec
