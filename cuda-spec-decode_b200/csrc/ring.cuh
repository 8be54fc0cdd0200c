// Warp-specialized CTA streaming ring for sm_100a (shared by the ring kernels).
//
// A persistent CTA has two roles:
//   - producer warp (lane 0): takes BLOCKS of BS * SE flattened elements from
//     a global atomic queue (or a static interleave) and keeps S shared-memory
//     stages in flight with cp.async.bulk; per stage it posts the stage's
//     flattened start in `sf0` and completes `full[slot]` (byte count);
//   - NC consumer warps: wait on `full[slot]`, each reduces / transforms its
//     own contiguous SE/NC sub-range of the stage from shared memory, then
//     arrives on `empty[slot]` so the producer can refill it.
// Forward kernels only stream: each consumer warp stores the partial of every
// (row, block) piece it saw with a plain store, at a slot fixed by (block
// index within the row, warp), so the result does not depend on which CTA
// took which block. A small finalize kernel, chained with programmatic
// dependent launch (PDL), merges the partials once the streaming grid is done.
// Dynamic blocks keep every SM busy to the end: equal bytes do not take equal
// time on a loaded memory system. Every wait is bounded (kWaitLimitNs).
#pragma once

#include <atomic>

#include "bulk_copy.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Global block queue: `ctr` hands out block indices; each CTA's producer stops
// after its first index >= nblocks. Every CTA then retires once; the last CTA
// to retire resets both words, leaving the counters zeroed for the next launch.
struct BlockQueue {
  unsigned* ctr;      // dynamic queue word (unused by the static interleave)
  unsigned* retired;  // CTAs retired; null: no counters at all (nothing to retire)
  unsigned nblocks;
  int dynamic;  // 0: block = blockIdx.x + k * gridDim.x (static interleave)

  // Every CTA's first block is its own index (no atomic on the way to the
  // first copy); the dynamic queue hands out the rest, from gridDim.x on.
  __device__ __forceinline__ unsigned first() const { return blockIdx.x; }
  __device__ __forceinline__ unsigned next(unsigned cur) const {
    return dynamic ? gridDim.x + atomicAdd(ctr, 1u) : cur + gridDim.x;
  }
  // Called once per CTA, after its last dequeue; true for the last CTA, which
  // has seen every earlier CTA's writes that preceded their retire.
  __device__ __forceinline__ bool retire() const {
    if (retired == nullptr) return false;
    __threadfence();
    if (atomicAdd(retired, 1u) + 1 == gridDim.x) {
      __threadfence();
      if (dynamic) *ctr = 0u;
      *retired = 0u;
      return true;
    }
    return false;
  }
};

// What a CTA may have left unfinished when one of its waits expired: the
// producer records the block of every stage it posts, the blocks it had
// dequeued but not yet fully posted and the stage count; each consumer warp
// records how many stages it finished. Read only after a timeout (the
// backward kernels then overwrite those blocks of the gradient with NaN).
template <int S>
struct RingTrack {
  unsigned sblk[S];   // block of the stage last posted in each slot
  unsigned held[2];   // dequeued, not fully posted (>= nblocks: none)
  int64_t posted;     // stages posted (or withheld), the end-of-work stage included
  int64_t done[8];    // per consumer warp: stages finished
  int timeout;        // a wait in this CTA expired
};

// Number of blocks of length BL that overlap row r (= slots of its partials).
__device__ __forceinline__ int blocks_in_row(int64_t r, int64_t V, int64_t BL) {
  return (int)(((r + 1) * V - 1) / BL - (r * V) / BL + 1);
}

// Programmatic dependent launch: a CTA that is done signals that the
// dependent (finalize) grid may start launching; the dependent waits for the
// whole primary grid to complete and flush before reading its results.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Row-liveness bitmask in shared memory (bit r = row r is read at all).
struct RowBits {
  const unsigned* words;
  bool valid;  // false: too many rows for the table, treat every row as live
  __device__ __forceinline__ bool live(int64_t r) const {
    return !valid || ((words[r >> 5] >> (r & 31)) & 1u);
  }
};

constexpr int kMaxRowWords = 1024;  // liveness bitmask capacity: 32768 rows

// Builds the liveness bitmask (all threads of the CTA, before the role split).
template <class LiveFn>
__device__ __forceinline__ RowBits build_row_bits(unsigned* words, int64_t R, int nwarps, LiveFn live) {
  RowBits rb;
  rb.words = words;
  rb.valid = R <= (int64_t)kMaxRowWords * 32;
  if (rb.valid) {
    // a warp takes kU consecutive words at a time and issues all their loads
    // before the first ballot: one memory round trip per kU words (the whole
    // table at the bench size) instead of one per word, ahead of the first copy
    constexpr int kU = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nwords = (R + 31) / 32;
    for (int64_t w0 = (int64_t)warp * kU; w0 < nwords; w0 += (int64_t)nwarps * kU) {
      bool lv[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t r = (w0 + u) * 32 + lane;
        lv[u] = r < R && live(r);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const unsigned bits = __ballot_sync(0xffffffffu, lv[u]);
        if (lane == 0 && w0 + u < nwords) words[w0 + u] = bits;
      }
    }
  }
  return rb;
}

// Elements of a stage that the bulk copy brought in: [f0, f0 + copied) with
// copied * sizeof(T) the stage's byte count rounded down to 16 bytes; the
// rest (at most 15 bytes, only at the very end of the data) is read from
// global memory.
template <class T>
__device__ __forceinline__ int64_t copied_end(int64_t f0, int64_t f1) {
  return f0 + ((((f1 - f0) * (int64_t)sizeof(T)) & ~int64_t(15)) / (int64_t)sizeof(T));
}

// 1: the forwards' producers post their first stage before the liveness table
// is built (ring_post_first); 0: after it, like the backwards.
#ifndef SPECDEC_EARLY_FIRST_STAGE
#define SPECDEC_EARLY_FIRST_STAGE 1
#endif

// The producer's first stage, posted before the CTA's liveness table exists
// (called by the producer lane right after it initialised the barriers): the
// first stage of block `first` is copied whatever its rows' liveness -- the
// consumers skip a dead row's stage by the table, so a dead copy costs only
// its bytes -- and the copy's latency overlaps the table's loads. Returns
// false (nothing posted; ring_produce starts from the beginning) when the
// block is past the end, is a single stage, or the test hook withholds it.
template <int NIN, int S, int SE, class T>
__device__ bool ring_post_first(const T* const* src, const BlockMap& bm, int64_t V, const BlockQueue& q, T* ring,
                                uint64_t* full, int64_t* sf0, int64_t* srow, unsigned first, bool withhold_first,
                                RingTrack<S>* trk) {
  if (withhold_first || first >= q.nblocks) return false;
  const int64_t blk_end = bm.end(first);
  const int64_t f0 = bm.start(first);
  const int64_t f1 = min(f0 + SE, blk_end);
  if (f1 == blk_end) return false;
  if (trk) trk->sblk[0] = first;
  sf0[0] = f0;
  srow[0] = f0 / V;
  const uint32_t vbytes = (uint32_t)(((f1 - f0) * (int64_t)sizeof(T)) & ~int64_t(15));
  if (vbytes) {
    mbar_arrive_expect_tx(full, vbytes * NIN);
#pragma unroll
    for (int i = 0; i < NIN; ++i) bulk_g2s(ring + (size_t)i * S * SE, src[i] + f0, vbytes, full);
  } else {
    mbar_arrive(full);
  }
  return true;
}

// Producer loop, lane 0 of the producer warp. NIN input streams of element
// type T share the flattened index space (ring k holds stream k's stages at
// ring + k*S*SE). A stage whose rows are all dead is posted without a copy.
// `first` is the CTA's first block (its own index; `first_posted`: its first
// stage was already posted by ring_post_first). The next block is
// dequeued only when the current block's last stage is posted, and taken up
// after the next slot wait: the atomic's latency hides behind that wait, and
// no CTA holds a whole unstarted block when the queue runs dry (which would
// leave the others idle at the end). Returns false on a wait timeout.
// `withhold_first` (failure-detection tests only) never posts the first
// stage: this CTA's consumers then see their bounded wait expire, which is
// the path under test. `trk` (or null) receives the progress record. The
// caller retires the CTA from the queue afterwards.
template <int NIN, int S, int SE, class T>
__device__ bool ring_produce(const T* const* src, const BlockMap& bm, int64_t V, const RowBits& rb,
                             const BlockQueue& q, T* ring, uint64_t* full, uint64_t* empty,
                             int64_t* sf0, int64_t* srow, unsigned first, bool withhold_first = false,
                             RingTrack<S>* trk = nullptr, bool first_posted = false) {
  unsigned b = first, nb = q.nblocks;
  bool have_nb = false, switch_pending = false;
  int64_t blk_start = 0, blk_end = 0, r_issue = 0;
  int k = first_posted ? 1 : 0;  // ring_post_first already posted stage 0 of block `first`
  auto enter_block = [&]() {
    if (b < q.nblocks) {
      blk_start = bm.start(b);
      blk_end = bm.end(b);
      r_issue = blk_start / V;
    }
  };
  enter_block();
  bool ok = true;
  int64_t it = first_posted ? 1 : 0;
  for (;; ++it) {
    const int slot = (int)(it % S);
    if (!mbar_wait(empty + slot, (uint32_t)(((it / S) & 1) ^ 1))) {
      ok = false;
      break;
    }
    if (switch_pending) {
      b = nb;
      have_nb = false;
      switch_pending = false;
      k = 0;
      enter_block();
    }
    if (trk) trk->sblk[slot] = b;
    if (withhold_first && it == 0) continue;  // neither copy nor arrive: full[0] stays incomplete
    if (b >= q.nblocks) {
      sf0[slot] = -1;
      mbar_arrive(full + slot);
      ++it;
      break;
    }
    const int64_t f0 = blk_start + (int64_t)k * SE;
    const int64_t f1 = min(f0 + SE, blk_end);
    if (f1 == blk_end) {  // the block's last stage: dequeue the next block now
      nb = q.next(b);
      have_nb = true;
    }
    sf0[slot] = f0;
    while ((r_issue + 1) * V <= f0) ++r_issue;
    srow[slot] = r_issue;
    bool live = !rb.valid;
    for (int64_t r = r_issue; !live && r * V < f1; ++r) live = rb.live(r);
    const uint32_t vbytes = (uint32_t)(((f1 - f0) * (int64_t)sizeof(T)) & ~int64_t(15));
    if (live && vbytes) {
      mbar_arrive_expect_tx(full + slot, vbytes * NIN);
#pragma unroll
      for (int i = 0; i < NIN; ++i)
        bulk_g2s(ring + (size_t)i * S * SE + (size_t)slot * SE, src[i] + f0, vbytes, full + slot);
    } else {
      mbar_arrive(full + slot);
    }
    if (f1 == blk_end) switch_pending = true;
    else ++k;
  }
  if (trk) {
    trk->held[0] = b;
    trk->held[1] = have_nb ? nb : q.nblocks;
    trk->posted = it;
  }
  return ok;
}

// After a timeout a consumer waits (bounded) for the next S stages so that no
// copy into this CTA's shared memory is left in flight when it exits.
template <int S>
__device__ __forceinline__ void ring_drain(uint64_t* full, int64_t it) {
  for (int64_t j = it; j < it + S; ++j) mbar_wait(full + (j % S), (uint32_t)((j / S) & 1));
}

// Shared-memory layout of a ring: NIN streams x S stages x SE elements, then
// the stage barriers, the posted stage starts and the liveness bitmask.
template <int NIN, int S, int SE, class T = float>
struct RingSmem {
  T ring[NIN * S * SE];  // first member: 128-byte aligned with the dynamic shared memory
  uint64_t full[S], empty[S];
  int64_t sf0[S];   // flattened start of the stage (-1: end of work)
  int64_t srow[S];  // row containing the stage's first element
  RingTrack<S> trk;
  unsigned bits[kMaxRowWords];
};

// Minimum CTAs per SM a ring kernel is compiled for (it caps the registers
// per thread): as many rings as fit in shared memory, at most 4 for CTAs of
// up to 160 threads and 2 for larger ones. Float kernels are compiled without
// a minimum unless 4 rings fit (their default allocation would otherwise
// leave room for 3).
template <int NC, int NIN, int S, int SE, class T>
constexpr int ring_min_ctas() {
  constexpr int by_smem = int((227 * 1024) / sizeof(RingSmem<NIN, S, SE, T>));
  // two-stage one-stream bf16 rings of up to 160 threads: 5 CTAs per SM (80
  // registers); the two-stream DFlash forward needs more registers and stays at 4
  constexpr int by_threads = (NC + 1) * 32 <= 160 ? (sizeof(T) == 2 && S <= 2 && NIN == 1 ? 5 : 4) : 2;
  constexpr int m = by_smem < by_threads ? (by_smem < 1 ? 1 : by_smem) : by_threads;
  return (sizeof(T) == 2 || m >= 4) ? m : 1;
}

template <int NIN, int S, int SE, class T>
__device__ __forceinline__ void ring_init(RingSmem<NIN, S, SE, T>& sm, int consumers, int init_thread = 0) {
  if ((int)threadIdx.x == init_thread) {
    for (int i = 0; i < S; ++i) {
      mbar_init(sm.full + i, 1);
      mbar_init(sm.empty + i, consumers);
    }
    sm.trk.timeout = 0;
    fence_mbar_init();
  }
}

// After a wait in this CTA expired (all threads, after a CTA-wide barrier):
// overwrites with NaN every block of dst that this CTA may have left
// unfinished -- the blocks of the stages some consumer warp had not finished
// (at most S stages: the producer never runs more than S ahead of the slowest
// consumer) and the blocks the producer had dequeued but not fully posted.
// With the static interleave (`stride` = the grid) this CTA also owns every
// later block of its sequence, held[1] + k * stride, which no other CTA will
// write: those are overwritten too. Blocks this CTA finished are left as
// written, so a gradient is never partly stale: every element is either
// correct or NaN.
template <class T, int S>
__device__ void ring_poison(T* dst, int64_t E, int64_t BL, unsigned nblocks, const RingTrack<S>& trk, int nc,
                            unsigned stride) {
  int64_t lo = trk.done[0];
  for (int w = 1; w < nc; ++w) lo = min(lo, trk.done[w]);
  unsigned ids[S + 2];
  int n = 0;
  for (int64_t st = max(lo, trk.posted - S); st < trk.posted; ++st) ids[n++] = trk.sblk[st % S];
  ids[n++] = trk.held[0];
  ids[n++] = trk.held[1];
  for (int i = 0; i < n; ++i) {
    const unsigned b = ids[i];
    bool seen = b >= nblocks;
    for (int j = 0; j < i; ++j) seen = seen || ids[j] == b;
    if (seen) continue;
    const int64_t f0 = (int64_t)b * BL, f1 = min(f0 + BL, E);
    for (int64_t x = f0 + threadIdx.x; x < f1; x += blockDim.x) store_elem(dst + x, __int_as_float(0x7fc00000));
  }
  if (stride != 0 && trk.held[1] < nblocks) {
    for (uint64_t b = (uint64_t)trk.held[1] + stride; b < nblocks; b += stride) {
      const int64_t f0 = (int64_t)b * BL, f1 = min(f0 + BL, E);
      for (int64_t x = f0 + threadIdx.x; x < f1; x += blockDim.x) store_elem(dst + x, __int_as_float(0x7fc00000));
    }
  }
}

// Accumulates smem elements [a, b) of a stage into the lane's (m, s).
__device__ __forceinline__ void warp_lse_smem(const float* sb, int a, int b, float& m, float& s) {
  const int lane = threadIdx.x & 31;
  const int a4 = (a + 3) & ~3, b4 = b & ~3;
  if (a4 >= b4) {
    for (int k = a + lane; k < b; k += 32) lse_push(m, s, sb[k]);
    return;
  }
  if (lane < a4 - a) lse_push(m, s, sb[a + lane]);
  if (lane < b - b4) lse_push(m, s, sb[b4 + lane]);
  const float4* q = reinterpret_cast<const float4*>(sb);
  int k = (a4 >> 2) + lane;
  const int kend = b4 >> 2;
  for (; k + 96 < kend; k += 128) {
    const float4 v0 = q[k], v1 = q[k + 32], v2 = q[k + 64], v3 = q[k + 96];
    const float cm = fmaxf(fmaxf(max4(v0), max4(v1)), fmaxf(max4(v2), max4(v3)));
    if (cm > m) {
      s *= exp_shift(m, cm);
      m = cm;
    }
    s += ((exp_shift(v0.x, m) + exp_shift(v0.y, m)) + (exp_shift(v0.z, m) + exp_shift(v0.w, m))) +
         ((exp_shift(v1.x, m) + exp_shift(v1.y, m)) + (exp_shift(v1.z, m) + exp_shift(v1.w, m))) +
         ((exp_shift(v2.x, m) + exp_shift(v2.y, m)) + (exp_shift(v2.z, m) + exp_shift(v2.w, m))) +
         ((exp_shift(v3.x, m) + exp_shift(v3.y, m)) + (exp_shift(v3.z, m) + exp_shift(v3.w, m)));
  }
  for (; k < kend; k += 32) {
    const float4 v = q[k];
    const float cm = max4(v);
    if (cm > m) {
      s *= exp_shift(m, cm);
      m = cm;
    }
    s += (exp_shift(v.x, m) + exp_shift(v.y, m)) + (exp_shift(v.z, m) + exp_shift(v.w, m));
  }
}

// Accumulates a full sub-range of KSUB floats (KSUB / 128 float4 per lane):
// all loads first, one max, then (the stage released to the producer when
// `empty` is given) one rescale and the exponentials from registers.
template <int KSUB>
__device__ __forceinline__ void warp_lse_full(const float* sb, float& m, float& s, uint64_t* empty = nullptr) {
  constexpr int U = KSUB / 128;
  static_assert(KSUB % 128 == 0, "sub-range must be a multiple of 128 floats");
  const int lane = threadIdx.x & 31;
  const float4* q = reinterpret_cast<const float4*>(sb) + lane;
  float4 v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) v[u] = q[32 * u];
  float cm = max4(v[0]);
#pragma unroll
  for (int u = 1; u < U; ++u) cm = fmaxf(cm, max4(v[u]));
  if (empty) release_stage(empty, cm);
  cm = warp_max(cm);  // one running maximum for the whole warp: the piece's close needs no rescale
  if (cm > m) {
    s *= exp_shift(m, cm);
    m = cm;
  }
  float acc[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    acc[u] = (exp_shift(v[u].x, m) + exp_shift(v[u].y, m)) + (exp_shift(v[u].z, m) + exp_shift(v[u].w, m));
#pragma unroll
  for (int w = 1; w < U; w <<= 1)
#pragma unroll
    for (int u = 0; u + w < U; u += 2 * w) acc[u] += acc[u + w];
  s += acc[0];
}

// bf16 stage, elements [a, b) (a stage cut by a row edge): scalar head and
// tail to 16-byte boundaries, then 16-byte vectors, four per lane per round.
__device__ __forceinline__ void warp_lse_smem(const bf16_t* sb, int a, int b, float& m, float& s) {
  const int lane = threadIdx.x & 31;
  const int a8 = (a + 7) & ~7, b8 = b & ~7;
  if (a8 >= b8) {
    for (int k = a + lane; k < b; k += 32) lse_push(m, s, to_f32(sb[k]));
    return;
  }
  if (lane < a8 - a) lse_push(m, s, to_f32(sb[a + lane]));
  if (lane < b - b8) lse_push(m, s, to_f32(sb[b8 + lane]));
  const uint4* q = reinterpret_cast<const uint4*>(sb);
  int k = (a8 >> 3) + lane;
  const int kend = b8 >> 3;
  for (; k + 96 < kend; k += 128) {
    const uint4 v0 = q[k], v1 = q[k + 32], v2 = q[k + 64], v3 = q[k + 96];
    const uint32_t mx = bmax2(bmax2(bmax8(v0), bmax8(v1)), bmax2(bmax8(v2), bmax8(v3)));
    const float cm = fmaxf(bf16_lo(mx), bf16_hi(mx));
    if (cm > m) {
      s *= exp_shift(m, cm);
      m = cm;
    }
    const float2 acc = fadd2(fadd2(vec8_expsum2(v0, m), vec8_expsum2(v1, m)),
                             fadd2(vec8_expsum2(v2, m), vec8_expsum2(v3, m)));
    s += acc.x + acc.y;
  }
  for (; k < kend; k += 32) {
    const uint4 v = q[k];
    const uint32_t mx = bmax8(v);
    const float cm = fmaxf(bf16_lo(mx), bf16_hi(mx));
    if (cm > m) {
      s *= exp_shift(m, cm);
      m = cm;
    }
    const float2 acc = vec8_expsum2(v, m);
    s += acc.x + acc.y;
  }
}

// bf16 full sub-range of KSUB elements (KSUB / 256 16-byte vectors per lane):
// the max is taken on the packed words, each element is widened once, and the
// arithmetic runs on fp32 pairs.
template <int KSUB>
__device__ __forceinline__ void warp_lse_full(const bf16_t* sb, float& m, float& s, uint64_t* empty = nullptr) {
  constexpr int U = KSUB / 256;
  static_assert(KSUB % 256 == 0, "sub-range must be a multiple of 256 bf16");
  const int lane = threadIdx.x & 31;
  const uint4* q = reinterpret_cast<const uint4*>(sb) + lane;
  uint4 v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) v[u] = q[32 * u];
  uint32_t mx = bmax8(v[0]);
#pragma unroll
  for (int u = 1; u < U; ++u) mx = bmax2(mx, bmax8(v[u]));
  float cm = fmaxf(bf16_lo(mx), bf16_hi(mx));
  if (empty) release_stage(empty, cm);
  cm = warp_max(cm);  // one running maximum for the whole warp: the piece's close needs no rescale
  if (cm > m) {
    s *= exp_shift(m, cm);
    m = cm;
  }
  float2 acc[U];
#pragma unroll
  for (int u = 0; u < U; ++u) acc[u] = vec8_expsum2(v[u], m);
#pragma unroll
  for (int w = 1; w < U; w <<= 1)
#pragma unroll
    for (int u = 0; u + w < U; u += 2 * w) acc[u] = fadd2(acc[u], acc[u + w]);
  s += acc[0].x + acc[0].y;
}

// End of a backward CTA (warp 0, after the CTA's poison writes, if any):
// folds this CTA's timeout into the launch's flag word and retires it; the
// last CTA to retire turns the flag into the status word (SPECDEC_ERR_CUDA =
// a wait expired somewhere; otherwise 0 unless `status_merge`, which only
// ever raises the word) and clears the flag. Without counters (no retire
// count) a timed-out CTA writes the status itself, over the 0 the entry point
// stored. With a loss epilogue (a forward_backward call whose finalize left
// the sum to this kernel) the last CTA also sums the per-sequence losses in
// index order -- the finalize's own arithmetic, so the same bits -- and
// writes the loss and the whole status word of the call.
template <class Args>
__device__ __forceinline__ void bwd_finish(const BlockQueue& q, const Args& a, bool timeout) {
  const int lane = threadIdx.x & 31;
  int last = 0;
  if (lane == 0) {
    if (timeout && a.flag) atomicOr(a.flag, 2);
    last = q.retire() ? 1 : 0;
  }
  last = __shfl_sync(kFullMask, last, 0);
  if (last) {
    float total = 0.f;
    if (a.loss) total = warp_sum_l2(a.seq_loss, a.nseq);
    if (lane == 0) {
      const int fb = a.flag ? atomicExch(a.flag, 0) : 0;
      if (a.loss) {
        const int f = atomicExch(a.fwd_flag, 0);
        a.loss[0] = (f & 2) ? __int_as_float(0x7fc00000) : total / (float)a.n_global;
        if (a.status)
          a.status[0] = ((f | fb) & 2) ? kStatusTimeout : ((f & 1) ? kStatusTargetRange : 0);
      } else if (a.status) {
        if (fb & 2) a.status[0] = kStatusTimeout;
        else if (!a.status_merge) a.status[0] = 0;
      }
    }
  } else if (lane == 0 && q.retired == nullptr && timeout && a.status) {
    a.status[0] = kStatusTimeout;
  }
}

// Launches a kernel chained to the previous kernel on the stream with
// programmatic dependent launch: it may become resident while that kernel
// drains, and waits for it inside with griddepcontrol.wait. Used only where
// the previous kernel is known: the finalize right after its own streaming
// kernel, enqueued by the same call. A chained grid that became resident
// early and waited on work ordered behind another stream (an event wait on a
// collective, say) could hold every SM that work needs, so kernels whose
// predecessor is the caller's are launched plainly.
template <class Kernel, class Args>
inline cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              const Args& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args);
}

// Raises `Kernel`'s dynamic shared-memory limit to `smem` once per device
// (the attribute is per device and per function); later launches, including
// ones under stream capture, skip the call.
template <auto Kernel>
inline cudaError_t ensure_smem_limit(size_t smem) {
  static std::atomic<unsigned long long> done{0};  // bit d: set on device d
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <class K>
inline int ring_occupancy_ctas(K kernel, int threads, size_t smem, int device, int cap) {
  int sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) return 0;
  if (cap > 0 && per_sm > cap) per_sm = cap;
  if (per_sm < 1) return 0;
  return sms * per_sm;
}

}  // namespace specdec
