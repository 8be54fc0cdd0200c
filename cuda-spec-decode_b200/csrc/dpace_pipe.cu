// D-PACE forward and backward in one cooperative launch that keeps every
// sequence's logits in shared memory between the two passes: HBM traffic is
// one read of the live logits and one write of the gradient (the separate
// forward and backward kernels read the live logits twice).
//
// Layout. One CTA per SM, all resident (cooperative launch): G CTAs. CTA c
// owns slice c of every sequence -- elements [c*SL, min((c+1)*SL, B*V)) of
// the sequence's B*V logits, SL = ceil(B*V / G) rounded up to 32 elements --
// and holds the slices of K consecutive sequences in a ring of K
// shared-memory slots (K = 4 for fp32 and 8 for bf16 at [N, 16, 128256]).
//
// Warp roles, all coordinated through shared-memory mbarriers per slot:
//   consumers (8 warps), iteration i = 0 .. N-1+L (L < K):
//     B(i-L): with the slot's row parameters posted, write
//             scale * (softmax - onehot) for the slice straight from shared
//             memory (streaming stores); release the slot.
//     F(i):   once the slice of sequence i has landed (bulk copy), each warp
//             leaves the (max, sum e^(x - max)) of its part of every row in
//             shared memory, and x[target] in global memory when the target
//             lies in its part.
//   producer lane: copies the live rows of sequence i's slice into slot
//     i % K once B(i-K) released it -- K-1-L iterations before F(i) needs
//     it, so that many slices per SM are in flight -- with the rows' live
//     flags and target offsets (read a sequence ahead).
//   publisher warp: merges the warps' row partials of F(i) in warp order into
//     the CTA's partials, stores them and counts the CTA done with sequence i
//     (release).
//   finalize warps (2, alternating sequences): once all G CTAs counted
//     sequence q (acquire) and the slot's previous B is done, merge each
//     row's partials in CTA order and compute lse, ce, the B-scan and scale
//     as dpace_finalize_kernel does -- every CTA computes the same bits, so
//     no finalized result has to travel back -- and post lse and scale of
//     the slice's rows for B(q). CTA q % G also writes q's outputs.
// Consumer warps touch no global memory on their critical path. B(q) runs
// L iterations after F(q): the finalize chain (the last CTA's F, its count,
// the partial loads, the finalize) has about L x (time of one sequence) to
// finish before a CTA would wait for it. Every wait is bounded (1 s); an expired one sets the
// flag and the call reports status 5 with a NaN loss. Warps keep following
// the shared-memory barrier phases after an expiry (so no barrier runs two
// phases ahead of a waiter) but compute nothing more, and a warp whose wait
// on another CTA expired waits on other CTAs no more. The merge tree (warps
// of a CTA, then CTAs in order) differs from the separate kernels', so
// results agree with them to float rounding, not bit for bit.
//
// Reference behaviour: losses/dpace.py:15-145; numbers follow
// losses/dpace_ref.py:8-51.
#include <cfloat>

#include "ring.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

constexpr int kPipeNC = 8;  // consumer warps

template <int NC>
struct PipeCtl {
  uint64_t full[kPipeMaxSlots];    // producer -> consumers: the slice landed
  uint64_t empty[kPipeMaxSlots];   // consumers -> producer, finalize warps: B done with the slot
  uint64_t fdone[kPipeMaxSlots];   // consumers -> publisher: F partials in wpart
  uint64_t pready[kPipeMaxSlots];  // finalize warps -> consumers: bparam posted
  float2 wpart[kPipeMaxSlots][NC][kPipeMaxRows];  // per-warp row partials of F
  int2 fmeta[kPipeMaxSlots][kPipeMaxRows];        // row live flag, target offset in the slot (-1: none)
  float2 bparam[kPipeMaxSlots][kPipeMaxRows];     // row lse, scale for B
  int last;                                       // exit: this CTA is the grid's last
};

// Bounded wait for *p == want (lane-uniform); every lane then loads the word
// with acquire semantics, ordering its own later loads.
__device__ __forceinline__ bool wait_word(const unsigned* p, unsigned want) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) {
    if (ld_acquire(p) != want) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire(p) != want) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  ok = __shfl_sync(kFullMask, ok, 0);
  if (ok) (void)ld_acquire(p);
  return ok;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded mbarrier wait by the whole warp.
__device__ __forceinline__ bool warp_mbar_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(kFullMask, mbar_wait(bar, parity));
}

// Gradient of slice elements [a, b) (offsets from the slot base): dst[x] =
// sc * (e^(x - l) - [x == tq]), or zeros. dst points at the slot's first
// element in the output.
template <class T>
__device__ __forceinline__ void pipe_grad(const T* sb, int a, int b, T* dst, bool zero, float sc, float l,
                                          int tq) {
  constexpr int kVec = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int av = (a + kVec - 1) & ~(kVec - 1), bv = b & ~(kVec - 1);
  auto scalar = [&](int x) {
    store_elem(dst + x, zero ? 0.f : sc * (exp_shift(to_f32(sb[x]), l) - (x == tq ? 1.f : 0.f)));
  };
  if (av >= bv) {
    for (int x = a + lane; x < b; x += 32) scalar(x);
    return;
  }
  if (lane < av - a) scalar(a + lane);
  if (lane < b - bv) scalar(bv + lane);
  const int nv = (bv - av) / kVec;
  uint4* d4 = reinterpret_cast<uint4*>(dst + av);
  if (zero) {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int k = lane; k < nv; k += 32) st_stream_u4(d4 + k, z);
    return;
  }
  const int tqv = tq - av;
  if constexpr (sizeof(T) == 4) {
    const float4* s4 = reinterpret_cast<const float4*>(sb + av);
    for (int k = lane; k < nv; k += 32) {
      const float4 v = s4[k];
      float4 y;
      y.x = exp_shift(v.x, l);
      y.y = exp_shift(v.y, l);
      y.z = exp_shift(v.z, l);
      y.w = exp_shift(v.w, l);
      const unsigned d = (unsigned)(tqv - 4 * k);
      if (d < 4u) {
        if (d == 0) y.x -= 1.f;
        else if (d == 1) y.y -= 1.f;
        else if (d == 2) y.z -= 1.f;
        else y.w -= 1.f;
      }
      y.x *= sc;
      y.y *= sc;
      y.z *= sc;
      y.w *= sc;
      st_stream(reinterpret_cast<float4*>(d4) + k, y);
    }
  } else {
    const uint4* s4 = reinterpret_cast<const uint4*>(sb + av);
    const float2 sc2 = make_float2(sc, sc);
    for (int k = lane; k < nv; k += 32) {
      const uint4 v = s4[k];
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
      float2 e[4], y[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        e[h] = exp_shift2(bf16x2_f32(wv[h]), l);
        y[h] = fmul2(e[h], sc2);
      }
      const unsigned d = (unsigned)(tqv - 8 * k);
      if (d < 8u) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (d == (unsigned)(2 * h)) y[h].x = sc * (e[h].x - 1.f);
          if (d == (unsigned)(2 * h + 1)) y[h].y = sc * (e[h].y - 1.f);
        }
      }
      st_stream_u4(d4 + k, make_uint4(pack_bf16x2(y[0].x, y[0].y), pack_bf16x2(y[1].x, y[1].y),
                                      pack_bf16x2(y[2].x, y[2].y), pack_bf16x2(y[3].x, y[3].y)));
    }
  }
}

// Finalize sequence n (one warp, lane j <-> row j): merge row j's CTA
// partials in CTA order, then the arithmetic of dpace_finalize_kernel. Every
// load (mask, target, x[target], the first kFinP partials) is issued before
// any of them is used: one round trip.
constexpr int kFinP = 16;
template <class T>
__device__ void pipe_finalize(const DpacePipeArgs& a, int64_t n, bool expired, bool outputs, float& lse_out,
                              float& scale_out) {
  const int lane = threadIdx.x & 31;
  const int B = a.f.B;
  const int64_t V = a.f.V, SL = a.SL;
  const int G = gridDim.x;
  const int j = lane;
  const bool in = j < B;
  const int64_t rj = n * B + (in ? j : 0);
  const int cf = (int)(((int64_t)j * V) / SL);
  const int cl = (int)min((int64_t)G - 1, (((int64_t)j + 1) * V - 1) / SL);
  const int k = in ? cl - cf + 1 : 0;
  const float2* part = a.f.part + rj * a.PM;
  const float mkj = in ? (a.f.mask ? a.f.mask[rj] : 1.f) : 0.f;
  const int64_t tj = in ? a.f.targets[rj] : 0;
  const float xt = in ? __ldcg(a.f.xtgt + rj) : 0.f;
  float2 v[kFinP];
#pragma unroll
  for (int u = 0; u < kFinP; ++u) v[u] = u < k ? __ldcg(part + u) : make_float2(kNegSeed, 0.f);
  const bool tvalid = tj >= 0 && tj < V;
  const bool live = in && mkj > 0.f;
  float lse = 0.f, ce = 0.f;
  if (live) {
    float m = v[0].x, s = v[0].y;
#pragma unroll
    for (int u = 1; u < kFinP; ++u)
      if (u < k) lse_merge(m, s, v[u].x, v[u].y);
    for (int u = kFinP; u < k; ++u) {
      const float2 w = __ldcg(part + u);
      lse_merge(m, s, w.x, w.y);
    }
    lse = __fadd_rn(m, logf(s));
    if (tvalid) ce = lse - xt;
  }
  if (expired) lse = ce = 0.f;
  if (outputs && in && !tvalid) atomicOr(a.f.flag, 1);
  if (outputs && in) a.f.lse[rj] = lse;
  const float mk = live ? 1.f : 0.f;
  const float sm = live ? __fadd_rn(__fmul_rn(a.f.one_minus_alpha, expf(-ce)), a.f.alpha) : 1.f;
  // prefix product and suffix sum in double, in sequence order (torch CPU
  // cumprod / cumsum accumulate in double); the factors are gathered first
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
  float Sx = 0.f;
#pragma unroll
  for (int i = 31; i >= 0; --i) {
    if (i < B) acc += (double)f[i];
    if (i == j) Sx = (float)acc;
  }
  float w = a.f.loss_type == 1 ? P : (a.f.loss_type == 2 ? __fdiv_rn(Sx, fmaxf(P, FLT_MIN)) : Sx);
  w = __fmul_rn(w, mk);
  const float contrib = live ? __fmul_rn(ce, w) : 0.f;
  const float scale = expired ? 0.f : __fmul_rn(w, a.f.inv_n);
  lse_out = lse;
  scale_out = scale;
  if (!outputs) return;
  if (in) a.f.scale[rj] = scale;
  const float loss_n = warp_sum(contrib);
  if (lane == 0) {
    if (a.f.loss_n) a.f.loss_n[n] = loss_n;
    a.f.seq_loss[n] = loss_n;
  }
  __syncwarp();
  unsigned last = 0;
  if (lane == 0) {
    __threadfence();  // seq_loss before the count
    last = atomicAdd(a.f.done_cnt, 1u) + 1 == (unsigned)a.f.N;
  }
  last = __shfl_sync(kFullMask, last, 0);
  if (last) {
    __threadfence();
    const float total = warp_sum_l2(a.f.seq_loss, a.f.N);
    if (lane == 0) a.f.loss[0] = total / (float)a.f.n_global;
  }
}

template <class T, int NC>
__global__ void __launch_bounds__((NC + 4) * 32, 1) dpace_pipe_kernel(const __grid_constant__ DpacePipeArgs a) {
  constexpr int kVec = 16 / sizeof(T);
  __shared__ PipeCtl<NC> ctl;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* slots = reinterpret_cast<T*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K, L = a.L;  // slots; the backward runs L (< K) sequences behind
  const int64_t N = a.f.N, V = a.f.V, SL = a.SL;
  const int B = a.f.B;
  const int64_t seq_len = (int64_t)B * V;
  const int G = gridDim.x, c = blockIdx.x;
  const int64_t lo = min((int64_t)c * SL, seq_len), hi = min(lo + SL, seq_len);  // the slice, in a sequence
  const int j0 = (int)(lo / V);
  const int nrows = hi > lo ? (int)((hi - 1) / V) - j0 + 1 : 0;  // <= kPipeMaxRows (host)
  const T* X = static_cast<const T*>(a.f.logits);
  T* D = static_cast<T*>(a.dlogits);

  if (threadIdx.x == 0) {
    for (int k = 0; k < K; ++k) {
      mbar_init(ctl.full + k, 1);
      mbar_init(ctl.empty + k, NC);
      mbar_init(ctl.fdone + k, NC);
      mbar_init(ctl.pready + k, 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp < NC) {
    // ---- consumers ------------------------------------------------------
    const int64_t sub = ((SL + NC - 1) / NC + 32 * kVec - 1) / (32 * kVec) * (32 * kVec);
    const int64_t w0 = min(lo + warp * sub, hi), w1 = min(w0 + sub, hi);  // this warp's part of the slice
    bool dead = false;  // a wait expired: keep following the barriers, compute nothing
    for (int64_t i = 0; i < N + L; ++i) {
      const int64_t q = i - L;
      if (q >= 0) {
        // B(q)
        const int slot = (int)(q % K);
        if (!warp_mbar_wait(ctl.pready + slot, (uint32_t)((q / K) & 1)) && !dead) {
          dead = true;
          if (lane == 0) atomicOr(a.f.flag, 2);
        }
        const T* sb = slots + (size_t)slot * SL;
        T* dq = D + q * seq_len + lo;
        for (int64_t j = w0 / V; w0 < w1 && j * V < w1; ++j) {
          const int jj = (int)(j - j0);
          const int64_t ra = max(w0, j * V), rb = min(w1, (j + 1) * V);
          const int2 meta = ctl.fmeta[slot][jj];
          const float2 prm = ctl.bparam[slot][jj];
          pipe_grad<T>(sb, (int)(ra - lo), (int)(rb - lo), dq, !meta.x || dead || prm.y == 0.f, prm.y, prm.x,
                       meta.y);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(ctl.empty + slot);
      }
      if (i < N) {
        // F(i)
        const int slot = (int)(i % K);
        if (!warp_mbar_wait(ctl.full + slot, (uint32_t)((i / K) & 1)) && !dead) {
          dead = true;
          if (lane == 0) atomicOr(a.f.flag, 2);
        }
        const T* sb = slots + (size_t)slot * SL;
        for (int jj = 0; jj < nrows; ++jj) {
          const int64_t j = j0 + jj;
          const int64_t ra = max(w0, j * V), rb = min(w1, (j + 1) * V);
          const int2 meta = ctl.fmeta[slot][jj];
          float m = kNegSeed, s = 0.f;
          if (ra < rb && meta.x && !dead) {
            warp_lse_smem(sb, (int)(ra - lo), (int)(rb - lo), m, s);
            if (lane == 0 && meta.y >= ra - lo && meta.y < rb - lo) a.f.xtgt[i * B + j] = to_f32(sb[meta.y]);
          }
          warp_lse(m, s);
          if (lane == 0) ctl.wpart[slot][warp][jj] = make_float2(m, s);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(ctl.fdone + slot);
      }
    }
  } else if (warp == NC) {
    // ---- producer -------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      // live flags and targets of the slice's rows, read a sequence ahead
      bool lv[kPipeMaxRows];
      int64_t tg[kPipeMaxRows];
      auto read_meta = [&](int64_t n) {
        for (int jj = 0; jj < kPipeMaxRows; ++jj) {
          const int64_t r = n * B + j0 + jj;
          lv[jj] = jj < nrows && (a.f.mask == nullptr || a.f.mask[r] > 0.f);
          tg[jj] = jj < nrows ? a.f.targets[r] : -1;
        }
      };
      if (N > 0) read_meta(0);
      for (int64_t i = 0; i < N; ++i) {
        const int slot = (int)(i % K);
        if (i >= K) {
          // the slot's previous sequence: released by B, and its own copy landed
          const uint32_t par = (uint32_t)(((i / K) - 1) & 1);
          ok = mbar_wait(ctl.empty + slot, par) && ok;
          ok = mbar_wait(ctl.full + slot, par) && ok;
        }
        if (i == 0 && a.withhold_stage && c == 0) {
          // failure-detection tests: the first copy comes after the consumers' wait expired
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < kWaitLimitNs + kWaitLimitNs / 8) __nanosleep(100000);
        }
        T* sb = slots + (size_t)slot * SL;
        const int64_t base = i * seq_len;
        int64_t runs[kPipeMaxRows][2];
        int nr = 0;
        int64_t run0 = -1;
        uint32_t bytes = 0;
        for (int jj = 0; jj < nrows; ++jj) {
          const int64_t j = j0 + jj;
          const int64_t r0 = max(lo, j * V), r1 = min(hi, (j + 1) * V);
          const int64_t t = tg[jj];
          ctl.fmeta[slot][jj] = make_int2(lv[jj] ? 1 : 0, lv[jj] && t >= 0 && t < V && j * V + t >= lo && j * V + t < hi
                                                              ? (int)(j * V + t - lo) : -1);
          if (lv[jj] && run0 < 0) run0 = r0;
          if (!lv[jj] && run0 >= 0) {
            runs[nr][0] = run0;
            runs[nr][1] = r0;
            ++nr;
            run0 = -1;
          }
          if (jj == nrows - 1 && run0 >= 0) {
            runs[nr][0] = run0;
            runs[nr][1] = r1;
            ++nr;
          }
        }
        for (int k = 0; k < nr; ++k) bytes += (uint32_t)((runs[k][1] - runs[k][0]) * (int64_t)sizeof(T));
        if (bytes) {
          mbar_arrive_expect_tx(ctl.full + slot, bytes);
          for (int k = 0; k < nr; ++k)
            bulk_g2s(sb + (runs[k][0] - lo), X + base + runs[k][0],
                     (uint32_t)((runs[k][1] - runs[k][0]) * (int64_t)sizeof(T)), ctl.full + slot);
        } else {
          mbar_arrive(ctl.full + slot);
        }
        if (i + 1 < N) read_meta(i + 1);
      }
      // no copy may be in flight when the CTA exits
      for (int64_t i = N - K < 0 ? 0 : N - K; i < N; ++i)
        ok = mbar_wait(ctl.full + (int)(i % K), (uint32_t)((i / K) & 1)) && ok;
      if (!ok) atomicOr(a.f.flag, 2);
    }
    __syncwarp();
  } else if (warp == NC + 1) {
    // ---- publisher ------------------------------------------------------
    // Takes F(i) and every later F already done (at most K), stores their
    // partials, and covers them with one fence before the counts.
    for (int64_t i = 0; i < N;) {
      if (!warp_mbar_wait(ctl.fdone + (int)(i % K), (uint32_t)((i / K) & 1)) && lane == 0) atomicOr(a.f.flag, 2);
      int64_t e = i + 1;
      while (e < N && e < i + K && __all_sync(kFullMask, mbar_test(ctl.fdone + (int)(e % K), (uint32_t)((e / K) & 1))))
        ++e;
      for (int64_t s = i; s < e; ++s) {
        const int slot = (int)(s % K);
        if (lane < nrows) {
          const int64_t j = j0 + lane;
          float m = ctl.wpart[slot][0][lane].x, sm = ctl.wpart[slot][0][lane].y;
#pragma unroll
          for (int w = 1; w < NC; ++w) lse_merge(m, sm, ctl.wpart[slot][w][lane].x, ctl.wpart[slot][w][lane].y);
          if (ctl.fmeta[slot][lane].x) a.f.part[(s * B + j) * a.PM + (c - (j * V) / SL)] = make_float2(m, sm);
        }
      }
      __syncwarp();
      if (lane == 0)  // release: the CTA's partials and x[target] before the counts
        for (int64_t s = i; s < e; ++s) red_release_add(a.seq_done + s, 1u);
      i = e;
    }
  } else {
    // ---- finalize warps -------------------------------------------------
    // Warp NC+2+w takes the sequences q = w, w+2, ...: once every CTA has
    // counted q, it merges all of q's row partials and runs the finalize
    // (every CTA computes the same bits), posts lse and scale of the slice's
    // rows for B(q), and in CTA q % G also writes q's outputs.
    const int w = warp - (NC + 2);
    bool gave_up = false;  // a wait on another CTA expired: post zeros from now on
    for (int64_t q = w; q < N; q += 2) {
      const int slot = (int)(q % K);
      if (q >= K && !warp_mbar_wait(ctl.empty + slot, (uint32_t)(((q / K) - 1) & 1)) && lane == 0)
        atomicOr(a.f.flag, 2);
      if (!gave_up && !wait_word(a.seq_done + q, (unsigned)G)) {
        gave_up = true;
        if (lane == 0) atomicOr(a.f.flag, 2);
      }
      float lse = 0.f, scale = 0.f;
      pipe_finalize<T>(a, q, gave_up, q % G == c, lse, scale);
      const float lse_r = __shfl_sync(kFullMask, lse, (j0 + lane) & 31);
      const float scale_r = __shfl_sync(kFullMask, scale, (j0 + lane) & 31);
      if (lane < nrows) ctl.bparam[slot][lane] = make_float2(lse_r, ctl.fmeta[slot][lane].x ? scale_r : 0.f);
      __syncwarp();
      if (lane == 0) mbar_arrive(ctl.pready + slot);
    }
  }

  // ---- exit: the grid's last CTA reports and resets the counters ----------
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    ctl.last = atomicAdd(a.exit_cnt, 1u) + 1 == (unsigned)G;
  }
  __syncthreads();
  if (ctl.last) {
    __threadfence();
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) a.seq_done[n] = 0u;
    if (threadIdx.x == 0) {
      const int fl = atomicExch(a.f.flag, 0);
      if (fl & 2) a.f.loss[0] = __int_as_float(0x7fc00000);  // a wait expired: no result
      if (a.f.status) a.f.status[0] = (fl & 2) ? kStatusTimeout : ((fl & 1) ? kStatusTargetRange : kStatusOk);
      *a.f.done_cnt = 0u;
      *a.exit_cnt = 0u;
    }
  }
}

template <class T>
cudaError_t pipe_launch_t(const DpacePipeArgs& a, int G, size_t smem, cudaStream_t st) {
  auto kern = dpace_pipe_kernel<T, kPipeNC>;
  cudaError_t e = ensure_smem_limit<dpace_pipe_kernel<T, kPipeNC>>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3((kPipeNC + 4) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <class T>
int pipe_resident_t(size_t smem) {
  int blocks = 0;
  if (ensure_smem_limit<dpace_pipe_kernel<T, kPipeNC>>(smem) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, dpace_pipe_kernel<T, kPipeNC>, (kPipeNC + 4) * 32,
                                                    smem) != cudaSuccess)
    return 0;
  return blocks;
}

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

PipePlan dpace_pipe_plan(int dtype, int64_t B, int64_t V, int device) {
  PipePlan p;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) return p;
  const int64_t esz = dtype == kDtypeBF16 ? 2 : 4;
  const int64_t seq_len = B * V;
  if (B < 1 || B > 32 || V < 1 || (V * esz) % 16 != 0) return p;
  const int64_t SL = ((seq_len + sms - 1) / sms + 31) / 32 * 32;
  if (SL > 3 * V) return p;  // a slice overlaps at most kPipeMaxRows rows
  const int64_t budget = kPipeSmemBudget;
  int64_t K = budget / (SL * esz);
  if (K > kPipeMaxSlots) K = kPipeMaxSlots;
  if (K < 3) return p;
  p.G = sms;
  p.SL = SL;
  p.K = (int)K;
  p.L = (int)(K / 2 > 2 ? K / 2 : 2);  // the rest of the slots prefetch
  p.PM = (int)((V - 1) / SL + 2);
  p.smem = (size_t)(K * SL * esz);
  p.ok = true;
  return p;
}

int dpace_pipe_resident(int dtype, size_t smem) {
  return dtype == kDtypeBF16 ? pipe_resident_t<bf16_t>(smem) : pipe_resident_t<float>(smem);
}

cudaError_t dpace_pipe_launch(int dtype, const DpacePipeArgs& a, int G, size_t smem, cudaStream_t st) {
  return dtype == kDtypeBF16 ? pipe_launch_t<bf16_t>(a, G, smem, st) : pipe_launch_t<float>(a, G, smem, st);
}

}  // namespace specdec
