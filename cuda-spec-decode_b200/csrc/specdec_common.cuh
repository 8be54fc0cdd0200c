// Device helpers shared by the drafter-loss kernels (sm_100a).
//
// Every kernel in this library streams rows of fp32 logits [rows, V] from HBM.
// The work is split the same way everywhere: the flattened element range
// [0, rows*V) is cut into `grid` equal contiguous chunks, one per CTA, and the
// grid is exactly (SM count x resident CTAs per SM), so one wave covers the
// whole problem with no tail. A chunk may start or end inside a row; the part
// of a row that one CTA sees is a "piece". Per-row reductions are produced per
// piece and combined later in a fixed order, so results are bitwise
// repeatable (no float atomics anywhere).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace specdec {

constexpr float kLog2e = 1.44269504088896340736f;
constexpr float kLn2 = 0.69314718055994530942f;
// Running-max seed. Finite on purpose: exp2(x - seed) of a -inf logit is 0, not NaN.
constexpr float kNegSeed = -1e30f;
constexpr unsigned kFullMask = 0xffffffffu;

// 2^x with the hardware MUFU.EX2 unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Read-only 128-bit load that does not allocate in L1 (the data is touched once
// per pass); L2 keeps normal priority so a following pass may still hit.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p));
  return v;
}

// L2 cache-policy descriptor that marks lines evict-first.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Last-use 128-bit load under an L2 policy (the backward pass never re-reads).
__device__ __forceinline__ float4 ld_last(const float4* p, uint64_t pol) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

// Streaming 128-bit store (cache-streaming, evict-first).
__device__ __forceinline__ void st_stream(float4* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float max4(const float4& v) {
  return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
}

// ---------------------------------------------------------------------------
// bfloat16 elements travel as their 16-bit patterns (bf16_t). Widening to
// float is exact (the pattern is the upper half of the float's); narrowing
// rounds to nearest even in hardware (cvt.rn.bf16[x2].f32). All arithmetic
// is float.
// ---------------------------------------------------------------------------
using bf16_t = uint16_t;

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(bf16_t x) { return __uint_as_float(uint32_t(x) << 16); }
// The two elements of a bf16x2 word: the lower address is the low half.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float ldg_f32(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ldg_f32(const bf16_t* p) { return to_f32(__ldg(p)); }

// Elementwise max of two bf16x2 words (NaN loses against a number, like fmaxf).
__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bmax8(const uint4& v) { return bmax2(bmax2(v.x, v.y), bmax2(v.z, v.w)); }

// Packs round-to-nearest-even bf16(lo) | bf16(hi) << 16.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void store_elem(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_elem(bf16_t* p, float v) {
  unsigned short h;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(v));
  *p = h;
}

// Streaming 128-bit store of raw words (cache-streaming, evict-first).
__device__ __forceinline__ void st_stream_u4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 FADD2 / FMUL2 / FFMA2 through the compiler's
// __fadd2_rn / __fmul2_rn / __ffma2_rn builtins): two IEEE round-to-nearest
// operations per issued instruction, bitwise equal to the scalar forms. The
// bf16 kernels move two elements per byte of fp32 data, so their instruction
// issue rate, not MUFU or HBM, is what the pairing relieves.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
// a - b is a + (-b) exactly (IEEE subtraction is defined so)
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) { return __fadd2_rn(a, make_float2(-b.x, -b.y)); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// The two elements of a bf16x2 word as an fp32 pair (low half first).
__device__ __forceinline__ float2 bf16x2_f32(uint32_t w) { return make_float2(bf16_lo(w), bf16_hi(w)); }

// ---------------------------------------------------------------------------
// Online log-sum-exp: the state (m, s) stands for s * e^m with m the running
// max; each element contributes e^(x - m) = 2^((x - m) * log2 e) (FADD, FMUL,
// MUFU.EX2). The max element contributes exactly 1, as in torch's
// log_softmax, and the max is refreshed once per loaded group, not per
// element. log-sum-exp(x) = m + log(s).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exp_shift(float x, float m) { return exp2_approx((x - m) * kLog2e); }

// exp_shift of a pair: (x - m) * log2 e in one packed subtract and multiply,
// bitwise equal to two exp_shift calls.
__device__ __forceinline__ float2 exp_shift2(float2 x, float m) {
  const float2 t = fmul2(fsub2(x, make_float2(m, m)), make_float2(kLog2e, kLog2e));
  return make_float2(exp2_approx(t.x), exp2_approx(t.y));
}

// Sum over the 8 elements of a bf16 vector of e^(x - m), as a pair: the
// exponent x log2 e - m log2 e is one packed fused multiply-add per pair
// (the separate subtract and multiply of exp_shift2 cost one more packed
// instruction; the exponent's error stays below an ulp of m log2 e).
__device__ __forceinline__ float2 vec8_expsum2(const uint4& v, float m) {
  const float mc = m * kLog2e;
  const float2 c2 = make_float2(kLog2e, kLog2e), n2 = make_float2(-mc, -mc);
  float2 t[4];
  t[0] = ffma2(bf16x2_f32(v.x), c2, n2);
  t[1] = ffma2(bf16x2_f32(v.y), c2, n2);
  t[2] = ffma2(bf16x2_f32(v.z), c2, n2);
  t[3] = ffma2(bf16x2_f32(v.w), c2, n2);
  float2 e[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) e[h] = make_float2(exp2_approx(t[h].x), exp2_approx(t[h].y));
  return fadd2(fadd2(e[0], e[1]), fadd2(e[2], e[3]));
}

// The rounding is spelled out (one product, then one fused multiply-add) so
// that every kernel that merges the same partials gets the same bits; left
// to the compiler, either product may be the one contracted.
__device__ __forceinline__ void lse_merge(float& m, float& s, float om, float os) {
  const float M = fmaxf(m, om);
  s = __fmaf_rn(s, exp_shift(m, M), __fmul_rn(os, exp_shift(om, M)));
  m = M;
}

__device__ __forceinline__ void lse_push(float& m, float& s, float x) {
  if (x > m) {
    s *= exp_shift(m, x);
    m = x;
  }
  s += exp_shift(x, m);
}

// Maximum over the warp's 32 lanes (one redux.sync on sm_100a; NaN inputs
// are ignored, as fmaxf ignores them).
__device__ __forceinline__ float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// Merges the 32 lanes' (m, s) into the warp's (max, sum of e^(x - max)),
// valid in every lane: the warp maximum M, each lane's s rescaled by
// e^(m - M), then a sum over a fixed butterfly. A lane whose m already is M
// is scaled by e^0 = 1 exactly, so the rescale is skipped when every lane
// holds M (the streaming kernels keep m warp-uniform on full stages): the
// bits are the same either way.
__device__ __forceinline__ void warp_lse(float& m, float& s) {
  const float M = warp_max(m);
  if (__any_sync(kFullMask, m != M)) s *= exp_shift(m, M);
  m = M;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
}

// Block-wide (m, s) merge in a fixed butterfly order. `sh` holds 2*NT/32
// floats. The result is valid in every lane of warp 0. Ends with a barrier.
template <int NT>
__device__ __forceinline__ void block_lse(float& m, float& s, float* sh) {
  constexpr int NW = NT / 32;
  warp_lse(m, s);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sh[w] = m;
    sh[NW + w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = lane < NW ? sh[lane] : kNegSeed;
    s = lane < NW ? sh[NW + lane] : 0.f;
    warp_lse(m, s);
  }
  __syncthreads();
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

// Fixed-order sum of x[0..n) by one warp: lane-strided partials, then a
// butterfly. Reads through L2 (the values were written by other CTAs).
__device__ __forceinline__ float warp_sum_l2(const float* x, int64_t n) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int64_t i = lane; i < n; i += 32) acc += __ldcg(x + i);
  return warp_sum(acc);
}

// ---------------------------------------------------------------------------
// Flattened, balanced split of [0, rows*V) into equal CTA chunks.
// ---------------------------------------------------------------------------
struct Partition {
  int64_t V = 0;      // row length in elements
  int64_t E = 0;      // rows * V
  int64_t chunk = 0;  // elements per CTA, a multiple of 4
  int64_t grid = 0;   // number of CTAs
  int pmax = 0;       // upper bound on the number of CTAs that touch one row
  // ring kernels: elements per stage, and the start of the one-stage queue
  // blocks at the end of the launch (-1: none; see BlockMap)
  int64_t stage = 0;
  int64_t split = -1;
  // partial slots per consumer warp in the workspace: rows * pmax, or for
  // the D-PACE ring forward blocks + rows (row r's slot s at index(r V) + r + s)
  int64_t nslots = 0;

  __host__ __device__ __forceinline__ int64_t first_cta(int64_t r) const { return (r * V) / chunk; }
  __host__ __device__ __forceinline__ int pieces(int64_t r) const {
    return int(((r + 1) * V - 1) / chunk - (r * V) / chunk + 1);
  }
};

// Queue geometry: blocks of BL = BS * SE elements below `split`, blocks of one
// stage (SE elements) from `split` to E. The D-PACE forward sets `split` so
// that its launch ends on short blocks: CTAs then finish within about a stage
// of one another instead of a whole block. `split` is a multiple of BL fixed
// by the problem size alone, never by the grid, so the partial slots -- and
// the results -- do not depend on the CTA count or the queue's schedule.
// Without short blocks split = ceil(E / BL) * BL. BL and SE are powers of two.
struct BlockMap {
  int64_t E = 0, split = 0;
  int lbl = 0, lse = 0;  // log2 of BL and SE
  unsigned nmain = 0, nblocks = 0;

  __host__ __device__ __forceinline__ int64_t start(unsigned b) const {
    return b < nmain ? (int64_t)b << lbl : split + ((int64_t)(b - nmain) << lse);
  }
  __host__ __device__ __forceinline__ int64_t end(unsigned b) const {
    const int64_t e = b < nmain ? (int64_t)(b + 1) << lbl : split + ((int64_t)(b - nmain + 1) << lse);
    return e < E ? e : E;
  }
  // the block containing element e (0 <= e < E)
  __host__ __device__ __forceinline__ int64_t index(int64_t e) const {
    return e < split ? e >> lbl : (int64_t)nmain + ((e - split) >> lse);
  }
  // blocks overlapping row r (= partial slots of the row)
  __host__ __device__ __forceinline__ int pieces(int64_t r, int64_t V) const {
    return (int)(index((r + 1) * V - 1) - index(r * V) + 1);
  }
};

__host__ __device__ __forceinline__ int ilog2_pow2(int64_t x) {
  int l = 0;
  while ((int64_t(1) << l) < x) ++l;
  return l;
}

// split: a multiple of BL (<= E rounded up to BL), or negative for none.
__host__ __device__ __forceinline__ BlockMap make_block_map(int64_t E, int64_t BL, int64_t SE, int64_t split) {
  BlockMap m;
  m.E = E;
  m.lbl = ilog2_pow2(BL);
  m.lse = ilog2_pow2(SE);
  const int64_t nb = (E + BL - 1) / BL;
  if (split < 0 || split >= E) {
    m.split = nb * BL;
    m.nmain = m.nblocks = (unsigned)nb;
  } else {
    m.split = split;
    m.nmain = (unsigned)(split / BL);
    m.nblocks = m.nmain + (unsigned)((E - split + SE - 1) / SE);
  }
  return m;
}

inline Partition make_partition(int64_t rows, int64_t V, int64_t ctas, int64_t min_chunk) {
  Partition p;
  p.V = V;
  p.E = rows * V;
  if (p.E <= 0) return p;
  if (ctas < 1) ctas = 1;
  int64_t c = (p.E + ctas - 1) / ctas;
  c = (c + 3) & ~int64_t(3);
  if (c < min_chunk) c = min_chunk;
  p.chunk = c;
  p.grid = (p.E + c - 1) / c;
  p.pmax = int((V - 1) / c + 2);
  p.nslots = rows * p.pmax;
  return p;
}

}  // namespace specdec
