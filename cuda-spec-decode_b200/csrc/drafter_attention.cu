// Attention of the DFlash drafter on the sm_100a tensor cores (tcgen05).
//
// Reference behaviour: models/dflash/model.py:25-53 (DFlashAttention:
// softmax(q k^T / sqrt(d) + mask) v per head) under the mask of
// models/dflash/model.py:123-131 (_build_dflash_mask), applied by its
// structure instead of a [T, T] tensor: query t < n_ctx sees keys j <= t
// (causal context), query t >= n_ctx (a block slot) sees every key j < T.
//
// Layout: q, k, v, o are bf16 [B, T, H, 64] -- the projections' own layout
// (row (b, t) holds the H heads' 64-element slices), so no transpose is
// needed on either side. lse is fp32 [B, H, T]: the natural-log
// log-sum-exp of each query row's scaled scores, kept for a backward.
//
// Forward: one CTA per (b, h, 128-query tile), 4 warps, four CTAs per SM;
// thread i owns query row i of the tile, which is TMEM lane i. The grid runs
// the heaviest query tiles (those that see the most keys) first. Per 64-key
// tile:
//   1. the K and V tiles are in shared memory in the canonical
//      128-byte-swizzled layout (rows of 128 bytes, 16-byte chunk c of row r
//      stored at chunk c ^ (r % 8), 8-row atoms of 1024 bytes), copied by
//      cp.async ahead of use: the next K tile as soon as this tile's QK^T has
//      read K, the next V tile as soon as P V has read V, so global-memory
//      latency overlaps the softmax and the products;
//   2. thread 0 issues S = Q K^T as four tcgen05.mma (M 128, N 64, K 16,
//      bf16 in, fp32 accumulate in TMEM columns 0..63) and commits them to an
//      mbarrier;
//   3. every thread reads its row of S from TMEM once (64 registers), takes
//      the tile maximum and forms p = 2^(s' - m_ref) in bf16 into shared
//      memory as the A operand of the next product (one 64-key atom row);
//      m_ref, the row's reference maximum, is raised only when a tile's
//      maximum exceeds it by more than 2^8, and only then is O rescaled (in
//      tensor memory: load, scale, store) -- every p stays <= 2^8;
//   4. thread 0 issues O += P V as four tcgen05.mma (M 128, N 64, K 16; V read
//      as an MN-major operand: d contiguous) into TMEM columns 64..127, the
//      output accumulator, and commits.
// The epilogue reads O from TMEM and divides by the row sum. Apart from the
// copies the stages run one after another; four CTAs per SM overlap one
// another's. Every mbarrier wait is bounded; a wait that expires sets
// *status and the CTA stops issuing work, waits (bounded) for what it issued
// and releases its TMEM.
#include <atomic>
#include <cstdint>

#include "bulk_copy.cuh"
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

constexpr int kHD = 64;        // head dimension
constexpr int kTM = 128;       // query rows per CTA (TMEM lanes)
constexpr int kThreads = 128;  // 4 warps

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + (((c ^ (r & 7u)) & 7u) << 4); }

// Shared-memory matrix descriptor, 128-byte swizzle: start address, leading
// byte offset (between 64-element chunks of the contiguous dimension; used
// by MN-major operands), stride byte offset (between 8-row atoms), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for tcgen05
  d |= (uint64_t)2u << 61;  // 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 D, M x N, majors.
constexpr uint32_t instr_desc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32-column loads (possibly from different column ranges) and one wait:
// the load latency is paid once for both.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, float (&a)[32], float (&b)[32]) {
  uint32_t r[32], t[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(t[0]), "=r"(t[1]), "=r"(t[2]), "=r"(t[3]), "=r"(t[4]), "=r"(t[5]), "=r"(t[6]), "=r"(t[7]),
        "=r"(t[8]), "=r"(t[9]), "=r"(t[10]), "=r"(t[11]), "=r"(t[12]), "=r"(t[13]), "=r"(t[14]), "=r"(t[15]),
        "=r"(t[16]), "=r"(t[17]), "=r"(t[18]), "=r"(t[19]), "=r"(t[20]), "=r"(t[21]), "=r"(t[22]), "=r"(t[23]),
        "=r"(t[24]), "=r"(t[25]), "=r"(t[26]), "=r"(t[27]), "=r"(t[28]), "=r"(t[29]), "=r"(t[30]), "=r"(t[31])
      : "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    a[i] = __uint_as_float(r[i]);
    b[i] = __uint_as_float(t[i]);
  }
}

__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Rows [t0, t0 + 128) of one head of a [B, T, H, 64] bf16 tensor into a
// swizzled shared tile through cp.async (16 bytes per thread and chunk; rows
// at or past T are zero-filled): the copies run while the thread goes on, and
// cp_async_wait<n>() waits for all but the n most recently committed groups.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int NT = kThreads, int ROWS = kTM>
__device__ __forceinline__ void load_tile_async(uint32_t tile, const bf16_t* base, int64_t row_stride, int t0,
                                                int T) {
#pragma unroll
  for (int j = 0; j < (ROWS * 8) / NT; ++j) {
    const int idx = threadIdx.x + j * NT;
    const int r = idx >> 3, c = idx & 7;
    const bool valid = t0 + r < T;
    const bf16_t* src = base + (valid ? (int64_t)(t0 + r) * row_stride + c * 8 : 0);
    cp_async16(tile + sw128((uint32_t)r, (uint32_t)c), src, valid);
  }
}

// Waits for the phase of `bar` with the given parity; false after the limit.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity) { return mbar_wait(bar, parity); }

// tcgen05.st of 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// Forward: 64-key tiles, four CTAs per SM. TMEM columns 0..63 hold S, 64..127
// the output accumulator O (the tensor core adds each tile's P V into it).
constexpr int kFN = 64;               // keys per forward tile
constexpr int kFCtas = 4;             // resident CTAs per SM (registers, TMEM, shared memory)
constexpr uint32_t kFTmemCols = 128;
constexpr uint32_t kFColO = 64;
constexpr uint32_t kFOffQ = 0;        // 128 rows x 128 B
constexpr uint32_t kFOffK = 16384;    // 64 rows x 128 B
constexpr uint32_t kFOffV = 24576;    // 64 rows x 128 B
constexpr uint32_t kFOffP = 32768;    // 128 rows x 128 B (one 64-key atom per row)
constexpr uint32_t kFOffBar = 49152;  // two mbarriers
constexpr uint32_t kFOffTmem = kFOffBar + 16;
constexpr uint32_t kSmemBytes = kFOffTmem + 16 + 1024;  // + alignment slack
// A row's probabilities are taken against a reference maximum that is
// raised only when the tile's maximum exceeds it by more than 2^8 (base-2
// exponent 8): p <= 2^8 then, fine for bf16 P and the fp32 sums, and O in
// tensor memory is rescaled only on those rare raises, not every tile.
constexpr float kRescaleLog2 = 8.f;

__global__ void __launch_bounds__(kThreads, kFCtas) dflash_attn_fwd_kernel(const bf16_t* __restrict__ q,
                                                                           const bf16_t* __restrict__ k,
                                                                           const bf16_t* __restrict__ v,
                                                                           bf16_t* __restrict__ o,
                                                                           float* __restrict__ lse, int T, int H,
                                                                           int n_ctx, float scale_log2, int* status,
                                                                           int withhold) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - smem_u32(smem_raw));
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(gbase + kFOffBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + kFOffTmem);

  const int warp = threadIdx.x >> 5;
  // heaviest query tiles first (the last tile sees every key): blocks are
  // dispatched in index order, x fastest
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int q0 = (gridDim.y - 1 - blockIdx.y) * kTM;
  const int64_t rs = (int64_t)H * kHD;  // row stride of [B, T, H, 64]
  const bf16_t* qb = q + (int64_t)b * T * rs + (int64_t)h * kHD;
  const bf16_t* kb = k + (int64_t)b * T * rs + (int64_t)h * kHD;
  const bf16_t* vb = v + (int64_t)b * T * rs + (int64_t)h * kHD;

  if (threadIdx.x == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kFTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // copies in flight: {Q, K tile 0}, then {V tile 0}
  load_tile_async<kThreads, kTM>(base + kFOffQ, qb, rs, q0, T);
  load_tile_async<kThreads, kFN>(base + kFOffK, kb, rs, 0, T);
  cp_async_commit();
  load_tile_async<kThreads, kFN>(base + kFOffV, vb, rs, 0, T);
  cp_async_commit();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  // key range of this query tile: up to its last context row, or every key
  // once the tile holds a block slot
  const int q_last = min(q0 + kTM, T) - 1;
  const int kv_end = q_last >= n_ctx ? T : q_last + 1;
  const int row = q0 + threadIdx.x;  // this thread's query row
  constexpr uint32_t kIdS = instr_desc(kTM, kFN, 0, 0);
  constexpr uint32_t kIdO = instr_desc(kTM, kHD, 0, 1);

  float m_ref = -INFINITY, l_run = 0.f;  // reference maximum (base-2 scaled), row sum against it
  uint32_t ph = 0;
  bool ok = true;

  for (int k0 = 0; k0 < kv_end && ok; k0 += kFN) {
    const bool more = k0 + kFN < kv_end;
    cp_async_wait<1>();  // this K tile (and Q) landed; the newest group, this V tile, may be in flight
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // failure-detection test hook: the grid's first CTA issues nothing for its
    // first tile, so its own wait runs into the limit
    if (threadIdx.x == 0 && !(withhold && k0 == 0 && blockIdx.x == 0 && blockIdx.y == 0)) {  // S = Q K^T
#pragma unroll
      for (int kk = 0; kk < kHD / 16; ++kk)
        umma_bf16(tmem, smem_desc(base + kFOffQ + kk * 32, 16, 1024), smem_desc(base + kFOffK + kk * 32, 16, 1024),
                  kIdS, kk > 0);
      umma_commit(bar_s);
    }
    if (__syncthreads_or(!wait_bar(bar_s, ph) ? 1 : 0)) {  // CTA-uniform: a wait expired
      ok = false;
      break;
    }
    tc_fence_after();
    // the product has read K: the next K tile streams in during the softmax and P V
    if (more) load_tile_async<kThreads, kFN>(base + kFOffK, kb, rs, k0 + kFN, T);
    cp_async_commit();
    // every row of this query tile sees every key of this key tile: no
    // per-element mask (a context row sees keys up to itself, a block row all
    // keys; rows past T are never stored)
    const bool full = k0 + kFN <= T && (q0 >= n_ctx || k0 + kFN - 1 <= q0);
    float s[2][32];  // this row's 64 scores, kept for both passes
    tmem_ld32x2(tmem + lane_base, tmem + lane_base + 32, s[0], s[1]);
    if (!full) {
#pragma unroll
      for (int i = 0; i < kFN; ++i) {
        const int j = k0 + i;
        if (!(j < T && (row >= n_ctx || j <= row))) s[i >> 5][i & 31] = -INFINITY;
      }
    }
    // the tile's maximum; the base-2 scale is positive, so scaling the
    // maximum equals the maximum of the scaled scores
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int i = 0; i < kFN; ++i) mx[i & 3] = fmaxf(mx[i & 3], s[i >> 5][i & 31]);
    const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
    // raise the reference maximum only by more than 2^8 (or the first time)
    const bool raise = mt > m_ref + kRescaleLog2;
    const float alpha = raise ? (m_ref == -INFINITY ? 0.f : exp2_approx(m_ref - mt)) : 1.f;
    if (raise) m_ref = mt;
    // p = 2^(s * scale_log2 - m_ref) (masked scores give exactly 0), row
    // sum, P in bf16 to shared memory (one 64-key atom row)
    const float nm = -m_ref;
    float ls[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t r = (uint32_t)threadIdx.x;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {  // 32 keys at a time: 16 packed words, four 16-byte chunks
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float p0 = exp2_approx(fmaf(s[hh][i], scale_log2, nm));
        const float p1 = exp2_approx(fmaf(s[hh][i + 1], scale_log2, nm));
        ls[(i >> 1) & 3] += p0 + p1;
        pk[i / 2] = pack_bf16x2(p0, p1);
      }
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4)
        st_shared_u4(base + kFOffP + sw128(r, (uint32_t)(hh * 4 + c4)),
                     make_uint4(pk[4 * c4], pk[4 * c4 + 1], pk[4 * c4 + 2], pk[4 * c4 + 3]));
    }
    l_run = fmaf(l_run, alpha, (ls[0] + ls[1]) + (ls[2] + ls[3]));
    // O holds earlier tiles' P V against the old reference: rescale it in
    // tensor memory before this tile's product adds to it (only the warps with
    // a raised row; the first tile writes O without accumulating)
    if (k0 > 0 && __any_sync(kFullMask, raise)) {
      float ot[2][32];
      tmem_ld32x2(tmem + lane_base + kFColO, tmem + lane_base + kFColO + 32, ot[0], ot[1]);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        ot[0][i] *= alpha;
        ot[1][i] *= alpha;
      }
      tmem_st32(tmem + lane_base + kFColO, ot[0]);
      tmem_st32(tmem + lane_base + kFColO + 32, ot[1]);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    cp_async_wait<1>();  // this V tile; the next K tile may be in flight
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {  // O += P V (the first tile writes O)
#pragma unroll
      for (int kk = 0; kk < kFN / 16; ++kk)
        umma_bf16(tmem + kFColO, smem_desc(base + kFOffP + (uint32_t)kk * 32u, 16, 1024),
                  smem_desc(base + kFOffV + (uint32_t)kk * 2048u, 16384, 1024), kIdO, (k0 > 0 || kk > 0) ? 1u : 0u);
      umma_commit(bar_o);
    }
    if (__syncthreads_or(!wait_bar(bar_o, ph) ? 1 : 0)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (more) load_tile_async<kThreads, kFN>(base + kFOffV, vb, rs, k0 + kFN, T);  // the product has read V
    cp_async_commit();
    ph ^= 1u;
  }

  cp_async_wait<0>();  // no copy outlives the CTA
  if (!ok) {
    if (threadIdx.x == 0 && status) atomicExch(status, kStatusTimeout);
    // wait (bounded) for the products this CTA may still have in flight
    wait_bar(bar_s, ph);
    wait_bar(bar_o, ph);
    // never a plausible wrong number: this CTA's rows of o and lse are NaN
    if (row < T) {
      bf16_t* orow = o + ((int64_t)b * T + row) * rs + (int64_t)h * kHD;
#pragma unroll
      for (int c = 0; c < kHD / 8; ++c)
        *reinterpret_cast<uint4*>(orow + 8 * c) = make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
      lse[((int64_t)b * H + h) * T + row] = __int_as_float(0x7fc00000);
    }
  } else {
    float ot[2][32];
    tmem_ld32x2(tmem + lane_base + kFColO, tmem + lane_base + kFColO + 32, ot[0], ot[1]);
    if (row < T) {
      const float inv = 1.f / l_run;
      bf16_t* orow = o + ((int64_t)b * T + row) * rs + (int64_t)h * kHD;
#pragma unroll
      for (int c = 0; c < kHD / 8; ++c) {
        const float* a = &ot[c >> 2][(c & 3) * 8];
        *reinterpret_cast<uint4*>(orow + 8 * c) =
            make_uint4(pack_bf16x2(a[0] * inv, a[1] * inv), pack_bf16x2(a[2] * inv, a[3] * inv),
                       pack_bf16x2(a[4] * inv, a[5] * inv), pack_bf16x2(a[6] * inv, a[7] * inv));
      }
      lse[((int64_t)b * H + h) * T + row] = (m_ref + log2f(l_run)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFTmemCols) : "memory");
}


// ---------------------------------------------------------------------------
// Backward, no atomics (every accumulation runs in a fixed order inside one
// CTA, so the gradients are bitwise repeatable). A small kernel first forms
// delta = sum_d dO * O per query row; then one grid runs both roles, dq and
// dk/dv tiles interleaved heaviest first, so their long tiles overlap:
//   dq role, one CTA per (b, h, 128-query tile), thread = query row: per
//     64-key tile: S = Q K^T and dP = dO V^T (tcgen05, TMEM columns 0..63 /
//     64..127), p = e^(s * scale - lse), dS = p * (dP - delta) * scale to
//     shared memory in bf16, dQ += dS K (K as an MN-major operand) in TMEM
//     columns 128..191.
//   dk/dv role, one CTA per (b, h, 128-key tile), thread = key row: per
//     64-query tile: S^T = K Q^T and dP^T = V dO^T, p^T and dS^T in bf16 to
//     shared memory, dV += P^T dO and dK += dS^T Q (dO and Q as MN-major
//     operands) in TMEM columns 128..191 / 192..255.
// 8 warps per CTA, two CTAs per SM (256 TMEM columns each). Warps w and w + 4
// share TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31 (one row each, thread t and
// t + 128) and split a tile's 64 columns into halves: with the row's
// log-sum-exp known, the halves are independent. Tiles arrive by cp.async one
// step ahead: the dq role double-buffers K and refills V once dP has read
// it; the dk/dv role double-buffers the query tile's Q, dO, lse and delta.
// ---------------------------------------------------------------------------

constexpr int kBN = 64;            // keys per dq tile, queries per dkv tile
constexpr int kBThreads = 256;     // 8 warps
constexpr int kBCtas = 2;          // resident CTAs per SM
constexpr uint32_t kBTmemCols = 256;
constexpr uint32_t kColS = 0, kColDP = 64, kColAcc0 = 128, kColAcc1 = 192;

// dq role shared memory (offsets from a 1024-byte-aligned base)
constexpr uint32_t kQOffQ = 0;        // 128 rows x 128 B
constexpr uint32_t kQOffG = 16384;    // dO, 128 rows
constexpr uint32_t kQOffK0 = 32768;   // K, even tiles, 64 rows
constexpr uint32_t kQOffK1 = 40960;   // K, odd tiles
constexpr uint32_t kQOffV = 49152;    // V, 64 rows
constexpr uint32_t kQOffS = 57344;    // dS, 128 rows x 64 keys (one atom per row)
constexpr uint32_t kQOffBar = 73728;
constexpr uint32_t kBSmemBytes = kQOffBar + 32 + 1024;

// dk/dv role shared memory
constexpr uint32_t kVOffK = 0;        // 128 rows
constexpr uint32_t kVOffV = 16384;    // 128 rows
constexpr uint32_t kVOffQ0 = 32768;   // query tile set 0: Q, 64 rows
constexpr uint32_t kVOffG0 = 40960;   //                   dO
constexpr uint32_t kVOffQ1 = 49152;   // query tile set 1
constexpr uint32_t kVOffG1 = 57344;
constexpr uint32_t kVOffP = 65536;    // P^T, 128 keys x 64 queries
constexpr uint32_t kVOffS = 81920;    // dS^T
constexpr uint32_t kVOffRow0 = 98304; // lse (64 floats) then delta (64 floats), set 0
constexpr uint32_t kVOffRow1 = 98816; // set 1
constexpr uint32_t kVOffBar = 99328;
constexpr uint32_t kBSmemBytesKV = kVOffBar + 32 + 1024;

__device__ __forceinline__ bool visible(int qrow, int key, int T, int n_ctx) {
  return qrow < T && key < T && (qrow >= n_ctx || key <= qrow);
}

// Writes 32 consecutive bf16 values (16 words) of row r of a one-atom (64
// columns) K-major operand at columns [32 hh, 32 hh + 32).
__device__ __forceinline__ void st_row32(uint32_t tile, uint32_t r, int hh, const uint32_t (&w)[16]) {
#pragma unroll
  for (int c4 = 0; c4 < 4; ++c4)
    st_shared_u4(tile + sw128(r, (uint32_t)(hh * 4 + c4)),
                 make_uint4(w[4 * c4], w[4 * c4 + 1], w[4 * c4 + 2], w[4 * c4 + 3]));
}

__device__ __forceinline__ void tmem_alloc_bwd(uint32_t* slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(kBTmemCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void cta_sync_tc() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// dq for query tile (n_tiles - 1 - rank): rank 0 is the heaviest (the last
// query tile sees every key). `fail_first`: the failure-detection test hook.
__device__ __forceinline__ void attn_bwd_dq(const bf16_t* __restrict__ q, const bf16_t* __restrict__ k,
                                            const bf16_t* __restrict__ v, const float* __restrict__ lse,
                                            const float* __restrict__ delta_in, const bf16_t* __restrict__ dO,
                                            bf16_t* __restrict__ dq, int T, int H, int n_ctx, float scale,
                                            int* status, int rank, bool fail_first) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - smem_u32(smem_raw));
  uint64_t* bar = reinterpret_cast<uint64_t*>(gbase + kQOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + kQOffBar + 16);
  const int warp = threadIdx.x >> 5;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int q0 = ((T + kTM - 1) / kTM - 1 - rank) * kTM;
  const int64_t rs = (int64_t)H * kHD;
  const int64_t head = (int64_t)b * T * rs + (int64_t)h * kHD;
  const int r_in = threadIdx.x & (kTM - 1), half = threadIdx.x >> 7;
  const int row = q0 + r_in;
  const float sl2 = scale * kLog2e;

  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc_bwd(tmem_slot);
  // one copy group: Q, dO and the first K and V tiles
  load_tile_async<kBThreads, kTM>(base + kQOffQ, q + head, rs, q0, T);
  load_tile_async<kBThreads, kTM>(base + kQOffG, dO + head, rs, q0, T);
  load_tile_async<kBThreads, kBN>(base + kQOffK0, k + head, rs, 0, T);
  load_tile_async<kBThreads, kBN>(base + kQOffV, v + head, rs, 0, T);
  cp_async_commit();
  // this row's delta = sum_d dO * O (the delta kernel) and its lse in base 2
  float delta = 0.f, lse2 = 0.f;
  if (row < T) {
    delta = delta_in[((int64_t)b * H + h) * T + row];
    lse2 = lse[((int64_t)b * H + h) * T + row] * kLog2e;
  }
  cta_sync_tc();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  const int q_last = min(q0 + kTM, T) - 1;
  const int kv_end = q_last >= n_ctx ? T : q_last + 1;
  constexpr uint32_t kIdS = instr_desc(kTM, kBN, 0, 0);
  constexpr uint32_t kIdQ = instr_desc(kTM, kHD, 0, 1);
  uint32_t ph = 0;
  bool ok = true;
  for (int k0 = 0, it = 0; k0 < kv_end; k0 += kBN, ++it) {
    const bool more = k0 + kBN < kv_end;
    const uint32_t kcur = (it & 1) ? kQOffK1 : kQOffK0, knext = (it & 1) ? kQOffK0 : kQOffK1;
    cp_async_wait<0>();  // this K and V tile
    cta_sync_tc();
    // the other K buffer was last read by the previous tile's dQ product: fill it now
    if (more) load_tile_async<kBThreads, kBN>(base + knext, k + head, rs, k0 + kBN, T);
    cp_async_commit();
    // failure-detection test hook: this CTA issues nothing for its first tile
    if (threadIdx.x == 0 && !(fail_first && k0 == 0)) {
#pragma unroll
      for (int kk = 0; kk < kHD / 16; ++kk) {  // S = Q K^T, dP = dO V^T
        umma_bf16(tmem + kColS, smem_desc(base + kQOffQ + kk * 32, 16, 1024),
                  smem_desc(base + kcur + kk * 32, 16, 1024), kIdS, kk > 0);
        umma_bf16(tmem + kColDP, smem_desc(base + kQOffG + kk * 32, 16, 1024),
                  smem_desc(base + kQOffV + kk * 32, 16, 1024), kIdS, kk > 0);
      }
      umma_commit(bar);
    }
    if (__syncthreads_or(!wait_bar(bar, ph) ? 1 : 0)) {
      ok = false;
      break;
    }
    ph ^= 1u;
    tc_fence_after();
    if (more) load_tile_async<kBThreads, kBN>(base + kQOffV, v + head, rs, k0 + kBN, T);  // dP has read V
    cp_async_commit();
    // every row of the query tile sees every key of the key tile: no per-element mask
    const bool full = k0 + kBN <= T && (q0 >= n_ctx || k0 + kBN - 1 <= q0);
    {
      float sv[32], dp[32];  // this thread's half of the tile's 64 columns
      tmem_ld32x2(tmem + lane_base + kColS + half * 32, tmem + lane_base + kColDP + half * 32, sv, dp);
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float p0 = exp2_approx(fmaf(sv[i], sl2, -lse2));
        float p1 = exp2_approx(fmaf(sv[i + 1], sl2, -lse2));
        if (!full) {
          const int j = k0 + half * 32 + i;
          p0 = visible(row, j, T, n_ctx) ? p0 : 0.f;
          p1 = visible(row, j + 1, T, n_ctx) ? p1 : 0.f;
        }
        w[i / 2] = pack_bf16x2(p0 * (dp[i] - delta) * scale, p1 * (dp[i + 1] - delta) * scale);
      }
      st_row32(base + kQOffS, (uint32_t)r_in, half, w);
    }
    cta_sync_tc();
    if (threadIdx.x == 0) {  // dQ += dS K
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk)
        umma_bf16(tmem + kColAcc0, smem_desc(base + kQOffS + (uint32_t)kk * 32u, 16, 1024),
                  smem_desc(base + kcur + (uint32_t)kk * 2048u, 16384, 1024), kIdQ, (k0 > 0 || kk > 0) ? 1u : 0u);
      umma_commit(bar);
    }
    if (__syncthreads_or(!wait_bar(bar, ph) ? 1 : 0)) {
      ok = false;
      break;
    }
    ph ^= 1u;
    cta_sync_tc();
  }
  cp_async_wait<0>();  // no copy outlives the CTA
  if (!ok) {
    if (threadIdx.x == 0 && status) atomicExch(status, kStatusTimeout);
    wait_bar(bar, ph);
    if (row < T) {  // never a plausible wrong number: this CTA's rows of dq are NaN
      bf16_t* drow = dq + head + (int64_t)row * rs + half * 32;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(drow + 8 * c) = make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
    }
  } else {
    tc_fence_after();
    float acc[32];  // this thread's half of the row's 64 dQ columns
    tmem_ld32(tmem + lane_base + kColAcc0 + half * 32, acc);
    if (row < T) {
      bf16_t* drow = dq + head + (int64_t)row * rs + half * 32;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float* a = acc + 8 * c;
        *reinterpret_cast<uint4*>(drow + 8 * c) = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                                              pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBTmemCols) : "memory");
}

// dk, dv for key tile kt (kt 0 is the heaviest: every query tile sees it).
__device__ __forceinline__ void attn_bwd_dkv(const bf16_t* __restrict__ q, const bf16_t* __restrict__ k,
                                             const bf16_t* __restrict__ v, const float* __restrict__ lse,
                                             const float* __restrict__ delta, const bf16_t* __restrict__ dO,
                                             bf16_t* __restrict__ dk, bf16_t* __restrict__ dv, int T, int H,
                                             int n_ctx, float scale, int* status, int kt, bool fail_first) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - smem_u32(smem_raw));
  uint64_t* bar = reinterpret_cast<uint64_t*>(gbase + kVOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + kVOffBar + 16);
  const int warp = threadIdx.x >> 5;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int k0 = kt * kTM;
  const int64_t rs = (int64_t)H * kHD;
  const int64_t head = (int64_t)b * T * rs + (int64_t)h * kHD;
  const int64_t rowv = ((int64_t)b * H + h) * T;
  const int r_in = threadIdx.x & (kTM - 1), half = threadIdx.x >> 7;
  const int key = k0 + r_in;
  const float sl2 = scale * kLog2e;

  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc_bwd(tmem_slot);
  // 64-query tiles that see a key of this tile: context queries from the
  // diagonal on, and every tile holding a block slot
  const int qt_first = (k0 < n_ctx ? k0 : n_ctx) / kBN;
  const int qt_end = (T + kBN - 1) / kBN;
  // Q, dO and the query rows' lse / delta of query tile qt sit in buffer set
  // (qt - qt_first) & 1; the next set is filled while this one is used.
  auto load_query_tile = [&](int qt, int set) {
    const int qq = qt * kBN;
    load_tile_async<kBThreads, kBN>(base + (set ? kVOffQ1 : kVOffQ0), q + head, rs, qq, T);
    load_tile_async<kBThreads, kBN>(base + (set ? kVOffG1 : kVOffG0), dO + head, rs, qq, T);
    if (r_in < kBN) {  // half 0 copies lse of query qq + r_in, half 1 its delta
      const int qr = qq + r_in;
      const uint32_t rows = base + (set ? kVOffRow1 : kVOffRow0);
      cp_async4(rows + 4u * (half * kBN + r_in), (half ? delta : lse) + rowv + (qr < T ? qr : 0), qr < T);
    }
  };
  load_tile_async<kBThreads, kTM>(base + kVOffK, k + head, rs, k0, T);
  load_tile_async<kBThreads, kTM>(base + kVOffV, v + head, rs, k0, T);
  if (qt_first < qt_end) load_query_tile(qt_first, 0);
  cp_async_commit();
  cta_sync_tc();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  constexpr uint32_t kIdS = instr_desc(kTM, kBN, 0, 0);
  constexpr uint32_t kIdKV = instr_desc(kTM, kHD, 0, 1);
  uint32_t ph = 0;
  bool ok = true;
  bool first = true;
  for (int qt = qt_first; qt < qt_end; ++qt) {
    const int q0 = qt * kBN;
    const int set = (qt - qt_first) & 1;
    const uint32_t offq = set ? kVOffQ1 : kVOffQ0, offg = set ? kVOffG1 : kVOffG0;
    const float* sh_lse = reinterpret_cast<const float*>(gbase + (set ? kVOffRow1 : kVOffRow0));
    const float* sh_delta = sh_lse + kBN;
    cp_async_wait<0>();  // this query tile's Q, dO, lse and delta
    cta_sync_tc();
    // the other set was last read by the previous tile's dV / dK products
    if (qt + 1 < qt_end) load_query_tile(qt + 1, set ^ 1);
    cp_async_commit();
    // failure-detection test hook: this CTA issues nothing for its first tile
    if (threadIdx.x == 0 && !(fail_first && first)) {
#pragma unroll
      for (int kk = 0; kk < kHD / 16; ++kk) {  // S^T = K Q^T, dP^T = V dO^T
        umma_bf16(tmem + kColS, smem_desc(base + kVOffK + kk * 32, 16, 1024),
                  smem_desc(base + offq + kk * 32, 16, 1024), kIdS, kk > 0);
        umma_bf16(tmem + kColDP, smem_desc(base + kVOffV + kk * 32, 16, 1024),
                  smem_desc(base + offg + kk * 32, 16, 1024), kIdS, kk > 0);
      }
      umma_commit(bar);
    }
    if (__syncthreads_or(!wait_bar(bar, ph) ? 1 : 0)) {
      ok = false;
      break;
    }
    ph ^= 1u;
    tc_fence_after();
    // every query of the tile sees every key of this CTA's tile: no per-element mask
    const bool full = k0 + kTM <= T && q0 + kBN <= T && (q0 >= n_ctx || k0 + kTM - 1 <= q0);
    {
      float sv[32], dp[32];  // this thread's half of the tile's 64 query columns
      tmem_ld32x2(tmem + lane_base + kColS + half * 32, tmem + lane_base + kColDP + half * 32, sv, dp);
      uint32_t wp[16], wd[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int c = half * 32 + i;
        float p0 = exp2_approx(fmaf(sv[i], sl2, -sh_lse[c] * kLog2e));
        float p1 = exp2_approx(fmaf(sv[i + 1], sl2, -sh_lse[c + 1] * kLog2e));
        if (!full) {
          p0 = visible(q0 + c, key, T, n_ctx) ? p0 : 0.f;
          p1 = visible(q0 + c + 1, key, T, n_ctx) ? p1 : 0.f;
        }
        wp[i / 2] = pack_bf16x2(p0, p1);
        wd[i / 2] = pack_bf16x2(p0 * (dp[i] - sh_delta[c]) * scale, p1 * (dp[i + 1] - sh_delta[c + 1]) * scale);
      }
      st_row32(base + kVOffP, (uint32_t)r_in, half, wp);
      st_row32(base + kVOffS, (uint32_t)r_in, half, wd);
    }
    cta_sync_tc();
    if (threadIdx.x == 0) {  // dV += P^T dO, dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk) {
        const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
        umma_bf16(tmem + kColAcc0, smem_desc(base + kVOffP + (uint32_t)kk * 32u, 16, 1024),
                  smem_desc(base + offg + (uint32_t)kk * 2048u, 16384, 1024), kIdKV, acc);
        umma_bf16(tmem + kColAcc1, smem_desc(base + kVOffS + (uint32_t)kk * 32u, 16, 1024),
                  smem_desc(base + offq + (uint32_t)kk * 2048u, 16384, 1024), kIdKV, acc);
      }
      umma_commit(bar);
    }
    if (__syncthreads_or(!wait_bar(bar, ph) ? 1 : 0)) {
      ok = false;
      break;
    }
    ph ^= 1u;
    first = false;
    cta_sync_tc();
  }
  cp_async_wait<0>();  // no copy outlives the CTA
  if (!ok) {
    if (threadIdx.x == 0 && status) atomicExch(status, kStatusTimeout);
    wait_bar(bar, ph);
    if (key < T) {  // never a plausible wrong number: this CTA's rows of dk and dv are NaN
      bf16_t* vr = dv + head + (int64_t)key * rs + half * 32;
      bf16_t* kr = dk + head + (int64_t)key * rs + half * 32;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        *reinterpret_cast<uint4*>(vr + 8 * c) = make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
        *reinterpret_cast<uint4*>(kr + 8 * c) = make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
      }
    }
  } else {
    tc_fence_after();
    // keys no query sees (none here: the qt loop covers every visible pair) still get zeros;
    // this thread writes its half of the row's 64 dV and dK columns
    float av[32], ak[32];
    tmem_ld32x2(tmem + lane_base + kColAcc0 + half * 32, tmem + lane_base + kColAcc1 + half * 32, av, ak);
    if (first) {
#pragma unroll
      for (int i = 0; i < 32; ++i) av[i] = ak[i] = 0.f;
    }
    if (key < T) {
      bf16_t* vr = dv + head + (int64_t)key * rs + half * 32;
      bf16_t* kr = dk + head + (int64_t)key * rs + half * 32;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float* a = av + 8 * c;
        const float* g = ak + 8 * c;
        *reinterpret_cast<uint4*>(vr + 8 * c) = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                                            pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
        *reinterpret_cast<uint4*>(kr + 8 * c) = make_uint4(pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]),
                                                            pack_bf16x2(g[4], g[5]), pack_bf16x2(g[6], g[7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBTmemCols) : "memory");
}

// delta[b, h, t] = sum_d dO * O of query row t (fp32, d in order): the
// rows' term of dS, read by both backward roles. One thread per row.
__global__ void __launch_bounds__(256) dflash_attn_delta_kernel(const bf16_t* __restrict__ o,
                                                                const bf16_t* __restrict__ dO,
                                                                float* __restrict__ delta, int B, int T, int H) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over [B, T, H], the inputs' row order
  if (i >= (int64_t)B * T * H) return;
  const int h = (int)(i % H), t = (int)((i / H) % T), b = (int)(i / ((int64_t)H * T));
  const bf16_t* orow = o + i * kHD;
  const bf16_t* grow = dO + i * kHD;
  float d = 0.f;
#pragma unroll
  for (int c = 0; c < kHD / 8; ++c) {
    const uint4 a = *reinterpret_cast<const uint4*>(orow + 8 * c);
    const uint4 g = *reinterpret_cast<const uint4*>(grow + 8 * c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      d = fmaf(bf16_lo(aw[j]), bf16_lo(gw[j]), d);
      d = fmaf(bf16_hi(aw[j]), bf16_hi(gw[j]), d);
    }
  }
  delta[((int64_t)b * H + h) * T + t] = d;
}

// Both backward roles in one grid: blockIdx.y even = dq for the query tile of
// rank y / 2, odd = dk / dv for key tile y / 2. Blocks are dispatched in index
// order and both roles run their heaviest tiles at rank 0, so the two roles'
// long tiles start first and their critical paths overlap.
__global__ void __launch_bounds__(kBThreads, kBCtas) dflash_attn_bwd_kernel(
    const bf16_t* __restrict__ q, const bf16_t* __restrict__ k, const bf16_t* __restrict__ v,
    const float* __restrict__ lse, const float* __restrict__ delta, const bf16_t* __restrict__ dO,
    bf16_t* __restrict__ dq, bf16_t* __restrict__ dk, bf16_t* __restrict__ dv, int T, int H, int n_ctx,
    float scale, int* status, int withhold) {
  const int idx = (int)(blockIdx.y >> 1);
  // failure-detection test hook: both roles' first CTA of (batch 0, head 0)
  const bool fail_first = withhold && blockIdx.x == 0 && idx == 0;
  if ((blockIdx.y & 1) == 0)
    attn_bwd_dq(q, k, v, lse, delta, dO, dq, T, H, n_ctx, scale, status, idx, fail_first);
  else
    attn_bwd_dkv(q, k, v, lse, delta, dO, dk, dv, T, H, n_ctx, scale, status, idx, fail_first);
}

}  // namespace

// Raises the kernel's dynamic shared-memory limit once per device.
static cudaError_t ensure_smem_limit_attn(size_t bytes) {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load() & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(dflash_attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

cudaError_t dflash_attn_fwd_launch(const void* q, const void* k, const void* v, void* o, float* lse, int batch, int T,
                                   int H, int n_ctx, float scale, int* status, int withhold, cudaStream_t st) {
  const cudaError_t e = ensure_smem_limit_attn(kSmemBytes);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)(batch * H), (unsigned)((T + kTM - 1) / kTM));
  dflash_attn_fwd_kernel<<<grid, kThreads, kSmemBytes, st>>>(
      static_cast<const bf16_t*>(q), static_cast<const bf16_t*>(k), static_cast<const bf16_t*>(v),
      static_cast<bf16_t*>(o), lse, T, H, n_ctx, scale * kLog2e, status, withhold);
  return cudaGetLastError();
}

cudaError_t dflash_attn_bwd_launch(const void* q, const void* k, const void* v, const void* o, const float* lse,
                                   const void* dO, void* dq, void* dk, void* dv, float* delta, int batch, int T, int H,
                                   int n_ctx, float scale, int* status, int withhold, cudaStream_t st) {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    // the grid's CTAs take the larger of the two roles' shared memory
    e = cudaFuncSetAttribute(dflash_attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(kBSmemBytesKV > kBSmemBytes ? kBSmemBytesKV : kBSmemBytes));
    if (e != cudaSuccess) return e;
    done.fetch_or(bit);
  }
  const int64_t rows = (int64_t)batch * T * H;
  dflash_attn_delta_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(
      static_cast<const bf16_t*>(o), static_cast<const bf16_t*>(dO), delta, batch, T, H);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)(batch * H), (unsigned)(2 * ((T + kTM - 1) / kTM)));
  dflash_attn_bwd_kernel<<<grid, kBThreads, (kBSmemBytesKV > kBSmemBytes ? kBSmemBytesKV : kBSmemBytes), st>>>(
      static_cast<const bf16_t*>(q), static_cast<const bf16_t*>(k), static_cast<const bf16_t*>(v), lse, delta,
      static_cast<const bf16_t*>(dO), static_cast<bf16_t*>(dq), static_cast<bf16_t*>(dk), static_cast<bf16_t*>(dv),
      T, H, n_ctx, scale, status, withhold);
  return cudaGetLastError();
}

}  // namespace specdec
