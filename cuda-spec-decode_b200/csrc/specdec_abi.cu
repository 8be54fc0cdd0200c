// extern "C" entry points of libspecdec.so (declared in include/specdec.h):
// argument checks, workspace layout, launch-shape selection and error codes.
// Nothing here allocates device memory or synchronises the stream.
#include "specdec.h"
#include "specdec_internal.h"
#include "bulk_copy.cuh"

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>

using namespace specdec;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return SPECDEC_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SPECDEC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Smallest CTA chunk in elements: below this, per-piece bookkeeping dominates.
constexpr int64_t kMinChunk = 1024;

// SPECDEC_SHAPE_DEFAULT (-1): the built-in choice per kernel and dtype (see
// ring_shape); any other value is the caller's.
std::atomic<int> g_shape[4] = {SPECDEC_SHAPE_DEFAULT, SPECDEC_SHAPE_DEFAULT, SPECDEC_SHAPE_DEFAULT,
                               SPECDEC_SHAPE_DEFAULT};
std::atomic<int> g_cap[4] = {0, 0, 0, 0};
std::atomic<int> g_static_queue{0};  // 1: ring kernels use a static block interleave
std::atomic<int> g_withhold_stage{0};  // failure-detection tests: launches left to withhold a stage

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

// Launch shapes 0..9 select a per-warp bulk-copy ring variant (used when the
// pointers are 16-byte aligned, else the 128-bit-load kernels run with their
// default shape); shapes 10..14 force the 128-bit-load kernels, variant
// shape - 10.
constexpr int kLdgShapeBase = 10;
// highest ring shape per kernel id (D-PACE fwd/bwd up to 8, DFlash up to 6)
constexpr int kMaxRingShape[4] = {8, 8, 6, 6};

bool has_ring_path(int kernel) { return kernel >= 0 && kernel <= 3; }

// Built-in ring shapes per element type and kernel (D-PACE fwd, D-PACE bwd,
// DFlash fwd, DFlash bwd), picked by graph-timed A/B at [64, 16, 128256]:
//  - D-PACE forward, shape 8 (two 16 KB stages per CTA: 4 CTAs per SM for
//    fp32, 5 for bf16). The bf16 forward is bound by its consumers'
//    exponentials and gains the warps (47.3 -> 46.1 us against shape 6); the
//    fp32 forward runs as fast as on shape 0 and leaves the shared memory that
//    lets the chained backward's CTAs move in while it drains (fused step
//    230.3 -> 227.1 us).
//  - bf16 D-PACE backward, shape 6 (fused step 126.0 -> 125.1 us; fp32 keeps
//    shape 0: 228.3 vs 229.1 us on shape 6).
//  - bf16 DFlash forward, shape 6 (two stages per stream, 4 CTAs per SM
//    instead of 3: 97.5 -> 92.4 us; fp32 151.7 vs 150.5 us keeps shape 0).
//  - fp32 DFlash backward, shape 6 (221.8 -> 221.0 us; bf16 116.2 vs 115.1 us
//    keeps shape 0).
constexpr int kDefaultRingShape[2][4] = {{8, 0, 0, 6}, {8, 6, 6, 0}};  // [fp32, bf16][kernel]
int default_ring_shape(int kernel, int dtype = kDtypeF32) {
  return has_ring_path(kernel) ? kDefaultRingShape[dtype == kDtypeBF16 ? 1 : 0][kernel] : 0;
}

// Variant id inside the chosen kernel family.
int kernel_shape(int kernel, bool tma) {
  const int raw = g_shape[kernel].load();
  if (raw < 0) return tma ? default_ring_shape(kernel) : 0;  // or the 128-bit-load kernels' shape 0
  if (tma) return raw;
  if (!has_ring_path(kernel)) return raw % kLdgShapeBase;
  return raw >= kLdgShapeBase ? raw - kLdgShapeBase : 0;
}

bool use_tma(int kernel, bool ptrs_aligned) {
  return g_shape[kernel].load() < kLdgShapeBase && ptrs_aligned && has_ring_path(kernel);
}

// bf16 has only the ring kernels: a shape that selects the 128-bit-load
// kernels falls back to ring shape 0. Default: default_ring_shape.
int bf16_shape(int kernel) {
  const int raw = g_shape[kernel].load();
  if (raw < 0) return default_ring_shape(kernel, kDtypeBF16);
  return raw < kLdgShapeBase ? raw : 0;
}

int ring_shape(int kernel, int dtype) {
  return dtype == kDtypeBF16 ? bf16_shape(kernel) : kernel_shape(kernel, true);
}

// Occupancy-derived CTA counts, cached per (kernel, dtype, kind, path,
// shape, cap, device). bf16 always takes the ring path.
int kernel_units(int kernel, int kind, bool tma, int device, int dtype = kDtypeF32) {
  static std::mutex mu;
  static std::map<uint64_t, int> cache;
  const int cap = g_cap[kernel].load();
  if (dtype == kDtypeBF16) tma = true;
  const int shape = tma ? ring_shape(kernel, dtype) : kernel_shape(kernel, false);
  const uint64_t key = (uint64_t(kernel) << 56) | (uint64_t(dtype & 1) << 55) | (uint64_t(kind & 0x3f) << 49) |
                       (uint64_t(tma) << 48) | (uint64_t(shape & 0xff) << 40) | (uint64_t(cap & 0xffff) << 24) |
                       uint64_t(device & 0xffffff);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int ctas = 0;
  switch (kernel) {
    case SPECDEC_KERNEL_DPACE_FWD:
      ctas = tma ? dpace_fwd_ring_ctas(dtype, shape, device, cap) : dpace_fwd_ctas(shape, device, cap);
      break;
    case SPECDEC_KERNEL_DPACE_BWD:
      ctas = tma ? dpace_bwd_ring_ctas(dtype, shape, device, cap) : dpace_bwd_ctas(shape, device, cap);
      break;
    case SPECDEC_KERNEL_DFLASH_FWD:
      ctas = tma ? dflash_fwd_ring_ctas(dtype, kind, shape, device, cap) : dflash_fwd_ctas(kind, shape, device, cap);
      break;
    case SPECDEC_KERNEL_DFLASH_BWD:
      ctas = tma ? dflash_bwd_ring_ctas(dtype, kind, shape, device, cap) : dflash_bwd_ctas(kind, shape, device, cap);
      break;
    default: ctas = 0;
  }
  if (ctas > 0) {
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = ctas;
  }
  return ctas;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- D-PACE workspace layout ----------------------------------------------
// counters: [done][flag][queue ctr][queue retired]
//           [backward queue ctr][backward retired][backward flag][-]  (forward_backward)
//           [seq_cnt u32 x N]
// scratch:  [part float2 x R*pmax*nc][xtgt f32 x R][seq_loss f32 x N]
struct DpaceLayout {
  size_t part = 0, xtgt = 0, seq_loss = 0, scratch = 0, counters = 0;
};

constexpr int kDpaceBwdWords = 4;  // word offset of the backward's three counter words
constexpr int kDpaceSeqWords = 8;  // word offset of seq_cnt

size_t dpace_counter_bytes(int64_t N, int64_t B) {
  (void)B;
  return align256(kDpaceSeqWords * sizeof(unsigned) + size_t(N) * sizeof(unsigned));
}

DpaceLayout dpace_layout(int64_t N, int64_t B, const Partition& pt, int nc) {
  DpaceLayout L;
  const size_t R = size_t(N) * size_t(B);
  L.part = 0;
  L.xtgt = align256(L.part + size_t(pt.nslots) * size_t(nc) * sizeof(float2));
  L.seq_loss = align256(L.xtgt + R * sizeof(float));
  L.scratch = align256(L.seq_loss + size_t(N) * sizeof(float));
  L.counters = dpace_counter_bytes(N, B);
  return L;
}

// Ring kernels: the unit of the partial table is a block of BL elements.
Partition ring_partition(int64_t rows, int64_t V, int64_t block_elems, int ctas) {
  Partition p;
  p.V = V;
  p.E = rows * V;
  p.chunk = block_elems;
  p.grid = ctas;
  p.pmax = int((V - 1) / block_elems + 2);
  p.nslots = rows * p.pmax;
  return p;
}

// D-PACE ring forward: one-stage queue blocks at the end of the launch
// (BlockMap) and the compact partial table -- row r's slot s at
// index(r V) + r + s, blocks + rows slots in all.
Partition dpace_ring_fwd_partition(int64_t rows, int64_t V, int dtype, int shape, int ctas) {
  Partition p = ring_partition(rows, V, dpace_ring_block_elems(dtype, shape), ctas);
  p.stage = dpace_ring_stage_elems(dtype, shape);
  p.split = dpace_fwd_split(p.E, p.chunk);
  const BlockMap bm = make_block_map(p.E, p.chunk, p.stage, p.split);
  if (bm.split < p.E) p.pmax = int((V - 1) / p.stage + 2);
  p.nslots = (int64_t)bm.nblocks + rows;
  return p;
}

// ---- DFlash workspace layout -----------------------------------------------
// counters: [done][flag][queue ctr][queue retired][row_cnt u32 x R]
// scratch:  [part DfPiece x R*pmax*nc][row_loss f32 x R][seq_loss f32 x N]
struct DflashLayout {
  size_t part = 0, row_loss = 0, seq_loss = 0, scratch = 0, counters = 0;
};

DflashLayout dflash_layout(int64_t N, int64_t B, const Partition& pt, int nc) {
  DflashLayout L;
  const size_t R = size_t(N) * size_t(B);
  L.part = 0;
  L.row_loss = align256(L.part + R * size_t(pt.pmax) * size_t(nc) * sizeof(DfPiece));
  L.seq_loss = align256(L.row_loss + R * sizeof(float));
  L.scratch = align256(L.seq_loss + size_t(N) * sizeof(float));
  L.counters = align256(16 + R * sizeof(unsigned));
  return L;
}

// A bf16 block (and stage) holds twice the elements of the float one of the
// same shape, so its partition has no more pieces per row.
Partition dpace_fwd_partition(int64_t N, int32_t B, int64_t V, bool tma, int device, int dtype = kDtypeF32) {
  const int units = kernel_units(SPECDEC_KERNEL_DPACE_FWD, 0, tma, device, dtype);
  if (tma || dtype == kDtypeBF16)
    return dpace_ring_fwd_partition(N * B, V, dtype, ring_shape(SPECDEC_KERNEL_DPACE_FWD, dtype), units);
  return make_partition(N * B, V, units, kMinChunk);
}

Partition dflash_fwd_partition(int64_t N, int32_t B, int64_t V, int kind, bool tma, int device,
                               int dtype = kDtypeF32) {
  const int units = kernel_units(SPECDEC_KERNEL_DFLASH_FWD, kind, tma, device, dtype);
  if (tma || dtype == kDtypeBF16)
    return ring_partition(N * B, V, dflash_ring_block_elems(dtype, ring_shape(SPECDEC_KERNEL_DFLASH_FWD, dtype)),
                          units);
  return make_partition(N * B, V, units, kMinChunk);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Failure-detection test hook: 1 if this ring forward launch should withhold a
// stage (consumes one of the launches armed by specdec_test_withhold_stage).
int take_withhold_stage() {
  int left = g_withhold_stage.load();
  while (left > 0 && !g_withhold_stage.compare_exchange_weak(left, left - 1)) {
  }
  return left > 0 ? 1 : 0;
}

}  // namespace

namespace specdec {
void set_last_error(const char* msg) { g_last_error = msg; }

// The checks of specdec_dpace_forward that need no workspace, in the order of
// losses/dpace.py:157-173 (_check); SPECDEC_OK with nothing to launch when N == 0.
int dpace_forward_check(int dtype, const void* logits, const int64_t* targets, int64_t N, int32_t B, int64_t V,
                        float alpha, int32_t loss_type, int64_t n_global, const float* loss, const float* lse,
                        const float* scale) {
  if (B < 1 || B > 32) return fail(SPECDEC_ERR_ARGUMENT, "kernel configured for block_size <= 32 (B=%d)", B);
  if (N < 0 || V < 0) return fail(SPECDEC_ERR_ARGUMENT, "negative shape N=%lld V=%lld", (long long)N, (long long)V);
  if (!(alpha >= 0.f && alpha <= 1.f))
    return fail(SPECDEC_ERR_VALUE, "dpace_alpha must be in [0, 1], got %g", (double)alpha);
  if (loss_type < 0 || loss_type > 2) return fail(SPECDEC_ERR_VALUE, "unknown loss_type %d", loss_type);
  if (N > 0 && (n_global < N || n_global < 1))
    return fail(SPECDEC_ERR_ARGUMENT, "n_global (%lld) must be >= N (%lld)", (long long)n_global, (long long)N);
  if (!loss) return fail(SPECDEC_ERR_ARGUMENT, "loss output is null");
  if (N == 0) return ok();
  if (V == 0) return fail(SPECDEC_ERR_TARGET_RANGE, "targets out of range [0, 0)");
  if (!logits || !targets || !lse || !scale) return fail(SPECDEC_ERR_ARGUMENT, "null input or output pointer");
  if (!aligned(logits, 4) || !aligned(targets, 8) || !aligned(lse, 4) || !aligned(scale, 4))
    return fail(SPECDEC_ERR_ARGUMENT, "misaligned input or output pointer");
  if (dtype == kDtypeBF16 && !aligned(logits, 16))
    return fail(SPECDEC_ERR_ARGUMENT, "bf16 logits must be 16-byte aligned");
  return ok();
}
}  // namespace specdec

extern "C" {

int specdec_version(void) { return 100; }

const char* specdec_last_error(void) { return g_last_error.c_str(); }

const char* specdec_status_string(int code) {
  switch (code) {
    case SPECDEC_OK: return "ok";
    case SPECDEC_ERR_ARGUMENT: return "invalid argument";
    case SPECDEC_ERR_VALUE: return "value out of domain";
    case SPECDEC_ERR_TARGET_RANGE: return "target id out of range";
    case SPECDEC_ERR_WORKSPACE: return "workspace too small";
    case SPECDEC_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

int specdec_set_launch_shape(int32_t kernel, int32_t shape, int32_t ctas_per_sm) {
  if (kernel < 0 || kernel > 3) return fail(SPECDEC_ERR_ARGUMENT, "unknown kernel id %d", kernel);
  if (shape < SPECDEC_SHAPE_DEFAULT || (shape > kMaxRingShape[kernel] && shape < kLdgShapeBase) ||
      shape > kLdgShapeBase + 4)
    return fail(SPECDEC_ERR_ARGUMENT, "unknown launch shape %d", shape);
  if (ctas_per_sm < 0 || ctas_per_sm > 32)
    return fail(SPECDEC_ERR_ARGUMENT, "ctas_per_sm must be in [0, 32], got %d", ctas_per_sm);
  g_shape[kernel].store(shape);
  g_cap[kernel].store(ctas_per_sm);
  return ok();
}

int specdec_set_block_queue(int32_t dynamic) {
  g_static_queue.store(dynamic ? 0 : 1);
  return ok();
}


int specdec_test_withhold_stage(int32_t launches) {
  if (launches < 0 || launches > 16) return fail(SPECDEC_ERR_ARGUMENT, "launches must be in [0, 16]");
  g_withhold_stage.store(launches);
  return ok();
}

int64_t specdec_launch_ctas(int32_t kernel, int64_t rows, int64_t V, int device) {
  if (kernel < 0 || kernel > 3 || rows <= 0 || V <= 0) return 0;
  const bool tma = use_tma(kernel, true);
  const int units = kernel_units(kernel, 0, tma, device);
  if (tma) return units;  // persistent ring CTAs
  return make_partition(rows, V, units, kMinChunk).grid;
}

// ---------------------------------------------------------------------------
// D-PACE
// ---------------------------------------------------------------------------

size_t specdec_dpace_scratch_bytes(int64_t N, int32_t B, int64_t V, int device) {
  if (N <= 0 || B <= 0 || V <= 0) return 256;
  // large enough for either kernel family (the call picks by pointer
  // alignment) and for either element type
  size_t best = dpace_layout(N, B, dpace_fwd_partition(N, B, V, false, device), 1).scratch;
  for (int dtype = kDtypeF32; dtype <= kDtypeBF16; ++dtype) {
    if (!(dtype == kDtypeF32 && !use_tma(SPECDEC_KERNEL_DPACE_FWD, true))) {
      const int nc = dpace_ring_consumers(ring_shape(SPECDEC_KERNEL_DPACE_FWD, dtype));
      const size_t b = dpace_layout(N, B, dpace_fwd_partition(N, B, V, true, device, dtype), nc).scratch;
      best = b > best ? b : best;
    }
  }
  return best;
}

size_t specdec_dpace_counter_bytes(int64_t N, int32_t B) {
  return dpace_counter_bytes(N > 0 ? N : 0, B > 0 ? B : 0);
}

size_t specdec_backward_counter_bytes(void) { return 256; }

}  // extern "C"

namespace {

// Where a forward whose finalize deferred its global loss keeps what the
// chained backward needs to finish it.
struct DeferredLoss {
  const float* seq_loss = nullptr;
  int* flag = nullptr;
};

int dpace_forward_impl(int dtype, const void* logits, const int64_t* targets, const float* mask, int64_t N,
                       int32_t B, int64_t V, float alpha, int32_t loss_type, int64_t n_global, float* loss,
                       float* loss_n, float* lse, float* scale, int32_t* status, void* scratch,
                       size_t scratch_bytes, void* counters, size_t counter_bytes, void* stream,
                       DeferredLoss* defer = nullptr) {
  const int rc = specdec::dpace_forward_check(dtype, logits, targets, N, B, V, alpha, loss_type, n_global, loss,
                                              lse, scale);
  if (rc != SPECDEC_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    // mean over an empty batch: NaN, as torch's mean of an empty tensor
    cudaError_t e = cudaMemsetAsync(loss, 0xff, sizeof(float), st);
    if (e == cudaSuccess && status) e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaMemsetAsync");
  }
  if (!scratch || !counters) return fail(SPECDEC_ERR_ARGUMENT, "null workspace pointer");
  if (!aligned(scratch, 256) || !aligned(counters, 16))
    return fail(SPECDEC_ERR_ARGUMENT, "misaligned workspace (scratch needs 256 B, counters 16 B)");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  const bool tma = dtype == kDtypeBF16 || use_tma(SPECDEC_KERNEL_DPACE_FWD, aligned(logits, 16));
  const Partition pt = dpace_fwd_partition(N, B, V, tma, dev, dtype);
  if (pt.grid <= 0) return fail(SPECDEC_ERR_CUDA, "occupancy query failed");
  const int shape = tma ? ring_shape(SPECDEC_KERNEL_DPACE_FWD, dtype) : kernel_shape(SPECDEC_KERNEL_DPACE_FWD, false);
  const int nc = tma ? dpace_ring_consumers(shape) : 1;
  const DpaceLayout L = dpace_layout(N, B, pt, nc);
  if (scratch_bytes < L.scratch)
    return fail(SPECDEC_ERR_WORKSPACE, "scratch needs %zu bytes, got %zu", L.scratch, scratch_bytes);
  if (counter_bytes < L.counters)
    return fail(SPECDEC_ERR_WORKSPACE, "counters need %zu bytes, got %zu", L.counters, counter_bytes);

  char* ws = static_cast<char*>(scratch);
  unsigned* cnt = static_cast<unsigned*>(counters);
  DpaceFwdArgs a;
  a.logits = logits;
  a.targets = targets;
  a.mask = mask;
  a.N = N;
  a.B = B;
  a.V = V;
  a.alpha = alpha;
  a.one_minus_alpha = (float)(1.0 - (double)alpha);
  a.loss_type = loss_type;
  a.n_global = n_global;
  a.inv_n = (float)(1.0 / (double)n_global);
  a.loss = loss;
  a.loss_n = loss_n;
  a.lse = lse;
  a.scale = scale;
  a.status = status;
  a.part = reinterpret_cast<float2*>(ws + L.part);
  a.xtgt = reinterpret_cast<float*>(ws + L.xtgt);
  a.seq_loss = reinterpret_cast<float*>(ws + L.seq_loss);
  a.nc = nc;
  a.done_cnt = cnt;
  a.flag = reinterpret_cast<int*>(cnt + 1);
  a.q_ctr = cnt + 2;
  a.q_retired = cnt + 3;
  a.q_dynamic = g_static_queue.load() ? 0 : 1;
  a.seq_cnt = cnt + kDpaceSeqWords;
  a.withhold_stage = tma ? take_withhold_stage() : 0;
  a.defer_loss = (defer != nullptr && tma) ? 1 : 0;
  if (defer) {
    defer->seq_loss = a.defer_loss ? a.seq_loss : nullptr;
    defer->flag = a.defer_loss ? a.flag : nullptr;
  }
  a.pt = pt;
  const cudaError_t e =
      tma ? dpace_fwd_ring_launch(dtype, shape, a, (int)pt.grid, st) : dpace_fwd_launch(shape, a, st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "dpace forward launch");
}

// The backward's counter block (specdec_backward_counter_bytes):
// [queue ctr][retired][flag]. `chained`: launched with programmatic dependent
// launch behind this library's own finalize, with row liveness from `mask`.
int dpace_backward_impl(int dtype, const void* logits, const int64_t* targets, const float* lse,
                        const float* scale, const float* dloss, void* dlogits, int64_t N, int32_t B, int64_t V,
                        int32_t* status, void* counters, size_t counter_bytes, void* stream,
                        bool status_merge = false, bool chained = false, const float* mask = nullptr,
                        const DeferredLoss* defer = nullptr, float* loss = nullptr, int64_t n_global = 1) {
  if (B < 1 || B > 32) return fail(SPECDEC_ERR_ARGUMENT, "kernel configured for block_size <= 32 (B=%d)", B);
  if (N < 0 || V < 0) return fail(SPECDEC_ERR_ARGUMENT, "negative shape");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0 || V == 0) {
    if (status && !status_merge) {
      const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
    return ok();
  }
  if (!logits || !targets || !lse || !scale || !dlogits)
    return fail(SPECDEC_ERR_ARGUMENT, "null input or output pointer");
  if (logits == dlogits) return fail(SPECDEC_ERR_ARGUMENT, "dlogits must not alias logits");
  if (dtype == kDtypeBF16 && !(aligned(logits, 16) && aligned(dlogits, 16)))
    return fail(SPECDEC_ERR_ARGUMENT, "bf16 logits and dlogits must be 16-byte aligned");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  const bool tma =
      dtype == kDtypeBF16 || use_tma(SPECDEC_KERNEL_DPACE_BWD, aligned(logits, 16) && aligned(dlogits, 16));
  const int units = kernel_units(SPECDEC_KERNEL_DPACE_BWD, 0, tma, dev, dtype);
  if (units <= 0) return fail(SPECDEC_ERR_CUDA, "occupancy query failed");
  const bool have_cnt = tma && counters != nullptr && counter_bytes >= 16 && aligned(counters, 16);
  // the 128-bit-load kernels have no waits; without a retire count the ring
  // kernel's CTAs only ever raise the word: start it at 0 on the stream
  if (status && !status_merge && !have_cnt) {
    const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  }
  DpaceBwdArgs a;
  a.logits = logits;
  a.targets = targets;
  a.lse = lse;
  a.scale = scale;
  a.dloss = dloss;
  a.dlogits = dlogits;
  unsigned* cnt = static_cast<unsigned*>(counters);
  a.q_ctr = have_cnt ? cnt : nullptr;
  a.q_retired = have_cnt ? cnt + 1 : nullptr;
  a.flag = have_cnt ? reinterpret_cast<int*>(cnt + 2) : nullptr;
  a.q_dynamic = have_cnt && !g_static_queue.load() ? 1 : 0;
  a.status = tma ? status : nullptr;
  a.status_merge = status_merge ? 1 : 0;
  a.chained = chained && tma ? 1 : 0;
  a.mask_liveness = a.chained;
  a.live_mask = mask;
  a.withhold_stage = tma ? take_withhold_stage() : 0;
  if (defer && defer->seq_loss && !(tma && have_cnt))
    return fail(SPECDEC_ERR_CUDA, "internal: a deferred loss needs the ring backward with counters");
  if (defer && defer->seq_loss) {  // finish the forward's loss when retiring
    a.loss = loss;
    a.seq_loss = defer->seq_loss;
    a.nseq = N;
    a.n_global = n_global;
    a.fwd_flag = defer->flag;
  }
  const int shape = tma ? ring_shape(SPECDEC_KERNEL_DPACE_BWD, dtype) : kernel_shape(SPECDEC_KERNEL_DPACE_BWD, false);
  a.pt = tma ? ring_partition(N * B, V, dpace_ring_block_elems(dtype, shape), units)
             : make_partition(N * B, V, units, kMinChunk);
  const cudaError_t e =
      tma ? dpace_bwd_ring_launch(dtype, shape, a, units, st) : dpace_bwd_launch(shape, a, st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "dpace backward launch");
}

int dpace_forward_backward_impl(int dtype, const void* logits, const int64_t* targets, const float* mask,
                                int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type, int64_t n_global,
                                float* loss, float* loss_n, float* lse, float* scale, void* dlogits,
                                int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                                size_t counter_bytes, void* stream) {
  if (B < 1 || B > 32) return fail(SPECDEC_ERR_ARGUMENT, "kernel configured for block_size <= 32 (B=%d)", B);
  if (N < 0 || V < 0) return fail(SPECDEC_ERR_ARGUMENT, "negative shape N=%lld V=%lld", (long long)N, (long long)V);
  if (!(alpha >= 0.f && alpha <= 1.f))
    return fail(SPECDEC_ERR_VALUE, "dpace_alpha must be in [0, 1], got %g", (double)alpha);
  if (loss_type < 0 || loss_type > 2) return fail(SPECDEC_ERR_VALUE, "unknown loss_type %d", loss_type);
  if (N > 0 && (n_global < N || n_global < 1))
    return fail(SPECDEC_ERR_ARGUMENT, "n_global (%lld) must be >= N (%lld)", (long long)n_global, (long long)N);
  if (!loss) return fail(SPECDEC_ERR_ARGUMENT, "loss output is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    cudaError_t e = cudaMemsetAsync(loss, 0xff, sizeof(float), st);
    if (e == cudaSuccess && status) e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaMemsetAsync");
  }
  if (V == 0) return fail(SPECDEC_ERR_TARGET_RANGE, "targets out of range [0, 0)");
  if (!logits || !targets || !lse || !scale || !dlogits || !scratch || !counters)
    return fail(SPECDEC_ERR_ARGUMENT, "null input, output or workspace pointer");
  if (logits == dlogits) return fail(SPECDEC_ERR_ARGUMENT, "dlogits must not alias logits");
  if (!aligned(targets, 8) || !aligned(lse, 4) || !aligned(scale, 4) || !aligned(scratch, 256) ||
      !aligned(counters, 16))
    return fail(SPECDEC_ERR_ARGUMENT, "misaligned pointer (scratch needs 256 B, counters 16 B)");
  const bool ptrs16 = aligned(logits, 16) && aligned(dlogits, 16);
  if (dtype == kDtypeBF16 && !ptrs16) return fail(SPECDEC_ERR_ARGUMENT, "bf16 logits and dlogits must be 16-byte aligned");
  // When both launches take the ring kernels, the finalize leaves the global
  // loss sum (and the status word) to the backward's last CTA, so the
  // backward, which waits for the finalize, is released sooner.
  const bool bwd_ring = dtype == kDtypeBF16 || use_tma(SPECDEC_KERNEL_DPACE_BWD, ptrs16);
  DeferredLoss defer;
  const int rc = dpace_forward_impl(dtype, logits, targets, mask, N, B, V, alpha, loss_type, n_global, loss, loss_n,
                                    lse, scale, status, scratch, scratch_bytes, counters, counter_bytes, stream,
                                    bwd_ring ? &defer : nullptr);
  if (rc != SPECDEC_OK) return rc;
  // The backward follows the finalize this call just enqueued, so it is
  // chained to it (programmatic dependent launch): its CTAs become resident
  // and start streaming logits -- rows chosen by the mask -- while the
  // finalize runs, and wait for lse / scale before computing. It uses its own
  // words of the counter block; its status only ever raises the forward's.
  unsigned* bcnt = static_cast<unsigned*>(counters) + kDpaceBwdWords;
  return dpace_backward_impl(dtype, logits, targets, lse, scale, nullptr, dlogits, N, B, V, status, bcnt,
                             counter_bytes - kDpaceBwdWords * sizeof(unsigned), stream, /*status_merge=*/true,
                             /*chained=*/true, mask, &defer, loss, n_global);
}

}  // namespace

extern "C" {

int specdec_dpace_forward_backward(const float* logits, const int64_t* targets, const float* mask, int64_t N,
                                   int32_t B, int64_t V, float alpha, int32_t loss_type, int64_t n_global,
                                   float* loss, float* loss_n, float* lse, float* scale, float* dlogits,
                                   int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                                   size_t counter_bytes, void* stream) {
  return dpace_forward_backward_impl(kDtypeF32, logits, targets, mask, N, B, V, alpha, loss_type, n_global, loss,
                                     loss_n, lse, scale, dlogits, status, scratch, scratch_bytes, counters,
                                     counter_bytes, stream);
}

int specdec_dpace_forward_backward_bf16(const uint16_t* logits, const int64_t* targets, const float* mask,
                                        int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                                        int64_t n_global, float* loss, float* loss_n, float* lse, float* scale,
                                        uint16_t* dlogits, int32_t* status, void* scratch, size_t scratch_bytes,
                                        void* counters, size_t counter_bytes, void* stream) {
  return dpace_forward_backward_impl(kDtypeBF16, logits, targets, mask, N, B, V, alpha, loss_type, n_global,
                                     loss, loss_n, lse, scale, dlogits, status, scratch, scratch_bytes, counters,
                                     counter_bytes, stream);
}

}  // extern "C"

namespace {
int scale_inplace_impl(int dtype, void* x, int64_t n, const float* factor, void* stream) {
  if (n < 0) return fail(SPECDEC_ERR_ARGUMENT, "negative length");
  if (n == 0) return ok();
  if (!x || !factor) return fail(SPECDEC_ERR_ARGUMENT, "null pointer");
  if (!aligned(x, 16)) return fail(SPECDEC_ERR_ARGUMENT, "x must be 16-byte aligned");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(SPECDEC_ERR_CUDA, "device query failed");
  const cudaError_t e = scale_inplace_launch(dtype, x, n, factor, sms * 4, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "scale launch");
}
}  // namespace

extern "C" {

int specdec_scale_inplace(float* x, int64_t n, const float* factor, void* stream) {
  return scale_inplace_impl(kDtypeF32, x, n, factor, stream);
}

int specdec_scale_inplace_bf16(uint16_t* x, int64_t n, const float* factor, void* stream) {
  return scale_inplace_impl(kDtypeBF16, x, n, factor, stream);
}

int specdec_dpace_forward(const float* logits, const int64_t* targets, const float* mask,
                          int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                          int64_t n_global, float* loss, float* loss_n, float* lse, float* scale,
                          int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                          size_t counter_bytes, void* stream) {
  return dpace_forward_impl(kDtypeF32, logits, targets, mask, N, B, V, alpha, loss_type, n_global, loss, loss_n,
                            lse, scale, status, scratch, scratch_bytes, counters, counter_bytes, stream);
}

int specdec_dpace_forward_bf16(const uint16_t* logits, const int64_t* targets, const float* mask,
                               int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                               int64_t n_global, float* loss, float* loss_n, float* lse, float* scale,
                               int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                               size_t counter_bytes, void* stream) {
  return dpace_forward_impl(kDtypeBF16, logits, targets, mask, N, B, V, alpha, loss_type, n_global, loss, loss_n,
                            lse, scale, status, scratch, scratch_bytes, counters, counter_bytes, stream);
}

int specdec_dpace_backward(const float* logits, const int64_t* targets, const float* lse,
                           const float* scale, const float* dloss, float* dlogits, int64_t N,
                           int32_t B, int64_t V, int32_t* status, void* counters, size_t counter_bytes,
                           void* stream) {
  return dpace_backward_impl(kDtypeF32, logits, targets, lse, scale, dloss, dlogits, N, B, V, status, counters,
                             counter_bytes, stream);
}

int specdec_dpace_backward_bf16(const uint16_t* logits, const int64_t* targets, const float* lse,
                                const float* scale, const float* dloss, uint16_t* dlogits, int64_t N,
                                int32_t B, int64_t V, int32_t* status, void* counters, size_t counter_bytes,
                                void* stream) {
  return dpace_backward_impl(kDtypeBF16, logits, targets, lse, scale, dloss, dlogits, N, B, V, status, counters,
                             counter_bytes, stream);
}

// ---------------------------------------------------------------------------
// DFlash
// ---------------------------------------------------------------------------

size_t specdec_dflash_scratch_bytes(int64_t N, int32_t B, int64_t V, int device) {
  if (N <= 0 || B <= 0 || V <= 0) return 256;
  // large enough for either kind, either kernel family and either element type
  size_t best = 0;
  for (int kind = 0; kind < 2; ++kind) {
    const size_t a = dflash_layout(N, B, dflash_fwd_partition(N, B, V, kind, false, device), 1).scratch;
    best = a > best ? a : best;
    for (int dtype = kDtypeF32; dtype <= kDtypeBF16; ++dtype) {
      if (dtype == kDtypeF32 && !use_tma(SPECDEC_KERNEL_DFLASH_FWD, true)) continue;
      const int nc = dflash_ring_consumers(ring_shape(SPECDEC_KERNEL_DFLASH_FWD, dtype));
      const size_t b = dflash_layout(N, B, dflash_fwd_partition(N, B, V, kind, true, device, dtype), nc).scratch;
      best = b > best ? b : best;
    }
  }
  return best;
}

size_t specdec_dflash_counter_bytes(int64_t N, int32_t B) {
  const int64_t R = (N > 0 && B > 0) ? N * B : 0;
  return align256(16 + size_t(R) * sizeof(unsigned));
}

}  // extern "C"

namespace {

int dflash_forward_impl(int dtype, const void* logits, const void* target_logits, const float* mask, int64_t N,
                        int32_t B, int64_t V, int32_t block_size, float gamma, int32_t sample_from_anchor,
                        int32_t kind, int64_t n_global, float* loss, float* loss_rows, float* scale, float* logzq,
                        float* logzp, int64_t* target_id, void* scratch, size_t scratch_bytes, void* counters,
                        size_t counter_bytes, void* stream) {
  // Mirrors models/dflash/loss.py:178-191 (_check) order of failures.
  if (N < 0 || B < 0 || V < 0) return fail(SPECDEC_ERR_ARGUMENT, "negative shape");
  if (V > INT32_MAX) return fail(SPECDEC_ERR_ARGUMENT, "V must be < 2^31");
  if (B > 0 && (block_size < 1 || block_size > B))
    return fail(SPECDEC_ERR_ARGUMENT, "block_size must be in [1, B] (block_size=%d, B=%d)", block_size, B);
  if (!(gamma > 0.f)) return fail(SPECDEC_ERR_VALUE, "gamma must be > 0, got %g", (double)gamma);
  if (kind != SPECDEC_DFLASH_KL && kind != SPECDEC_DFLASH_CE)
    return fail(SPECDEC_ERR_VALUE, "unknown loss kind %d, expected 0 (kl) or 1 (ce)", kind);
  if (N > 0 && (n_global < N)) return fail(SPECDEC_ERR_ARGUMENT, "n_global must be >= N");
  if (!loss) return fail(SPECDEC_ERR_ARGUMENT, "loss output is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0 || B == 0 || V == 0) {
    // sum over no rows / N: NaN for N == 0 (0/0), 0 otherwise
    const cudaError_t e = cudaMemsetAsync(loss, N == 0 ? 0xff : 0, sizeof(float), st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaMemsetAsync");
  }
  if (!logits || !target_logits || !scale || !logzq || !logzp || !scratch || !counters)
    return fail(SPECDEC_ERR_ARGUMENT, "null input, output or workspace pointer");
  if (kind == SPECDEC_DFLASH_CE && !target_id) return fail(SPECDEC_ERR_ARGUMENT, "CE needs target_id output");
  if (!aligned(scratch, 256) || !aligned(counters, 16))
    return fail(SPECDEC_ERR_ARGUMENT, "misaligned workspace (scratch 256 B, counters 16 B)");
  if (dtype == kDtypeBF16 && !(aligned(logits, 16) && aligned(target_logits, 16)))
    return fail(SPECDEC_ERR_ARGUMENT, "bf16 logits and target_logits must be 16-byte aligned");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  const bool tma = dtype == kDtypeBF16 ||
                   use_tma(SPECDEC_KERNEL_DFLASH_FWD, aligned(logits, 16) && aligned(target_logits, 16));
  const Partition pt = dflash_fwd_partition(N, B, V, kind, tma, dev, dtype);
  if (pt.grid <= 0) return fail(SPECDEC_ERR_CUDA, "occupancy query failed");
  const int shape =
      tma ? ring_shape(SPECDEC_KERNEL_DFLASH_FWD, dtype) : kernel_shape(SPECDEC_KERNEL_DFLASH_FWD, false);
  const int nc = tma ? dflash_ring_consumers(shape) : 1;
  const DflashLayout L = dflash_layout(N, B, pt, nc);
  if (scratch_bytes < L.scratch)
    return fail(SPECDEC_ERR_WORKSPACE, "scratch needs %zu bytes, got %zu", L.scratch, scratch_bytes);
  if (counter_bytes < L.counters)
    return fail(SPECDEC_ERR_WORKSPACE, "counters need %zu bytes, got %zu", L.counters, counter_bytes);
  char* ws = static_cast<char*>(scratch);
  unsigned* cnt = static_cast<unsigned*>(counters);
  DflashFwdArgs a;
  a.logits = logits;
  a.target_logits = target_logits;
  a.mask = mask;
  a.N = N;
  a.B = B;
  a.V = V;
  a.block_size = block_size;
  a.gamma = gamma;
  a.sfa = sample_from_anchor ? 1 : 0;
  a.kind = kind;
  a.n_global = n_global;
  a.loss = loss;
  a.loss_rows = loss_rows;
  a.scale = scale;
  a.logzq = logzq;
  a.logzp = logzp;
  a.target_id = target_id;
  a.part = reinterpret_cast<DfPiece*>(ws + L.part);
  a.row_loss = reinterpret_cast<float*>(ws + L.row_loss);
  a.seq_loss = reinterpret_cast<float*>(ws + L.seq_loss);
  a.done_cnt = cnt;
  a.flag = reinterpret_cast<int*>(cnt + 1);
  a.q_ctr = cnt + 2;
  a.q_retired = cnt + 3;
  a.q_dynamic = g_static_queue.load() ? 0 : 1;
  a.row_cnt = cnt + 4;
  a.nc = nc;
  a.withhold_stage = tma ? take_withhold_stage() : 0;
  a.pt = pt;
  const cudaError_t e =
      tma ? dflash_fwd_ring_launch(dtype, shape, a, (int)pt.grid, st) : dflash_fwd_launch(shape, a, st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "dflash forward launch");
}

int dflash_backward_impl(int dtype, const void* logits, const void* target_logits, const float* scale,
                         const float* logzq, const float* logzp, const int64_t* target_id, const float* dloss,
                         void* dlogits, int64_t N, int32_t B, int64_t V, int32_t kind, int32_t* status,
                         void* counters, size_t counter_bytes, void* stream) {
  if (N < 0 || B < 0 || V < 0) return fail(SPECDEC_ERR_ARGUMENT, "negative shape");
  if (kind != SPECDEC_DFLASH_KL && kind != SPECDEC_DFLASH_CE)
    return fail(SPECDEC_ERR_VALUE, "unknown loss kind %d", kind);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0 || B == 0 || V == 0) {
    if (status) {
      const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
    return ok();
  }
  if (!logits || !scale || !logzq || !logzp || !dlogits)
    return fail(SPECDEC_ERR_ARGUMENT, "null input or output pointer");
  if (kind == SPECDEC_DFLASH_KL && !target_logits) return fail(SPECDEC_ERR_ARGUMENT, "KL needs target_logits");
  if (kind == SPECDEC_DFLASH_CE && !target_id) return fail(SPECDEC_ERR_ARGUMENT, "CE needs target_id");
  if (logits == dlogits || target_logits == dlogits)
    return fail(SPECDEC_ERR_ARGUMENT, "dlogits must not alias an input");
  const bool ptrs16 = aligned(logits, 16) && aligned(dlogits, 16) &&
                      (kind == SPECDEC_DFLASH_CE || aligned(target_logits, 16));
  if (dtype == kDtypeBF16 && !ptrs16)
    return fail(SPECDEC_ERR_ARGUMENT, "bf16 logits, target_logits and dlogits must be 16-byte aligned");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  const bool tma = dtype == kDtypeBF16 || use_tma(SPECDEC_KERNEL_DFLASH_BWD, ptrs16);
  const int ctas = kernel_units(SPECDEC_KERNEL_DFLASH_BWD, kind, tma, dev, dtype);
  if (ctas <= 0) return fail(SPECDEC_ERR_CUDA, "occupancy query failed");
  const bool have_cnt = tma && counters != nullptr && counter_bytes >= 16 && aligned(counters, 16);
  if (status && !have_cnt) {
    const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  }
  DflashBwdArgs a;
  a.logits = logits;
  a.target_logits = target_logits;
  a.scale = scale;
  a.logzq = logzq;
  a.logzp = logzp;
  a.target_id = target_id;
  a.dloss = dloss;
  a.dlogits = dlogits;
  a.kind = kind;
  unsigned* cnt = static_cast<unsigned*>(counters);
  a.q_ctr = have_cnt ? cnt : nullptr;
  a.q_retired = have_cnt ? cnt + 1 : nullptr;
  a.flag = have_cnt ? reinterpret_cast<int*>(cnt + 2) : nullptr;
  a.q_dynamic = have_cnt && !g_static_queue.load() ? 1 : 0;
  a.status = tma ? status : nullptr;
  a.status_merge = 0;
  a.withhold_stage = tma ? take_withhold_stage() : 0;
  const int shape =
      tma ? ring_shape(SPECDEC_KERNEL_DFLASH_BWD, dtype) : kernel_shape(SPECDEC_KERNEL_DFLASH_BWD, false);
  a.pt = tma ? ring_partition(N * B, V, dflash_ring_block_elems(dtype, shape), ctas)
             : make_partition(N * B, V, ctas, kMinChunk);
  const cudaError_t e =
      tma ? dflash_bwd_ring_launch(dtype, shape, a, ctas, st) : dflash_bwd_launch(shape, a, st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "dflash backward launch");
}

}  // namespace

extern "C" {

int specdec_dflash_forward(const float* logits, const float* target_logits, const float* mask,
                           int64_t N, int32_t B, int64_t V, int32_t block_size, float gamma,
                           int32_t sample_from_anchor, int32_t kind, int64_t n_global, float* loss,
                           float* loss_rows, float* scale, float* logzq, float* logzp,
                           int64_t* target_id, void* scratch, size_t scratch_bytes, void* counters,
                           size_t counter_bytes, void* stream) {
  return dflash_forward_impl(kDtypeF32, logits, target_logits, mask, N, B, V, block_size, gamma,
                             sample_from_anchor, kind, n_global, loss, loss_rows, scale, logzq, logzp, target_id,
                             scratch, scratch_bytes, counters, counter_bytes, stream);
}

int specdec_dflash_forward_bf16(const uint16_t* logits, const uint16_t* target_logits, const float* mask,
                                int64_t N, int32_t B, int64_t V, int32_t block_size, float gamma,
                                int32_t sample_from_anchor, int32_t kind, int64_t n_global, float* loss,
                                float* loss_rows, float* scale, float* logzq, float* logzp,
                                int64_t* target_id, void* scratch, size_t scratch_bytes, void* counters,
                                size_t counter_bytes, void* stream) {
  return dflash_forward_impl(kDtypeBF16, logits, target_logits, mask, N, B, V, block_size, gamma,
                             sample_from_anchor, kind, n_global, loss, loss_rows, scale, logzq, logzp, target_id,
                             scratch, scratch_bytes, counters, counter_bytes, stream);
}

int specdec_dflash_backward(const float* logits, const float* target_logits, const float* scale,
                            const float* logzq, const float* logzp, const int64_t* target_id,
                            const float* dloss, float* dlogits, int64_t N, int32_t B, int64_t V,
                            int32_t kind, int32_t* status, void* counters, size_t counter_bytes, void* stream) {
  return dflash_backward_impl(kDtypeF32, logits, target_logits, scale, logzq, logzp, target_id, dloss, dlogits,
                              N, B, V, kind, status, counters, counter_bytes, stream);
}

int specdec_dflash_backward_bf16(const uint16_t* logits, const uint16_t* target_logits, const float* scale,
                                 const float* logzq, const float* logzp, const int64_t* target_id,
                                 const float* dloss, uint16_t* dlogits, int64_t N, int32_t B, int64_t V,
                                 int32_t kind, int32_t* status, void* counters, size_t counter_bytes,
                                 void* stream) {
  return dflash_backward_impl(kDtypeBF16, logits, target_logits, scale, logzq, logzp, target_id, dloss,
                              dlogits, N, B, V, kind, status, counters, counter_bytes, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// DFlash drafter layers
// ---------------------------------------------------------------------------

extern "C" {

int specdec_rmsnorm_forward(const void* x, const float* weight, void* y, float* rstd, int64_t rows, int32_t D,
                            float eps, int32_t dtype, void* stream) {
  if (rows < 0 || D < 1) return fail(SPECDEC_ERR_ARGUMENT, "bad shape rows=%lld D=%d", (long long)rows, D);
  if (dtype != kDtypeF32 && dtype != kDtypeBF16) return fail(SPECDEC_ERR_ARGUMENT, "unknown dtype %d", dtype);
  if (!(eps >= 0.f)) return fail(SPECDEC_ERR_VALUE, "eps must be >= 0, got %g", (double)eps);
  if (rows == 0) return ok();
  if (!x || !weight || !y) return fail(SPECDEC_ERR_ARGUMENT, "null input or output pointer");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(SPECDEC_ERR_CUDA, "device query failed");
  const cudaError_t e = rmsnorm_fwd_launch(dtype, x, weight, y, rstd, rows, D, eps, sms,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "rmsnorm forward launch");
}

size_t specdec_rmsnorm_workspace_bytes(int64_t rows, int32_t D, int device) {
  if (rows <= 0 || D <= 0) return 256;
  return align256((size_t)rmsnorm_bwd_ctas(rows, D, device) * (size_t)D * sizeof(float));
}

int specdec_rmsnorm_backward(const void* x, const float* weight, const float* rstd, const void* dy, void* dx,
                             float* dweight, int64_t rows, int32_t D, int32_t dtype, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (rows < 0 || D < 1) return fail(SPECDEC_ERR_ARGUMENT, "bad shape rows=%lld D=%d", (long long)rows, D);
  if (dtype != kDtypeF32 && dtype != kDtypeBF16) return fail(SPECDEC_ERR_ARGUMENT, "unknown dtype %d", dtype);
  if (rmsnorm_bwd_warps(D) < 1) return fail(SPECDEC_ERR_ARGUMENT, "D=%d too large for the backward", D);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (!dweight) return fail(SPECDEC_ERR_ARGUMENT, "null dweight");
    const cudaError_t e = cudaMemsetAsync(dweight, 0, (size_t)D * sizeof(float), st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaMemsetAsync");
  }
  if (!x || !weight || !rstd || !dy || !dx || !dweight || !workspace)
    return fail(SPECDEC_ERR_ARGUMENT, "null input, output or workspace pointer");
  const int dev = current_device();
  if (dev < 0) return fail(SPECDEC_ERR_CUDA, "cudaGetDevice failed");
  const int ctas = rmsnorm_bwd_ctas(rows, D, dev);
  if (ctas <= 0) return fail(SPECDEC_ERR_CUDA, "device query failed");
  const size_t need = (size_t)ctas * (size_t)D * sizeof(float);
  if (workspace_bytes < need) return fail(SPECDEC_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  const cudaError_t e = rmsnorm_bwd_launch(dtype, x, weight, rstd, dy, dx, dweight, static_cast<float*>(workspace),
                                           rows, D, ctas, st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "rmsnorm backward launch");
}

int specdec_dflash_attention_forward(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                                     float* lse, int32_t batch, int32_t T, int32_t heads, int32_t head_dim,
                                     int32_t n_ctx, float scale, int32_t* status, void* stream) {
  if (head_dim != 64) return fail(SPECDEC_ERR_ARGUMENT, "head_dim must be 64, got %d", head_dim);
  if (batch < 0 || T < 0 || heads < 1) return fail(SPECDEC_ERR_ARGUMENT, "bad shape");
  if (n_ctx < 0 || n_ctx > T) return fail(SPECDEC_ERR_ARGUMENT, "n_ctx must be in [0, T] (n_ctx=%d, T=%d)", n_ctx, T);
  if ((int64_t)batch * heads > INT32_MAX) return fail(SPECDEC_ERR_ARGUMENT, "batch * heads must fit in int32");
  if ((T + 127) / 128 > 65535) return fail(SPECDEC_ERR_ARGUMENT, "T must be <= 65535 * 128");
  if (!(scale > 0.f)) return fail(SPECDEC_ERR_VALUE, "scale must be > 0");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (batch == 0 || T == 0) return ok();
  if (!q || !k || !v || !o || !lse) return fail(SPECDEC_ERR_ARGUMENT, "null input or output pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(o, 16))
    return fail(SPECDEC_ERR_ARGUMENT, "q, k, v and o must be 16-byte aligned");
  const cudaError_t e =
      dflash_attn_fwd_launch(q, k, v, o, lse, batch, T, heads, n_ctx, scale, status, take_withhold_stage(), st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "attention forward launch");
}

size_t specdec_dflash_attention_workspace_bytes(int32_t batch, int32_t T, int32_t heads) {
  if (batch <= 0 || T <= 0 || heads <= 0) return 256;
  return align256((size_t)batch * (size_t)heads * (size_t)T * sizeof(float));
}

int specdec_dflash_attention_backward(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                                      const float* lse, const uint16_t* dout, uint16_t* dq, uint16_t* dk,
                                      uint16_t* dv, int32_t batch, int32_t T, int32_t heads, int32_t head_dim,
                                      int32_t n_ctx, float scale, int32_t* status, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (head_dim != 64) return fail(SPECDEC_ERR_ARGUMENT, "head_dim must be 64, got %d", head_dim);
  if (batch < 0 || T < 0 || heads < 1) return fail(SPECDEC_ERR_ARGUMENT, "bad shape");
  if (n_ctx < 0 || n_ctx > T) return fail(SPECDEC_ERR_ARGUMENT, "n_ctx must be in [0, T] (n_ctx=%d, T=%d)", n_ctx, T);
  if ((int64_t)batch * heads > INT32_MAX) return fail(SPECDEC_ERR_ARGUMENT, "batch * heads must fit in int32");
  if ((T + 127) / 128 > 65535) return fail(SPECDEC_ERR_ARGUMENT, "T must be <= 65535 * 128");
  if (!(scale > 0.f)) return fail(SPECDEC_ERR_VALUE, "scale must be > 0");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (batch == 0 || T == 0) return ok();
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv || !workspace)
    return fail(SPECDEC_ERR_ARGUMENT, "null input, output or workspace pointer");
  const void* ptrs[] = {q, k, v, o, dout, dq, dk, dv};
  for (const void* p : ptrs)
    if (!aligned(p, 16)) return fail(SPECDEC_ERR_ARGUMENT, "attention tensors must be 16-byte aligned");
  const size_t need = (size_t)batch * (size_t)heads * (size_t)T * sizeof(float);
  if (workspace_bytes < need) return fail(SPECDEC_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  const cudaError_t e = dflash_attn_bwd_launch(q, k, v, o, lse, dout, dq, dk, dv, static_cast<float*>(workspace), batch,
                                               T, heads, n_ctx, scale, status, take_withhold_stage(), st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "attention backward launch");
}

}  // extern "C"
