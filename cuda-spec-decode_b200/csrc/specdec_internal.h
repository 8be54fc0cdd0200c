// Internal launch interface between the C-ABI layer (specdec_abi.cu) and the
// kernels (dpace_kernels.cu, dflash_kernels.cu). Not part of the public ABI.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "specdec_common.cuh"

namespace specdec {

constexpr int kStatusOk = 0;
constexpr int kStatusTargetRange = 3;  // equals SPECDEC_ERR_TARGET_RANGE in include/specdec.h
// kStatusTimeout (= SPECDEC_ERR_CUDA) is defined in bulk_copy.cuh

constexpr int kKindKL = 0;
constexpr int kKindCE = 1;

// Element type of the logits (and of the gradient written for them).
constexpr int kDtypeF32 = 0;
constexpr int kDtypeBF16 = 1;

// Per-piece partial of the DFlash forward (32 bytes, two float4 stores).
struct alignas(16) DfPiece {
  float m2q, sq, m2p, sp, t, bx, bl;
  int bi;
};

struct DpaceFwdArgs {
  const void* logits;      // [N, B, V] float, or bf16 for the bf16 ring kernels
  const int64_t* targets;  // [N, B]
  const float* mask;       // [N, B] or null (all positions scored); scored iff > 0
  int64_t N;               // sequences in this launch
  int B;                   // positions per sequence, 1..32
  int64_t V;
  float alpha, one_minus_alpha;
  int loss_type;           // 0 = S (dpace), 1 = P (cumulative confidence), 2 = S/P (continuation value)
  int64_t n_global;        // divisor: sequences across all shards
  float inv_n;             // 1 / n_global
  float* loss;             // [1]  sum_n loss_n / n_global
  float* loss_n;           // [N]  sum_j w_j * ce_j, or null
  float* lse;              // [N, B]
  float* scale;            // [N, B]  w_j / n_global
  int* status;             // [1]  device status word, or null
  // workspace
  float2* part;            // [N*B, pt.pmax, nc] (max, sum) per row piece (and consumer warp)
  float* xtgt;             // [N*B] logit at the target id
  float* seq_loss;         // [N]
  unsigned* seq_cnt;       // [N]  128-bit-load kernel: CTA pieces per sequence; zero on entry/exit
  unsigned* done_cnt;      // [1]  zero on entry, zero on exit
  int* flag;               // [1]  zero on entry, zero on exit
  unsigned* q_ctr;         // [1]  ring kernel block queue; zero on entry/exit
  unsigned* q_retired;     // [1]
  int q_dynamic;           // 1: atomic block queue, 0: static interleave
  int nc;                  // partials per (row, slot): consumer warps (ring) or 1
  int withhold_stage;      // failure-detection tests: CTA 0 never posts its first stage
  int defer_loss = 0;      // 1: the chained backward sums seq_loss into loss and writes status
  Partition pt;            // ring kernel: chunk = block length, pmax from it
};

struct DpaceBwdArgs {
  const void* logits;      // element type as the forward's
  const int64_t* targets;
  const float* lse;
  const float* scale;
  const float* dloss;      // [1] upstream gradient, or null for 1
  void* dlogits;           // element type of logits
  int* status = nullptr;   // [1] or null: 0, or kStatusTimeout if a wait expired
  int status_merge = 0;    // 1: only ever raise *status (it holds the forward's word)
  int* flag;               // [1] or null (no counters): bit 2 set if a copy wait timed out
  unsigned* q_ctr;         // ring kernel block queue word
  unsigned* q_retired;     // null: no counters (static interleave, no retire count)
  int q_dynamic;
  int mask_liveness = 0;   // 1: rows are read iff live_mask > 0 (null: all), known before lse/scale
  const float* live_mask = nullptr;  // [N, B] position mask, with mask_liveness
  int chained = 0;         // 1: launched with programmatic dependent launch after the finalize
  int withhold_stage = 0;  // failure-detection tests: CTA 0 never posts its first stage
  // loss epilogue of a forward whose finalize deferred it (null loss: none)
  float* loss = nullptr;   // [1] sum_n seq_loss[n] / n_global, NaN if the forward timed out
  const float* seq_loss = nullptr;  // [nseq] the finalize's per-sequence losses
  int64_t nseq = 0;
  int64_t n_global = 1;
  int* fwd_flag = nullptr; // the forward's flag word: bit 1 target out of range, bit 2 timeout
  Partition pt;
};

struct DflashFwdArgs {
  const void* logits;          // draft [N, B, V] (float, or bf16 for the bf16 ring kernels)
  const void* target_logits;   // verifier [N, B, V], same element type
  const float* mask;           // [N, B] raw float mask, or null for all ones
  int64_t N;
  int B;
  int64_t V;
  int block_size;              // decay position = j % block_size
  float gamma;
  int sfa;                     // sample_from_anchor
  int kind;                    // kKindKL or kKindCE
  int64_t n_global;
  float* loss;                 // [1]
  float* loss_rows;            // [N*B] or null
  float* scale;                // [N*B]
  float* logzq;                // [N*B]
  float* logzp;                // [N*B]
  int64_t* target_id;          // [N*B] argmax(verifier) for CE, or null
  // workspace
  DfPiece* part;               // [N*B, pt.pmax, nc]
  float* row_loss;             // [N*B] 128-bit-load kernel
  float* seq_loss;             // [N]   ring kernel
  unsigned* row_cnt;           // [N*B] 128-bit-load kernel; zero on entry, zero on exit
  unsigned* done_cnt;          // [1]   zero on entry, zero on exit
  int* flag;                   // [1]   bit 2: a copy wait timed out
  unsigned* q_ctr;             // ring kernel block queue; zero on entry/exit
  unsigned* q_retired;
  int q_dynamic;
  int nc;                      // partials per (row, slot)
  int withhold_stage;          // failure-detection tests: CTA 0 never posts its first stage
  Partition pt;                // ring kernel: chunk = block length
};

struct DflashBwdArgs {
  const void* logits;
  const void* target_logits;   // read for KL only
  const float* scale;
  const float* logzq;
  const float* logzp;
  const int64_t* target_id;    // read for CE only
  const float* dloss;
  void* dlogits;               // element type of logits
  int kind;
  int* status = nullptr;       // [1] or null: 0, or kStatusTimeout if a wait expired
  int status_merge = 0;        // 1: only ever raise *status
  int* flag;                   // [1] or null (no counters)
  unsigned* q_ctr;             // ring kernel block queue word
  unsigned* q_retired;         // null: no counters (static interleave, no retire count)
  int q_dynamic;
  int withhold_stage = 0;      // failure-detection tests: CTA 0 never posts its first stage
  // no loss epilogue (the DFlash forward always completes its own loss)
  float* loss = nullptr;
  const float* seq_loss = nullptr;
  int64_t nseq = 0;
  int64_t n_global = 1;
  int* fwd_flag = nullptr;
  Partition pt;
};

// Launch shapes: 0 = default; others select alternative (threads, unroll)
// instantiations (see the switch tables in the kernel files).
int dpace_fwd_ctas(int shape, int device, int cap_per_sm);
int dpace_bwd_ctas(int shape, int device, int cap_per_sm);
cudaError_t dpace_fwd_launch(int shape, const DpaceFwdArgs& a, cudaStream_t st);
cudaError_t dpace_bwd_launch(int shape, const DpaceBwdArgs& a, cudaStream_t st);

// Warp-specialized ring kernels (dpace_ring.cu); sizes in CTAs. `dtype` is
// kDtypeF32 or kDtypeBF16; a bf16 shape moves the same bytes per stage as the
// float shape of the same number (twice the elements).
int dpace_ring_block_elems(int dtype, int shape);
int dpace_ring_stage_elems(int dtype, int shape);
// start of the D-PACE forward's one-stage queue blocks for E elements in
// blocks of BL (-1: none)
int64_t dpace_fwd_split(int64_t E, int64_t BL);
int dpace_ring_consumers(int shape);
int dpace_fwd_ring_ctas(int dtype, int shape, int device, int cap_per_sm);
int dpace_bwd_ring_ctas(int dtype, int shape, int device, int cap_per_sm);
cudaError_t dpace_fwd_ring_launch(int dtype, int shape, const DpaceFwdArgs& a, int ctas, cudaStream_t st);
cudaError_t dpace_bwd_ring_launch(int dtype, int shape, const DpaceBwdArgs& a, int ctas, cudaStream_t st);

// Warp-specialized ring kernels (dflash_ring.cu); sizes in CTAs.
int dflash_ring_block_elems(int dtype, int shape);
int dflash_ring_consumers(int shape);
int dflash_fwd_ring_ctas(int dtype, int kind, int shape, int device, int cap_per_sm);
int dflash_bwd_ring_ctas(int dtype, int kind, int shape, int device, int cap_per_sm);
cudaError_t dflash_fwd_ring_launch(int dtype, int shape, const DflashFwdArgs& a, int ctas, cudaStream_t st);
cudaError_t dflash_bwd_ring_launch(int dtype, int shape, const DflashBwdArgs& a, int ctas, cudaStream_t st);

// In-place dloss scaling of a gradient (dpace_scale.cu).
cudaError_t scale_inplace_launch(int dtype, void* x, int64_t n, const float* factor, int ctas, cudaStream_t st);

// RMSNorm of the drafter (drafter_norm.cu).
int rmsnorm_bwd_ctas(int64_t rows, int D, int device);
int rmsnorm_bwd_warps(int D);
cudaError_t rmsnorm_fwd_launch(int dtype, const void* x, const float* w, void* y, float* rstd, int64_t rows, int D,
                               float eps, int sms, cudaStream_t st);
cudaError_t rmsnorm_bwd_launch(int dtype, const void* x, const float* w, const float* rstd, const void* dy,
                               void* dx, float* dw, float* part, int64_t rows, int D, int ctas, cudaStream_t st);

// Attention of the drafter on the tensor cores (drafter_attention.cu):
// bf16 q/k/v/o [B, T, H, 64], lse fp32 [B, H, T].
cudaError_t dflash_attn_fwd_launch(const void* q, const void* k, const void* v, void* o, float* lse, int batch, int T,
                                   int H, int n_ctx, float scale, int* status, int withhold, cudaStream_t st);
// Backward: delta [B, H, T] fp32 is scratch written by the first kernel.
cudaError_t dflash_attn_bwd_launch(const void* q, const void* k, const void* v, const void* o, const float* lse,
                                   const void* dO, void* dq, void* dk, void* dv, float* delta, int batch, int T, int H,
                                   int n_ctx, float scale, int* status, int withhold, cudaStream_t st);

// Sets the calling thread's specdec_last_error() text.
void set_last_error(const char* msg);

// specdec_dpace_forward's checks that need no workspace (status code; sets
// the error text).
int dpace_forward_check(int dtype, const void* logits, const int64_t* targets, int64_t N, int32_t B, int64_t V,
                        float alpha, int32_t loss_type, int64_t n_global, const float* loss, const float* lse,
                        const float* scale);

int dflash_fwd_ctas(int kind, int shape, int device, int cap_per_sm);
int dflash_bwd_ctas(int kind, int shape, int device, int cap_per_sm);
cudaError_t dflash_fwd_launch(int shape, const DflashFwdArgs& a, cudaStream_t st);
cudaError_t dflash_bwd_launch(int shape, const DflashBwdArgs& a, cudaStream_t st);

}  // namespace specdec
