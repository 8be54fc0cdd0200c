/*
 * specdec.h -- C ABI of the B200 drafter-loss library (libspecdec.so).
 *
 * Fused training losses for speculative-decoding drafters over fp32 (or
 * bf16) logits [N, B, V] (N sequences, B draft positions, V vocabulary):
 *   - D-PACE: cross entropy weighted by the detached, alpha-smoothed
 *     acceptance prefix/suffix scan of each sequence;
 *   - DFlash: KL(softmax(verifier) || softmax(draft)) or CE against
 *     argmax(verifier), weighted by an exponential slot decay.
 *
 * Conventions (all entry points):
 *   - every pointer is a device pointer unless stated otherwise; tensors are
 *     C-contiguous; no entry point allocates device memory or synchronises;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); all work is
 *     enqueued on it;
 *   - return value: SPECDEC_OK or an error code; specdec_last_error() gives a
 *     message for the calling thread;
 *   - `scratch` is device memory of at least the queried size with no
 *     initialisation requirement; `counters` is device memory of at least the
 *     queried size that must be all-zero before the first call and is left
 *     all-zero by every call that completes on the GPU (zero it once, e.g.
 *     cudaMemset at allocation, then reuse). Calls that may run concurrently
 *     on the GPU must not share scratch or counters.
 *   - results are bitwise repeatable: all reductions run in a fixed order.
 *
 * Each entry point cites the reference interface it replaces
 * (harvestingmoon/cuda-spec-decode, path:line).
 */
#ifndef SPECDEC_H_
#define SPECDEC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SPECDEC_OK 0
#define SPECDEC_ERR_ARGUMENT 1     /* shape, pointer or size contract broken (reference: AssertionError) */
#define SPECDEC_ERR_VALUE 2        /* alpha, loss_type, gamma or kind out of domain (reference: ValueError) */
#define SPECDEC_ERR_TARGET_RANGE 3 /* a target id outside [0, V); reported through *status on the device */
#define SPECDEC_ERR_WORKSPACE 4    /* scratch or counters smaller than the queried size */
#define SPECDEC_ERR_CUDA 5         /* CUDA runtime or launch failure */

/* D-PACE loss_type values (reference: losses/dpace.py:148 _LOSS_TYPES). */
#define SPECDEC_DPACE 0                      /* "dpace": w = S_j */
#define SPECDEC_DPACE_CUMULATIVE_CONFIDENCE 1 /* "dpace-cumulative-confidence-only": w = P_j */
#define SPECDEC_DPACE_CONTINUATION_VALUE 2   /* "dpace-continuation-value-only": w = S_j / P_j */

/* DFlash kind values (reference: models/dflash/loss.py:169 _KINDS). */
#define SPECDEC_DFLASH_KL 0
#define SPECDEC_DFLASH_CE 1

/* Library version, major * 10000 + minor * 100 + patch. */
int specdec_version(void);

/* Message for the last error on the calling thread ("" when none). */
const char* specdec_last_error(void);

/* Static name of a status code. */
const char* specdec_status_string(int code);

/* ------------------------------------------------------------------------- */
/* D-PACE                                                                     */
/* ------------------------------------------------------------------------- */

/* Workspace sizes for specdec_dpace_forward on `device` (CUDA ordinal). */
size_t specdec_dpace_scratch_bytes(int64_t N, int32_t B, int64_t V, int device);
size_t specdec_dpace_counter_bytes(int64_t N, int32_t B);

/*
 * D-PACE forward. Replaces the launch of dpace_megakernel in
 * losses/dpace.py:176-187 (_forward) and its host check losses/dpace.py:157-173
 * (_check), returning what losses/dpace.py:215 returns (the mean over N).
 *
 *   logits    [N, B, V] fp32           targets [N, B] int64
 *   mask      [N, B] fp32 or NULL      (NULL = every position scored; a
 *                                       position is scored iff mask > 0)
 *   n_global  divisor of the loss (N for one shard; the total sequence count
 *             when N is one shard of a larger batch)
 * Outputs (device):
 *   loss      [1]     sum_n sum_j w_j * ce_j / n_global
 *   loss_n    [N]     sum_j w_j * ce_j per sequence, or NULL
 *   lse       [N, B]  row log-sum-exp (0 for unscored rows)
 *   scale     [N, B]  w_j / n_global (dLoss/dce_j), 0 for unscored rows
 *   status    [1]     int32: SPECDEC_OK, or SPECDEC_ERR_TARGET_RANGE when a
 *                     target id lies outside [0, V) (the reference raises
 *                     ValueError, losses/dpace.py:172-173); may be NULL
 * Host-side errors: SPECDEC_ERR_ARGUMENT for B outside [1, 32], N < 0,
 * V < 1, null required pointers; SPECDEC_ERR_VALUE for alpha outside [0, 1]
 * or an unknown loss_type.
 */
int specdec_dpace_forward(const float* logits, const int64_t* targets, const float* mask,
                          int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                          int64_t n_global, float* loss, float* loss_n, float* lse, float* scale,
                          int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                          size_t counter_bytes, void* stream);

/* Counter bytes for the block queue and status of both backward entry points. */
size_t specdec_backward_counter_bytes(void);

/*
 * D-PACE backward. Replaces the launch of dpace_backward in
 * losses/dpace.py:217-226 (DPACELoss.backward):
 *   dlogits = scale[n, j] * dloss[0] * (softmax(logits[n, j]) - onehot(targets[n, j]))
 * dloss may be NULL (treated as 1). dlogits must not alias logits.
 * counters (zeroed once, left zeroed; specdec_backward_counter_bytes())
 * enable the dynamic block queue; NULL selects a static block interleave.
 * status [1] int32 (device, may be NULL): SPECDEC_OK, or SPECDEC_ERR_CUDA when
 * a bounded wait inside the launch expired. The reference's backward has no
 * device waits; this failure mode is this design's, so it is reported two
 * ways: through *status, and in the gradient itself -- every block of
 * dlogits the failed part of the launch may have left unfinished is
 * overwritten with NaN, so a gradient is never partly stale. A forward whose
 * wait expired writes NaN lse/scale, so a backward from it is NaN throughout.
 */
int specdec_dpace_backward(const float* logits, const int64_t* targets, const float* lse,
                           const float* scale, const float* dloss, float* dlogits, int64_t N,
                           int32_t B, int64_t V, int32_t* status, void* counters, size_t counter_bytes,
                           void* stream);

/*
 * D-PACE forward and backward in one call, for callers that want the loss and
 * the gradient together (dloss = 1): the loss, lse, scale (and loss_n) of
 * specdec_dpace_forward and the dlogits of specdec_dpace_backward with a
 * NULL dloss -- the same kernels on `stream`, so the same bits. Because the
 * call owns both launches, the backward is chained to the forward's last
 * kernel (programmatic dependent launch): it starts streaming the logits of
 * the scored rows while the forward finishes. No single counterpart in the
 * reference (losses/dpace.py:176-187 + :217-226 in one call). Arguments as in
 * specdec_dpace_forward plus `dlogits` [N, B, V] (same element type as
 * logits, must not alias it); same workspace queries. *status is the
 * forward's word, raised to SPECDEC_ERR_CUDA if a wait of the backward expired.
 */
int specdec_dpace_forward_backward(const float* logits, const int64_t* targets, const float* mask, int64_t N,
                                   int32_t B, int64_t V, float alpha, int32_t loss_type, int64_t n_global,
                                   float* loss, float* loss_n, float* lse, float* scale, float* dlogits,
                                   int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                                   size_t counter_bytes, void* stream);
int specdec_dpace_forward_backward_bf16(const uint16_t* logits, const int64_t* targets, const float* mask,
                                        int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                                        int64_t n_global, float* loss, float* loss_n, float* lse, float* scale,
                                        uint16_t* dlogits, int32_t* status, void* scratch, size_t scratch_bytes,
                                        void* counters, size_t counter_bytes, void* stream);

/*
 * x[i] *= *factor for i < n, on the device (16-byte-aligned x); returns
 * without touching x when *factor == 1 (checked on the device). Applies an
 * upstream gradient to a gradient computed with dloss = 1. No counterpart in
 * the reference.
 */
int specdec_scale_inplace(float* x, int64_t n, const float* factor, void* stream);
int specdec_scale_inplace_bf16(uint16_t* x, int64_t n, const float* factor, void* stream);

/*
 * D-PACE forward without any caller-provided workspace. No counterpart in the
 * reference: it serves callers that cannot allocate device memory -- plugin
 * hosts that pass only input and output buffers, and processes whose device
 * memory is all reserved by their own pool -- so it calls no cudaMalloc,
 * cudaFree or other allocating routine. Same arguments, kernels and results
 * as specdec_dpace_forward minus scratch/counters: its scratch is a 4 MiB
 * array built into the library (held on every GPU that loads the library
 * until exit): 64 KiB of counters and 4 MiB - 64 KiB of scratch. A problem
 * fits when specdec_dpace_counter_bytes(N, B) <= 64 KiB (N <= 16376) and
 * specdec_dpace_scratch_bytes(N, B, V, device) <= 4 MiB - 64 KiB -- at
 * V = 128256 about 14000 rows of N*B (about 287 bytes of scratch per row
 * plus 48 KiB for the forward's short final queue blocks). Larger problems
 * return SPECDEC_ERR_WORKSPACE before any launch; invalid arguments return
 * the same codes as specdec_dpace_forward, checked first. The first call on
 * a device looks up the array's address with that device current; make it
 * before any stream capture. The address is kept for the life of the
 * process: do not call this entry point on a device after cudaDeviceReset
 * (or any other destruction of its primary context). All calls on a device
 * share the array: its counters are cleared on `stream` before each launch,
 * and calls that overlap on the GPU race.
 */
int specdec_dpace_forward_noalloc(const float* logits, const int64_t* targets, const float* mask,
                                  int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                                  int64_t n_global, float* loss, float* loss_n, float* lse,
                                  float* scale, int32_t* status, void* stream);

/* ------------------------------------------------------------------------- */
/* DFlash objective                                                           */
/* ------------------------------------------------------------------------- */

size_t specdec_dflash_scratch_bytes(int64_t N, int32_t B, int64_t V, int device);
size_t specdec_dflash_counter_bytes(int64_t N, int32_t B);

/*
 * DFlash forward. Replaces the launch of dflash_loss_fwd in
 * models/dflash/loss.py:194-212 (_forward, including the denominator of
 * loss.py:200) and its host check models/dflash/loss.py:178-191 (_check),
 * returning what models/dflash/loss.py:257 returns (sum over rows / N).
 *
 *   logits, target_logits  [N, B, V] fp32 (draft, verifier)
 *   mask        [N, B] fp32 or NULL (all ones); used as a raw weight
 *   block_size  decay position of slot j is j % block_size, 1 <= block_size <= B
 *   gamma > 0; sample_from_anchor 0/1; kind SPECDEC_DFLASH_KL or _CE
 * Outputs: loss [1] (= sum_rows w * elementwise / n_global), loss_rows [N, B]
 * or NULL, scale [N, B] (= w / n_global), logzq / logzp [N, B] (log-normalisers
 * of draft / verifier; logzp is 0 for CE), target_id [N, B] int64 argmax of
 * the verifier row (CE only; may be NULL for KL). Rows with weight 0 have
 * zeros in every per-row output.
 */
int specdec_dflash_forward(const float* logits, const float* target_logits, const float* mask,
                           int64_t N, int32_t B, int64_t V, int32_t block_size, float gamma,
                           int32_t sample_from_anchor, int32_t kind, int64_t n_global, float* loss,
                           float* loss_rows, float* scale, float* logzq, float* logzp,
                           int64_t* target_id, void* scratch, size_t scratch_bytes, void* counters,
                           size_t counter_bytes, void* stream);

/*
 * DFlash backward. Replaces the launch of dflash_loss_bwd in
 * models/dflash/loss.py:259-269 (DFlashLoss.backward):
 *   KL: dlogits = scale * dloss * (softmax(logits) - softmax(target_logits))
 *   CE: dlogits = scale * dloss * (softmax(logits) - onehot(target_id))
 * target_logits is read for KL only (may be NULL for CE); target_id for CE only.
 * counters and status: as for specdec_dpace_backward (NULL counters = static
 * block interleave; an expired wait gives SPECDEC_ERR_CUDA and NaN blocks).
 */
int specdec_dflash_backward(const float* logits, const float* target_logits, const float* scale,
                            const float* logzq, const float* logzp, const int64_t* target_id,
                            const float* dloss, float* dlogits, int64_t N, int32_t B, int64_t V,
                            int32_t kind, int32_t* status, void* counters, size_t counter_bytes,
                            void* stream);

/* ------------------------------------------------------------------------- */
/* bfloat16 logits                                                            */
/* ------------------------------------------------------------------------- */

/*
 * bf16 variants of the four entry points above. No counterpart in the
 * reference, whose kernels take fp32 only (README.md:263, asserted by
 * losses/dpace.py:158 and models/dflash/loss.py:179): `logits`,
 * `target_logits` and `dlogits` hold bfloat16 values as their 16-bit
 * patterns; everything else (mask, per-row outputs, loss, workspace) is as
 * in the fp32 entry point of the same name, and the workspace sizes queried
 * for fp32 cover bf16. Every element is widened exactly to fp32 and all
 * arithmetic is fp32, so the loss and per-row outputs equal the fp32 entry
 * point's on the widened logits; the backward writes each gradient element
 * rounded to nearest even. logits, target_logits and dlogits must be
 * 16-byte aligned (SPECDEC_ERR_ARGUMENT otherwise).
 */
int specdec_dpace_forward_bf16(const uint16_t* logits, const int64_t* targets, const float* mask,
                               int64_t N, int32_t B, int64_t V, float alpha, int32_t loss_type,
                               int64_t n_global, float* loss, float* loss_n, float* lse, float* scale,
                               int32_t* status, void* scratch, size_t scratch_bytes, void* counters,
                               size_t counter_bytes, void* stream);
int specdec_dpace_backward_bf16(const uint16_t* logits, const int64_t* targets, const float* lse,
                                const float* scale, const float* dloss, uint16_t* dlogits, int64_t N,
                                int32_t B, int64_t V, int32_t* status, void* counters, size_t counter_bytes,
                                void* stream);
int specdec_dflash_forward_bf16(const uint16_t* logits, const uint16_t* target_logits, const float* mask,
                                int64_t N, int32_t B, int64_t V, int32_t block_size, float gamma,
                                int32_t sample_from_anchor, int32_t kind, int64_t n_global, float* loss,
                                float* loss_rows, float* scale, float* logzq, float* logzp,
                                int64_t* target_id, void* scratch, size_t scratch_bytes, void* counters,
                                size_t counter_bytes, void* stream);
int specdec_dflash_backward_bf16(const uint16_t* logits, const uint16_t* target_logits, const float* scale,
                                 const float* logzq, const float* logzp, const int64_t* target_id,
                                 const float* dloss, uint16_t* dlogits, int64_t N, int32_t B, int64_t V,
                                 int32_t kind, int32_t* status, void* counters, size_t counter_bytes,
                                 void* stream);

/* ------------------------------------------------------------------------- */
/* DFlash drafter layers                                                      */
/* ------------------------------------------------------------------------- */

/* Element types of the drafter-layer entry points. */
#define SPECDEC_DTYPE_F32 0
#define SPECDEC_DTYPE_BF16 1

/*
 * RMSNorm over the last dimension of x [rows, D] (fp32 or bf16, `dtype`),
 * fp32 weight [D]: y = x / sqrt(mean(x^2) + eps) * weight, in x's dtype, all
 * arithmetic fp32. Replaces torch.nn.RMSNorm in models/dflash/model.py:60,62
 * (norm1 / norm2), :111 (norm_out) and :114 (final_norm). rstd [rows] (or
 * NULL) receives 1 / sqrt(mean(x^2) + eps) for the backward.
 */
int specdec_rmsnorm_forward(const void* x, const float* weight, void* y, float* rstd, int64_t rows, int32_t D,
                            float eps, int32_t dtype, void* stream);

/* Workspace bytes of specdec_rmsnorm_backward (partial weight gradients). */
size_t specdec_rmsnorm_workspace_bytes(int64_t rows, int32_t D, int device);

/*
 * RMSNorm backward: dx [rows, D] (x's dtype) and dweight [D] (fp32, summed
 * over rows in a fixed order: bitwise repeatable) from x, weight, the
 * forward's rstd and dy (x's dtype). The gradient torch.nn.RMSNorm's
 * autograd computes for models/dflash/model.py's norms. D <= 51200.
 */
int specdec_rmsnorm_backward(const void* x, const float* weight, const float* rstd, const void* dy, void* dx,
                             float* dweight, int64_t rows, int32_t D, int32_t dtype, void* workspace,
                             size_t workspace_bytes, void* stream);

/*
 * DFlash attention forward on the tensor cores, bf16. Replaces the per-head
 * softmax(q k^T * scale + mask) v of models/dflash/model.py:25-53 under the
 * mask of models/dflash/model.py:123-131, applied by its structure: query
 * t < n_ctx sees keys j <= t, query t >= n_ctx sees every key j < T.
 *   q, k, v, o  [batch, T, heads, head_dim] bfloat16 bit patterns (the
 *               projections' own layout), 16-byte aligned; head_dim = 64
 *   lse         [batch, heads, T] fp32: log-sum-exp of each query row's
 *               scaled scores (natural log), for a backward
 *   status      [1] int32 or NULL: set to SPECDEC_ERR_CUDA if a bounded
 *               wait of the kernel expired, never cleared by the call (zero
 *               it first for a per-call report); the rows of o and lse the
 *               failed part owned are then NaN, never a plausible value
 * P = softmax is rounded to bf16 before the second product, the
 * accumulation is fp32. 0 <= n_ctx <= T <= 65535 * 128.
 */
int specdec_dflash_attention_forward(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                                     float* lse, int32_t batch, int32_t T, int32_t heads, int32_t head_dim,
                                     int32_t n_ctx, float scale, int32_t* status, void* stream);

/* Workspace bytes of specdec_dflash_attention_backward ([batch, heads, T] fp32). */
size_t specdec_dflash_attention_workspace_bytes(int32_t batch, int32_t T, int32_t heads);

/*
 * DFlash attention backward on the tensor cores, bf16: dq, dk, dv
 * [batch, T, heads, 64] from q, k, v, the forward's o and lse, and dout (the
 * gradient of o). The gradient autograd computes through
 * models/dflash/model.py:25-53 under the mask of :123-131. Probabilities
 * are recomputed from lse; dS = P * (dP - rowsum(dout * o)) * scale;
 * products in bf16 with fp32 accumulation, every sum in a fixed order (no
 * atomics: bitwise repeatable). workspace: specdec_dflash_attention_
 * workspace_bytes() of device memory, no initialisation required. status
 * as in the forward (sticky; the failed part's rows of dq / dk / dv NaN).
 */
int specdec_dflash_attention_backward(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                                      const float* lse, const uint16_t* dout, uint16_t* dq, uint16_t* dk,
                                      uint16_t* dv, int32_t batch, int32_t T, int32_t heads, int32_t head_dim,
                                      int32_t n_ctx, float scale, int32_t* status, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* Launch tuning                                                              */
/* ------------------------------------------------------------------------- */

/* Kernel ids for specdec_set_launch_shape. */
#define SPECDEC_KERNEL_DPACE_FWD 0
#define SPECDEC_KERNEL_DPACE_BWD 1
#define SPECDEC_KERNEL_DFLASH_FWD 2
#define SPECDEC_KERNEL_DFLASH_BWD 3

/* specdec_set_launch_shape: the built-in choice (ring shape 8 for the
 * D-PACE forward; ring shape 6 for the bf16 D-PACE backward, the bf16 DFlash
 * forward and the fp32 DFlash backward; ring shape 0 otherwise). */
#define SPECDEC_SHAPE_DEFAULT (-1)

/*
 * Selects a kernel variant and caps resident CTAs per SM (0 = occupancy
 * limit) for one kernel, process-wide. Shapes 0..6 (0..8 for the D-PACE
 * kernels) are warp-specialized bulk-copy ring variants (used when the
 * streamed pointers are 16-byte
 * aligned; otherwise the 128-bit-load kernels run with their default shape);
 * 10..14 force the 128-bit-load kernels, variant shape - 10 (bf16 entry
 * points, which have only the ring kernels, then use ring shape 0);
 * SPECDEC_SHAPE_DEFAULT restores the built-in choice. Workspace sizes depend
 * on it: query sizes after changing it.
 */
int specdec_set_launch_shape(int32_t kernel, int32_t shape, int32_t ctas_per_sm);

/* Number of CTAs the kernel would launch for a problem of rows x V on device. */
int64_t specdec_launch_ctas(int32_t kernel, int64_t rows, int64_t V, int device);

/*
 * Ring kernels hand out blocks through a global atomic queue (dynamic = 1,
 * default) or a static interleave (dynamic = 0), process-wide.
 */
int specdec_set_block_queue(int32_t dynamic);

/*
 * Failure-detection test hook (no counterpart in the reference). The next
 * `launches` D-PACE or DFlash launches on the ring path (forward or backward)
 * make CTA 0's producer withhold its first stage, so that CTA's consumers
 * reach the 1 s limit of their bounded wait: they record the timeout, wait
 * (bounded) for their own copies, and return. The launch completes in about
 * 2 s. A forward so failed gives a NaN loss and NaN per-row lse/scale/logz
 * (and, for D-PACE, *status = SPECDEC_ERR_CUDA); a backward gives
 * *status = SPECDEC_ERR_CUDA and NaN over the blocks CTA 0 held. The context
 * stays usable and the next launch is normal. Drafter attention launches
 * (forward, backward) consume armed launches too: the grid's first CTA
 * issues no product for its first tile, its wait expires, *status is set and
 * its rows of the outputs are NaN. 0 cancels. Not for production use. The
 * same reports follow any wait that expires for a real reason.
 */
int specdec_test_withhold_stage(int32_t launches);

#ifdef __cplusplus
}
#endif

#endif /* SPECDEC_H_ */
