/*
 * A C host of libspecdec.so: no Python, only include/specdec.h and the CUDA
 * runtime. Reads a problem from a file, runs the forward and backward
 * through the C ABI, writes the loss and the gradient.
 *
 *   abi_host <in.bin> <out.bin>
 *   in : int32 family (0 D-PACE, 1 DFlash), int64 N, int32 B, int64 V,
 *        int32 loss_type or kind, float alpha or gamma,
 *        float logits[N*B*V], then int64 targets[N*B] + float mask[N*B]
 *        (D-PACE) or float target_logits[N*B*V] (DFlash, no mask)
 *   out: float loss, float dlogits[N*B*V]
 * Exit status: 0 ok, 2 I/O, 3 C ABI error (message on stderr), 4 CUDA error,
 * 5 device status word not OK.
 */
#include <stdio.h>
#include <stdlib.h>

#include <cuda_runtime.h>

#include "specdec.h"

#define CUDA(call)                                                          \
  do {                                                                      \
    cudaError_t e_ = (call);                                                \
    if (e_ != cudaSuccess) {                                                \
      fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));           \
      return 4;                                                             \
    }                                                                       \
  } while (0)
#define ABI(call)                                                           \
  do {                                                                      \
    int rc_ = (call);                                                       \
    if (rc_ != SPECDEC_OK) {                                                \
      fprintf(stderr, "%s: %s (%s)\n", #call, specdec_status_string(rc_),   \
              specdec_last_error());                                        \
      return 3;                                                             \
    }                                                                       \
  } while (0)

static int read_all(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }

int main(int argc, char** argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: %s in.bin out.bin\n", argv[0]);
    return 2;
  }
  FILE* in = fopen(argv[1], "rb");
  if (!in) return 2;
  int32_t family, B, code;
  int64_t N, V;
  float param;
  if (!read_all(in, &family, 4) || !read_all(in, &N, 8) || !read_all(in, &B, 4) || !read_all(in, &V, 8) ||
      !read_all(in, &code, 4) || !read_all(in, &param, 4))
    return 2;
  const size_t E = (size_t)N * (size_t)B * (size_t)V, R = (size_t)N * (size_t)B;
  float* h_x = (float*)malloc(E * 4);
  float* h_g = (float*)malloc(E * 4);
  float* h_y = family == 1 ? (float*)malloc(E * 4) : NULL;
  int64_t* h_t = family == 0 ? (int64_t*)malloc(R * 8) : NULL;
  float* h_m = family == 0 ? (float*)malloc(R * 4) : NULL;
  if (!h_x || !h_g || !read_all(in, h_x, E * 4)) return 2;
  if (family == 0 && (!read_all(in, h_t, R * 8) || !read_all(in, h_m, R * 4))) return 2;
  if (family == 1 && !read_all(in, h_y, E * 4)) return 2;
  fclose(in);

  cudaStream_t st;
  CUDA(cudaStreamCreate(&st));
  int dev;
  CUDA(cudaGetDevice(&dev));
  float *x, *y = NULL, *g, *mask = NULL, *loss, *r0, *r1, *r2, *r3;
  int64_t *t = NULL, *tid = NULL;
  int32_t* status;  /* forward (D-PACE) */
  int32_t* bstatus; /* backward */
  CUDA(cudaMalloc((void**)&x, E * 4));
  CUDA(cudaMalloc((void**)&g, E * 4));
  CUDA(cudaMalloc((void**)&loss, 4));
  CUDA(cudaMalloc((void**)&r0, R * 4));
  CUDA(cudaMalloc((void**)&r1, R * 4));
  CUDA(cudaMalloc((void**)&r2, R * 4));
  CUDA(cudaMalloc((void**)&r3, R * 4));
  CUDA(cudaMalloc((void**)&tid, R * 8));
  CUDA(cudaMalloc((void**)&status, 4));
  CUDA(cudaMalloc((void**)&bstatus, 4));
  CUDA(cudaMemcpy(x, h_x, E * 4, cudaMemcpyHostToDevice));
  const size_t bwd_cb = specdec_backward_counter_bytes();
  void *scratch, *counters, *bwd_counters;
  size_t sb, cb;
  if (family == 0) {
    sb = specdec_dpace_scratch_bytes(N, B, V, dev);
    cb = specdec_dpace_counter_bytes(N, B);
  } else {
    sb = specdec_dflash_scratch_bytes(N, B, V, dev);
    cb = specdec_dflash_counter_bytes(N, B);
  }
  CUDA(cudaMalloc(&scratch, sb));
  CUDA(cudaMalloc(&counters, cb));
  CUDA(cudaMalloc(&bwd_counters, bwd_cb));
  CUDA(cudaMemset(counters, 0, cb)); /* once: every launch leaves them zero */
  CUDA(cudaMemset(bwd_counters, 0, bwd_cb));

  if (family == 0) {
    CUDA(cudaMalloc((void**)&t, R * 8));
    CUDA(cudaMalloc((void**)&mask, R * 4));
    CUDA(cudaMemcpy(t, h_t, R * 8, cudaMemcpyHostToDevice));
    CUDA(cudaMemcpy(mask, h_m, R * 4, cudaMemcpyHostToDevice));
    ABI(specdec_dpace_forward(x, t, mask, N, B, V, param, code, N, loss, NULL, r0, r1, status, scratch, sb,
                              counters, cb, st));
    ABI(specdec_dpace_backward(x, t, r0, r1, NULL, g, N, B, V, bstatus, bwd_counters, bwd_cb, st));
  } else {
    CUDA(cudaMalloc((void**)&y, E * 4));
    CUDA(cudaMemcpy(y, h_y, E * 4, cudaMemcpyHostToDevice));
    ABI(specdec_dflash_forward(x, y, NULL, N, B, V, B, param, 0, code, N, loss, NULL, r1, r2, r3, tid, scratch,
                               sb, counters, cb, st));
    ABI(specdec_dflash_backward(x, code == SPECDEC_DFLASH_KL ? y : NULL, r1, r2, r3, tid, NULL, g, N, B, V, code,
                                bstatus, bwd_counters, bwd_cb, st));
    CUDA(cudaMemsetAsync(status, 0, 4, st));
  }
  CUDA(cudaStreamSynchronize(st));
  int32_t h_status, h_bstatus;
  float h_loss;
  CUDA(cudaMemcpy(&h_status, status, 4, cudaMemcpyDeviceToHost));
  CUDA(cudaMemcpy(&h_bstatus, bstatus, 4, cudaMemcpyDeviceToHost));
  if (h_status != SPECDEC_OK || h_bstatus != SPECDEC_OK) {
    fprintf(stderr, "device status %d / %d: %s\n", h_status, h_bstatus,
            specdec_status_string(h_status != SPECDEC_OK ? h_status : h_bstatus));
    return 5;
  }
  CUDA(cudaMemcpy(&h_loss, loss, 4, cudaMemcpyDeviceToHost));
  CUDA(cudaMemcpy(h_g, g, E * 4, cudaMemcpyDeviceToHost));
  FILE* out = fopen(argv[2], "wb");
  if (!out || fwrite(&h_loss, 4, 1, out) != 1 || fwrite(h_g, 4, E, out) != E) return 2;
  fclose(out);
  printf("libspecdec %d: loss %.9g\n", specdec_version(), h_loss);
  return 0;
}
