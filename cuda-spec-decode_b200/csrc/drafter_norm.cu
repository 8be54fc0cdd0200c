// RMSNorm of the DFlash drafter, forward and backward.
//
// Reference behaviour: models/dflash/model.py:60,62 (norm1 / norm2 of
// DFlashTransformerLayer), :111 (norm_out) and :114 (final_norm), all
// torch.nn.RMSNorm(d):
//     y = x / sqrt(mean(x^2) + eps) * w
// with eps = finfo(x.dtype).eps when the module leaves it unset. Rows are
// [rows, D] C-contiguous; x and y are fp32 or bf16 (the weight is fp32, as
// the module keeps it under autocast), all arithmetic fp32. The per-row
// 1/rms is saved for the backward:
//     g = dy * w,  dx = rstd * g - x * rstd^3 * sum(g * x) / D,
//     dw = sum over rows of dy * x * rstd
// HBM-bound: one read of x (and dy) and one write of y (dx) per pass.
//
// Three row layouts, picked by D (16-byte vectors: 4 floats or 8 bf16; rows
// and pointers 16-byte aligned, D a whole number of vectors):
//   warp per row   D <= 1024: a lane holds up to 8 vectors of its row in
//                  registers, every load of the row in flight at once;
//   CTA per row    1024 < D <= 8192: 256 threads hold the row, a block
//                  reduction per row;
//   generic        anything else (unaligned, ragged D): a warp per row,
//                  element loops.
// dw is reduced deterministically: every CTA sums its rows into its own
// partial row (fixed row order), and a second kernel sums the partial rows
// in a fixed order (32 interleaved chains, then the chains in order).
#include <algorithm>
#include <initializer_list>

#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

constexpr int kNormThreads = 256;  // 8 warps
constexpr int kWarpRowMaxD = 1024;
constexpr int kCtaRowMaxD = 8192;

__device__ __forceinline__ float load_elem(const float* p) { return *p; }
__device__ __forceinline__ float load_elem(const bf16_t* p) { return to_f32(*p); }

// 16-byte vector of the row: 4 floats or 8 bf16 -> fp32 values.
template <class T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void load(const float* p, float* v) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  }
  __device__ __forceinline__ static void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct Vec<bf16_t> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void load(const bf16_t* p, float* v) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = bf16_lo(w[i]);
      v[2 * i + 1] = bf16_hi(w[i]);
    }
  }
  __device__ __forceinline__ static void store(bf16_t* p, const float* v) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                              pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
};

// NV consecutive weights (fp32, 16-byte aligned).
template <int NV>
__device__ __forceinline__ void load_w(const float* w, float* v) {
#pragma unroll
  for (int i = 0; i < NV; i += 4) {
    const float4 q = *reinterpret_cast<const float4*>(w + i);
    v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
  }
}

__device__ __forceinline__ void st_elem(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_elem(bf16_t* p, float v) { store_elem(p, v); }

// Sum over the CTA's 8 warps, valid in every thread; `red` holds 8 floats.
// Ends with a barrier, so `red` may be reused right away.
__device__ __forceinline__ float cta_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

// ---- forward ---------------------------------------------------------------

// Warp per row; lane holds vectors lane + 32 i (i < VPL) of the row.
template <class T, int VPL>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_warp(const T* __restrict__ x, const float* __restrict__ w,
                                                                 T* __restrict__ y, float* __restrict__ rstd,
                                                                 int64_t rows, int D, float eps) {
  constexpr int NV = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int nvec = D / NV;
  const int64_t warps = (int64_t)gridDim.x * (kNormThreads / 32);
  for (int64_t r = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* xr = x + r * D;
    float v[VPL][NV];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) {
        Vec<T>::load(xr + (size_t)k * NV, v[i]);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) v[i][j] = 0.f;
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int j = 0; j < NV; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rstd) rstd[r] = rs;
    T* yr = y + r * D;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) {
        float wv[NV], o[NV];
        load_w<NV>(w + (size_t)k * NV, wv);
#pragma unroll
        for (int j = 0; j < NV; ++j) o[j] = v[i][j] * rs * wv[j];
        Vec<T>::store(yr + (size_t)k * NV, o);
      }
    }
  }
}

// CTA per row; thread holds vectors tid + 256 i (i < VPT) of the row.
template <class T, int VPT>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_cta(const T* __restrict__ x, const float* __restrict__ w,
                                                                T* __restrict__ y, float* __restrict__ rstd,
                                                                int64_t rows, int D, float eps) {
  constexpr int NV = Vec<T>::N;
  __shared__ float red[kNormThreads / 32];
  const int nvec = D / NV;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * D;
    float v[VPT][NV];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int k = threadIdx.x + kNormThreads * i;
      if (k < nvec) {
        Vec<T>::load(xr + (size_t)k * NV, v[i]);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) v[i][j] = 0.f;
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < NV; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    ss = cta_sum(ss, red);
    const float rs = rsqrtf(ss / (float)D + eps);
    if (threadIdx.x == 0 && rstd) rstd[r] = rs;
    T* yr = y + r * D;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int k = threadIdx.x + kNormThreads * i;
      if (k < nvec) {
        float wv[NV], o[NV];
        load_w<NV>(w + (size_t)k * NV, wv);
#pragma unroll
        for (int j = 0; j < NV; ++j) o[j] = v[i][j] * rs * wv[j];
        Vec<T>::store(yr + (size_t)k * NV, o);
      }
    }
  }
}

// Generic rows (any D, any alignment): warp per row, element loops.
template <class T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_generic(const T* __restrict__ x,
                                                                    const float* __restrict__ w, T* __restrict__ y,
                                                                    float* __restrict__ rstd, int64_t rows, int D,
                                                                    float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kNormThreads / 32);
  for (int64_t r = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* xr = x + r * D;
    float ss = 0.f;
    for (int k = lane; k < D; k += 32) {
      const float v = load_elem(xr + k);
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rstd) rstd[r] = rs;
    T* yr = y + r * D;
    for (int k = lane; k < D; k += 32) st_elem(yr + k, load_elem(xr + k) * rs * w[k]);
  }
}

// ---- backward --------------------------------------------------------------

// Warp per row over this CTA's contiguous row range (warps interleaved); each
// lane keeps the weight-gradient partial of its columns in registers. At the
// end the CTA sums its warps' partials in warp order into part[blockIdx.x].
template <class T, int VPL>
__global__ void __launch_bounds__(kNormThreads, 2) rmsnorm_bwd_warp(const T* __restrict__ x, const float* __restrict__ w,
                                                                 const float* __restrict__ rstd,
                                                                 const T* __restrict__ dy, T* __restrict__ dx,
                                                                 float* __restrict__ part, int64_t rows, int D) {
  constexpr int NV = Vec<T>::N;
  __shared__ float sh[(kNormThreads / 32) * kWarpRowMaxD];  // [warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = D / NV;
  float acc[VPL][NV];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int j = 0; j < NV; ++j) acc[i][j] = 0.f;
  const int64_t per = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per, r1 = min(rows, r0 + per);
  for (int64_t r = r0 + warp; r < r1; r += kNormThreads / 32) {
    const T* xr = x + r * D;
    const T* gr = dy + r * D;
    float xv[VPL][NV], gv[VPL][NV];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) {
        Vec<T>::load(xr + (size_t)k * NV, xv[i]);
        Vec<T>::load(gr + (size_t)k * NV, gv[i]);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) xv[i][j] = gv[i][j] = 0.f;
      }
    }
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) {
        float wv[NV];
        load_w<NV>(w + (size_t)k * NV, wv);
#pragma unroll
        for (int j = 0; j < NV; ++j) dot = fmaf(gv[i][j] * wv[j], xv[i][j], dot);
      }
    }
    dot = warp_sum(dot);
    const float c = rs * rs * rs * dot / (float)D;
    T* dr = dx + r * D;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) {
        float wv[NV], o[NV];
        load_w<NV>(w + (size_t)k * NV, wv);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          o[j] = rs * gv[i][j] * wv[j] - xv[i][j] * c;
          acc[i][j] = fmaf(gv[i][j], xv[i][j] * rs, acc[i][j]);
        }
        Vec<T>::store(dr + (size_t)k * NV, o);
      }
    }
  }
  float* my = sh + warp * kWarpRowMaxD;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int k = lane + 32 * i;
    if (k < nvec)
#pragma unroll
      for (int j = 0; j < NV; ++j) my[k * NV + j] = acc[i][j];
  }
  __syncthreads();
  for (int k = threadIdx.x; k < D; k += kNormThreads) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kNormThreads / 32; ++q) s += sh[q * kWarpRowMaxD + k];
    part[(size_t)blockIdx.x * D + k] = s;
  }
}

// CTA per row over rows blockIdx.x, blockIdx.x + gridDim.x, ...; each thread
// keeps the weight-gradient partial of its columns in registers and writes
// it to part[blockIdx.x] at the end.
template <class T, int VPT>
__global__ void __launch_bounds__(kNormThreads, 2) rmsnorm_bwd_cta(const T* __restrict__ x, const float* __restrict__ w,
                                                                const float* __restrict__ rstd,
                                                                const T* __restrict__ dy, T* __restrict__ dx,
                                                                float* __restrict__ part, int64_t rows, int D) {
  constexpr int NV = Vec<T>::N;
  __shared__ float red[kNormThreads / 32];
  const int nvec = D / NV;
  float acc[VPT][NV];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int j = 0; j < NV; ++j) acc[i][j] = 0.f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * D;
    const T* gr = dy + r * D;
    float xv[VPT][NV], gv[VPT][NV];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int k = threadIdx.x + kNormThreads * i;
      if (k < nvec) {
        Vec<T>::load(xr + (size_t)k * NV, xv[i]);
        Vec<T>::load(gr + (size_t)k * NV, gv[i]);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) xv[i][j] = gv[i][j] = 0.f;
      }
    }
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int k = threadIdx.x + kNormThreads * i;
      if (k < nvec) {
        float wv[NV];
        load_w<NV>(w + (size_t)k * NV, wv);
#pragma unroll
        for (int j = 0; j < NV; ++j) dot = fmaf(gv[i][j] * wv[j], xv[i][j], dot);
      }
    }
    dot = cta_sum(dot, red);
    const float c = rs * rs * rs * dot / (float)D;
    T* dr = dx + r * D;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int k = threadIdx.x + kNormThreads * i;
      if (k < nvec) {
        float wv[NV], o[NV];
        load_w<NV>(w + (size_t)k * NV, wv);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          o[j] = rs * gv[i][j] * wv[j] - xv[i][j] * c;
          acc[i][j] = fmaf(gv[i][j], xv[i][j] * rs, acc[i][j]);
        }
        Vec<T>::store(dr + (size_t)k * NV, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int k = threadIdx.x + kNormThreads * i;
    if (k < nvec)
#pragma unroll
      for (int j = 0; j < NV; ++j) part[(size_t)blockIdx.x * D + (size_t)k * NV + j] = acc[i][j];
  }
}

// Generic rows: warp per row, element loops; each warp keeps its partial in
// shared memory ([warps][D] floats: the launch picks as many warps, up to 8,
// as fit in 200 KB); the CTA sums its warps in warp order at the end.
template <class T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_generic(const T* __restrict__ x,
                                                                    const float* __restrict__ w,
                                                                    const float* __restrict__ rstd,
                                                                    const T* __restrict__ dy, T* __restrict__ dx,
                                                                    float* __restrict__ part, int64_t rows, int D) {
  extern __shared__ float sh_dw[];  // [warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = blockDim.x >> 5;
  float* my = sh_dw + (size_t)warp * D;
  for (int k = lane; k < D; k += 32) my[k] = 0.f;
  const int64_t per = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per, r1 = min(rows, r0 + per);
  for (int64_t r = r0 + warp; r < r1; r += W) {
    const T* xr = x + r * D;
    const T* gr = dy + r * D;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int k = lane; k < D; k += 32) {
      const float g = load_elem(gr + k) * w[k];
      dot = fmaf(g, load_elem(xr + k), dot);
    }
    dot = warp_sum(dot);
    const float c = rs * rs * rs * dot / (float)D;
    T* dr = dx + r * D;
    for (int k = lane; k < D; k += 32) {
      const float xv = load_elem(xr + k), gv = load_elem(gr + k);
      st_elem(dr + k, rs * gv * w[k] - xv * c);
      my[k] = fmaf(gv, xv * rs, my[k]);
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < D; k += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < W; ++q) s += sh_dw[(size_t)q * D + k];
    part[(size_t)blockIdx.x * D + k] = s;
  }
}

// dw[k] = sum over partial rows p of part[p * D + k]: 32 chains per column
// (p = y, y + 32, ...), then the chains in order. blockDim (32, 32).
__global__ void __launch_bounds__(1024) rmsnorm_dw_kernel(const float* __restrict__ part, float* __restrict__ dw,
                                                          int nparts, int D) {
  __shared__ float sh[32][33];
  const int k = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (k < D)
    for (int p = threadIdx.y; p < nparts; p += 32) s += part[(size_t)p * D + k];
  sh[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && k < D) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 32; ++q) t += sh[q][threadIdx.x];
    dw[k] = t;
  }
}

// Vectors per lane (warp rows) or per thread (CTA rows): 1, 2, 4 or 8; 0 = too many.
int per_thread(int nvec, int threads) {
  const int n = (nvec + threads - 1) / threads;
  return n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : n <= 8 ? 8 : 0;
}

bool vec_ok(int dtype, int D, std::initializer_list<const void*> ptrs) {
  const int nv = dtype == kDtypeBF16 ? 8 : 4;
  if (D % nv != 0) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return false;
  return true;
}

template <class T>
cudaError_t fwd_dispatch(const T* x, const float* w, T* y, float* rstd, int64_t rows, int D, float eps, int sms,
                         bool vec, cudaStream_t st) {
  constexpr int NV = Vec<T>::N;
  const int nvec = D / NV;
  const int64_t by_rows = (rows + 7) / 8;
  if (vec && D <= kWarpRowMaxD) {
    const int ctas = (int)(by_rows < (int64_t)sms * 8 ? by_rows : (int64_t)sms * 8);
    switch (per_thread(nvec, 32)) {
      case 1: rmsnorm_fwd_warp<T, 1><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps); break;
      case 2: rmsnorm_fwd_warp<T, 2><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps); break;
      case 4: rmsnorm_fwd_warp<T, 4><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps); break;
      default:
        if constexpr (NV == 4) rmsnorm_fwd_warp<T, 8><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps);
        break;
    }
  } else if (vec && D <= kCtaRowMaxD) {
    const int ctas = (int)(rows < (int64_t)sms * 4 ? rows : (int64_t)sms * 4);
    switch (per_thread(nvec, kNormThreads)) {
      case 1: rmsnorm_fwd_cta<T, 1><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps); break;
      case 2: rmsnorm_fwd_cta<T, 2><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps); break;
      case 4: rmsnorm_fwd_cta<T, 4><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps); break;
      default:
        if constexpr (NV == 4) rmsnorm_fwd_cta<T, 8><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps);
        break;
    }
  } else {
    const int ctas = (int)(by_rows < (int64_t)sms * 8 ? by_rows : (int64_t)sms * 8);
    rmsnorm_fwd_generic<T><<<ctas, kNormThreads, 0, st>>>(x, w, y, rstd, rows, D, eps);
  }
  return cudaGetLastError();
}

template <class T>
cudaError_t bwd_dispatch(const T* x, const float* w, const float* rstd, const T* dy, T* dx, float* part,
                         int64_t rows, int D, int ctas, bool vec, cudaStream_t st) {
  constexpr int NV = Vec<T>::N;
  const int nvec = D / NV;
  if (vec && D <= kWarpRowMaxD) {
    switch (per_thread(nvec, 32)) {
      case 1: rmsnorm_bwd_warp<T, 1><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D); break;
      case 2: rmsnorm_bwd_warp<T, 2><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D); break;
      case 4: rmsnorm_bwd_warp<T, 4><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D); break;
      default:
        if constexpr (NV == 4)
          rmsnorm_bwd_warp<T, 8><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D);
        break;
    }
  } else if (vec && D <= kCtaRowMaxD) {
    switch (per_thread(nvec, kNormThreads)) {
      case 1: rmsnorm_bwd_cta<T, 1><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D); break;
      case 2: rmsnorm_bwd_cta<T, 2><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D); break;
      case 4: rmsnorm_bwd_cta<T, 4><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D); break;
      default:
        if constexpr (NV == 4)
          rmsnorm_bwd_cta<T, 8><<<ctas, kNormThreads, 0, st>>>(x, w, rstd, dy, dx, part, rows, D);
        break;
    }
  } else {
    const int W = rmsnorm_bwd_warps(D);
    if (W < 1) return cudaErrorInvalidValue;
    const size_t smem = (size_t)W * D * sizeof(float);
    if (smem > 48 * 1024) {
      const cudaError_t e =
          cudaFuncSetAttribute(rmsnorm_bwd_generic<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    rmsnorm_bwd_generic<T><<<ctas, 32 * W, smem, st>>>(x, w, rstd, dy, dx, part, rows, D);
  }
  return cudaGetLastError();
}

}  // namespace

// Partial weight-gradient rows of the backward (one per CTA): warp rows
// (D <= 1024) take 8 rows per CTA up to 4 CTAs per SM; CTA rows up to 2 CTAs
// per SM. The generic layout uses the same count for the same D.
int rmsnorm_bwd_ctas(int64_t rows, int D, int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  const int64_t c = D <= kWarpRowMaxD ? std::min<int64_t>((rows + 7) / 8, (int64_t)sms * 4)
                                      : std::min<int64_t>(rows, (int64_t)sms * 2);
  return (int)(c < 1 ? 1 : c);
}

// Warps per CTA of the generic backward: up to 8, as many [D] float partials
// as fit in 200 KB of shared memory (0: D too large).
int rmsnorm_bwd_warps(int D) {
  const int w = (int)((200 * 1024) / ((size_t)D * sizeof(float)));
  return w > 8 ? 8 : w;
}

cudaError_t rmsnorm_fwd_launch(int dtype, const void* x, const float* w, void* y, float* rstd, int64_t rows, int D,
                               float eps, int sms, cudaStream_t st) {
  const bool vec = vec_ok(dtype, D, {x, y, w});
  if (dtype == kDtypeBF16)
    return fwd_dispatch<bf16_t>(static_cast<const bf16_t*>(x), w, static_cast<bf16_t*>(y), rstd, rows, D, eps, sms,
                                vec, st);
  return fwd_dispatch<float>(static_cast<const float*>(x), w, static_cast<float*>(y), rstd, rows, D, eps, sms, vec,
                             st);
}

cudaError_t rmsnorm_bwd_launch(int dtype, const void* x, const float* w, const float* rstd, const void* dy,
                               void* dx, float* dw, float* part, int64_t rows, int D, int ctas, cudaStream_t st) {
  const bool vec = vec_ok(dtype, D, {x, w, dy, dx});
  cudaError_t e;
  if (dtype == kDtypeBF16)
    e = bwd_dispatch<bf16_t>(static_cast<const bf16_t*>(x), w, rstd, static_cast<const bf16_t*>(dy),
                             static_cast<bf16_t*>(dx), part, rows, D, ctas, vec, st);
  else
    e = bwd_dispatch<float>(static_cast<const float*>(x), w, rstd, static_cast<const float*>(dy),
                            static_cast<float*>(dx), part, rows, D, ctas, vec, st);
  if (e != cudaSuccess) return e;
  rmsnorm_dw_kernel<<<(D + 31) / 32, dim3(32, 32), 0, st>>>(part, dw, ctas, D);
  return cudaGetLastError();
}

}  // namespace specdec
