// RMSNorm of the DFlash drafter, forward and backward, one warp per row.
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
// dw is reduced deterministically: every CTA sums its rows into its own
// partial row (fixed row order), and a second kernel sums the partials in CTA
// order. HBM-bound: one read of x (and dy) and one write of y (dx) per pass.
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

constexpr int kNormThreads = 256;  // 8 warps, one row each at a time

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

__device__ __forceinline__ void st_elem(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_elem(bf16_t* p, float v) { store_elem(p, v); }

// Row r of D elements: lanes take 16-byte vectors in order (vector path, D a
// multiple of the vector width and 16-byte aligned rows) or single elements.
template <class T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(const T* __restrict__ x,
                                                                   const float* __restrict__ w,
                                                                   T* __restrict__ y, float* __restrict__ rstd,
                                                                   int64_t rows, int D, float eps, int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kNormThreads / 32);
  constexpr int NV = Vec<T>::N;
  for (int64_t r = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* xr = x + r * D;
    float ss = 0.f;
    if (vec) {
      for (int k = lane * NV; k < D; k += 32 * NV) {
        float v[NV];
        Vec<T>::load(xr + k, v);
#pragma unroll
        for (int i = 0; i < NV; ++i) ss = fmaf(v[i], v[i], ss);
      }
    } else {
      for (int k = lane; k < D; k += 32) {
        const float v = load_elem(xr + k);
        ss = fmaf(v, v, ss);
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rstd) rstd[r] = rs;
    T* yr = y + r * D;
    if (vec) {
      for (int k = lane * NV; k < D; k += 32 * NV) {
        float v[NV], g[NV];
        Vec<T>::load(xr + k, v);
#pragma unroll
        for (int i = 0; i < NV; ++i) g[i] = v[i] * rs * w[k + i];
        Vec<T>::store(yr + k, g);
      }
    } else {
      for (int k = lane; k < D; k += 32) st_elem(yr + k, load_elem(xr + k) * rs * w[k]);
    }
  }
}

// Backward: dx per row, and this CTA's partial dw (sum over its rows, in
// row order) in part[blockIdx.x * D + k]. Each warp keeps its own partial in
// shared memory ([warps][D] floats: the launch picks as many warps, up to 8,
// as fit); the CTA sums its warps in warp order at the end.
template <class T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(const T* __restrict__ x,
                                                                   const float* __restrict__ w,
                                                                   const float* __restrict__ rstd,
                                                                   const T* __restrict__ dy, T* __restrict__ dx,
                                                                   float* __restrict__ part, int64_t rows, int D) {
  extern __shared__ float sh_dw[];  // [warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = blockDim.x >> 5;
  float* my = sh_dw + (size_t)warp * D;
  for (int k = lane; k < D; k += 32) my[k] = 0.f;
  // rows of this CTA: a contiguous range, warps interleaved inside it
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

// dw[k] = sum over CTAs c of part[c * D + k], in CTA order.
__global__ void rmsnorm_dw_kernel(const float* __restrict__ part, float* __restrict__ dw, int ctas, int D) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= D) return;
  float s = 0.f;
  for (int c = 0; c < ctas; ++c) s += part[(size_t)c * D + k];
  dw[k] = s;
}

}  // namespace

int rmsnorm_bwd_ctas(int64_t rows, int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  const int64_t by_rows = (rows + 7) / 8, by_sms = (int64_t)sms * 4;
  const int64_t c = by_rows < by_sms ? by_rows : by_sms;
  return (int)(c < 1 ? 1 : c);
}

cudaError_t rmsnorm_fwd_launch(int dtype, const void* x, const float* w, void* y, float* rstd, int64_t rows, int D,
                               float eps, int ctas, cudaStream_t st) {
  const int vec = (D % (dtype == kDtypeBF16 ? 8 : 4) == 0) &&
                  (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
  if (dtype == kDtypeBF16)
    rmsnorm_fwd_kernel<bf16_t><<<ctas, kNormThreads, 0, st>>>(static_cast<const bf16_t*>(x), w,
                                                              static_cast<bf16_t*>(y), rstd, rows, D, eps, vec);
  else
    rmsnorm_fwd_kernel<float><<<ctas, kNormThreads, 0, st>>>(static_cast<const float*>(x), w,
                                                             static_cast<float*>(y), rstd, rows, D, eps, vec);
  return cudaGetLastError();
}

// Warps per backward CTA: up to 8, as many [D] float partials as fit in
// 200 KB of shared memory (0: D too large).
int rmsnorm_bwd_warps(int D) {
  const int w = (int)((200 * 1024) / ((size_t)D * sizeof(float)));
  return w > 8 ? 8 : w;
}

cudaError_t rmsnorm_bwd_launch(int dtype, const void* x, const float* w, const float* rstd, const void* dy,
                               void* dx, float* dw, float* part, int64_t rows, int D, int ctas, cudaStream_t st) {
  const int W = rmsnorm_bwd_warps(D);
  if (W < 1) return cudaErrorInvalidValue;
  const size_t smem = (size_t)W * D * sizeof(float);
  if (dtype == kDtypeBF16) {
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<bf16_t>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    rmsnorm_bwd_kernel<bf16_t><<<ctas, 32 * W, smem, st>>>(
        static_cast<const bf16_t*>(x), w, rstd, static_cast<const bf16_t*>(dy), static_cast<bf16_t*>(dx), part,
        rows, D);
  } else {
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<float>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    rmsnorm_bwd_kernel<float><<<ctas, 32 * W, smem, st>>>(static_cast<const float*>(x), w, rstd,
                                                                static_cast<const float*>(dy),
                                                                static_cast<float*>(dx), part, rows, D);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  rmsnorm_dw_kernel<<<(D + 255) / 256, 256, 0, st>>>(part, dw, ctas, D);
  return cudaGetLastError();
}

}  // namespace specdec
