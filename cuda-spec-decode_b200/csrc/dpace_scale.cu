// In-place scaling of a gradient by the upstream dloss, for callers that
// computed the gradient for dloss = 1 (specdec_dpace_forward_backward) and
// receive the real dloss later (the autograd backward).
#include "specdec_common.cuh"
#include "specdec_internal.h"

namespace specdec {

namespace {

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

}  // namespace specdec
