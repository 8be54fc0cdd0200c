// D-PACE loss, forward and backward, for sm_100a.
//
// Reference behaviour (harvestingmoon/cuda-spec-decode):
//   losses/dpace.py:15-118    dpace_megakernel  (per-row lse / CE / q, then the B-scan)
//   losses/dpace.py:120-145   dpace_backward    ((w_j/N) * dloss * (softmax - onehot))
//   losses/dpace_ref.py:8-51  torch oracle whose numbers this file reproduces
//
// Forward, one launch:
//   1. every CTA streams its chunk of the flattened logits once, keeping an
//      online log-sum-exp per row piece, and writes (max, sum) per piece to
//      the workspace; the CTA whose piece holds the target id also stores
//      x[target];
//   2. a per-sequence arrival counter elects the CTA that lands last on
//      sequence n; it merges the pieces of the B rows in slot order, forms
//      ce_j = lse_j - x[target_j], q_j = exp(-ce_j), the alpha-smoothed prefix
//      product P_j, the suffix sum S_j and the detached weights w_j, and
//      writes loss_n, lse and scale = w_j / N_global;
//   3. a global counter elects the CTA that finalises the last sequence; it
//      sums loss_n in index order and writes loss = sum / N_global.
// Rows whose position mask is 0 are never read: their weight is exactly 0,
// so neither the loss nor the gradient depends on their logits.
//
// Backward, one launch: dlogits = scale * dloss * (exp(x - lse) - onehot), one read and one write per element; rows with scale 0 are written
// as zeros without being read.
#include "specdec_common.cuh"
#include "specdec_internal.h"

#include <cfloat>

namespace specdec {

namespace {

// Sum over the B rows of sequence n of the number of CTA pieces per row: the
// count the per-sequence arrival counter must reach.
__device__ __forceinline__ unsigned seq_piece_count(const Partition& pt, int64_t n, int B) {
  unsigned total = 0;
  for (int j = 0; j < B; ++j) total += (unsigned)pt.pieces(n * B + j);
  return total;
}

template <int NT, int U>
__device__ __forceinline__ void stream_lse(const float* __restrict__ p, int64_t n, float& m,
                                           float& s) {
  const int tid = threadIdx.x;
  int64_t head = ((16 - (reinterpret_cast<uintptr_t>(p) & 15)) & 15) >> 2;
  if (head > n) head = n;
  const int64_t body = (n - head) >> 2;
  const int64_t tail0 = head + (body << 2);
  if (tid < head) lse_push(m, s, p[tid]);
  if (tail0 + tid < n) lse_push(m, s, p[tail0 + tid]);
  const float4* q = reinterpret_cast<const float4*>(p + head);
  int64_t i = tid;
  for (; i + (U - 1) * NT < body; i += U * NT) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ld_stream(q + i + u * NT);
    float cm = max4(v[0]);
#pragma unroll
    for (int u = 1; u < U; ++u) cm = fmaxf(cm, max4(v[u]));
    if (cm > m) {
      s *= exp_shift(m, cm);
      m = cm;
    }
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      acc += exp_shift(v[u].x, m) + exp_shift(v[u].y, m) + exp_shift(v[u].z, m) +
             exp_shift(v[u].w, m);
    }
    s += acc;
  }
  for (; i < body; i += NT) {
    const float4 v = ld_stream(q + i);
    const float cm = max4(v);
    if (cm > m) {
      s *= exp_shift(m, cm);
      m = cm;
    }
    s += (exp_shift(v.x, m) + exp_shift(v.y, m)) + (exp_shift(v.z, m) + exp_shift(v.w, m));
  }
}

// Runs in the CTA elected for sequence n (all NT threads).
template <int NT>
__device__ void dpace_finalize_sequence(const DpaceFwdArgs& a, int64_t n, float* sh_lse,
                                        float* sh_ce, float* sh_sm, float* sh_mk, float* sh_p,
                                        float* sh_s, int* sh_last) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int B = a.B;
  __threadfence();
  // Phase A: log-sum-exp of each live row, pieces merged in slot order.
  for (int j = w; j < B; j += NW) {
    const int64_t r = n * B + j;
    const bool live = a.mask == nullptr || a.mask[r] > 0.f;
    float m = kNegSeed, s = 0.f;
    if (live) {
      const int k = a.pt.pieces(r);
      const float2* part = a.part + r * a.pt.pmax;
      for (int q = lane; q < k; q += 32) {
        const float2 v = __ldcg(part + q);
        lse_merge(m, s, v.x, v.y);
      }
      warp_lse(m, s);
    }
    if (lane == 0) sh_lse[j] = live ? m + logf(s) : 0.f;
  }
  __syncthreads();
  // Phase B: the B-scan (B <= 32) in warp 0. The prefix product and the
  // suffix sum accumulate in double, as torch's CPU cumprod/cumsum do.
  if (w == 0) {
    const int j = lane;
    const int64_t r = n * B + j;
    const bool in = j < B;
    const bool live = in && (a.mask == nullptr || a.mask[r] > 0.f);
    const int64_t t = in ? a.targets[r] : 0;
    const bool tvalid = t >= 0 && t < a.V;
    if (in && !tvalid) atomicOr(a.flag, 1);
    float ce = 0.f;
    if (live && tvalid) ce = sh_lse[j] - __ldcg(a.xtgt + r);
    if (in) {
      const float q = expf(-ce);
      sh_ce[j] = ce;
      sh_mk[j] = live ? 1.f : 0.f;
      sh_sm[j] = live ? __fadd_rn(__fmul_rn(a.one_minus_alpha, q), a.alpha) : 1.f;
    }
    __syncwarp();
    if (lane == 0) {
      double run = 1.0;
      for (int i = 0; i < B; ++i) {
        run *= (double)sh_sm[i];
        sh_p[i] = (float)run;
      }
      double acc = 0.0;
      for (int i = B - 1; i >= 0; --i) {
        acc += (double)__fmul_rn(sh_p[i], sh_mk[i]);
        sh_s[i] = (float)acc;
      }
    }
    __syncwarp();
    float contrib = 0.f;
    if (in) {
      const float P = sh_p[j], S = sh_s[j];
      float wt = a.loss_type == 1 ? P : (a.loss_type == 2 ? S / fmaxf(P, FLT_MIN) : S);
      wt = __fmul_rn(wt, sh_mk[j]);
      if (live) contrib = __fmul_rn(ce, wt);
      a.scale[r] = __fmul_rn(wt, a.inv_n);
      a.lse[r] = sh_lse[j];
    }
    const float loss_n = warp_sum(contrib);
    if (lane == 0) {
      if (a.loss_n) a.loss_n[n] = loss_n;
      a.seq_loss[n] = loss_n;
      a.seq_cnt[n] = 0u;  // leave the workspace zeroed for the next launch
      __threadfence();
      const unsigned prev = atomicAdd(a.done_cnt, 1u);
      *sh_last = (prev + 1 == (unsigned)a.N);
    }
  }
  __syncthreads();
  if (*sh_last) {
    // Global finaliser: loss = sum_n loss_n / N_global, in index order.
    if (w == 0) {
      __threadfence();
      const float total = warp_sum_l2(a.seq_loss, a.N);
      if (lane == 0) {
        a.loss[0] = total / (float)a.n_global;
        const int f = atomicExch(a.flag, 0);
        if (a.status) a.status[0] = f ? kStatusTargetRange : kStatusOk;
        *a.done_cnt = 0u;
      }
    }
  }
  __syncthreads();
}

template <int NT, int U>
__global__ void __launch_bounds__(NT) dpace_fwd_kernel(const __grid_constant__ DpaceFwdArgs a) {
  constexpr int NW = NT / 32;
  __shared__ float sh_red[2 * NW];
  __shared__ float sh_lse[32], sh_ce[32], sh_sm[32], sh_mk[32], sh_p[32], sh_s[32];
  __shared__ int sh_flag;
  __shared__ int sh_last;
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const Partition& pt = a.pt;
  const int64_t e_begin = c * pt.chunk;
  const int64_t e_end = min(e_begin + pt.chunk, pt.E);
  int64_t r = e_begin / pt.V;
  for (int64_t e = e_begin; e < e_end; ++r) {
    const int64_t row0 = r * pt.V;
    const int64_t lo = e - row0;
    const int64_t hi = min(e_end, row0 + pt.V) - row0;
    e = row0 + hi;
    const int64_t n = r / a.B;
    const bool live = a.mask == nullptr || a.mask[r] > 0.f;
    if (live) {
      const float* row = static_cast<const float*>(a.logits) + row0;
      float m = kNegSeed, s = 0.f;
      stream_lse<NT, U>(row + lo, hi - lo, m, s);
      block_lse<NT>(m, s, sh_red);
      if (tid == 0) {
        a.part[r * pt.pmax + (c - pt.first_cta(r))] = make_float2(m, s);
        const int64_t t = a.targets[r];
        if (t >= lo && t < hi) a.xtgt[r] = row[t];
      }
    }
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(a.seq_cnt + n, 1u);
      sh_flag = (prev + 1 == seq_piece_count(pt, n, a.B));
    }
    __syncthreads();
    if (sh_flag) dpace_finalize_sequence<NT>(a, n, sh_lse, sh_ce, sh_sm, sh_mk, sh_p, sh_s, &sh_last);
    __syncthreads();
  }
}

template <int NT, int U>
__global__ void __launch_bounds__(NT) dpace_bwd_kernel(const __grid_constant__ DpaceBwdArgs a) {
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const Partition& pt = a.pt;
  const int64_t e_begin = c * pt.chunk;
  const int64_t e_end = min(e_begin + pt.chunk, pt.E);
  const float g = a.dloss ? __ldg(a.dloss) : 1.f;
  const uint64_t pol = policy_evict_first();
  int64_t r = e_begin / pt.V;
  for (int64_t e = e_begin; e < e_end; ++r) {
    const int64_t row0 = r * pt.V;
    const int64_t lo = e - row0;
    const int64_t hi = min(e_end, row0 + pt.V) - row0;
    e = row0 + hi;
    const int64_t n = hi - lo;
    const float sc = __fmul_rn(a.scale[r], g);
    const float* src = static_cast<const float*>(a.logits) + row0 + lo;
    float* dst = static_cast<float*>(a.dlogits) + row0 + lo;
    const int64_t t = a.targets[r] - lo;  // target position relative to the piece
    const float l = a.lse[r];
    // Vector path when source and destination share 16-byte phase.
    const bool vec = ((reinterpret_cast<uintptr_t>(src) ^ reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
    int64_t head = vec ? (((16 - (reinterpret_cast<uintptr_t>(src) & 15)) & 15) >> 2) : n;
    if (head > n) head = n;
    const int64_t body = (n - head) >> 2;
    const int64_t tail0 = head + (body << 2);
    if (sc == 0.f) {
      for (int64_t i = tid; i < head; i += NT) dst[i] = 0.f;
      for (int64_t i = tail0 + tid; i < n; i += NT) dst[i] = 0.f;
      float4* q = reinterpret_cast<float4*>(dst + head);
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t i = tid; i < body; i += NT) st_stream(q + i, z);
      continue;
    }
    for (int64_t i = tid; i < head; i += NT)
      dst[i] = sc * (exp_shift(src[i], l) - (i == t ? 1.f : 0.f));
    for (int64_t i = tail0 + tid; i < n; i += NT)
      dst[i] = sc * (exp_shift(src[i], l) - (i == t ? 1.f : 0.f));
    const float4* qs = reinterpret_cast<const float4*>(src + head);
    float4* qd = reinterpret_cast<float4*>(dst + head);
    const int64_t tb = t - head;  // target relative to the vector body
    int64_t i = tid;
    for (; i + (U - 1) * NT < body; i += U * NT) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = ld_last(qs + i + u * NT, pol);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t k = i + u * NT;
        float4 y;
        y.x = exp_shift(v[u].x, l);
        y.y = exp_shift(v[u].y, l);
        y.z = exp_shift(v[u].z, l);
        y.w = exp_shift(v[u].w, l);
        const uint64_t d = (uint64_t)(tb - 4 * k);
        if (d < 4) {
          if (d == 0) y.x -= 1.f;
          else if (d == 1) y.y -= 1.f;
          else if (d == 2) y.z -= 1.f;
          else y.w -= 1.f;
        }
        y.x *= sc;
        y.y *= sc;
        y.z *= sc;
        y.w *= sc;
        st_stream(qd + k, y);
      }
    }
    for (; i < body; i += NT) {
      const float4 v = ld_last(qs + i, pol);
      float4 y;
      y.x = exp_shift(v.x, l);
      y.y = exp_shift(v.y, l);
      y.z = exp_shift(v.z, l);
      y.w = exp_shift(v.w, l);
      const uint64_t d = (uint64_t)(tb - 4 * i);
      if (d < 4) {
        if (d == 0) y.x -= 1.f;
        else if (d == 1) y.y -= 1.f;
        else if (d == 2) y.z -= 1.f;
        else y.w -= 1.f;
      }
      y.x *= sc;
      y.y *= sc;
      y.z *= sc;
      y.w *= sc;
      st_stream(qd + i, y);
    }
  }
}

template <class K>
int occupancy_grid(K kernel, int nt, int device, int cap_per_sm) {
  static int cached_sms[64] = {0};
  int sms = device >= 0 && device < 64 ? cached_sms[device] : 0;
  if (sms == 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    if (device >= 0 && device < 64) cached_sms[device] = sms;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, nt, 0) != cudaSuccess) return 0;
  if (cap_per_sm > 0 && per_sm > cap_per_sm) per_sm = cap_per_sm;
  if (per_sm < 1) per_sm = 1;
  return sms * per_sm;
}

template <int NT, int U>
struct DpaceVariant {
  static int fwd_ctas(int device, int cap) { return occupancy_grid(dpace_fwd_kernel<NT, U>, NT, device, cap); }
  static int bwd_ctas(int device, int cap) { return occupancy_grid(dpace_bwd_kernel<NT, U>, NT, device, cap); }
  static cudaError_t fwd(const DpaceFwdArgs& a, cudaStream_t st) {
    dpace_fwd_kernel<NT, U><<<(unsigned)a.pt.grid, NT, 0, st>>>(a);
    return cudaGetLastError();
  }
  static cudaError_t bwd(const DpaceBwdArgs& a, cudaStream_t st) {
    dpace_bwd_kernel<NT, U><<<(unsigned)a.pt.grid, NT, 0, st>>>(a);
    return cudaGetLastError();
  }
};

}  // namespace

// Launch-shape table: index = LaunchShape id (see specdec_internal.h).
int dpace_fwd_ctas(int shape, int device, int cap) {
  switch (shape) {
    case 1: return DpaceVariant<256, 4>::fwd_ctas(device, cap);
    case 2: return DpaceVariant<512, 8>::fwd_ctas(device, cap);
    case 3: return DpaceVariant<256, 8>::fwd_ctas(device, cap);
    case 4: return DpaceVariant<512, 2>::fwd_ctas(device, cap);
    default: return DpaceVariant<512, 4>::fwd_ctas(device, cap);
  }
}

int dpace_bwd_ctas(int shape, int device, int cap) {
  switch (shape) {
    case 1: return DpaceVariant<256, 4>::bwd_ctas(device, cap);
    case 2: return DpaceVariant<512, 8>::bwd_ctas(device, cap);
    case 3: return DpaceVariant<256, 8>::bwd_ctas(device, cap);
    case 4: return DpaceVariant<512, 2>::bwd_ctas(device, cap);
    default: return DpaceVariant<512, 4>::bwd_ctas(device, cap);
  }
}

cudaError_t dpace_fwd_launch(int shape, const DpaceFwdArgs& a, cudaStream_t st) {
  switch (shape) {
    case 1: return DpaceVariant<256, 4>::fwd(a, st);
    case 2: return DpaceVariant<512, 8>::fwd(a, st);
    case 3: return DpaceVariant<256, 8>::fwd(a, st);
    case 4: return DpaceVariant<512, 2>::fwd(a, st);
    default: return DpaceVariant<512, 4>::fwd(a, st);
  }
}

cudaError_t dpace_bwd_launch(int shape, const DpaceBwdArgs& a, cudaStream_t st) {
  switch (shape) {
    case 1: return DpaceVariant<256, 4>::bwd(a, st);
    case 2: return DpaceVariant<512, 8>::bwd(a, st);
    case 3: return DpaceVariant<256, 8>::bwd(a, st);
    case 4: return DpaceVariant<512, 2>::bwd(a, st);
    default: return DpaceVariant<512, 4>::bwd(a, st);
  }
}

}  // namespace specdec
