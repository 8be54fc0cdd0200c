// D-PACE forward for callers that cannot allocate device memory.
//
// specdec_dpace_forward asks its caller for scratch and for zeroed counters.
// Some callers have no way to provide them: plugin hosts whose interface hands
// a plugin only its input and output buffers (no workspace argument), and
// processes that reserve all free device memory for their own pool at start-up,
// where a later cudaMalloc fails or fragments the pool. For them,
// specdec_dpace_forward_noalloc keeps its scratch in a fixed array compiled
// into this library (kNoAllocBytes = 4 MiB, held on every GPU that loads the
// library until the process exits) and otherwise runs exactly the same
// kernels as specdec_dpace_forward.
//
// Rules, also stated in include/specdec.h:
//   - nothing here calls cudaMalloc, cudaFree or any allocating routine;
//   - the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture. The address is kept for the life of the
//     process, so the entry point must not be used on a device after
//     cudaDeviceReset (or another destruction of its primary context);
//   - every call on a device shares the one array, which keeps the last
//     call's contents: the counter region is cleared on the caller's stream
//     before each launch, and calls that overlap on the GPU (different
//     streams, no ordering between them) race on the array;
//   - the arguments are checked first, exactly as specdec_dpace_forward
//     checks them; then problems whose scratch does not fit are rejected
//     with SPECDEC_ERR_WORKSPACE; nothing is enqueued for either.
#include "specdec.h"
#include "specdec_internal.h"

#include <cstdio>
#include <mutex>

namespace {

constexpr size_t kNoAllocBytes = size_t(4) << 20;    // the whole array
constexpr size_t kCounterRegion = size_t(64) << 10;  // counters at its start, scratch after
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_setup_mu;
unsigned char* g_device_ptr[kMaxDevices] = {};

// Device address of the array on `device` (which must be current); looked up
// once per device. Returns nullptr and sets the error text on failure.
unsigned char* noalloc_base(int device) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_device_ptr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[256];
      snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the built-in scratch failed: %s",
               cudaGetErrorString(e));
      specdec::set_last_error(msg);
      return nullptr;
    }
    g_device_ptr[device] = static_cast<unsigned char*>(p);
  }
  return g_device_ptr[device];
}

}  // namespace

extern "C" int specdec_dpace_forward_noalloc(const float* logits, const int64_t* targets,
                                             const float* mask, int64_t N, int32_t B, int64_t V,
                                             float alpha, int32_t loss_type, int64_t n_global,
                                             float* loss, float* loss_n, float* lse, float* scale,
                                             int32_t* status, void* stream) {
  // argument errors first, in the allocating entry point's order, before
  // anything touches the shared array
  const int rc = specdec::dpace_forward_check(specdec::kDtypeF32, logits, targets, N, B, V, alpha, loss_type,
                                              n_global, loss, lse, scale);
  if (rc != SPECDEC_OK) return rc;
  if (N == 0) {
    // an empty batch: the allocating entry point writes the NaN loss and
    // touches no scratch
    return specdec_dpace_forward(logits, targets, mask, N, B, V, alpha, loss_type, n_global, loss,
                                 loss_n, lse, scale, status, nullptr, 0, nullptr, 0, stream);
  }
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    specdec::set_last_error("cudaGetDevice failed or device ordinal out of range");
    return SPECDEC_ERR_CUDA;
  }
  const size_t counter_bytes = specdec_dpace_counter_bytes(N, B);
  const size_t scratch_bytes = specdec_dpace_scratch_bytes(N, B, V, device);
  if (counter_bytes > kCounterRegion || scratch_bytes > kNoAllocBytes - kCounterRegion) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "problem [N=%lld, B=%d, V=%lld] needs %zu scratch + %zu counter bytes; the "
             "no-allocation entry point holds %zu + %zu",
             (long long)N, B, (long long)V, scratch_bytes, counter_bytes, kNoAllocBytes - kCounterRegion,
             kCounterRegion);
    specdec::set_last_error(msg);
    return SPECDEC_ERR_WORKSPACE;
  }
  unsigned char* base = noalloc_base(device);
  if (base == nullptr) return SPECDEC_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // counters must start at zero; a call that completes leaves them zero, this
  // also covers one that did not
  const cudaError_t e = cudaMemsetAsync(base, 0, counter_bytes, st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "clearing the built-in counters failed: %s", cudaGetErrorString(e));
    specdec::set_last_error(msg);
    return SPECDEC_ERR_CUDA;
  }
  return specdec_dpace_forward(logits, targets, mask, N, B, V, alpha, loss_type, n_global, loss,
                               loss_n, lse, scale, status, base + kCounterRegion,
                               kNoAllocBytes - kCounterRegion, base, kCounterRegion, stream);
}
