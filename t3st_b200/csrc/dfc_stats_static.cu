// dfc_grad_stats_noalloc: the gradient statistics of dfc_grad_stats for
// callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc (or any allocating
// routine, torch's caching allocator included) at the point where they want
// gradient statistics: a host runtime that has handed all device memory to
// its own pool, or a plugin whose host forbids device allocations while a
// training step runs.  This entry point takes only the gradients and the
// output records; the per-tile partial records that dfc_grad_stats keeps in
// a caller-provided scratch buffer live here instead in a file-scope device
// array of DFC_GRAD_STATS_STATIC_RECORDS records (24 bytes each, 1.5 MiB),
// which every GPU that loads the library holds until the process exits.
//
// Host code must not pass the array's name to a kernel: on the host it is a
// stand-in symbol, not a device address.  The first call on each device
// (with that device current) looks the address up once with
// cudaGetSymbolAddress and caches it; that first call should therefore come
// before any stream capture.  The cached address belongs to the device's
// primary context: after cudaDeviceReset on a device this entry point must
// not be called again on it in the same process.  Every call shares the one array per device and
// it keeps the last call's contents; nothing needs clearing, because each
// call writes every partial record before its second pass reads it.  Calls
// whose kernels overlap on the GPU (different streams, no ordering) race on
// the array; order them on one stream.
#include <mutex>

#include "dfc_common.cuh"

namespace dfc {

// Shared with dfc_grad_stats (dfc_stats.cu).
int grad_stats_launch(const DfcGradRef* grads, int32_t n_grads, DfcGradStats* out,
                      DfcGradStats* partial, cudaStream_t st);
size_t grad_stats_records(const DfcGradRef* grads, int32_t n_grads);
int grad_stats_validate(const DfcGradRef* grads, int32_t n_grads);

namespace {

static __device__ __align__(256) DfcGradStats g_partial_records[DFC_GRAD_STATS_STATIC_RECORDS];

constexpr int kMaxDevices = 256;
std::mutex g_setup_mutex;
DfcGradStats* g_partial_ptr[kMaxDevices] = {};

// Device address of g_partial_records on the current device (set-up on the
// first call per device).
int partial_records(DfcGradStats** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return DFC_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return DFC_ERR_SIZE;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_partial_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_partial_records);
    if (e != cudaSuccess || p == nullptr) {
      set_cuda_error(e);
      return DFC_ERR_CUDA;
    }
    g_partial_ptr[dev] = static_cast<DfcGradStats*>(p);
  }
  *out = g_partial_ptr[dev];
  return DFC_OK;
}

}  // namespace
}  // namespace dfc

extern "C" int dfc_grad_stats_noalloc(const DfcGradRef* grads, int32_t n_grads, DfcGradStats* out,
                                      void* stream) {
  using namespace dfc;
  int rc = grad_stats_validate(grads, n_grads);
  if (rc != DFC_OK) return rc;
  if (n_grads == 0) return DFC_OK;
  if (!out) return DFC_ERR_NULL;
  if (!aligned(out, 8)) return DFC_ERR_ALIGN;
  if (grad_stats_records(grads, n_grads) > static_cast<size_t>(DFC_GRAD_STATS_STATIC_RECORDS))
    return DFC_ERR_SCRATCH;
  DfcGradStats* partial = nullptr;
  rc = partial_records(&partial);
  if (rc != DFC_OK) return rc;
  return grad_stats_launch(grads, n_grads, out, partial, static_cast<cudaStream_t>(stream));
}
