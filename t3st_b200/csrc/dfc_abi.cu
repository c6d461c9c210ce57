// Version, status strings, the per-thread CUDA error slot of the C ABI and
// the SM-count cache used to size persistent grids.
#include <atomic>

#include "dfc_common.cuh"

namespace dfc {
namespace {
thread_local int g_last_cuda_error = 0;
constexpr int kMaxDevices = 256;
std::atomic<int> g_sm_count[kMaxDevices];  // 0 until read
}  // namespace

void set_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return 148;
  }
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 148;
    }
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace dfc

extern "C" int dfc_abi_version(void) { return DFC_ABI_VERSION; }

extern "C" int dfc_last_cuda_error(void) { return dfc::g_last_cuda_error; }

extern "C" const char* dfc_strerror(int status) {
  switch (status) {
    case DFC_OK: return "ok";
    case DFC_ERR_NULL: return "required pointer is NULL";
    case DFC_ERR_ALIGN: return "pointer not aligned to its element size";
    case DFC_ERR_SIZE: return "negative, inconsistent or too large size";
    case DFC_ERR_DTYPE: return "unsupported gradient element type";
    case DFC_ERR_MODE: return "unknown moment-word format";
    case DFC_ERR_HYPER: return "hyper-set index out of range";
    case DFC_ERR_CUDA: return "CUDA runtime error";
    case DFC_ERR_RANGE: return "fiber range out of bounds";
    case DFC_ERR_SCRATCH: return "scratch buffer too small";
    default: return "unknown status";
  }
}
