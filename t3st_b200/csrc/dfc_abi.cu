// Version, status strings and the per-thread CUDA error slot of the C ABI.
#include "dfc_common.cuh"

namespace dfc {
namespace {
thread_local int g_last_cuda_error = 0;
}  // namespace

void set_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

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
