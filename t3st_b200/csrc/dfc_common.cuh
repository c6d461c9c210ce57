// Shared device helpers of libdfc_b200.so: FP32 bit views, the packed moment
// word, and the status bookkeeping of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "dfc_b200.h"

namespace dfc {

// Status of the last CUDA failure on this host thread (dfc_last_cuda_error).
void set_cuda_error(cudaError_t e);

// Number of SMs of the current device (read once per device, then cached).
int sm_count();

// CTAs of `kernel` (threads per CTA, no dynamic shared memory) that are
// resident at once on the current device: the largest grid a grid-stride
// kernel should get, so that no CTA waits for a second wave.
template <typename Kernel>
int resident_ctas(Kernel kernel, int threads) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  return sm_count() * per_sm;
}

// Check for a launch error after queueing kernels.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return DFC_ERR_CUDA;
  }
  return DFC_OK;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// ---- packed moment word -------------------------------------------------
// For a 31-bit FP32 magnitude a:
//   enc(a) = a + ((a & 0x8000) << 1)   (a <= +Inf: the high half becomes a
//            rounded to the nearest bf16, ties away from zero, and the low
//            half -- unchanged -- read as int16 is the residual in ulps)
//   enc(a) = 0x7FC00000                (NaN: the canonical quiet NaN, so the
//            CPU and GPU words agree whatever NaN the arithmetic produced)
// dec(w) = (hi << 16) + (int16)lo, clamped to [0, +Inf]; hi > 0x7F80 is a NaN
// and decodes to itself.  dec(enc(a)) == a for every non-NaN a.
__device__ __forceinline__ uint32_t enc_mag(uint32_t a) {
  return a > 0x7F800000u ? 0x7FC00000u : a + ((a & 0x8000u) << 1);
}

// Signed value bits -> packed word; a NaN becomes the canonical +NaN word.
__device__ __forceinline__ uint32_t enc_signed_bits(uint32_t b) {
  const uint32_t a = b & 0x7FFFFFFFu;
  return a > 0x7F800000u ? 0x7FC00000u : (b & 0x80000000u) | (a + ((a & 0x8000u) << 1));
}

__device__ __forceinline__ uint32_t dec_mag(uint32_t w) {
  int32_t r = static_cast<int32_t>(w & 0xFFFF0000u) + (static_cast<int32_t>(w << 16) >> 16);
  r = min(max(r, 0), 0x7F800000);
  return (w >> 16) > 0x7F80u ? w : static_cast<uint32_t>(r);
}

__device__ __forceinline__ uint32_t pack_signed(float x) { return enc_signed_bits(f2u(x)); }

__device__ __forceinline__ float unpack_signed(uint32_t w) {
  return u2f((w & 0x80000000u) | dec_mag(w & 0x7FFFFFFFu));
}

// Residual carried by a (bf16 value, residual field) pair of the compressed
// gradient: dec(c:q) - c, exact (Sterbenz); zero when c is Inf/NaN.
__device__ __forceinline__ float ef_residual(uint32_t c, uint32_t q) {
  uint32_t hm = c & 0x7FFFu;
  float s = u2f(((c & 0x8000u) << 16) | dec_mag((hm << 16) | (q & 0xFFFFu)));
  float r = __fsub_rn(s, bf16_bits_to_f32(c));
  return hm >= 0x7F80u ? 0.0f : r;
}

}  // namespace dfc
