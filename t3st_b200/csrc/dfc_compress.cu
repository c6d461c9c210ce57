// bf16 gradient compression with per-element error feedback (the arithmetic
// is in dfc_compress_elem.cuh).  12 bytes of HBM traffic per element: g (4 B
// read), comp and resid (2+2 B read, 2+2 B written).  Streaming
// 128-bit/64-bit accesses.
//
// Two grid shapes.  Alone on the GPU (ctas_per_sm <= 0): one CTA per tile of
// 2048 elements, CTAs dispatched in address order, so the accesses in flight
// stay in one compact window of the buffer -- 1.07 of the measured copy
// bandwidth on B200 over 2^28 elements.  A persistent grid-stride form of the
// same arithmetic reached 0.86 at 8 CTAs per SM (its warps drift apart over
// the whole buffer) and 0.93 at 4.  Beside another kernel (ctas_per_sm > 0,
// the ZeRO-1 pipeline's fused step) the persistent form keeps a fixed number
// of CTAs per SM, so that the other kernel always finds room.
#include <algorithm>

#include "dfc_compress_elem.cuh"

namespace dfc {
namespace {

constexpr int kThreads = 256;

// Grid-stride over quads, two quads (a grid stride apart) per thread per
// iteration: both quads' loads are issued before either is used, so a
// capped grid (a few CTAs per SM) still keeps enough bytes in flight.  Each
// warp-wide access covers 32 consecutive quads.
__global__ void __launch_bounds__(kThreads)
    compress_vec_kernel(const float* __restrict__ g, uint16_t* __restrict__ comp,
                        uint16_t* __restrict__ resid, int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  uint2* c2 = reinterpret_cast<uint2*>(comp);
  uint2* q2 = reinterpret_cast<uint2*>(resid);
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; j < n4; j += 2 * stride) {
    const int64_t k = j + stride;
    const bool two = k < n4;
    const float4 G0 = __ldcs(g4 + j);
    uint2 C0 = __ldcs(c2 + j);
    uint2 Q0 = __ldcs(q2 + j);
    float4 G1 = make_float4(0.f, 0.f, 0.f, 0.f);
    uint2 C1 = make_uint2(0u, 0u), Q1 = make_uint2(0u, 0u);
    if (two) {
      G1 = __ldcs(g4 + k);
      C1 = __ldcs(c2 + k);
      Q1 = __ldcs(q2 + k);
    }
    compress_quad(G0, C0, Q0);
    __stcs(c2 + j, C0);
    __stcs(q2 + j, Q0);
    if (two) {
      compress_quad(G1, C1, Q1);
      __stcs(c2 + k, C1);
      __stcs(q2 + k, Q1);
    }
  }
}

// One tile of 2 x kThreads quads per CTA (compress_tile).
__global__ void __launch_bounds__(kThreads)
    compress_tile_kernel(const float* __restrict__ g, uint16_t* __restrict__ comp,
                         uint16_t* __restrict__ resid, int64_t n4) {
  compress_tile<kThreads>(g, comp, resid, n4, blockIdx.x);
}

__global__ void __launch_bounds__(kThreads)
    compress_scalar_kernel(const float* __restrict__ g, uint16_t* __restrict__ comp,
                           uint16_t* __restrict__ resid, int64_t begin, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += stride) {
    uint32_t c = comp[i], q = resid[i];
    compress1(g[i], c, q);
    comp[i] = static_cast<uint16_t>(c);
    resid[i] = static_cast<uint16_t>(q);
  }
}

// ctas_per_sm CTAs per SM (8, the whole SM at 256 threads, by default);
// fewer for small buffers.  A smaller figure leaves room on every SM for a
// kernel that runs beside this one (the ZeRO-1 fused step).
// (never more than are resident at once: a grid-stride CTA that waits for a
// second wave would finish its share late).
template <typename Kernel>
int grid_for(Kernel kernel, int64_t work, int32_t ctas_per_sm) {
  const int64_t per_sm = ctas_per_sm > 0 ? std::min(ctas_per_sm, 8) : 8;
  const int64_t cap = std::min<int64_t>(sm_count() * per_sm, resident_ctas(kernel, kThreads));
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + kThreads - 1) / kThreads, cap)));
}

}  // namespace
}  // namespace dfc

extern "C" int dfc_compress_ef(const float* grad, uint16_t* comp, uint16_t* resid, int64_t n,
                               int32_t ctas_per_sm, void* stream) {
  using namespace dfc;
  if (n < 0) return DFC_ERR_SIZE;
  if (n == 0) return DFC_OK;
  if (!grad || !comp || !resid) return DFC_ERR_NULL;
  if (!aligned(grad, 4) || !aligned(comp, 2) || !aligned(resid, 2)) return DFC_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t done = 0;
  if (aligned(grad, 16) && aligned(comp, 8) && aligned(resid, 8)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      if (ctas_per_sm <= 0) {
        const int64_t tiles = (n4 + 2 * kThreads - 1) / (2 * kThreads);
        if (tiles > INT32_MAX) return DFC_ERR_SIZE;
        compress_tile_kernel<<<static_cast<unsigned>(tiles), kThreads, 0, st>>>(grad, comp, resid, n4);
      } else {
        compress_vec_kernel<<<grid_for(compress_vec_kernel, n4, ctas_per_sm), kThreads, 0, st>>>(grad, comp, resid, n4);
      }
    }
    done = n4 * 4;
  }
  if (done < n)
    compress_scalar_kernel<<<grid_for(compress_scalar_kernel, n - done, ctas_per_sm), kThreads, 0, st>>>(grad, comp, resid, done, n);
  return launch_status();
}
