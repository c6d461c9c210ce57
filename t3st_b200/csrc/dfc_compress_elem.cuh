// bf16 error-feedback compression, element and tile arithmetic shared by the
// compression kernels (dfc_compress.cu) and the ZeRO-1 fused step, whose grid
// compresses the next bucket beside its own tiles (dfc_peer.cu).
//
// Per element: s = g + e (e recovered exactly from the previous call's
// (comp, resid) pair), then the packed-word encoding of s is split into its
// two halves: comp = bf16 of s (round to nearest, ties away from zero),
// resid = signed 16-bit residual in FP32 ulps, so that s == dec(comp:resid)
// bit for bit.
#pragma once

#include "dfc_common.cuh"

namespace dfc {

__device__ __forceinline__ void compress1(float g, uint32_t& c, uint32_t& q) {
  const float s = __fadd_rn(g, ef_residual(c, q));
  const uint32_t w = enc_signed_bits(f2u(s));
  c = w >> 16;
  q = w & 0xFFFFu;
}

// Four elements (one float4 of g, one 8-byte word each of comp and resid)
// per quad; bits of lane u in the 16-bit halves of the words.
__device__ __forceinline__ void compress_quad(const float4& G, uint2& C, uint2& Q) {
  uint32_t c0 = C.x & 0xFFFFu, c1 = C.x >> 16, c2 = C.y & 0xFFFFu, c3 = C.y >> 16;
  uint32_t q0 = Q.x & 0xFFFFu, q1 = Q.x >> 16, q2 = Q.y & 0xFFFFu, q3 = Q.y >> 16;
  compress1(G.x, c0, q0);
  compress1(G.y, c1, q1);
  compress1(G.z, c2, q2);
  compress1(G.w, c3, q3);
  C = make_uint2(c0 | (c1 << 16), c2 | (c3 << 16));
  Q = make_uint2(q0 | (q1 << 16), q2 | (q3 << 16));
}

// Tile `tile` of 2 x THREADS quads of a buffer of n4 quads, by a CTA of
// THREADS threads: thread t takes quads t and t + THREADS of the tile (each
// warp-wide access covers 32 consecutive quads), both quads' loads issued
// before either is used.  grad 16-byte aligned, comp and resid 8-byte aligned.
template <int THREADS>
__device__ __forceinline__ void compress_tile(const float* __restrict__ g,
                                              uint16_t* __restrict__ comp,
                                              uint16_t* __restrict__ resid, int64_t n4,
                                              int64_t tile) {
  const float4* g4 = reinterpret_cast<const float4*>(g);
  uint2* c2 = reinterpret_cast<uint2*>(comp);
  uint2* q2 = reinterpret_cast<uint2*>(resid);
  const int64_t j = tile * (2 * THREADS) + threadIdx.x;
  const int64_t k = j + THREADS;
  float4 G0 = make_float4(0.f, 0.f, 0.f, 0.f), G1 = G0;
  uint2 C0 = make_uint2(0u, 0u), C1 = C0, Q0 = C0, Q1 = C0;
  if (j < n4) {
    G0 = __ldcs(g4 + j);
    C0 = __ldcs(c2 + j);
    Q0 = __ldcs(q2 + j);
  }
  if (k < n4) {
    G1 = __ldcs(g4 + k);
    C1 = __ldcs(c2 + k);
    Q1 = __ldcs(q2 + k);
  }
  if (j < n4) {
    compress_quad(G0, C0, Q0);
    __stcs(c2 + j, C0);
    __stcs(q2 + j, Q0);
  }
  if (k < n4) {
    compress_quad(G1, C1, Q1);
    __stcs(c2 + k, C1);
    __stcs(q2 + k, Q1);
  }
}

}  // namespace dfc
