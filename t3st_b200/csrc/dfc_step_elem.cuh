// Element arithmetic of the DFC-AdamW step, shared by dfc_mt_step and the
// fused ZeRO-1 kernel.  Restates remote/torch_fiber.py:90-116 with explicit
// rounding (no contraction: -fmad=false and __f*_rn intrinsics):
//   g   = (g * grad_scale) * device_scale
//   m'  = fma(g, 1-b1, m*b1)            :98   mul_ then add_(alpha)
//   v'  = fma((1-b2)*g, g, v*b2)        :99   mul_ then addcmul_
//   den = sqrt(v')/sqrt(bc2) + eps      :112  IEEE sqrt and divide
//   p'  = p*decay + (-lr/bc1 * m')/den  :114-116 mul_, addcdiv_
// Sign fiber (:90-107): bit 31 of v is masked off before and restored after.
// Packed words: decoded before and re-encoded after with integer bit ops.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "dfc_common.cuh"

namespace dfc {

// ---- 16-bit parameter types ----------------------------------------------
// Round to nearest even with the hardware conversions (cvt.rn.bf16.f32 /
// cvt.rn.f16.f32; subnormals kept, -ftz=false); a NaN that is stored becomes
// the type's canonical quiet NaN (bf16 0x7FC0, fp16 0x7E00), as PyTorch's CPU
// conversions produce.
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float x) {
  return x != x ? 0x7FC0u : static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x)));
}

__device__ __forceinline__ uint32_t f32_to_f16_bits(float x) {
  return x != x ? 0x7E00u : static_cast<uint32_t>(__half_as_ushort(__float2half_rn(x)));
}

template <int DT>
__device__ __forceinline__ uint32_t to_bits16(float x) {
  return DT == DFC_DTYPE_BF16 ? f32_to_bf16_bits(x) : f32_to_f16_bits(x);
}

template <int DT>
__device__ __forceinline__ float from_bits16(uint32_t h) {
  return DT == DFC_DTYPE_BF16 ? u2f(h << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// x rounded to the parameter type (identity for FP32), as an intermediate
// value: a NaN stays a NaN (which one does not matter: every NaN that reaches
// a stored parameter is canonicalised by to_bits16).
template <int DT>
__device__ __forceinline__ float round_to(float x) {
  if (DT == DFC_DTYPE_F32) return x;
  if (DT == DFC_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return __half2float(__float2half_rn(x));
}

struct Scalars {
  float b1, omb1, b2, omb2, sbc2, eps, decay, nstep, gscale, dscale;
};

// p holds the parameter's value as FP32 (exact for 16-bit types) and comes
// back rounded to PDT.
template <int MODE, int PDT = DFC_DTYPE_F32>
__device__ __forceinline__ void step_elem(const Scalars& s, float& p, float gin, uint32_t& mw,
                                          uint32_t& vw) {
  const float g = __fmul_rn(__fmul_rn(gin, s.gscale), s.dscale);
  float m, v;
  uint32_t payload = 0u;
  if (MODE == DFC_MODE_PACKED) {
    m = unpack_signed(mw);
    payload = vw & 0x80000000u;
    v = u2f(dec_mag(vw & 0x7FFFFFFFu));
  } else if (MODE == DFC_MODE_SIGNFIBER) {
    m = u2f(mw);
    payload = vw & 0x80000000u;
    v = u2f(vw & 0x7FFFFFFFu);
  } else {
    m = u2f(mw);
    v = u2f(vw);
  }
  const float m_new = __fmaf_rn(g, s.omb1, __fmul_rn(m, s.b1));
  const float v_new = __fmaf_rn(__fmul_rn(s.omb2, g), g, __fmul_rn(v, s.b2));
  float v_upd;
  if (MODE == DFC_MODE_PLAIN) {
    v_upd = v_new;
    vw = f2u(v_new);
  } else {
    const uint32_t mag = f2u(v_new) & 0x7FFFFFFFu;
    v_upd = u2f(mag);
    vw = payload | (MODE == DFC_MODE_PACKED ? enc_mag(mag) : mag);
  }
  const float den = __fadd_rn(__fdiv_rn(__fsqrt_rn(v_upd), s.sbc2), s.eps);
  if (PDT == DFC_DTYPE_F32) {
    const float upd = __fdiv_rn(__fmul_rn(s.nstep, m_new), den);
    p = __fadd_rn(__fmul_rn(p, s.decay), upd);
  } else {
    const float p1 = round_to<PDT>(__fmul_rn(p, s.decay));
    const float upd = __fdiv_rn(__fmul_rn(s.nstep, round_to<PDT>(m_new)), round_to<PDT>(den));
    p = round_to<PDT>(__fadd_rn(p1, upd));
  }
  mw = MODE == DFC_MODE_PACKED ? pack_signed(m_new) : f2u(m_new);
}

__device__ __forceinline__ Scalars load_scalars(const DfcHyper& h, const float* dev_scale) {
  Scalars s;
  s.b1 = h.beta1;
  s.omb1 = h.one_minus_beta1;
  s.b2 = h.beta2;
  s.omb2 = h.one_minus_beta2;
  s.sbc2 = h.sqrt_bc2;
  s.eps = h.eps;
  s.decay = h.decay;
  s.nstep = h.neg_step_size;
  s.gscale = h.grad_scale;
  s.dscale = dev_scale ? *dev_scale : 1.0f;
  return s;
}

}  // namespace dfc
