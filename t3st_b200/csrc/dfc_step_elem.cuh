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

#include "dfc_common.cuh"

namespace dfc {

struct Scalars {
  float b1, omb1, b2, omb2, sbc2, eps, decay, nstep, gscale, dscale;
};

template <int MODE>
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
  const float upd = __fdiv_rn(__fmul_rn(s.nstep, m_new), den);
  p = __fadd_rn(__fmul_rn(p, s.decay), upd);
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
