"""The reference's DFC-AdamW step as eager PyTorch CPU ops -- TEST
INFRASTRUCTURE / CPU BASELINE ONLY (bench.py's cpu_baseline leg and
``--impl reference`` arm time it; the product never imports it).

``step_fp32`` follows remote/torch_fiber.py:68-117 op for op (sign-fiber
decode with bitwise_and / abs, mul_ + add_(alpha), mul_ + addcmul_, sqrt /
div_ / add_, mul_ + addcdiv_, payload re-embedding), on the host's cores
with PyTorch's intra-op threads -- the reference's own CPU path restated.
``step_packed`` wraps the same ops with the packed-word decode/encode
(integer tensor ops), the CPU counterpart of the B200 packed format, which
the reference itself does not have.
"""

from __future__ import annotations

import math

import torch

SIGN = -2147483648
MAG = 2147483647


def _dec_mag(w: torch.Tensor) -> torch.Tensor:
    """Packed 31-bit magnitude word -> FP32 magnitude bits (int32 ops)."""
    hi = w >> 16
    r = (w & -65536) + ((w << 16) >> 16)
    r = torch.clamp(r, 0, 0x7F800000)
    return torch.where(hi > 0x7F80, w, r)


def _enc_mag(a: torch.Tensor) -> torch.Tensor:
    return torch.where(a > 0x7F800000, torch.full_like(a, 0x7FC00000), a + ((a & 0x8000) << 1))


def _enc_signed(b: torch.Tensor) -> torch.Tensor:
    a = b & MAG
    return torch.where(a > 0x7F800000, torch.full_like(a, 0x7FC00000), (b & SIGN) | _enc_mag(a))


def step_fp32(p, g, m, v, lr, betas, eps, weight_decay, step, fiber=True):
    """remote/torch_fiber.py:83-116 on CPU FP32 tensors, in place."""
    beta1, beta2 = betas
    g = g.float()
    if fiber:
        payload = torch.bitwise_and(v.view(torch.int32), SIGN)
        second = v.abs()
    else:
        second = v
    m.mul_(beta1).add_(g, alpha=1.0 - beta1)
    second.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    if fiber:
        bits = torch.bitwise_or(torch.bitwise_and(second.view(torch.int32), MAG), payload)
        v.copy_(bits.view(torch.float32))
        upd = v.abs()
    else:
        upd = v
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    den = upd.sqrt().div_(math.sqrt(bc2)).add_(eps)
    if weight_decay:
        p.mul_(1.0 - lr * weight_decay)
    p.addcdiv_(m, den, value=-(lr / bc1))


def step_packed(p, g, mw, vw, lr, betas, eps, weight_decay, step):
    """Packed-word moments (int32 tensors): decode, the reference's update,
    re-encode; bit 31 of vw is the payload and is kept."""
    beta1, beta2 = betas
    g = g.float()
    m = ((mw & SIGN) | _dec_mag(mw & MAG)).view(torch.float32)
    payload = vw & SIGN
    v = _dec_mag(vw & MAG).view(torch.float32)
    m.mul_(beta1).add_(g, alpha=1.0 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    vb = v.view(torch.int32) & MAG
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    den = vb.view(torch.float32).sqrt().div_(math.sqrt(bc2)).add_(eps)
    if weight_decay:
        p.mul_(1.0 - lr * weight_decay)
    p.addcdiv_(m, den, value=-(lr / bc1))
    mw.copy_(_enc_signed(m.view(torch.int32)))
    vw.copy_(payload | _enc_mag(vb))
