"""Seeded synthetic workloads for the DFC-AdamW step (shapes and value
distributions only; no datasets, no checkpoints).

resnet18_cifar_shapes   62 parameter shapes of ResNet-18 with a 3x3 stem,
                        no max-pool and a 10-class head (11,173,962 elements)
ragged_sizes            4096 sizes log-uniform in [1, 4M] with forced sizes
                        that are not multiples of 4 or 8
"""

from __future__ import annotations

import math

import numpy as np
import torch


def resnet18_cifar_shapes(num_classes: int = 10) -> list[tuple[int, ...]]:
    """Parameter shapes in ``model.parameters()`` order for torchvision's
    BasicBlock ResNet-18 with conv1 = 3x3/stride 1 and no max-pool."""
    shapes: list[tuple[int, ...]] = [(64, 3, 3, 3), (64,), (64,)]
    cin = 64
    for cout, stride in ((64, 1), (128, 2), (256, 2), (512, 2)):
        for block in range(2):
            s = stride if block == 0 else 1
            shapes += [(cout, cin, 3, 3), (cout,), (cout,), (cout, cout, 3, 3), (cout,), (cout,)]
            if s != 1 or cin != cout:
                shapes += [(cout, cin, 1, 1), (cout,), (cout,)]
            cin = cout
    shapes += [(num_classes, 512), (num_classes,)]
    return shapes


RESNET18_CIFAR_NUMEL = 11_173_962


def ragged_sizes(seed: int = 0, n: int = 4096, max_size: int = 4 * 1024 * 1024) -> list[int]:
    """Sizes floor(exp(U(0, ln max_size))) >= 1, the first 64 forced to
    awkward values (1..8, 4k+-1, 8k+-3, odd millions)."""
    rng = np.random.default_rng(seed)
    sizes = np.floor(np.exp(rng.uniform(0.0, math.log(max_size), n))).astype(np.int64)
    sizes = np.maximum(sizes, 1)
    forced = [1, 2, 3, 5, 6, 7, 9, 11, 13, 15, 17, 4095, 4097, 4099, 8189, 8195, 12291,
              65537, 65539, 131071, 262147, 1048573, 1048579, 2097149, 3999999, 4194301]
    sizes[: len(forced)] = forced[: n]
    return [int(s) for s in sizes]


def normal_(t: torch.Tensor, std: float, gen: torch.Generator) -> torch.Tensor:
    return t.normal_(0.0, std, generator=gen)


def student_t_grads_(t: torch.Tensor, gen: torch.Generator, scale: float = 1e-3,
                     zero_frac: float = 0.05, denormal_frac: float = 0.001) -> torch.Tensor:
    """Student-t(3) * scale with exact zeros and FP32 denormals mixed in, in place."""
    n = t.numel()
    z = torch.randn(n, 4, device=t.device, generator=gen)
    chi2 = (z[:, 1:] ** 2).sum(dim=1)
    val = z[:, 0] / torch.sqrt(chi2 / 3.0) * scale
    u = torch.rand(n, device=t.device, generator=gen)
    val = torch.where(u < zero_frac, torch.zeros_like(val), val)
    den_bits = torch.randint(1, 1 << 23, (n,), device=t.device, generator=gen, dtype=torch.int32)
    sign = torch.randint(0, 2, (n,), device=t.device, generator=gen, dtype=torch.int32) << 31
    den = (den_bits | sign).view(torch.float32)
    val = torch.where(u > 1.0 - denormal_frac, den, val)
    t.view(-1).copy_(val)
    return t


def random_residual_fields_(words: torch.Tensor, gen: torch.Generator) -> torch.Tensor:
    """Replace the low 16 bits of every word with uniform random bits."""
    lo = torch.randint(0, 1 << 16, words.shape, device=words.device, generator=gen,
                       dtype=torch.int32)
    w = words.view(torch.int32)
    w.copy_((w & -65536) | lo)
    return words


def random_payload_(words: torch.Tensor, gen: torch.Generator) -> torch.Tensor:
    """Set bit 31 of every word to a uniform random bit."""
    bit = torch.randint(0, 2, words.shape, device=words.device, generator=gen, dtype=torch.int32)
    w = words.view(torch.int32)
    w.copy_((w & 0x7FFFFFFF) | (bit << 31))
    return words
