"""Seeded synthetic AWQ tensors with the shapes and value distributions of the
benchmark configurations (the reference publishes no checkpoint or dataset
for this path):

* qweight / qzeros: uniform random 32-bit words, i.e. eight independent
  uniform nibbles 0..15 per word (so the packing order does not change the
  distribution),
* scales ~ U(0.001, 0.02),
* activations ~ N(0, 1).

Tensors are generated directly on the target device with a seeded
``torch.Generator``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class AWQWeights:
    qweight: torch.Tensor  # int32 [K, N/8]
    qzeros: torch.Tensor   # int32 [K/g, N/8]
    scales: torch.Tensor   # dtype [K/g, N]
    group_size: int

    @property
    def k(self) -> int:
        return self.qweight.shape[0]

    @property
    def n(self) -> int:
        return self.qweight.shape[1] * 8

    def nbytes(self) -> int:
        """Bytes the fused GEMM must read for the weights (packed + zeros + scales)."""
        return (self.qweight.numel() * 4 + self.qzeros.numel() * 4
                + self.scales.numel() * self.scales.element_size())


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def random_words(shape, device, gen: torch.Generator) -> torch.Tensor:
    return torch.randint(-(2 ** 31), 2 ** 31, shape, dtype=torch.int64, device=device,
                         generator=gen).to(torch.int32)


def make_weights(k: int, n: int, group_size: int, dtype: torch.dtype = torch.float16,
                 device="cuda", seed: int = 0x5EED, scale_lo: float = 0.001,
                 scale_hi: float = 0.02) -> AWQWeights:
    g = _gen(device, seed)
    qweight = random_words((k, n // 8), device, g)
    qzeros = random_words((k // group_size, n // 8), device, g)
    scales = (torch.rand((k // group_size, n), device=device, generator=g, dtype=torch.float32)
              * (scale_hi - scale_lo) + scale_lo).to(dtype)
    return AWQWeights(qweight, qzeros, scales, group_size)


def make_input(rows: int, k: int, dtype: torch.dtype = torch.float16, device="cuda",
               seed: int = 0x1234, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    g = _gen(device, seed)
    x = torch.randn((rows, k), device=device, generator=g, dtype=torch.float32).to(dtype)
    if out is not None:
        out.copy_(x)
        return out
    return x
