"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

Weights are drawn ~N(0, 0.02) in bf16 and quantised; activations ~N(0, 1) in
bf16.  Seed 0 is used for weights and seed 1 for activations unless a caller
passes others.  The CPU generator is used here; GPU tests draw on the device
with a CUDA generator of the same seeds and copy what the oracle needs.
"""

from __future__ import annotations

import torch

from . import codec
from .moe import MoEBanks

WEIGHT_STD = 0.02


def generator(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def weight(shape: tuple[int, ...], gen: torch.Generator) -> torch.Tensor:
    return (torch.randn(shape, generator=gen) * WEIGHT_STD).to(torch.bfloat16)


def activations(shape: tuple[int, ...], gen: torch.Generator) -> torch.Tensor:
    return torch.randn(shape, generator=gen).to(torch.bfloat16)


def quantised(n: int, k: int, group: int, gen: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
    return codec.quantise(weight((n, k), gen), group)


def bank(experts: int, n: int, k: int, group: int, gen: torch.Generator):
    packed, scales = zip(*(quantised(n, k, group, gen) for _ in range(experts)))
    return torch.stack(packed), torch.stack(scales)


def moe_banks(
    hidden: int, experts: int, inter: int, group: int, seed: int = 0, top_k: int = 8,
    scaling: float = 2.446,
) -> MoEBanks:
    """Router + (experts + 1 shared) expert banks, all from one seeded generator."""
    gen = generator(seed)
    router = weight((experts, hidden), gen)
    w1p, w1s = bank(experts + 1, inter, hidden, group, gen)
    w2p, w2s = bank(experts + 1, hidden, inter, group, gen)
    w3p, w3s = bank(experts + 1, inter, hidden, group, gen)
    return MoEBanks(router, torch.zeros(experts), w1p, w1s, w2p, w2s, w3p, w3s, top_k, scaling)
