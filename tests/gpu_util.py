"""Helpers for the GPU parity tests: seeded device inputs and oracle copies."""

from __future__ import annotations

import torch

from local_kimi_b200 import ops

WEIGHT_STD = 0.02


def cuda_gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def rand_weight(shape, gen, std: float = WEIGHT_STD) -> torch.Tensor:
    return (torch.randn(shape, generator=gen, device="cuda") * std).to(torch.bfloat16)


def rand_act(shape, gen) -> torch.Tensor:
    return torch.randn(shape, generator=gen, device="cuda").to(torch.bfloat16)


def quant_matrix(n: int, k: int, group: int, gen, std: float = WEIGHT_STD):
    """Quantise a seeded N(0, std) matrix on the device (packed, scales)."""
    return ops.quantise(rand_weight((n, k), gen, std), group)


def quant_bank(experts: int, n: int, k: int, group: int, gen, std: float = WEIGHT_STD):
    w = rand_weight((experts * n, k), gen, std)
    packed, scales = ops.quantise(w, group)
    return packed.view(experts, n, k // 2), scales.view(experts, n, k // group)


def zipf_indices(tokens: int, experts: int, top_k: int, s: float, seed: int,
                 max_load: int | None = None) -> torch.Tensor:
    """Per token, top_k distinct experts drawn with Zipf(s) popularity over a
    seeded permutation of the experts (CPU int64 [tokens, top_k])."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(experts, generator=g)
    ranks = torch.arange(1, experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    load = torch.zeros(experts, dtype=torch.long)
    rows = []
    for _ in range(tokens):
        probs = p.clone()
        if max_load is not None:
            full = load[perm] >= max_load
            probs[full] = 0
        pick = torch.multinomial(probs, top_k, replacement=False, generator=g)
        chosen = perm[pick]
        load[chosen] += 1
        rows.append(chosen)
    return torch.stack(rows)
