"""Kimi-Linear MoE decode layer on the B200 kernels.

The composition of KLinearMoE.forward with grouped W4A16 banks
(engine/klinear/moe.py:278-334, :375-398) in three launches:

  1. moe_router          fp32 logits, sigmoid, biased top-k, renormalised and
                         scaled weights (engine/klinear/router.py:47-85); it also
                         appends the shared expert (bank slot E) as the last
                         route (engine/klinear/moe.py:23-36, :284-286)
  2. w4a16_swiglu        gate/up for the k routed experts and the shared expert
  3. moe_down_combine    down projection of every route + weighted combine,
                         shared route added with weight 1

Banks follow the reference layout: [E+1, N, K/2] uint8 codes and
[E+1, N, K/group] bf16 scales, slot E holding the shared expert.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class MoELayerWeights:
    router_weight: torch.Tensor  # bf16 [E, H]
    router_bias: torch.Tensor | None  # fp32 [E] (e_score_correction_bias)
    w1_packed: torch.Tensor  # uint8 [E+1, I, H/2]
    w1_scales: torch.Tensor  # bf16 [E+1, I, H/g]
    w2_packed: torch.Tensor  # uint8 [E+1, H, I/2]
    w2_scales: torch.Tensor  # bf16 [E+1, H, I/g]
    w3_packed: torch.Tensor
    w3_scales: torch.Tensor
    top_k: int = 8
    scaling: float = 2.446

    @property
    def num_experts(self) -> int:
        return int(self.router_weight.shape[0])

    @property
    def intermediate(self) -> int:
        return int(self.w1_packed.shape[1])


def stable_indices(idx: torch.Tensor, shared_id: int) -> torch.Tensor:
    """Append the shared expert as the last route of every token."""
    shared = torch.full((idx.shape[0], 1), shared_id, dtype=idx.dtype, device=idx.device)
    return torch.cat((idx, shared), dim=1)


def moe_forward(
    hidden: torch.Tensor, layer: MoELayerWeights
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """hidden bf16 [T, H] -> (output bf16 [T, H], indices [T, k], weights fp32 [T, k])."""
    stable, weights = ops.moe_router(
        hidden, layer.router_weight, layer.router_bias, layer.top_k,
        routed_scaling_factor=layer.scaling, append_expert=layer.num_experts,
    )
    idx = stable[:, : layer.top_k]
    activated = ops.w4a16_swiglu(
        hidden, stable, layer.w1_packed, layer.w1_scales, layer.w3_packed, layer.w3_scales
    )
    out = ops.moe_down_combine(activated, stable, weights, layer.w2_packed, layer.w2_scales)
    return out, idx, weights
