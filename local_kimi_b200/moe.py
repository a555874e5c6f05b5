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


# From this many tokens on, the shared expert (every token's last route) runs
# on the tcgen05 tensor-core path and the routed experts on the projection
# engine; below it the fused three-launch layer is faster.
SHARED_TC_TOKENS = 64


def moe_forward(
    hidden: torch.Tensor, layer: MoELayerWeights
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """hidden bf16 [T, H] -> (output bf16 [T, H], indices [T, k], weights fp32 [T, k])."""
    stable, weights = ops.moe_router(
        hidden, layer.router_weight, layer.router_bias, layer.top_k,
        routed_scaling_factor=layer.scaling, append_expert=layer.num_experts,
    )
    idx = stable[:, : layer.top_k]
    if hidden.shape[0] >= SHARED_TC_TOKENS and _shared_on_tc(hidden, layer):
        return _moe_forward_batched(hidden, layer, stable, weights), idx, weights
    activated = ops.w4a16_swiglu(
        hidden, stable, layer.w1_packed, layer.w1_scales, layer.w3_packed, layer.w3_scales
    )
    out = ops.moe_down_combine(activated, stable, weights, layer.w2_packed, layer.w2_scales)
    return out, idx, weights


def _shared_on_tc(hidden: torch.Tensor, layer: MoELayerWeights) -> bool:
    t, h = hidden.shape
    i = layer.intermediate
    g1 = h // layer.w1_scales.shape[2]
    g2 = i // layer.w2_scales.shape[2]
    return ops.tc_supported(t, i, h, g1) and ops.tc_supported(t, h, i, g2)


def _moe_forward_batched(hidden: torch.Tensor, layer: MoELayerWeights, stable: torch.Tensor,
                         weights: torch.Tensor) -> torch.Tensor:
    """The same layer for many tokens: the shared expert's gate/up and down on
    the tensor cores (it sees every token), the routed experts' on the
    projection engine (a few rows each), then the route combine
    bf16(sum_r w_r y_r) + y_shared in route order (moe_combine.py:209-261)."""
    t, width = hidden.shape
    k = layer.top_k
    routed = stable[:, :k].contiguous()
    shared = stable[:, k:].contiguous()
    act_r = ops.w4a16_swiglu(hidden, routed, layer.w1_packed, layer.w1_scales,
                             layer.w3_packed, layer.w3_scales)
    act_s = ops.w4a16_swiglu_tc(hidden, shared, layer.w1_packed, layer.w1_scales,
                                layer.w3_packed, layer.w3_scales)
    inter = act_r.shape[-1]
    y_r = ops.w4a16_grouped(act_r.view(t * k, inter), routed.view(t * k, 1), layer.w2_packed,
                            layer.w2_scales)
    y_s = ops.w4a16_grouped_tc(act_s.view(t, inter), shared, layer.w2_packed, layer.w2_scales)
    routes = torch.cat((y_r.view(t, k, width), y_s), dim=1)
    return ops.moe_combine_routes(routes, weights)
