"""One Kimi-Linear MoE decode layer in the reference's grouped structure (test oracle).

Restates KLinearMoE.forward with grouped W4A16 banks
(engine/klinear/moe.py:278-334 and :375-398):
  router top-k -> append the shared expert as route R-1 (bank slot E)
  -> w4a16_swiglu over all routes -> w4a16_grouped down projection
  -> bf16(sum_r float(y_r) * w_r) + y_shared.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class MoEBanks:
    router_weight: torch.Tensor  # bf16 [E, H]
    router_bias: torch.Tensor  # fp32 [E]
    w1_packed: torch.Tensor  # uint8 [E+1, I, H/2]
    w1_scales: torch.Tensor
    w2_packed: torch.Tensor  # uint8 [E+1, H, I/2]
    w2_scales: torch.Tensor
    w3_packed: torch.Tensor
    w3_scales: torch.Tensor
    top_k: int = 8
    scaling: float = 2.446

    @property
    def num_experts(self) -> int:
        return self.router_weight.shape[0]


def moe_layer(hidden: torch.Tensor, banks: MoEBanks, *, return_parts: bool = False,
              lane_order: bool = False):
    """hidden bf16 [T, H] -> (output bf16 [T, H], indices [T, k], weights fp32 [T, k]).

    With ``return_parts`` a fourth element gives the per-element rounding bound
    of the combine (ops.combine_rounding_bound).  With ``lane_order`` the router
    logits are summed in the fixed order of ops.router_logits_lanes instead of
    the BLAS order.
    """
    logits = (ops.router_logits_lanes(hidden, banks.router_weight) if lane_order else None)
    idx, weights, _ = ops.router_topk(
        hidden, banks.router_weight, banks.router_bias, banks.top_k, scaling=banks.scaling,
        logits=logits,
    )
    stable = ops.shape_stable_indices(idx, banks.num_experts)
    activated = ops.swiglu(
        hidden, stable, banks.w1_packed, banks.w1_scales, banks.w3_packed, banks.w3_scales
    )
    out, bound = ops.w2_combine(
        activated, stable, weights, banks.w2_packed, banks.w2_scales, return_parts=True
    )
    if return_parts:
        return out, idx, weights, bound
    return out, idx, weights
