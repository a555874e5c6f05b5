"""W4A16 codec restated with the group size as a parameter (test oracle).

Follows engine/quant/w4a16.py:
  quantise    :68-105  scale = bf16(absmax / 7), all-zero group -> 1, scale
                       clamped to the smallest normal, codes = round(w / scale)
                       (ties to even) clamped to [-7, 7], two codes per byte,
                       even index in the low nibble.
  dequantise  :108-129 nibble >= 8 -> nibble - 16, times float(scale).
The kernels round the decoded value to bf16 before the dot product
(engine/kernels/w4a16_gemv.py:146-158); ``decode_bf16`` gives that value.
"""

from __future__ import annotations

import torch

QMIN, QMAX = -7, 7
REFERENCE_GROUP = 32


def quantise(weight: torch.Tensor, group: int = REFERENCE_GROUP) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [N, K] -> (packed uint8 [N, K/2], scales bf16 [N, K/group])."""
    if weight.ndim != 2:
        raise ValueError("weight must have shape [out_features, in_features]")
    if weight.dtype != torch.bfloat16:
        raise TypeError("weight must have dtype torch.bfloat16")
    n, k = weight.shape
    if k % group:
        raise ValueError(f"the reduction axis must be divisible by group size {group}")
    if not bool(torch.isfinite(weight).all()):
        raise ValueError("weight must contain only finite values")
    groups = weight.detach().reshape(n, k // group, group).float()
    absmax = groups.abs().amax(dim=-1)
    stored = (absmax / float(QMAX)).to(torch.bfloat16).float()
    tiny = torch.finfo(torch.bfloat16).tiny
    scales = torch.where(absmax == 0, torch.ones_like(stored), stored.clamp_min(tiny))
    scales = scales.to(torch.bfloat16)
    codes = torch.round(groups / scales.float().unsqueeze(-1)).clamp(QMIN, QMAX)
    codes = codes.to(torch.int16).reshape(n, k)
    nib = torch.bitwise_and(codes, 0xF).to(torch.uint8)
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    return packed.contiguous(), scales.contiguous()


def unpack_codes(packed: torch.Tensor) -> torch.Tensor:
    """uint8 [..., K/2] -> signed int16 codes [..., K] (nibble >= 8 -> nibble - 16)."""
    low = packed & 0xF
    high = packed >> 4
    nib = torch.stack((low, high), dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    signed = nib.to(torch.int16)
    return torch.where(signed >= 8, signed - 16, signed)


def dequantise(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Exact fp32 decode code * scale (no bf16 rounding), any leading dims."""
    codes = unpack_codes(packed)
    k = codes.shape[-1]
    group = k // scales.shape[-1]
    idx = torch.arange(k) // group
    return codes.float() * scales.float()[..., idx]


def decode_bf16(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Decoded weights as the kernels use them: bf16(code * scale), returned as fp32."""
    return dequantise(packed, scales).to(torch.bfloat16).float()
