"""KDA decode preparation restated on the CPU (test oracle, not product code).

Between the q/k/v projections and the KDA recurrent step, a decode token goes
through (engine/klinear/attention.py:192-230, fused path):

  short_conv3   the width-4 depthwise causal convolution of each of q, k and v
                (engine/kernels/kda_prepare.py:426-472): the state [B, C, 4]
                shifts left by one and takes the new token last; the output is
                silu(sum_w float(state'[w]) * float(weight[w])) rounded to the
                input dtype; the state is updated in place;
  gates         (engine/kernels/kda_prepare.py:581-615, attention.py:167-172):
                decay = -exp(A_log[h]) * softplus(raw_decay + dt_bias) in fp32
                (softplus(x) = x above 20, log(1 + exp(x)) otherwise, as
                F.softplus), beta = sigmoid(raw_beta), q and k per head
                multiplied by rsqrt(sum of squares + eps) in fp32.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def short_conv(values: torch.Tensor, state: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """One width-4 decode convolution: values [B, 1, C] (or [B, C]), state
    [B, C, 4] updated in place, weight [C, 1, 4] or [C, 4] -> [B, 1, C] in
    the values' dtype (engine/kernels/kda_prepare.py:426-436)."""
    token = values.reshape(values.shape[0], -1)
    shifted = torch.cat((state[:, :, 1:], token.unsqueeze(-1)), dim=-1)
    w = weight[:, 0, :] if weight.ndim == 3 else weight
    convolved = F.silu((shifted.float() * w.float().unsqueeze(0)).sum(dim=-1))
    state.copy_(shifted)
    return convolved.to(values.dtype).unsqueeze(1)


def short_conv3(q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight, v_weight):
    """The three convolutions of q, k and v (kda_prepare.py:439-472)."""
    return (short_conv(q_in, q_state, q_weight), short_conv(k_in, k_state, k_weight),
            short_conv(v_in, v_state, v_weight))


def gates(raw_decay: torch.Tensor, dt_bias: torch.Tensor, a_log: torch.Tensor,
          raw_beta: torch.Tensor, q: torch.Tensor, k: torch.Tensor, *, num_heads: int,
          head_dim: int, eps: float = 1e-6):
    """(decay fp32 [B,1,H,D], beta fp32 [B,1,H], q and k normalised fp32
    [B,1,H,D]) -- kda_prepare.py:581-615."""
    batch = raw_decay.shape[0]
    biased = raw_decay.float().reshape(batch, 1, num_heads, head_dim) + dt_bias.float().view(
        num_heads, head_dim)
    rate = a_log.float().reshape(1, 1, num_heads, 1).exp()
    decay = -rate * F.softplus(biased)
    beta = torch.sigmoid(raw_beta.float().reshape(batch, 1, num_heads))
    qn = q.reshape(batch, 1, num_heads, head_dim).float()
    kn = k.reshape(batch, 1, num_heads, head_dim).float()
    qn = qn * torch.rsqrt(qn.square().sum(dim=-1, keepdim=True) + eps)
    kn = kn * torch.rsqrt(kn.square().sum(dim=-1, keepdim=True) + eps)
    return decay, beta, qn, kn


def prepare(q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight, v_weight,
            raw_decay, dt_bias, a_log, raw_beta, *, num_heads: int, head_dim: int,
            eps: float = 1e-6):
    """Convolutions then gates: (q, k, v fp32 [B,H,D], decay fp32 [B,H,D],
    beta fp32 [B,H]) -- the inputs of the KDA step (attention.py:192-230)."""
    q, k, v = short_conv3(q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight,
                          v_weight)
    decay, beta, qn, kn = gates(raw_decay, dt_bias, a_log, raw_beta, q, k,
                                num_heads=num_heads, head_dim=head_dim, eps=eps)
    batch = q_in.shape[0]
    return (qn[:, 0], kn[:, 0], v.reshape(batch, num_heads, head_dim).float(), decay[:, 0],
            beta[:, 0])
