"""The hot-path decode step chained through the oracle (test infrastructure).

Restates one decode step of the synthetic Kimi-Linear hot path layer by layer
with the oracle's operators, so that a whole multi-layer program of the B200
decode-step executor can be checked against the CPU, not only against the
per-operation path.  The step follows the reference model's order of INT4
operations (engine/klinear/model.py:412 and the layer bodies of
engine/klinear/attention.py and engine/klinear/moe.py:278-334):

  KDA layer:  q/k/v projections of x (w4a16_fused_qkv.py:257-271); with
              ``prepare`` their short convolutions and the gates
              (oracle.kda_prep, attention.py:192-230), else fixed prepared
              inputs; the KDA recurrent step (kda_step.py:173-196); o_proj of
              the step's output rounded to bf16;
  MLA layer:  q_proj of x and kv_b of the latent; o_proj of the attention
              output;
  then the layer's MLP: the dense SwiGLU MLP of layer 0 (gate/up with the
  SwiGLU rounding contract, then down) or the MoE block (oracle.moe);
  finally the INT4 lm_head (engine/klinear/model.py:134-160).

The parts of the model that are not on the path (norms, MLA softmax
attention, the BF16 gate projections and -- without ``prepare`` -- the KDA
input preparation) enter as the same fixed tensors the product's synthetic
step uses; the caller passes them in ``inputs``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import kda_prep
from . import moe as omoe
from . import ops


@dataclass
class OracleLayer:
    kind: str                                   # "kda" or "mla"
    qkv: list[tuple[torch.Tensor, torch.Tensor]] | None = None
    q_proj: tuple[torch.Tensor, torch.Tensor] | None = None
    kv_b: tuple[torch.Tensor, torch.Tensor] | None = None
    o_proj: tuple[torch.Tensor, torch.Tensor] | None = None
    kda_state: torch.Tensor | None = None       # fp32 [B, H, Dk, Dv], mutated
    moe: omoe.MoEBanks | None = None
    dense_mlp: tuple | None = None              # ((w1p, w1s), (w3p, w3s), (w2p, w2s)), 2-D
    conv_w: list[torch.Tensor] | None = None    # KDA preparation (bf16 [C, 4] x 3)
    conv_state: list[torch.Tensor] | None = None  # bf16 [B, C, 4] x 3, mutated
    dt_bias: torch.Tensor | None = None
    a_log: torch.Tensor | None = None


@dataclass
class StepTrace:
    """Intermediates of one oracle step, for per-layer checks."""

    layer_out: list[torch.Tensor] = field(default_factory=list)
    routes: list[torch.Tensor] = field(default_factory=list)
    weights: list[torch.Tensor] = field(default_factory=list)
    bounds: list[torch.Tensor] = field(default_factory=list)


def decode_step(layers: list[OracleLayer], lm_head: tuple[torch.Tensor, torch.Tensor],
                inputs: dict[str, torch.Tensor], x: torch.Tensor, *, kda_scale: float,
                trace: StepTrace | None = None, prepare: bool = False,
                heads: int = 0) -> torch.Tensor:
    """x bf16 [B, hidden] -> logits bf16 [B, vocab]; KDA states are updated in place.

    ``inputs`` holds the fixed tensors of the parts off the path:
    ``kda_q``, ``kda_k``, ``kda_v``, ``kda_decay``, ``kda_beta`` (fp32
    [B, H, D] / [B, H]) without ``prepare``, ``raw_decay`` and ``raw_beta``
    (bf16 outputs of the gate projections) with it, ``mla_latent`` and
    ``mla_attn`` (bf16).
    Router logits are summed in the kernels' stated lane order
    (ops.router_logits_lanes).
    """
    for lw in layers:
        if lw.kind == "kda":
            qkv = [ops.dense(x, p, s) for p, s in lw.qkv]
            if prepare:
                d = qkv[0].shape[1] // heads
                kin = kda_prep.prepare(*qkv, *lw.conv_state, *lw.conv_w, inputs["raw_decay"],
                                       lw.dt_bias, lw.a_log, inputs["raw_beta"],
                                       num_heads=heads, head_dim=d)
            else:   # the projections are computed by the step, consumed off the path
                kin = (inputs["kda_q"], inputs["kda_k"], inputs["kda_v"], inputs["kda_decay"],
                       inputs["kda_beta"])
            out = ops.kda_step(lw.kda_state, *kin, scale=kda_scale)
            h = ops.dense(out.reshape(out.shape[0], -1).to(torch.bfloat16), *lw.o_proj)
        else:
            ops.dense(x, *lw.q_proj)
            ops.dense(inputs["mla_latent"], *lw.kv_b)
            h = ops.dense(inputs["mla_attn"], *lw.o_proj)
        if lw.dense_mlp is not None:
            (w1p, w1s), (w3p, w3s), (w2p, w2s) = lw.dense_mlp
            idx0 = torch.zeros((h.shape[0], 1), dtype=torch.long)
            act = ops.swiglu(h, idx0, w1p[None], w1s[None], w3p[None], w3s[None])[:, 0]
            x = ops.dense(act, w2p, w2s)
        else:
            x, idx, wts, bound = omoe.moe_layer(h, lw.moe, return_parts=True, lane_order=True)
            if trace is not None:
                trace.routes.append(idx)
                trace.weights.append(wts)
                trace.bounds.append(bound)
        if trace is not None:
            trace.layer_out.append(x)
    return ops.dense(x, *lm_head)
