"""One MoE decode layer end to end on the GPU against the oracle (GPU).

Config 1 (one token) and config 3 (64 tokens with a skewed router) shapes:
hidden 2304, 256 routed experts + 1 shared (bank slot 256), top-8,
intermediate 1024, group 128 (and 32).
"""

from __future__ import annotations

import pytest
import torch

from local_kimi_b200 import moe as kmoe
from oracle import moe as omoe
from tests.conftest import assert_close
from tests.gpu_util import cuda_gen, quant_bank, rand_act, rand_weight

pytestmark = pytest.mark.gpu


def _layer(group: int, skew: float = 0.0) -> kmoe.MoELayerWeights:
    gen = cuda_gen(0)
    router = rand_weight((256, 2304), gen)
    w1p, w1s = quant_bank(257, 1024, 2304, group, gen)
    w2p, w2s = quant_bank(257, 2304, 1024, group, gen)
    w3p, w3s = quant_bank(257, 1024, 2304, group, gen)
    bias = torch.zeros(256, device="cuda")
    if skew:
        # Zipf-like popularity: a seeded permutation of the experts gets a
        # correction bias decreasing with log-rank (choice only, not weights).
        perm = torch.randperm(256, generator=torch.Generator().manual_seed(7))
        ranks = torch.empty(256)
        ranks[perm] = torch.arange(1, 257, dtype=torch.float32)
        bias = (-skew * torch.log(ranks)).to("cuda") * 0.05
    return kmoe.MoELayerWeights(router, bias, w1p, w1s, w2p, w2s, w3p, w3s, top_k=8,
                                scaling=2.446)


def _oracle_layer(layer: kmoe.MoELayerWeights, used: torch.Tensor) -> omoe.MoEBanks:
    sel = used.to("cuda")
    return omoe.MoEBanks(
        layer.router_weight.cpu(), layer.router_bias.cpu(),
        layer.w1_packed.cpu(), layer.w1_scales.cpu(),
        layer.w2_packed.cpu(), layer.w2_scales.cpu(),
        layer.w3_packed.cpu(), layer.w3_scales.cpu(), layer.top_k, layer.scaling,
    ) if sel.numel() > 64 else omoe.MoEBanks(
        layer.router_weight.cpu(), layer.router_bias.cpu(),
        *_subset(layer, sel), layer.top_k, layer.scaling,
    )


def _subset(layer, sel):
    # Keep the full bank shape but only the used experts' data (others zero)
    # so that the oracle's index arithmetic is unchanged and the copy is small.
    out = []
    for t in (layer.w1_packed, layer.w1_scales, layer.w2_packed, layer.w2_scales,
              layer.w3_packed, layer.w3_scales):
        z = torch.zeros_like(t, device="cpu")
        z[sel.cpu()] = t[sel].cpu()
        out.append(z)
    return out


@pytest.mark.parametrize("tokens,group,skew", [(1, 128, 0.0), (1, 32, 0.0), (64, 128, 1.1)])
def test_moe_layer_matches_oracle(cuda, tokens, group, skew):
    layer = _layer(group, skew)
    hidden = rand_act((tokens, 2304), cuda_gen(1))
    out, idx, w = kmoe.moe_forward(hidden, layer)
    used = torch.unique(torch.cat((idx.flatten().cpu(), torch.tensor([256]))))
    banks = _oracle_layer(layer, used)
    ref_out, ref_idx, ref_w, bound = omoe.moe_layer(hidden.cpu(), banks, return_parts=True,
                                                    lane_order=True)
    assert torch.equal(idx.cpu(), ref_idx), "router indices differ"
    torch.testing.assert_close(w.cpu(), ref_w, rtol=1e-5, atol=1e-6)
    # Where the routed sum and the shared output cancel, each element is also
    # allowed the rounding bound of the oracle's bf16 intermediates.
    assert_close(out, ref_out, what=f"moe layer T={tokens} g{group}", allowance=bound)
    again, _, _ = kmoe.moe_forward(hidden, layer)
    assert torch.equal(out, again)
