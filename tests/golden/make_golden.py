"""Generate golden vectors by running the reference implementation on the CPU.

Usage (in a checkout that has the reference package available):
    python tests/golden/make_golden.py [REFERENCE_DIR]
REFERENCE_DIR defaults to the KIMI_REFERENCE_DIR environment variable.  The
script imports the reference's own functions -- the codec
(engine/quant/w4a16.py), fused_w2_combine_reference
(engine/kernels/moe_combine.py:209-261), kda_decode_step_reference
(engine/kernels/kda_step.py:173-196), fused_short_conv_triple_reference and
fused_kda_gates_reference (engine/kernels/kda_prepare.py:426-472, 581-615),
KLinearRouter (engine/klinear/router.py)
and KLinearMoE's eager expert path with an expert provider returning
dequantised weights (engine/klinear/moe.py:336-398) -- runs them on seeded
inputs at the reference group size 32, and writes every input and output to
``reference_g32.pt`` next to this file.  The fixtures are small (tens of KB)
and are committed; tests never import the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_g32.pt"


def _load_reference(ref_dir: str):
    sys.path.insert(0, ref_dir)
    from engine.kernels.kda_prepare import (fused_kda_gates_reference,
                                            fused_short_conv_triple_reference)
    from engine.kernels.kda_step import kda_decode_step_reference
    from engine.kernels.moe_combine import fused_w2_combine_reference
    from engine.klinear.moe import KLinearMoE
    from engine.klinear.router import KLinearRouter
    from engine.quant.w4a16 import W4A16Tensor, dequantise, quantise

    return {
        "quantise": quantise,
        "dequantise": dequantise,
        "W4A16Tensor": W4A16Tensor,
        "combine": fused_w2_combine_reference,
        "kda": kda_decode_step_reference,
        "conv3": fused_short_conv_triple_reference,
        "gates": fused_kda_gates_reference,
        "router": KLinearRouter,
        "moe": KLinearMoE,
    }


def _ref_linear(R, x, packed, scales):
    """Kernel contract with the reference codec: bf16-rounded decode, fp32 dot, bf16 out."""
    n, half = packed.shape
    enc = R["W4A16Tensor"](packed=packed, scales=scales, original_shape=(n, half * 2))
    w = R["dequantise"](enc).float()  # bf16 restore, as the kernels decode
    return F.linear(x.float(), w).to(torch.bfloat16)


def main(ref_dir: str) -> None:
    R = _load_reference(ref_dir)
    gold: dict[str, object] = {}

    # -- codec ---------------------------------------------------------------
    torch.manual_seed(20260801)
    w = (torch.randn(24, 256) * 0.02).to(torch.bfloat16)
    w[3, 32:64] = 0  # an all-zero group -> scale 1
    w[5, 0:32] = torch.linspace(-1, 1, 32).to(torch.bfloat16)
    enc = R["quantise"](w)
    gold["codec.w"] = w
    gold["codec.packed"] = enc.packed
    gold["codec.scales"] = enc.scales
    gold["codec.dequant_bf16"] = R["dequantise"](enc)
    gold["codec.dequant_f32"] = R["dequantise"](enc, dtype=torch.float32)

    # -- dense (M = 1 and M = 3) ------------------------------------------------
    torch.manual_seed(20260802)
    wd = (torch.randn(48, 256) * 0.02).to(torch.bfloat16)
    encd = R["quantise"](wd)
    for m in (1, 3):
        x = torch.randn(m, 256).to(torch.bfloat16)
        gold[f"dense.m{m}.x"] = x
        gold[f"dense.m{m}.y"] = _ref_linear(R, x, encd.packed, encd.scales)
    gold["dense.packed"] = encd.packed
    gold["dense.scales"] = encd.scales

    # -- grouped + swiglu ------------------------------------------------------
    torch.manual_seed(20260803)
    E, N, K, T, Rt = 5, 40, 128, 4, 3
    banks = {}
    for name in ("w1", "w3"):
        ps, ss = [], []
        for _ in range(E):
            e = R["quantise"]((torch.randn(N, K) * 0.05).to(torch.bfloat16))
            ps.append(e.packed)
            ss.append(e.scales)
        banks[name] = (torch.stack(ps), torch.stack(ss))
    xg = torch.randn(T, K).to(torch.bfloat16)
    idx = torch.tensor([[0, 3, 4], [1, 3, 2], [4, 0, 1], [2, 2, 4]], dtype=torch.long)
    gate = torch.empty(T, Rt, N, dtype=torch.bfloat16)
    up = torch.empty(T, Rt, N, dtype=torch.bfloat16)
    for t in range(T):
        for r in range(Rt):
            e = int(idx[t, r])
            gate[t, r] = _ref_linear(R, xg[t : t + 1], banks["w1"][0][e], banks["w1"][1][e])[0]
            up[t, r] = _ref_linear(R, xg[t : t + 1], banks["w3"][0][e], banks["w3"][1][e])[0]
    gold["grouped.x"] = xg
    gold["grouped.idx"] = idx
    gold["grouped.w1_packed"], gold["grouped.w1_scales"] = banks["w1"]
    gold["grouped.w3_packed"], gold["grouped.w3_scales"] = banks["w3"]
    gold["grouped.gate"] = gate
    gold["grouped.up"] = up
    gold["grouped.swiglu"] = F.silu(gate) * up  # engine/kernels/__init__.py:196-197

    # -- down projection + combine ----------------------------------------------
    torch.manual_seed(20260729)
    tokens, routes, experts, out_size, red = 2, 3, 4, 5, 64
    act = torch.randn((tokens, routes, red), dtype=torch.bfloat16)
    cidx = torch.tensor([[0, 1, 3], [2, 0, 3]], dtype=torch.long)
    cw = torch.tensor([[0.25, 0.75, 0.125], [0.6, 0.4, 7.0]], dtype=torch.float32)
    w2p = torch.randint(0, 256, (experts, out_size, red // 2), dtype=torch.uint8)
    w2s = (torch.rand((experts, out_size, red // 32)) * 0.05 + 0.001).to(torch.bfloat16)
    gold["combine.act"], gold["combine.idx"], gold["combine.w"] = act, cidx, cw
    gold["combine.w2_packed"], gold["combine.w2_scales"] = w2p, w2s
    gold["combine.out"] = R["combine"](act, cidx, cw, w2p, w2s)
    # larger seeded case: 3 tokens, 9 routes (8 routed + shared), 12 experts
    torch.manual_seed(20260804)
    act2 = torch.randn((3, 9, 128), dtype=torch.bfloat16)
    idx2 = torch.stack([torch.cat((torch.randperm(11)[:8], torch.tensor([11]))) for _ in range(3)])
    w2 = torch.rand(3, 9, dtype=torch.float32)
    p2, s2 = [], []
    for _ in range(12):
        e = R["quantise"]((torch.randn(96, 128) * 0.05).to(torch.bfloat16))
        p2.append(e.packed)
        s2.append(e.scales)
    w2p2, w2s2 = torch.stack(p2), torch.stack(s2)
    gold["combine2.act"], gold["combine2.idx"], gold["combine2.w"] = act2, idx2, w2
    gold["combine2.w2_packed"], gold["combine2.w2_scales"] = w2p2, w2s2
    gold["combine2.out"] = R["combine"](act2, idx2, w2, w2p2, w2s2)

    # -- router ---------------------------------------------------------------------
    torch.manual_seed(20260805)
    router = R["router"](64, 16, 4, routed_scaling_factor=2.446, dtype=torch.bfloat16).eval()
    with torch.no_grad():
        router.weight.copy_((torch.randn(16, 64) * 0.3).to(torch.bfloat16))
        router.e_score_correction_bias.copy_((torch.randn(16) * 0.05).to(torch.bfloat16))
    hid = torch.randn(6, 64).to(torch.bfloat16)
    ridx, rw = router(hid)
    order = torch.argsort(ridx, dim=-1)
    gold["router.hidden"] = hid
    gold["router.weight"] = router.weight.detach().clone()
    gold["router.bias"] = router.e_score_correction_bias.detach().clone()
    gold["router.idx_sorted"] = torch.gather(ridx, 1, order)
    gold["router.w_sorted"] = torch.gather(rw, 1, order)

    # -- KDA --------------------------------------------------------------------------
    torch.manual_seed(20260806)
    B, H, Dk, Dv = 2, 3, 16, 8
    st = 0.05 * torch.randn(B, H, Dk, Dv)
    q = F.normalize(torch.randn(B, H, Dk), dim=-1)
    k = F.normalize(torch.randn(B, H, Dk), dim=-1)
    v = 0.2 * torch.randn(B, H, Dv)
    decay = -(0.005 + 0.075 * torch.rand(B, H, Dk))
    beta = torch.sigmoid(torch.randn(B, H))
    gold["kda.state_in"] = st.clone()
    gold["kda.q"], gold["kda.k"], gold["kda.v"] = q, k, v
    gold["kda.decay"], gold["kda.beta"] = decay, beta
    out = R["kda"](st, q, k, v, decay, beta, scale=Dk**-0.5)
    gold["kda.state_out"] = st
    gold["kda.out"] = out

    # -- one MoE layer (small config), reference eager expert path ---------------
    torch.manual_seed(20260807)
    H2, E2, I2, K2 = 128, 16, 64, 4
    experts = {}
    for e in range(E2):
        experts[e] = tuple(
            R["quantise"]((torch.randn(shape) * 0.05).to(torch.bfloat16))
            for shape in ((I2, H2), (H2, I2), (I2, H2))
        )

    def provider(layer_idx, expert_id, device, dtype):
        return tuple(R["dequantise"](encx) for encx in experts[expert_id])

    moe = R["moe"](1, H2, I2, E2, K2, num_shared_experts=1, routed_scaling_factor=2.446,
                   expert_provider=provider, dtype=torch.bfloat16).eval()
    shared = tuple(
        R["quantise"]((torch.randn(shape) * 0.05).to(torch.bfloat16))
        for shape in ((I2, H2), (H2, I2), (I2, H2))
    )
    with torch.no_grad():
        moe.gate.weight.copy_((torch.randn(E2, H2) * 0.1).to(torch.bfloat16))
        moe.gate.e_score_correction_bias.zero_()
        moe.shared_experts.gate_proj.weight.copy_(R["dequantise"](shared[0]))
        moe.shared_experts.down_proj.weight.copy_(R["dequantise"](shared[1]))
        moe.shared_experts.up_proj.weight.copy_(R["dequantise"](shared[2]))
    hm = torch.randn(3, H2).to(torch.bfloat16)
    with torch.no_grad():
        mo, midx, mw = moe(hm, return_router=True)
    gold["moe.hidden"] = hm
    gold["moe.router_weight"] = moe.gate.weight.detach().clone()
    gold["moe.out"] = mo
    morder = torch.argsort(midx, dim=-1)
    gold["moe.idx_sorted"] = torch.gather(midx, 1, morder)
    gold["moe.w_sorted"] = torch.gather(mw, 1, morder)
    for j, name in enumerate(("w1", "w2", "w3")):
        gold[f"moe.{name}_packed"] = torch.stack(
            [experts[e][j].packed for e in range(E2)] + [shared[j].packed]
        )
        gold[f"moe.{name}_scales"] = torch.stack(
            [experts[e][j].scales for e in range(E2)] + [shared[j].scales]
        )

    # KDA decode preparation: the width-4 short convolutions of q/k/v (states
    # updated in place) and the gates, bf16 inputs as in the model.
    gp = torch.Generator().manual_seed(20260729)
    B, C, NH, HD = 2, 256, 2, 128
    vals = [torch.randn(B, 1, C, generator=gp).to(torch.bfloat16) for _ in range(3)]
    states = [torch.randn(B, C, 4, generator=gp).to(torch.bfloat16) for _ in range(3)]
    weights = [(0.5 * torch.randn(C, 1, 4, generator=gp)).to(torch.bfloat16) for _ in range(3)]
    for j, name in enumerate("qkv"):
        gold[f"prep.{name}_in"] = vals[j].clone()
        gold[f"prep.{name}_state_in"] = states[j].clone()
        gold[f"prep.{name}_weight"] = weights[j].clone()
    conv = R["conv3"](*vals, *states, *weights)
    for j, name in enumerate("qkv"):
        gold[f"prep.{name}_conv"] = conv[j].clone()
        gold[f"prep.{name}_state_out"] = states[j].clone()
    raw_decay = torch.randn(B, 1, NH, HD, generator=gp).to(torch.bfloat16)
    dt_bias = torch.randn(NH * HD, generator=gp)
    a_log = torch.log(1.0 + 15.0 * torch.rand(NH, generator=gp)).view(1, 1, NH, 1)
    raw_beta = torch.randn(B, 1, NH, generator=gp).to(torch.bfloat16)
    raw_decay[0, 0, 0, :4] = torch.tensor([30.0, -30.0, 0.0, 19.0])   # softplus branches
    gates = R["gates"](raw_decay, dt_bias, a_log, raw_beta, conv[0], conv[1], num_heads=NH,
                       head_dim=HD, eps=1e-6)
    gold.update({"prep.raw_decay": raw_decay, "prep.dt_bias": dt_bias, "prep.a_log": a_log,
                 "prep.raw_beta": raw_beta, "prep.decay": gates[0], "prep.beta": gates[1],
                 "prep.q": gates[2], "prep.k": gates[3]})

    torch.save(gold, OUT)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(gold)} tensors)")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KIMI_REFERENCE_DIR", "")
    if not ref:
        raise SystemExit("pass the reference checkout directory (or set KIMI_REFERENCE_DIR)")
    main(ref)
