"""Decode-step executor (kb_step_*) against the oracle and the per-operation path (GPU).

Every operation kind runs inside a program (one persistent launch) and is
checked against the CPU oracle at the north-star tolerance; a small
Kimi-Linear-shaped model checks a whole multi-layer program against the
per-operation step; relaunching checks that the device counters reset.
"""

from __future__ import annotations

import pytest
import torch

from local_kimi_b200 import moe as kmoe
from local_kimi_b200 import ops
from local_kimi_b200.decode import HotPathDecoder, KimiLinearShape
from local_kimi_b200.step import StepProgram
from oracle import moe as omoe
from oracle import ops as oref
from tests.conftest import assert_close
from tests.gpu_util import cuda_gen, quant_bank, quant_matrix, rand_act, rand_weight

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,group", [(1, 128), (3, 32), (8, 128)])
def test_step_dense_swiglu_and_chunked(cuda, tokens, group):
    gen = cuda_gen(10 + tokens)
    x = rand_act((tokens, 2304), gen)
    lat = rand_act((tokens, 512), gen)
    wq = quant_matrix(4096, 2304, group, gen)
    wkv = quant_matrix(8192, 512, group, gen)
    w1 = quant_matrix(1024, 2304, group, gen)
    w3 = quant_matrix(1024, 2304, group, gen)
    big = quant_matrix(256, 9216, group, gen)           # reduction split into chunks
    xbig = rand_act((tokens, 9216), gen)
    yq = torch.empty((tokens, 4096), dtype=torch.bfloat16, device=cuda)
    ykv = torch.empty((tokens, 8192), dtype=torch.bfloat16, device=cuda)
    act = torch.empty((tokens, 1024), dtype=torch.bfloat16, device=cuda)
    ybig = torch.empty((tokens, 256), dtype=torch.bfloat16, device=cuda)
    prog = StepProgram(tokens)
    a = prog.dense([(x, *wq, yq), (lat, *wkv, ykv)])
    b = prog.swiglu(x, w1, w3, act, deps=[a])
    prog.dense([(xbig, *big, ybig)], deps=[b])
    prog.finalize()
    prog.launch()
    torch.cuda.synchronize()
    xc, latc = x.cpu(), lat.cpu()
    assert_close(yq, oref.dense(xc, wq[0].cpu(), wq[1].cpu()), what="q_proj")
    assert_close(ykv, oref.dense(latc, wkv[0].cpu(), wkv[1].cpu()), what="kv_b")
    idx0 = torch.zeros((tokens, 1), dtype=torch.long)
    ref = oref.swiglu(xc, idx0, w1[0].cpu()[None], w1[1].cpu()[None], w3[0].cpu()[None],
                      w3[1].cpu()[None])[:, 0]
    assert_close(act, ref, what="dense swiglu")
    assert_close(ybig, oref.dense(xbig.cpu(), big[0].cpu(), big[1].cpu()), what="K=9216")
    # The same program again: counters were reset by the first launch.
    prev = (yq.clone(), act.clone(), ybig.clone())
    prog.launch()
    torch.cuda.synchronize()
    assert torch.equal(yq, prev[0]) and torch.equal(act, prev[1]) and torch.equal(ybig, prev[2])


def _moe_layer(group: int, gen) -> kmoe.MoELayerWeights:
    router = rand_weight((256, 2304), gen)
    w1p, w1s = quant_bank(257, 1024, 2304, group, gen)
    w2p, w2s = quant_bank(257, 2304, 1024, group, gen)
    w3p, w3s = quant_bank(257, 1024, 2304, group, gen)
    bias = 0.01 * torch.randn(256, generator=gen, device="cuda")
    return kmoe.MoELayerWeights(router, bias, w1p, w1s, w2p, w2s, w3p, w3s, top_k=8,
                                scaling=2.446)


def _oracle_banks(layer: kmoe.MoELayerWeights, used: torch.Tensor) -> omoe.MoEBanks:
    out = []
    for t in (layer.w1_packed, layer.w1_scales, layer.w2_packed, layer.w2_scales,
              layer.w3_packed, layer.w3_scales):
        z = torch.zeros_like(t, device="cpu")
        z[used] = t[used.to(t.device)].cpu()
        out.append(z)
    return omoe.MoEBanks(layer.router_weight.cpu(), layer.router_bias.cpu(), *out, layer.top_k,
                         layer.scaling)


@pytest.mark.parametrize("tokens", [1, 4, 8])
def test_step_moe_layer_matches_oracle_and_per_op(cuda, tokens):
    gen = cuda_gen(20 + tokens)
    layer = _moe_layer(128, gen)
    h = rand_act((tokens, 2304), gen)
    lg = StepProgram.router_scratch(tokens, 256, cuda)
    idx = torch.empty((tokens, 9), dtype=torch.long, device=cuda)
    wts = torch.empty((tokens, 8), dtype=torch.float32, device=cuda)
    act = torch.empty((tokens * 9, 1024), dtype=torch.bfloat16, device=cuda)
    routed = torch.empty((tokens * 9, 2304), dtype=torch.bfloat16, device=cuda)
    out = torch.empty((tokens, 2304), dtype=torch.bfloat16, device=cuda)
    prog = StepProgram(tokens)
    r = prog.router(h, layer.router_weight, layer.router_bias, 8, 2.446, lg, idx, wts)
    prog.moe(r, h, layer, act, routed, out)
    prog.finalize()
    prog.launch()
    torch.cuda.synchronize()

    # Routing equals the per-operation router bit for bit (same logit order).
    ref_stable, ref_w = ops.moe_router(h, layer.router_weight, layer.router_bias, 8,
                                       routed_scaling_factor=2.446, append_expert=256)
    assert torch.equal(idx, ref_stable)
    assert torch.equal(wts, ref_w)

    used = torch.unique(torch.cat((idx.flatten().cpu(), torch.tensor([256]))))
    banks = _oracle_banks(layer, used)
    ref_out, ref_idx, ref_wts, bound = omoe.moe_layer(h.cpu(), banks, return_parts=True,
                                                     lane_order=True)
    assert torch.equal(idx[:, :8].cpu(), ref_idx)
    torch.testing.assert_close(wts.cpu(), ref_wts, rtol=1e-5, atol=1e-6)
    assert_close(out, ref_out, what=f"step moe T={tokens}", allowance=bound)
    # Step and per-operation path each sit within the oracle's rounding bound
    # where routed and shared outputs cancel, so they may differ by twice it.
    per_op, _, _ = kmoe.moe_forward(h, layer)
    assert_close(out, per_op, what="step vs per-op", allowance=2 * bound)

    prog.launch()
    torch.cuda.synchronize()
    again = out.clone()
    prog.launch()
    torch.cuda.synchronize()
    assert torch.equal(out, again)


@pytest.mark.parametrize("batch", [1, 3])
def test_step_kda_equals_kernel(cuda, batch):
    gen = cuda_gen(30 + batch)
    H, D = 32, 128
    q = torch.nn.functional.normalize(torch.randn((batch, H, D), generator=gen, device=cuda), dim=-1)
    k = torch.nn.functional.normalize(torch.randn((batch, H, D), generator=gen, device=cuda), dim=-1)
    v = 0.2 * torch.randn((batch, H, D), generator=gen, device=cuda)
    decay = -(0.005 + 0.075 * torch.rand((batch, H, D), generator=gen, device=cuda))
    beta = torch.sigmoid(torch.randn((batch, H), generator=gen, device=cuda))
    s0 = 0.05 * torch.randn((batch, H, D, D), generator=gen, device=cuda)
    st_prog, st_kern = s0.clone(), s0.clone()
    out = torch.empty((batch, H, D), dtype=torch.float32, device=cuda)
    out16 = torch.empty((batch, H * D), dtype=torch.bfloat16, device=cuda)
    prog = StepProgram(1)
    prog.kda(st_prog, q, k, v, decay, beta, D ** -0.5, out=out, out_bf16=out16)
    prog.finalize()
    prog.launch()
    ref16 = torch.empty_like(out16)
    ref = ops.kda_decode_step(st_kern, q, k, v, decay, beta, scale=D ** -0.5, out_bf16=ref16)
    torch.cuda.synchronize()
    assert torch.equal(out, ref.reshape(out.shape))
    assert torch.equal(st_prog, st_kern)
    assert torch.equal(out16, ref16)
    st_cpu = s0.cpu()
    o_cpu = oref.kda_step(st_cpu, q.cpu(), k.cpu(), v.cpu(), decay.cpu(), beta.cpu(),
                          scale=D ** -0.5)
    torch.testing.assert_close(out.cpu(), o_cpu, rtol=3e-5, atol=3e-5)


def _small_shape() -> KimiLinearShape:
    return KimiLinearShape(vocab_size=8192, hidden=1024, layers=4, kda_heads=4, mla_heads=4,
                           experts=64, moe_intermediate=256, dense_intermediate=2048,
                           mla_layers=(4,))


@pytest.mark.parametrize("batch", [1, 5])
def test_step_program_matches_per_op_step(cuda, batch):
    model = HotPathDecoder(batch, shape=_small_shape(), kda_prepare=False)
    x = model.x0.clone()
    states = [lw.kda_state.clone() if lw.kda_state is not None else None for lw in model.layers]
    prog, buf = model.build_program(x)
    prog.launch()
    torch.cuda.synchronize()
    step_logits = buf["logits"].clone()
    step_states = [lw.kda_state.clone() if lw.kda_state is not None else None
                   for lw in model.layers]
    # The per-operation step from the same states.
    for lw, st in zip(model.layers, states):
        if st is not None:
            lw.kda_state.copy_(st)
    ref_logits = model.step(x)
    torch.cuda.synchronize()
    for lw, st in zip(model.layers, step_states):
        if st is not None:
            assert torch.equal(lw.kda_state, st), "KDA states differ"
    assert_close(step_logits, ref_logits, what=f"program logits B={batch}")
    n_moe = sum(1 for lw in model.layers if lw.moe is not None)
    assert len(buf["idx"]) == n_moe
    for idx in buf["idx"]:
        assert int(idx.min()) >= 0 and int(idx[:, :-1].max()) < model.shape.experts
        assert bool((idx[:, -1] == model.shape.experts).all())


def _oracle_model(model: HotPathDecoder, states: list) -> list:
    from oracle.decode import OracleLayer

    def cpu(pair):
        return (pair[0].cpu(), pair[1].cpu())

    layers = []
    for lw, st in zip(model.layers, states):
        ol = OracleLayer(kind=lw.kind)
        if lw.kind == "kda":
            ol.qkv = [cpu(p) for p in lw.qkv]
            ol.kda_state = st.cpu().clone()
        else:
            ol.q_proj, ol.kv_b = cpu(lw.q_proj), cpu(lw.kv_b)
        ol.o_proj = cpu(lw.o_proj)
        if lw.dense_mlp is not None:
            (w1p, w1s), (w3p, w3s), (w2p, w2s) = lw.dense_mlp
            ol.dense_mlp = ((w1p[0].cpu(), w1s[0].cpu()), (w3p[0].cpu(), w3s[0].cpu()),
                            (w2p.cpu(), w2s.cpu()))
        else:
            m = lw.moe
            ol.moe = omoe.MoEBanks(m.router_weight.cpu(), m.router_bias.cpu(),
                                   m.w1_packed.cpu(), m.w1_scales.cpu(), m.w2_packed.cpu(),
                                   m.w2_scales.cpu(), m.w3_packed.cpu(), m.w3_scales.cpu(),
                                   m.top_k, m.scaling)
        layers.append(ol)
    return layers


@pytest.mark.parametrize("batch", [1, 5])
def test_step_program_matches_oracle_chain(cuda, batch):
    # The whole multi-layer program against the CPU oracle chained layer by
    # layer (oracle.decode): routing of every MoE layer exact, KDA states at
    # the reference's single-step tolerance, logits at the north-star
    # tolerance.
    from oracle.decode import StepTrace, decode_step

    model = HotPathDecoder(batch, shape=_small_shape(), seed=7, kda_prepare=False)
    x = model.x0.clone()
    states = [lw.kda_state.clone() if lw.kda_state is not None else None for lw in model.layers]
    layers = _oracle_model(model, states)
    prog, buf = model.build_program(x)
    prog.launch()
    torch.cuda.synchronize()
    inputs = {"kda_q": model.kda_q.cpu(), "kda_k": model.kda_k.cpu(), "kda_v": model.kda_v.cpu(),
              "kda_decay": model.kda_decay.cpu(), "kda_beta": model.kda_beta.cpu(),
              "mla_latent": model.mla_latent.cpu(), "mla_attn": model.mla_attn.cpu()}
    trace = StepTrace()
    ref_logits = decode_step(layers, (model.lm_head[0].cpu(), model.lm_head[1].cpu()), inputs,
                             x.cpu(), kda_scale=model.shape.kda_head_dim ** -0.5, trace=trace)
    for lw, ol in zip(model.layers, layers):
        if lw.kda_state is not None:
            torch.testing.assert_close(lw.kda_state.cpu(), ol.kda_state, rtol=3e-5, atol=3e-5)
    assert len(buf["idx"]) == len(trace.routes)
    for idx, wts, ref_idx, ref_w in zip(buf["idx"], buf["weights"], trace.routes,
                                        trace.weights):
        assert torch.equal(idx[:, :-1].cpu(), ref_idx)
        torch.testing.assert_close(wts.cpu(), ref_w, rtol=1e-5, atol=1e-6)
    assert_close(buf["logits"], ref_logits, what=f"program logits vs oracle B={batch}")


@pytest.mark.parametrize("batch", [1, 6])
def test_per_op_step_with_kda_prepare_matches_oracle_chain(cuda, batch):
    # The per-operation step with the KDA decode preparation (q/k/v from the
    # layer's projections through the short convolutions and gates) against
    # the oracle chain: logits, KDA and convolution states.
    from oracle.decode import StepTrace, decode_step

    model = HotPathDecoder(batch, shape=_small_shape(), seed=11)
    assert model.kda_prepare
    x = model.x0.clone()
    states = [lw.kda_state.clone() if lw.kda_state is not None else None for lw in model.layers]
    layers = _oracle_model(model, states)
    for lw, ol in zip(model.layers, layers):
        if lw.kind == "kda":
            ol.conv_w = [w.cpu() for w in lw.conv_w]
            ol.conv_state = [c.cpu().clone() for c in lw.conv_state]
            ol.dt_bias, ol.a_log = lw.dt_bias.cpu(), lw.a_log.cpu()
    logits = model.step(x)
    torch.cuda.synchronize()
    inputs = {"raw_decay": model.raw_decay.cpu(), "raw_beta": model.raw_beta.cpu(),
              "mla_latent": model.mla_latent.cpu(), "mla_attn": model.mla_attn.cpu()}
    trace = StepTrace()
    ref = decode_step(layers, (model.lm_head[0].cpu(), model.lm_head[1].cpu()), inputs,
                      x.cpu(), kda_scale=model.shape.kda_head_dim ** -0.5, trace=trace,
                      prepare=True, heads=model.shape.kda_heads)
    for lw, ol in zip(model.layers, layers):
        if lw.kda_state is not None:
            torch.testing.assert_close(lw.kda_state.cpu(), ol.kda_state, rtol=1e-3, atol=1e-4)
            # the newest token of each state is the layer's projection output,
            # itself within one bf16 rounding of the oracle's
            for c, rc in zip(lw.conv_state, ol.conv_state):
                assert_close(c, rc, what="conv state")
    assert_close(logits, ref, what=f"per-op step with KDA preparation B={batch}")
