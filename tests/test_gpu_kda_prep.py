"""KDA decode preparation (kb_kda_prepare) against the oracle (GPU).

Tolerances are the reference's own for the fused preparation
(tests/test_kda_prepare.py:128-204): the bf16 convolution outputs within 2e-2,
the gates and normalised q/k within 2e-3; the convolution states bit-exact.
"""

from __future__ import annotations

import pytest
import torch

from local_kimi_b200 import ops
from oracle import kda_prep
from oracle import ops as oref

pytestmark = pytest.mark.gpu

GATE_TOL = 2e-3


def _run(cuda, q_in, k_in, v_in, states, weights, raw_decay, dt_bias, a_log, raw_beta, heads,
         dim):
    dev_states = [s.to(cuda).contiguous() for s in states]
    out = ops.kda_prepare(q_in.to(cuda), k_in.to(cuda), v_in.to(cuda), *dev_states,
                          *(w.to(cuda) for w in weights), raw_decay.to(cuda), dt_bias.to(cuda),
                          a_log.to(cuda), raw_beta.to(cuda), num_heads=heads, head_dim=dim)
    torch.cuda.synchronize()
    return [o.cpu() for o in out], [s.cpu() for s in dev_states]


def test_kda_prepare_matches_reference_golden(cuda, golden):
    g = golden
    states = [g[f"prep.{n}_state_in"] for n in "qkv"]
    out, new_states = _run(cuda, *(g[f"prep.{n}_in"] for n in "qkv"), states,
                           [g[f"prep.{n}_weight"] for n in "qkv"], g["prep.raw_decay"],
                           g["prep.dt_bias"], g["prep.a_log"], g["prep.raw_beta"], 2, 128)
    for n, st in zip("qkv", new_states):
        assert torch.equal(st, g[f"prep.{n}_state_out"]), f"{n} state"
    q, k, v, decay, beta = out
    torch.testing.assert_close(q, g["prep.q"][:, 0], atol=GATE_TOL, rtol=GATE_TOL)
    torch.testing.assert_close(k, g["prep.k"][:, 0], atol=GATE_TOL, rtol=GATE_TOL)
    torch.testing.assert_close(v, g["prep.v_conv"].float().view(2, 2, 128), atol=2e-2,
                               rtol=2e-2)
    torch.testing.assert_close(decay, g["prep.decay"][:, 0], atol=GATE_TOL, rtol=GATE_TOL)
    torch.testing.assert_close(beta, g["prep.beta"][:, 0], atol=GATE_TOL, rtol=GATE_TOL)


@pytest.mark.parametrize("batch", [1, 5, 64])
def test_kda_prepare_real_shape_then_step(cuda, batch):
    # 32 heads x 128: the preparation, then the KDA step on its outputs,
    # against the oracle chain.
    gen = torch.Generator().manual_seed(20260729 + batch)
    heads, dim = 32, 128
    c = heads * dim
    x = [torch.randn(batch, c, generator=gen).to(torch.bfloat16) for _ in range(3)]
    states = [torch.randn(batch, c, 4, generator=gen).to(torch.bfloat16) for _ in range(3)]
    weights = [(0.3 * torch.randn(c, 4, generator=gen)).to(torch.bfloat16) for _ in range(3)]
    raw_decay = torch.randn(batch, c, generator=gen).to(torch.bfloat16)
    dt_bias = torch.randn(c, generator=gen)
    a_log = torch.log(1.0 + 15.0 * torch.rand(heads, generator=gen))
    raw_beta = torch.randn(batch, heads, generator=gen).to(torch.bfloat16)
    out, new_states = _run(cuda, *x, states, weights, raw_decay, dt_bias, a_log, raw_beta, heads,
                           dim)
    ref_states = [s.clone() for s in states]
    ref = kda_prep.prepare(*x, *ref_states, *weights, raw_decay, dt_bias, a_log, raw_beta,
                           num_heads=heads, head_dim=dim)
    for st, rs in zip(new_states, ref_states):
        assert torch.equal(st, rs)
    tols = (GATE_TOL, GATE_TOL, 2e-2, GATE_TOL, GATE_TOL)
    for name, a, e, tol in zip(("q", "k", "v", "decay", "beta"), out, ref, tols):
        torch.testing.assert_close(a, e, atol=tol, rtol=tol, msg=f"{name} differs")
    # The step on the prepared inputs (reference tolerance of a single step).
    s0 = 0.05 * torch.randn(batch, heads, dim, dim, generator=gen)
    st_dev = s0.to(cuda)
    o = ops.kda_decode_step(st_dev, *(t.to(cuda) for t in out[:4]), out[4].to(cuda),
                            scale=dim ** -0.5)
    st_cpu = s0.clone()
    o_ref = oref.kda_step(st_cpu, *ref[:4], ref[4], scale=dim ** -0.5)
    torch.testing.assert_close(o.cpu(), o_ref, atol=1e-3, rtol=1e-3)


def test_kda_prepare_rejects_bad_inputs(cuda):
    x = torch.zeros(2, 256, dtype=torch.bfloat16, device=cuda)
    st = torch.zeros(2, 256, 4, dtype=torch.bfloat16, device=cuda)
    w = torch.zeros(256, 4, dtype=torch.bfloat16, device=cuda)
    rd = torch.zeros(2, 256, dtype=torch.bfloat16, device=cuda)
    dt = torch.zeros(256, device=cuda)
    a = torch.zeros(2, device=cuda)
    rb = torch.zeros(2, 2, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(TypeError):
        ops.kda_prepare(x.float(), x, x, st, st.clone(), st.clone(), w, w, w, rd, dt, a, rb,
                        num_heads=2, head_dim=128)
    with pytest.raises(ValueError):
        ops.kda_prepare(x, x, x, st[:, :128], st.clone(), st.clone(), w, w, w, rd, dt, a, rb,
                        num_heads=2, head_dim=128)


@pytest.mark.parametrize("batch", [1, 13, 40])
def test_kda_prepare_step_equals_the_two_calls(cuda, batch):
    # The fused preparation + step against kb_kda_prepare then
    # kb_kda_decode_step on the same inputs: identical convolution states, and
    # identical KDA state and outputs where both step with the streaming
    # kernel; and against the oracle chain within tolerance.
    gen = torch.Generator().manual_seed(20261202 + batch)
    heads, dim = 32, 128
    c = heads * dim
    qkv = torch.randn(batch, 3 * c, generator=gen).to(torch.bfloat16)
    x = [qkv[:, i * c:(i + 1) * c] for i in range(3)]        # one row stride, as the model
    states = [torch.randn(batch, c, 4, generator=gen).to(torch.bfloat16) for _ in range(3)]
    weights = [(0.3 * torch.randn(c, 4, generator=gen)).to(torch.bfloat16) for _ in range(3)]
    raw_decay = torch.randn(batch, c, generator=gen).to(torch.bfloat16)
    dt_bias = torch.randn(c, generator=gen)
    a_log = torch.log(1.0 + 15.0 * torch.rand(heads, generator=gen))
    raw_beta = torch.randn(batch, heads, generator=gen).to(torch.bfloat16)
    s0 = 0.05 * torch.randn(batch, heads, dim, dim, generator=gen)
    scale = dim ** -0.5
    dx = [t.to(cuda) for t in x]
    dev = [t.to(cuda) for t in (raw_decay, dt_bias, a_log, raw_beta)]
    dw = [w.to(cuda) for w in weights]
    st_a = [t.to(cuda) for t in states]
    kda_a = s0.to(cuda)
    ob_a = torch.empty(batch, heads, dim, dtype=torch.bfloat16, device=cuda)
    out_a = ops.kda_prepare_step(kda_a, *dx, *st_a, *dw, *dev, num_heads=heads, head_dim=dim,
                                 scale=scale, out_bf16=ob_a)
    st_b = [t.to(cuda) for t in states]
    kda_b = s0.to(cuda)
    kin = ops.kda_prepare(*dx, *st_b, *dw, *dev, num_heads=heads, head_dim=dim)
    ob_b = torch.empty(batch, heads, dim, dtype=torch.bfloat16, device=cuda)
    out_b = ops.kda_decode_step(kda_b, *kin, scale=scale, out_bf16=ob_b)
    torch.cuda.synchronize()
    for sa, sb in zip(st_a, st_b):
        assert torch.equal(sa, sb)
    if batch * heads >= 296:
        # Both paths run the streaming step: identical bits.
        assert torch.equal(kda_a, kda_b)
        assert torch.equal(out_a, out_b)
        assert torch.equal(ob_a, ob_b)
    else:
        # The two-call path steps with the column-slice kernel (another order).
        torch.testing.assert_close(kda_a, kda_b, atol=3e-5, rtol=3e-5)
        torch.testing.assert_close(out_a, out_b, atol=3e-5, rtol=3e-5)
    ref_states = [s.clone() for s in states]
    ref = kda_prep.prepare(*x, *ref_states, *weights, raw_decay, dt_bias, a_log, raw_beta,
                           num_heads=heads, head_dim=dim)
    s_ref = s0.clone()
    o_ref = oref.kda_step(s_ref, *ref[:4], ref[4], scale=scale)
    torch.testing.assert_close(out_a.cpu(), o_ref, atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(kda_a.cpu(), s_ref, atol=1e-3, rtol=1e-3)
