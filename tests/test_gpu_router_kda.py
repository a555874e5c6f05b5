"""Parity of the router, KDA step and on-device quantiser against the oracle (GPU)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from local_kimi_b200 import ops
from oracle import codec
from oracle import ops as oref
from tests.gpu_util import cuda_gen, rand_act, rand_weight

pytestmark = pytest.mark.gpu

# Tolerances of the reference's own KDA tests (tests/test_kda_step.py:12-15).
SINGLE_STEP_TOL = 3e-5
RECURRENT_TOL = 5e-4


# ---------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------


def _sorted(idx: torch.Tensor, w: torch.Tensor):
    order = torch.argsort(idx, dim=-1)
    return torch.gather(idx, 1, order), torch.gather(w, 1, order)


def test_router_matches_reference_golden(cuda, golden):
    idx, w = ops.moe_router(golden["router.hidden"].to(cuda), golden["router.weight"].to(cuda),
                            golden["router.bias"].to(cuda), 4, routed_scaling_factor=2.446)
    si, sw = _sorted(idx.cpu(), w.cpu())
    assert torch.equal(si, golden["router.idx_sorted"])
    torch.testing.assert_close(sw, golden["router.w_sorted"], rtol=1e-5, atol=1e-6)


def _router_with_logits(hidden, weight, bias, top_k, scaling):
    """kb_router_topk through the C ABI with a caller workspace, so that the
    fp32 logits it leaves at the start of the workspace can be read back."""
    from ctypes import c_float, c_int64, c_size_t, c_void_p

    from local_kimi_b200 import _lib

    tokens, width = hidden.shape
    experts = weight.shape[0]
    need = int(_lib.lib().kb_router_workspace_size(tokens, experts))
    ws = torch.zeros(need, dtype=torch.uint8, device=hidden.device)
    idx = torch.empty((tokens, top_k), dtype=torch.long, device=hidden.device)
    wts = torch.empty((tokens, top_k), dtype=torch.float32, device=hidden.device)
    _lib.call("kb_router_topk", c_void_p(hidden.data_ptr()), c_int64(hidden.stride(0)),
              c_int64(tokens), c_int64(width), c_void_p(weight.data_ptr()),
              c_void_p(bias.data_ptr()), c_int64(experts), c_int64(top_k), 1, c_float(scaling),
              c_void_p(idx.data_ptr()), c_int64(-1), c_void_p(wts.data_ptr()),
              c_void_p(ws.data_ptr()), c_size_t(need),
              c_void_p(torch.cuda.current_stream(hidden.device).cuda_stream))
    logits = ws[: tokens * experts * 4].view(torch.float32).view(tokens, experts)
    return idx, wts, logits


@pytest.mark.parametrize("tokens,width,seed", [(1, 2304, 0), (32, 2304, 0), (64, 2304, 0),
                                               (200, 2304, 5), (16, 7168, 6), (9, 520, 7)])
def test_router_bit_exact_logits_and_indices(cuda, tokens, width, seed):
    # The oracle sums the logits in the kernel's stated lane order
    # (oracle.ops.router_logits_lanes), so logits and indices must be
    # identical, with no near-tie exemption.  Widths cover whole lane rounds
    # (2304 = 9 x 32 words), a long row (7168) and a ragged last round (520).
    weight = rand_weight((256, width), cuda_gen(seed))
    bias = (torch.randn(256, generator=torch.Generator().manual_seed(4)) * 1e-3).to(cuda)
    hidden = rand_act((tokens, width), cuda_gen(seed + 1))
    idx, w, logits = _router_with_logits(hidden, weight, bias, 8, 2.446)
    ref_logits = oref.router_logits_lanes(hidden.cpu(), weight.cpu())
    assert torch.equal(logits.cpu(), ref_logits)
    ridx, rw, _ = oref.router_topk(hidden.cpu(), weight.cpu(), bias.cpu(), 8, scaling=2.446,
                                   logits=ref_logits)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, rtol=1e-5, atol=1e-6)
    # The torch-facing op gives the same routing, shared route appended.
    sidx, sw = ops.moe_router(hidden, weight, bias, 8, routed_scaling_factor=2.446,
                              append_expert=256)
    assert torch.equal(sidx[:, :8], idx) and bool((sidx[:, 8] == 256).all())
    assert torch.equal(sw, w)


def test_router_ties_go_to_lower_index_and_nan_stays_in_range(cuda):
    weight = torch.zeros((64, 128), dtype=torch.bfloat16, device=cuda)
    weight[10] = 1.0
    weight[20] = 1.0  # ties with 10
    hidden = torch.ones((2, 128), dtype=torch.bfloat16, device=cuda)
    idx, _ = ops.moe_router(hidden, weight, None, 4)
    assert idx[0].tolist() == [10, 20, 0, 1]
    hidden[1, 3] = float("nan")
    idx, _ = ops.moe_router(hidden, weight, None, 4)
    assert bool(((idx >= 0) & (idx < 64)).all())


def test_router_known_answer(cuda):
    weight = torch.tensor([[3.0, 0.0], [2.0, 0.0], [1.0, 0.0], [0.0, 0.0]])
    weight = F.pad(weight, (0, 6)).to(torch.bfloat16).to(cuda)
    hidden = F.pad(torch.tensor([[1.0, 0.0]]), (0, 6)).to(torch.bfloat16).to(cuda)
    idx, w = ops.moe_router(hidden, weight, None, 2, routed_scaling_factor=2.446)
    assert idx[0].tolist() == [0, 1]
    raw = torch.sigmoid(torch.tensor([3.0, 2.0]))
    torch.testing.assert_close(w[0].cpu(), raw / raw.sum() * 2.446)


# ---------------------------------------------------------------------------
# KDA
# ---------------------------------------------------------------------------


def test_kda_matches_reference_golden(cuda, golden):
    st = golden["kda.state_in"].to(cuda).clone()
    out = ops.kda_decode_step(st, *(golden[f"kda.{n}"].to(cuda) for n in
                                    ("q", "k", "v", "decay", "beta")), scale=16 ** -0.5)
    torch.testing.assert_close(st.cpu(), golden["kda.state_out"], atol=SINGLE_STEP_TOL,
                               rtol=SINGLE_STEP_TOL)
    torch.testing.assert_close(out.cpu(), golden["kda.out"], atol=SINGLE_STEP_TOL,
                               rtol=SINGLE_STEP_TOL)


def _real_inputs(batch: int, seed: int = 20260729):
    g = torch.Generator().manual_seed(seed)
    state = 0.05 * torch.randn(batch, 32, 128, 128, generator=g)
    q = F.normalize(torch.randn(batch, 32, 128, generator=g), dim=-1)
    k = F.normalize(torch.randn(batch, 32, 128, generator=g), dim=-1)
    v = 0.2 * torch.randn(batch, 32, 128, generator=g)
    decay = -(0.005 + 0.075 * torch.rand(batch, 32, 128, generator=g))
    beta = torch.sigmoid(torch.randn(batch, 32, generator=g))
    return state, q, k, v, decay, beta


# batch 1 runs the column-slice kernel, 13 and 32 (416 and 1024 heads) the
# streaming kernel (uneven and several passes per CTA over its three stages).
@pytest.mark.parametrize("batch", [1, 13, 32])
def test_kda_real_shape_single_step(cuda, batch):
    state, q, k, v, decay, beta = _real_inputs(batch)
    dev = [t.to(cuda) for t in (state, q, k, v, decay, beta)]
    st = dev[0].clone()
    out_bf16 = torch.empty((batch, 32, 128), dtype=torch.bfloat16, device=cuda)
    out = ops.kda_decode_step(st, *dev[1:], scale=128 ** -0.5, out_bf16=out_bf16)
    ref_state = state.clone()
    ref_out = oref.kda_step(ref_state, q, k, v, decay, beta, scale=128 ** -0.5)
    torch.testing.assert_close(st.cpu(), ref_state, atol=SINGLE_STEP_TOL, rtol=SINGLE_STEP_TOL)
    torch.testing.assert_close(out.cpu(), ref_out, atol=SINGLE_STEP_TOL, rtol=SINGLE_STEP_TOL)
    assert torch.equal(out_bf16, out.to(torch.bfloat16))


def test_kda_256_recurrent_steps(cuda):
    state, *_ = _real_inputs(1)
    st_gpu = state.to(cuda)
    st_ref = state.clone()
    g = torch.Generator().manual_seed(99)
    for _ in range(256):
        q = F.normalize(torch.randn(1, 32, 128, generator=g), dim=-1)
        k = F.normalize(torch.randn(1, 32, 128, generator=g), dim=-1)
        v = 0.2 * torch.randn(1, 32, 128, generator=g)
        decay = -(0.005 + 0.075 * torch.rand(1, 32, 128, generator=g))
        beta = torch.sigmoid(torch.randn(1, 32, generator=g))
        out = ops.kda_decode_step(st_gpu, q.to(cuda), k.to(cuda), v.to(cuda), decay.to(cuda),
                                  beta.to(cuda), scale=128 ** -0.5)
        ref = oref.kda_step(st_ref, q, k, v, decay, beta, scale=128 ** -0.5)
    torch.testing.assert_close(st_gpu.cpu(), st_ref, atol=RECURRENT_TOL, rtol=RECURRENT_TOL)
    torch.testing.assert_close(out.cpu(), ref, atol=RECURRENT_TOL, rtol=RECURRENT_TOL)


def test_kda_streaming_recurrent_steps_strided_heads(cuda):
    # 24 sequences (768 heads) whose states are every other head of a larger
    # buffer: the streaming kernel with head and batch strides, 8 steps.
    state, *_ = _real_inputs(24)
    big = torch.zeros(24, 64, 128, 128, device=cuda)
    view = big[:, ::2]
    view.copy_(state.to(cuda))
    st_ref = state.clone()
    g = torch.Generator().manual_seed(7)
    for _ in range(8):
        q = F.normalize(torch.randn(24, 32, 128, generator=g), dim=-1)
        k = F.normalize(torch.randn(24, 32, 128, generator=g), dim=-1)
        v = 0.2 * torch.randn(24, 32, 128, generator=g)
        decay = -(0.005 + 0.075 * torch.rand(24, 32, 128, generator=g))
        beta = torch.sigmoid(torch.randn(24, 32, generator=g))
        out = ops.kda_decode_step(view, q.to(cuda), k.to(cuda), v.to(cuda), decay.to(cuda),
                                  beta.to(cuda), scale=128 ** -0.5)
        ref = oref.kda_step(st_ref, q, k, v, decay, beta, scale=128 ** -0.5)
    torch.testing.assert_close(view.cpu(), st_ref, atol=RECURRENT_TOL, rtol=RECURRENT_TOL)
    torch.testing.assert_close(out.cpu(), ref, atol=RECURRENT_TOL, rtol=RECURRENT_TOL)
    assert float(big[:, 1::2].abs().max()) == 0.0


def test_kda_noncontiguous_state_is_updated_in_place(cuda):
    state, q, k, v, decay, beta = _real_inputs(2)
    big = torch.zeros(2, 32, 128, 160, device=cuda)
    view = big[..., :128]
    view.copy_(state.to(cuda))
    out = ops.kda_decode_step(view, q.to(cuda), k.to(cuda), v.to(cuda), decay.to(cuda),
                              beta.to(cuda), scale=128 ** -0.5)
    ref_state = state.clone()
    ref = oref.kda_step(ref_state, q, k, v, decay, beta, scale=128 ** -0.5)
    torch.testing.assert_close(view.cpu(), ref_state, atol=SINGLE_STEP_TOL, rtol=SINGLE_STEP_TOL)
    torch.testing.assert_close(out.cpu(), ref, atol=SINGLE_STEP_TOL, rtol=SINGLE_STEP_TOL)
    assert float(big[..., 128:].abs().max()) == 0.0


# ---------------------------------------------------------------------------
# quantiser
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("group", [32, 128])
def test_quantise_bit_exact(cuda, group):
    w = rand_weight((512, 2304), cuda_gen(0))
    w[7, :group] = 0
    w[9, :group] = torch.linspace(-3, 3, group, device=cuda).to(torch.bfloat16)
    packed, scales = ops.quantise(w, group)
    ref_p, ref_s = codec.quantise(w.cpu(), group)
    assert torch.equal(packed.cpu(), ref_p)
    assert torch.equal(scales.cpu(), ref_s)


def test_quantise_rejects_nonfinite(cuda):
    w = torch.zeros((4, 128), dtype=torch.bfloat16, device=cuda)
    w[1, 5] = float("inf")
    with pytest.raises(ValueError, match="finite"):
        ops.quantise(w, 128)
