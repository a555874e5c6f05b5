"""Pin the CPU oracle to the reference: golden vectors and known answers (CPU).

The golden vectors in tests/golden/reference_g32.pt were produced by running
the reference implementation (tests/golden/make_golden.py).  The known-answer
cases restate the values asserted by the reference's own tests.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import codec, moe, ops


# ---------------------------------------------------------------------------
# codec
# ---------------------------------------------------------------------------


def test_quantise_matches_reference_bit_for_bit(golden):
    packed, scales = codec.quantise(golden["codec.w"], 32)
    assert torch.equal(packed, golden["codec.packed"])
    assert torch.equal(scales, golden["codec.scales"])


def test_dequantise_matches_reference(golden):
    f32 = codec.dequantise(golden["codec.packed"], golden["codec.scales"])
    assert torch.equal(f32, golden["codec.dequant_f32"])
    bf = codec.decode_bf16(golden["codec.packed"], golden["codec.scales"])
    assert torch.equal(bf, golden["codec.dequant_bf16"].float())


def test_nibble_sign_and_group_known_answers():
    # tests/test_w4a16_gemv.py:26-43 of the reference
    nibbles = torch.arange(64, dtype=torch.uint8) % 16
    packed = (nibbles[0::2] | (nibbles[1::2] << 4)).reshape(1, 32)
    scales = torch.tensor([[1.0, 10.0]], dtype=torch.bfloat16)
    actual = codec.dequantise(packed, scales)
    assert actual[0, 0].item() == 0.0
    assert actual[0, 7].item() == 7.0
    assert actual[0, 8].item() == -8.0
    assert actual[0, 15].item() == -1.0
    assert actual[0, 33].item() == 10.0
    assert actual[0, 40].item() == -80.0


def test_two_row_known_answers():
    # tests/test_w4a16_dense_gemv.py:25-45 of the reference
    first = torch.arange(64, dtype=torch.uint8) % 16
    second = torch.flip(first, dims=(0,))
    nib = torch.stack((first, second))
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    scales = torch.tensor([[1.0, 10.0], [0.5, 2.0]], dtype=torch.bfloat16)
    actual = codec.dequantise(packed, scales)
    assert actual[0, 7].item() == 7.0
    assert actual[0, 8].item() == -8.0
    assert actual[0, 15].item() == -1.0
    assert actual[0, 33].item() == 10.0
    assert actual[1, 0].item() == -0.5


def _grid_weight(scales: torch.Tensor, group: int) -> torch.Tensor:
    pattern = torch.tensor([i % 15 - 7 for i in range(group)], dtype=torch.bfloat16)
    codes = pattern.reshape(1, 1, group).expand(scales.shape[0], scales.shape[1], group)
    return (codes * scales.unsqueeze(-1)).reshape(scales.shape[0], -1)


def test_grid_round_trip_and_per_group_scales_g32_and_g128():
    # tests/test_quant_w4a16.py:32-53 of the reference, and the same at group 128
    for group in (32, 128):
        expected = torch.tensor([[0.25, 8.0], [2.0, 0.5]], dtype=torch.bfloat16)
        weight = _grid_weight(expected, group)
        packed, scales = codec.quantise(weight, group)
        assert torch.equal(scales, expected)
        assert torch.equal(codec.dequantise(packed, scales).to(torch.bfloat16), weight)


def test_zero_group_scale_one_and_nonfinite_rejected():
    # tests/test_quant_w4a16.py:135-151 of the reference
    packed, scales = codec.quantise(torch.zeros((3, 64), dtype=torch.bfloat16), 32)
    assert torch.equal(scales, torch.ones_like(scales))
    assert torch.equal(codec.dequantise(packed, scales), torch.zeros(3, 64))
    bad = torch.zeros((1, 32), dtype=torch.bfloat16)
    bad[0, 0] = float("inf")
    try:
        codec.quantise(bad, 32)
    except ValueError as error:
        assert "finite" in str(error)
    else:
        raise AssertionError("non-finite weight accepted")


def test_packing_is_eight_codes_per_int32():
    # The byte layout [N, K/2] viewed as little-endian int32 [N, K/8] holds code
    # k % 8 at bits 4 * (k % 8).
    packed = torch.randint(0, 256, (4, 64), dtype=torch.uint8)
    codes = codec.unpack_codes(packed)
    words = packed.view(torch.int32)
    for k in range(0, 128, 13):
        nib = (words[:, k // 8] >> (4 * (k % 8))) & 0xF
        expect = torch.where(nib >= 8, nib - 16, nib)
        assert torch.equal(expect.to(torch.int16), codes[:, k])


# ---------------------------------------------------------------------------
# operators
# ---------------------------------------------------------------------------


def test_dense_matches_reference(golden):
    for m in (1, 3):
        y = ops.dense(golden[f"dense.m{m}.x"], golden["dense.packed"], golden["dense.scales"])
        assert torch.equal(y, golden[f"dense.m{m}.y"])


def test_grouped_and_swiglu_match_reference(golden):
    g = golden
    gate = ops.grouped(g["grouped.x"], g["grouped.idx"], g["grouped.w1_packed"], g["grouped.w1_scales"])
    up = ops.grouped(g["grouped.x"], g["grouped.idx"], g["grouped.w3_packed"], g["grouped.w3_scales"])
    assert torch.equal(gate, g["grouped.gate"])
    assert torch.equal(up, g["grouped.up"])
    sw = ops.swiglu(g["grouped.x"], g["grouped.idx"], g["grouped.w1_packed"], g["grouped.w1_scales"],
                    g["grouped.w3_packed"], g["grouped.w3_scales"])
    assert torch.equal(sw, g["grouped.swiglu"])


def test_swiglu_rounds_projection_outputs_before_silu():
    # tests/test_moe_swiglu.py:13-34 of the reference
    acc = torch.tensor([1.003], dtype=torch.float32)
    bf16_first = F.silu(acc.to(torch.bfloat16)) * acc.to(torch.bfloat16)
    through = (F.silu(acc) * acc).to(torch.bfloat16)
    assert not torch.equal(bf16_first, through)


def test_combine_matches_reference(golden):
    for key in ("combine", "combine2"):
        out = ops.w2_combine(golden[f"{key}.act"], golden[f"{key}.idx"], golden[f"{key}.w"],
                             golden[f"{key}.w2_packed"], golden[f"{key}.w2_scales"])
        assert torch.equal(out, golden[f"{key}.out"]), key


def test_shared_expert_added_with_weight_one():
    # tests/test_moe_combine.py:65-90 of the reference: routed 32*0.25 = 8, shared 64 -> 72
    red = 32
    act = torch.ones((1, 2, red), dtype=torch.bfloat16)
    idx = torch.tensor([[0, 1]])
    w = torch.tensor([[0.25, 0.0]])
    p = torch.stack([torch.full((1, red // 2), v | (v << 4), dtype=torch.uint8) for v in (1, 2)])
    s = torch.ones((2, 1, 1), dtype=torch.bfloat16)
    out = ops.w2_combine(act, idx, w, p, s)
    assert torch.equal(out, torch.tensor([[72.0]], dtype=torch.bfloat16))


def test_router_matches_reference(golden):
    idx, w, _ = ops.router_topk(golden["router.hidden"], golden["router.weight"],
                                golden["router.bias"], 4, scaling=2.446)
    order = torch.argsort(idx, dim=-1)
    assert torch.equal(torch.gather(idx, 1, order), golden["router.idx_sorted"])
    torch.testing.assert_close(torch.gather(w, 1, order), golden["router.w_sorted"],
                               rtol=1e-6, atol=1e-7)


def test_lane_order_router_matches_reference(golden):
    # The fixed lane summation order changes the logits only in the last fp32
    # bits of the BLAS sum; it routes the reference's golden tokens the same.
    lanes = ops.router_logits_lanes(golden["router.hidden"], golden["router.weight"])
    blas = ops.router_logits(golden["router.hidden"], golden["router.weight"])
    torch.testing.assert_close(lanes, blas, rtol=1e-5, atol=1e-5)
    idx, w, _ = ops.router_topk(golden["router.hidden"], golden["router.weight"],
                                golden["router.bias"], 4, scaling=2.446, logits=lanes)
    order = torch.argsort(idx, dim=-1)
    assert torch.equal(torch.gather(idx, 1, order), golden["router.idx_sorted"])
    torch.testing.assert_close(torch.gather(w, 1, order), golden["router.w_sorted"],
                               rtol=1e-6, atol=1e-6)


def test_lane_order_logits_follow_the_stated_order():
    # A row whose exact sum depends on the order: large terms that cancel
    # with small ones between them.  The stated order is computed here by
    # hand for K = 512 (64 words, two per lane).
    k = 512
    h = torch.ones((1, k), dtype=torch.bfloat16)
    w = torch.zeros((1, k), dtype=torch.bfloat16)
    w[0, 0] = 2.0 ** 24          # word 0, lane 0, pair 0, first value
    w[0, 1] = 1.0                # lost against 2^24 in the same partial sum
    w[0, 8 * 32] = -(2.0 ** 24)  # word 32: lane 0 again, pair 0
    w[0, 2] = 1.0                # pair 1 of word 0: its own partial, kept
    got = ops.router_logits_lanes(h, w)
    # partial 0: (2^24 + 1) rounds to 2^24, then - 2^24 -> 0; partial 1 = 1.
    assert got.item() == 1.0
    assert float((h.double() * w.double()).sum()) == 2.0   # the exact sum differs


def test_router_known_answer_and_tie_break():
    # tests/test_klinear_forward.py:43-75 of the reference
    weight = torch.tensor([[3.0, 0.0], [2.0, 0.0], [1.0, 0.0], [0.0, 0.0]]).to(torch.bfloat16)
    idx, w, _ = ops.router_topk(torch.tensor([[1.0, 0.0]]).to(torch.bfloat16), weight, None, 2,
                                scaling=2.446)
    assert set(idx[0].tolist()) == {0, 1}
    raw = torch.sigmoid(torch.tensor([3.0, 2.0]))
    torch.testing.assert_close(w[0], raw / raw.sum() * 2.446)
    # Equal scores: the lower expert index wins.
    tie = torch.zeros(5, 2).to(torch.bfloat16)
    idx, _, _ = ops.router_topk(torch.tensor([[1.0, 0.0]]).to(torch.bfloat16), tie, None, 3)
    assert idx[0].tolist() == [0, 1, 2]


def test_kda_matches_reference(golden):
    st = golden["kda.state_in"].clone()
    out = ops.kda_step(st, golden["kda.q"], golden["kda.k"], golden["kda.v"], golden["kda.decay"],
                       golden["kda.beta"], scale=16 ** -0.5)
    assert torch.equal(st, golden["kda.state_out"])
    assert torch.equal(out, golden["kda.out"])


def test_kda_hand_computed_two_head_case():
    # tests/test_kda_step.py:18-91 of the reference
    state = torch.tensor([[[[1.0, 2.0, 3.0, 4.0], [5.0, 6.0, 7.0, 8.0], [9.0, 10.0, 11.0, 12.0],
                            [13.0, 14.0, 15.0, 16.0]],
                           [[2.0, 0.0, 1.0, -1.0], [1.0, 3.0, -2.0, 4.0], [0.0, 5.0, 2.0, 1.0],
                            [4.0, -1.0, 0.0, 2.0]]]])
    q = torch.tensor([[[1.0, -1.0, 0.0, 0.0], [0.0, 1.0, 0.0, -1.0]]])
    k = torch.tensor([[[1.0, 1.0, 0.0, 0.0], [0.0, 1.0, 0.0, 1.0]]])
    v = torch.tensor([[[4.5, 7.0, 9.5, 12.0], [7.0, -1.0, 2.0, 4.0]]])
    decay = torch.tensor([[[1.0, 0.5, 2.0, 0.25], [0.5, 1.0, 0.25, 2.0]]]).log()
    beta = torch.tensor([[0.5, 0.25]])
    expected_state = torch.tensor([[[[1.5, 3.0, 4.5, 6.0], [3.0, 4.0, 5.0, 6.0],
                                     [18.0, 20.0, 22.0, 24.0], [3.25, 3.5, 3.75, 4.0]],
                                    [[1.0, 0.0, 0.5, -0.5], [0.5, 2.5, -1.0, 3.0],
                                     [0.0, 1.25, 0.5, 0.25], [7.5, -2.5, 1.0, 3.0]]]])
    expected_out = torch.tensor([[[-0.375, -0.25, -0.125, 0.0], [-1.75, 1.25, -0.5, 0.0]]])
    out = ops.kda_step(state, q, k, v, decay, beta, scale=0.25)
    torch.testing.assert_close(state, expected_state, atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(out, expected_out, atol=1e-6, rtol=1e-6)


def test_moe_layer_matches_reference_eager_path(golden):
    g = golden
    banks = moe.MoEBanks(g["moe.router_weight"], torch.zeros(16), g["moe.w1_packed"],
                         g["moe.w1_scales"], g["moe.w2_packed"], g["moe.w2_scales"],
                         g["moe.w3_packed"], g["moe.w3_scales"], top_k=4, scaling=2.446)
    out, idx, w = moe.moe_layer(g["moe.hidden"], banks)
    order = torch.argsort(idx, dim=-1)
    assert torch.equal(torch.gather(idx, 1, order), g["moe.idx_sorted"])
    torch.testing.assert_close(torch.gather(w, 1, order), g["moe.w_sorted"], rtol=1e-6, atol=1e-7)
    # The reference's eager path multiplies bf16 matrices on the CPU (its own
    # accumulation order); the grouped structure here must agree to within
    # one bf16 rounding of each projection.
    from tests.conftest import assert_close

    assert_close(out, g["moe.out"], what="moe layer")


def test_shape_stable_indices_append_shared_route():
    # tests/test_decode_equivalence.py:70-87 of the reference
    idx = torch.tensor([[4, 1, 7], [2, 6, 0]])
    stable = ops.shape_stable_indices(idx, 8)
    assert torch.equal(stable[:, :-1], idx)
    assert torch.equal(stable[:, -1], torch.full((2,), 8))


def test_kda_prepare_matches_reference(golden):
    # kda_prepare.py:426-472 and 581-615, recorded from the reference.
    from oracle import kda_prep

    g = golden
    states = [g[f"prep.{n}_state_in"].clone() for n in "qkv"]
    conv = kda_prep.short_conv3(*(g[f"prep.{n}_in"] for n in "qkv"), *states,
                                *(g[f"prep.{n}_weight"] for n in "qkv"))
    for j, n in enumerate("qkv"):
        assert torch.equal(conv[j], g[f"prep.{n}_conv"])
        assert torch.equal(states[j], g[f"prep.{n}_state_out"])
    decay, beta, q, k = kda_prep.gates(g["prep.raw_decay"], g["prep.dt_bias"], g["prep.a_log"],
                                       g["prep.raw_beta"], conv[0], conv[1], num_heads=2,
                                       head_dim=128)
    assert torch.equal(decay, g["prep.decay"])
    assert torch.equal(beta, g["prep.beta"])
    assert torch.equal(q, g["prep.q"])
    assert torch.equal(k, g["prep.k"])


def test_kda_prepare_known_answers():
    # tests/test_kda_prepare.py:26-123 of the reference (hand-computed cases).
    import math

    from oracle import kda_prep

    silu = lambda v: v / (1.0 + math.exp(-v))  # noqa: E731
    states = [torch.tensor([[[1.0, 2.0, 3.0, 4.0]]]), torch.tensor([[[4.0, 3.0, 2.0, 1.0]]]),
              torch.tensor([[[-1.0, -2.0, -3.0, -4.0]]])]
    weights = [torch.tensor([[[1.0, 0.0, 0.0, 0.0]]]), torch.tensor([[[0.0, 0.0, 1.0, 0.0]]]),
               torch.tensor([[[1.0, 1.0, 1.0, 1.0]]])]
    out = kda_prep.short_conv3(torch.tensor([[[5.0]]]), torch.tensor([[[0.0]]]),
                               torch.tensor([[[6.0]]]), *states, *weights)
    for actual, expected in zip(out, (silu(2.0), silu(1.0), silu(-3.0))):
        torch.testing.assert_close(actual, torch.tensor([[[expected]]]), atol=1e-6, rtol=1e-6)
    assert torch.equal(states[0], torch.tensor([[[2.0, 3.0, 4.0, 5.0]]]))
    assert torch.equal(states[2], torch.tensor([[[-2.0, -3.0, -4.0, 6.0]]]))
    eps = 1e-6
    decay, beta, q, k = kda_prep.gates(
        torch.tensor([[[[0.0, 1.0], [-1.0, 2.0]]]]), torch.tensor([0.5, -0.5, 1.0, -1.0]),
        torch.log(torch.tensor([2.0, 0.5])).view(1, 1, 2, 1),
        torch.tensor([[[0.0, math.log(3.0)]]]), torch.tensor([[[3.0, 4.0, 0.0, 2.0]]]),
        torch.tensor([[[5.0, 12.0, 8.0, 15.0]]]), num_heads=2, head_dim=2, eps=eps)
    sp = lambda v: math.log1p(math.exp(v))  # noqa: E731
    torch.testing.assert_close(decay, torch.tensor(
        [[[[-2.0 * sp(0.5), -2.0 * sp(0.5)], [-0.5 * sp(0.0), -0.5 * sp(1.0)]]]]),
        atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(beta, torch.tensor([[[0.5, 0.75]]]), atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(q, torch.tensor(
        [[[[3.0 / math.sqrt(25 + eps), 4.0 / math.sqrt(25 + eps)],
           [0.0, 2.0 / math.sqrt(4 + eps)]]]]), atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(k, torch.tensor(
        [[[[5.0 / math.sqrt(169 + eps), 12.0 / math.sqrt(169 + eps)],
           [8.0 / math.sqrt(289 + eps), 15.0 / math.sqrt(289 + eps)]]]]), atol=1e-6, rtol=1e-6)
