"""Tensor-core (tcgen05/TMEM) W4A16 projections against the oracle (GPU).

The many-token forms of the dense, grouped and SwiGLU projections
(kb_w4a16_dense_tc / kb_w4a16_grouped_tc / kb_w4a16_swiglu_tc) at the
north-star tolerance, at the decode shapes, ragged sizes and both group
sizes; the grouped forms with duplicate, skewed and single-expert routing.
"""

from __future__ import annotations

import pytest
import torch

from local_kimi_b200 import ops
from oracle import ops as oref
from tests.conftest import assert_close
from tests.gpu_util import cuda_gen, quant_bank, quant_matrix, rand_act, zipf_indices

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k,group", [
    (1, 512, 1024, 128),      # fewer token rows than one activation copy box
    (5, 1024, 2304, 128),
    (16, 4096, 2304, 128),
    (32, 4096, 2304, 128),
    (64, 2304, 4096, 128),
    (100, 2048, 2304, 128),
    (128, 1024, 2304, 32),
    (200, 1000, 1024, 128),   # ragged N (partial tiles) and two token blocks
    (64, 8192, 512, 128),     # MLA kv_b shape
])
def test_dense_tc_matches_oracle(cuda, m, n, k, group):
    gen = cuda_gen(100 + m)
    packed, scales = quant_matrix(n, k, group, gen)
    x = rand_act((m, k), gen)
    y = ops.w4a16_dense_tc(x, packed, scales)
    torch.cuda.synchronize()
    ref = oref.dense(x.cpu(), packed.cpu(), scales.cpu())
    assert_close(y, ref, what=f"dense tc M={m} N={n} K={k} g{group}")
    # Deterministic run to run.
    again = ops.w4a16_dense_tc(x, packed, scales)
    assert torch.equal(y, again)


def test_dense_tc_strided_activations_and_output(cuda):
    gen = cuda_gen(7)
    packed, scales = quant_matrix(2048, 2304, 128, gen)
    big = rand_act((48, 2304 + 64), gen)
    x = big[:, 32:32 + 2304]
    out = torch.zeros((48, 2048 + 16), dtype=torch.bfloat16, device=cuda)
    ops.w4a16_dense_tc(x, packed, scales, out=out[:, :2048])
    torch.cuda.synchronize()
    ref = oref.dense(x.cpu(), packed.cpu(), scales.cpu())
    assert_close(out[:, :2048], ref, what="strided")
    assert bool((out[:, 2048:] == 0).all())


def test_dense_tc_agrees_with_gemv_engine(cuda):
    gen = cuda_gen(9)
    packed, scales = quant_matrix(4096, 2304, 128, gen)
    x = rand_act((32, 2304), gen)
    a = ops.w4a16_dense_tc(x, packed, scales)
    b = ops.w4a16_dense_engine(x, packed, scales)
    assert_close(a, b, what="tc vs gemv")


@pytest.mark.parametrize("tokens,skew", [(64, 1.1), (16, 0.0), (200, 0.0)])
def test_swiglu_tc_matches_oracle(cuda, tokens, skew):
    gen = cuda_gen(200 + tokens)
    experts = 33
    w1 = quant_bank(experts, 1024, 2304, 128, gen)
    w3 = quant_bank(experts, 1024, 2304, 128, gen)
    x = rand_act((tokens, 2304), gen)
    routed = zipf_indices(tokens, experts - 1, 4, skew, seed=tokens)
    idx = torch.cat((routed, torch.full((tokens, 1), experts - 1)), dim=1).to(cuda)
    y = ops.w4a16_swiglu_tc(x, idx, *w1, *w3)
    torch.cuda.synchronize()
    ref = oref.swiglu(x.cpu(), idx.cpu(), w1[0].cpu(), w1[1].cpu(), w3[0].cpu(), w3[1].cpu())
    assert_close(y, ref, what=f"swiglu tc T={tokens}")
    per_op = ops.w4a16_swiglu(x, idx, *w1, *w3)
    assert_close(y, per_op, what="swiglu tc vs gemv engine")


@pytest.mark.parametrize("rows,group", [(576, 128), (64, 32)])
def test_grouped_tc_down_projection_pattern(cuda, rows, group):
    # The down projection's call pattern: one route per row (R = 1), rows of
    # several tokens' routes, K = 1024 -> N = 2304.
    gen = cuda_gen(300 + rows)
    experts = 17
    w2 = quant_bank(experts, 2304, 1024, group, gen)
    x = rand_act((rows, 1024), gen)
    idx = torch.randint(0, experts, (rows, 1), generator=torch.Generator().manual_seed(rows))
    idx = idx.to(cuda)
    y = ops.w4a16_grouped_tc(x, idx, *w2)
    torch.cuda.synchronize()
    ref = oref.grouped(x.cpu(), idx.cpu(), w2[0].cpu(), w2[1].cpu())
    assert_close(y, ref, what=f"grouped tc rows={rows} g{group}")


def test_grouped_tc_single_expert_many_rows(cuda):
    # Every assignment on one expert: the shared-expert case over a batch
    # (more rows than one unit takes, so it is split into token blocks).
    gen = cuda_gen(400)
    w = quant_bank(3, 1024, 2304, 128, gen)
    x = rand_act((300, 2304), gen)
    idx = torch.full((300, 1), 2, dtype=torch.long, device=cuda)
    y = ops.w4a16_grouped_tc(x, idx, *w)
    torch.cuda.synchronize()
    ref = oref.dense(x.cpu(), w[0][2].cpu(), w[1][2].cpu())
    assert_close(y[:, 0], ref, what="single expert")


def test_tc_reports_no_device_errors(cuda):
    from local_kimi_b200 import _lib

    gen = cuda_gen(500)
    packed, scales = quant_matrix(1024, 2304, 128, gen)
    x = rand_act((64, 2304), gen)
    ops.w4a16_dense_tc(x, packed, scales)
    torch.cuda.synchronize()
    assert _lib.device_errors() == 0


def test_single_expert_swiglu_and_down(cuda):
    # One expert and 300 rows (a dense MLP through the grouped modes): SwiGLU,
    # then the down projection on its output, in token blocks of 64 rows.
    gen = cuda_gen(500)
    w1 = quant_bank(1, 1024, 2304, 128, gen)
    w3 = quant_bank(1, 1024, 2304, 128, gen)
    w2 = quant_bank(1, 2304, 1024, 128, gen)
    x = rand_act((300, 2304), gen)
    idx = torch.zeros((300, 1), dtype=torch.long, device=cuda)
    act = ops.w4a16_swiglu_tc(x, idx, *w1, *w3)
    y = ops.w4a16_grouped_tc(act[:, 0], idx, *w2)
    torch.cuda.synchronize()
    ref_act = oref.swiglu(x.cpu(), idx.cpu(), w1[0].cpu(), w1[1].cpu(), w3[0].cpu(),
                          w3[1].cpu())
    assert_close(act, ref_act, what="swiglu, one expert, 300 rows")
    ref = oref.dense(act[:, 0].cpu(), w2[0][0].cpu(), w2[1][0].cpu())
    assert_close(y[:, 0], ref, what="down, one expert, 300 rows")
