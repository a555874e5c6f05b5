"""kb_router_topk_static: the router entry point that allocates nothing.

It keeps its scratch in a fixed device array instead of a caller workspace.
It is called here through the C ABI and compared with kb_router_topk (the
workspace entry point, through ops.moe_router) and with the CPU oracle (logits
summed in the kernels' stated lane order) on the same inputs, two calls in a
row per shape, and across shapes, so that counters left by one call are seen
by the next.  The file is named to be collected last, so that the same checks
also run after every other GPU test in one process.
"""

from __future__ import annotations

from ctypes import c_float, c_int64, c_void_p

import pytest
import torch

from local_kimi_b200 import _lib, ops
from oracle import ops as oref

from tests.conftest import assert_close
from tests.gpu_util import cuda_gen, rand_act, rand_weight

pytestmark = pytest.mark.gpu

KB_ERR_WORKSPACE = 5


def static_router(hidden, weight, bias, top_k, scaling, append_id=-1):
    tokens, width = hidden.shape
    experts = weight.shape[0]
    extra = 1 if append_id >= 0 else 0
    idx = torch.empty((tokens, top_k + extra), dtype=torch.long, device=hidden.device)
    wts = torch.empty((tokens, top_k), dtype=torch.float32, device=hidden.device)
    stream = c_void_p(torch.cuda.current_stream(hidden.device).cuda_stream)
    _lib.call(
        "kb_router_topk_static",
        c_void_p(hidden.data_ptr()), c_int64(hidden.stride(0)), c_int64(tokens),
        c_int64(width), c_void_p(weight.data_ptr()),
        c_void_p(0 if bias is None else bias.data_ptr()), c_int64(experts), c_int64(top_k), 1,
        c_float(scaling), c_void_p(idx.data_ptr()), c_int64(append_id),
        c_void_p(wts.data_ptr()), stream,
    )
    return idx, wts


def check_against_workspace_entry(cuda, tokens, experts, width, top_k, seed, append):
    gen = cuda_gen(seed)
    hidden = rand_act((tokens, width), gen)
    weight = rand_weight((experts, width), gen, std=0.05)
    bias = torch.randn(experts, generator=gen, device=cuda) * 0.1
    want_idx, want_w = ops.moe_router(hidden, weight, bias, top_k, routed_scaling_factor=2.446,
                                      append_expert=experts if append else None)
    ref_idx, ref_w, _ = oref.router_topk(
        hidden.cpu(), weight.cpu(), bias.cpu(), top_k, scaling=2.446,
        logits=oref.router_logits_lanes(hidden.cpu(), weight.cpu()))
    for _ in range(2):
        idx, w = static_router(hidden, weight, bias, top_k, 2.446, experts if append else -1)
        torch.cuda.synchronize()
        assert torch.equal(idx, want_idx)
        assert_close(w, want_w, what="static router weights")
        assert torch.equal(idx[:, :top_k].cpu(), ref_idx)
        torch.testing.assert_close(w.cpu(), ref_w, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("tokens,experts,width,top_k,append", [
    (1, 256, 2304, 8, True),
    (32, 256, 2304, 8, True),
    (64, 256, 2304, 8, False),
    (5, 1024, 512, 32, False),
])
def test_static_router_matches_workspace_router(cuda, tokens, experts, width, top_k, append):
    check_against_workspace_entry(cuda, tokens, experts, width, top_k, 1000 + tokens, append)


def test_static_router_shape_sequence(cuda):
    # Alternating shapes share one scratch array; each call must leave its
    # counters at zero for the next.
    for tokens in (64, 1, 17, 512, 3):
        check_against_workspace_entry(cuda, tokens, 256, 2304, 8, 2000 + tokens, True)


def test_static_router_rejects_oversize_calls(cuda):
    limit = int(_lib.lib().kb_router_static_scratch_bytes())
    assert limit >= 256 * 512 * 4
    gen = cuda_gen(7)
    tokens, experts = 513, 256  # T*E = 131328 logits, above the fixed scratch
    hidden = rand_act((tokens, 64), gen)
    weight = rand_weight((experts, 64), gen)
    with pytest.raises(_lib.KernelError) as err:
        static_router(hidden, weight, None, 8, 1.0)
    assert err.value.status == KB_ERR_WORKSPACE
    assert "kb_router_topk" in str(err.value) and "T*E" in str(err.value)
    # Few experts, many tokens: within the logit space but above the 1024
    # token blocks of 8 that the fixed arrival counters cover.
    tokens, experts = 8200, 8
    hidden = rand_act((tokens, 64), gen)
    weight = rand_weight((experts, 64), gen)
    with pytest.raises(_lib.KernelError) as err:
        static_router(hidden, weight, None, 2, 1.0)
    assert err.value.status == KB_ERR_WORKSPACE
    assert "arrival counters" in str(err.value) and "T*E" not in str(err.value)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_static_router_on_a_second_device():
    # The scratch and its set-up are per device.
    dev = torch.device("cuda", 1)
    with torch.cuda.device(dev):
        gen = torch.Generator(device=dev).manual_seed(3000)
        hidden = torch.randn((16, 2304), generator=gen, device=dev).to(torch.bfloat16)
        weight = (torch.randn((256, 2304), generator=gen, device=dev) * 0.05).to(torch.bfloat16)
        want_idx, want_w = ops.moe_router(hidden, weight, None, 8, routed_scaling_factor=2.446)
        for _ in range(2):
            idx, w = static_router(hidden, weight, None, 8, 2.446)
            torch.cuda.synchronize(dev)
            assert torch.equal(idx, want_idx)
            assert torch.equal(w, want_w)
