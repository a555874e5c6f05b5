"""kb_router_topk_static: the router entry point that allocates nothing.

It keeps its scratch in a fixed device array instead of a caller workspace.
It is called here through the C ABI and compared with kb_router_topk (the
workspace entry point, through ops.moe_router) on the same inputs, two calls
in a row per shape, and across shapes, so that counters left by one call are
seen by the next.  The file is named to be collected last, so that the same
checks also run after every other GPU test in one process.
"""

from __future__ import annotations

from ctypes import c_float, c_int64, c_void_p

import pytest
import torch

from local_kimi_b200 import _lib, ops

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
    for _ in range(2):
        idx, w = static_router(hidden, weight, bias, top_k, 2.446, experts if append else -1)
        torch.cuda.synchronize()
        assert torch.equal(idx, want_idx)
        assert_close(w, want_w, what="static router weights")


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
    assert "kb_router_topk" in str(err.value)
