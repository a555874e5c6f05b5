"""Argument checks of the torch-facing ops that run before any launch (CPU)."""

from __future__ import annotations

import pytest
import torch

from local_kimi_b200 import ops


def test_combine_routes_rejects_weights_on_another_device(monkeypatch):
    # routes sits on a non-CPU device (meta stands in for a GPU here); a CPU
    # weights tensor must be refused before its pointer reaches the kernel.
    monkeypatch.setattr(ops, "_require_cuda", lambda tensor, what: None)
    routes = torch.empty((2, 9, 16), dtype=torch.bfloat16, device="meta")
    weights = torch.ones((2, 8), dtype=torch.float32)
    with pytest.raises(ValueError, match="same CUDA device"):
        ops.moe_combine_routes(routes, weights)


def test_combine_routes_type_and_shape_errors():
    routes = torch.zeros((2, 9, 16), dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        ops.moe_combine_routes(routes.float(), torch.ones((2, 8)))
    with pytest.raises(ValueError, match="T rows"):
        ops.moe_combine_routes(routes, torch.ones((2, 7)))
    with pytest.raises(ValueError, match="requires CUDA"):
        ops.moe_combine_routes(routes, torch.ones((2, 8)))
