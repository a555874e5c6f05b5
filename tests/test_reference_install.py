"""The drop-in, installed into the reference's own kernel registry (CPU).

``local_kimi_b200.kernels.install()`` registers the ``b200`` variants inside
``engine.kernels.registry`` (engine/kernels/registry.py:34-204, populated by
engine/kernels/__init__.py:21-223) and rebinds
``engine.kernels.kda_step.kda_decode_step``, the function KDAAttention imports
by module path (engine/klinear/attention.py:153-165).  These checks import the
reference from its source tree when it is present (the build container) and
skip otherwise; no kernel runs.
"""

from __future__ import annotations

import inspect
import os
import sys
from pathlib import Path

import pytest
import torch

REFERENCE_ROOT = Path(os.environ.get("KIMI_REFERENCE_ROOT", "/root/reference"))

pytestmark = pytest.mark.skipif(not (REFERENCE_ROOT / "engine" / "kernels").is_dir(),
                                reason="reference source tree not present")


@pytest.fixture(scope="module")
def reference():
    if str(REFERENCE_ROOT) not in sys.path:
        sys.path.insert(0, str(REFERENCE_ROOT))
    try:
        import engine.kernels  # noqa: F401
        import engine.kernels.kda_step as kda_module
        from engine.kernels import registry
    except Exception as exc:  # pragma: no cover - depends on the reference's imports
        pytest.skip(f"reference kernels do not import here: {exc}")
    from local_kimi_b200 import kernels

    original_kda = kda_module.kda_decode_step
    kernels.install(registry, kda_module=kda_module)
    return registry, kda_module, original_kda


def test_b200_is_the_shipped_default(reference, monkeypatch):
    registry, _, _ = reference
    monkeypatch.delenv("KIMI_KERNELS", raising=False)
    for op in ("w4a16_dense", "w4a16_grouped", "w4a16_swiglu"):
        assert "b200" in registry.variants(op)
        assert registry.default_of(op) == "b200"
        assert registry.active(op) == "b200"
        # The reference variant is still registered and still the reference.
        assert registry.reference_of(op).name == "reference"


def test_environment_and_programmatic_overrides_still_win(reference, monkeypatch):
    registry, _, _ = reference
    monkeypatch.setenv("KIMI_KERNELS", "w4a16_dense=triton_gemv")
    assert registry.active("w4a16_dense") == "triton_gemv"
    assert registry.active("w4a16_grouped") == "b200"
    monkeypatch.delenv("KIMI_KERNELS")
    with registry.using("w4a16_swiglu", "reference"):
        assert registry.active("w4a16_swiglu") == "reference"
    assert registry.active("w4a16_swiglu") == "b200"


def test_unwired_ops_get_registry_entries(reference):
    registry, _, _ = reference
    from engine.kernels import moe_combine, w4a16_fused_qkv

    assert registry.variants("moe_combine") == ("reference", "b200")
    assert registry.reference_of("moe_combine").fn is moe_combine.fused_w2_combine_reference
    assert registry.variants("w4a16_qkv") == ("reference", "b200")
    assert registry.reference_of("w4a16_qkv").fn is w4a16_fused_qkv.fused_qkv_w4a16_reference
    assert registry.active("moe_combine") == "b200"


def test_install_is_idempotent(reference):
    registry, kda_module, _ = reference
    from local_kimi_b200 import kernels

    before = {op: registry.variants(op) for op in ("w4a16_dense", "moe_combine", "w4a16_qkv")}
    kernels.install(registry, kda_module=kda_module)
    after = {op: registry.variants(op) for op in before}
    assert before == after


def test_kda_step_is_rebound_with_the_reference_signature(reference):
    _, kda_module, original = reference
    from local_kimi_b200 import ops

    assert kda_module.kda_decode_step is ops.kda_decode_step
    assert kda_module._reference_kda_decode_step is original
    ours = inspect.signature(ops.kda_decode_step).parameters
    theirs = inspect.signature(original).parameters
    for name in ("state", "q", "k", "v", "decay", "beta"):
        assert list(ours).index(name) == list(theirs).index(name)
    assert ours["scale"].kind is inspect.Parameter.KEYWORD_ONLY
    assert theirs["scale"].kind is inspect.Parameter.KEYWORD_ONLY


def test_resolve_refuses_without_cuda_and_cpu_tensors_raise_value_error(reference):
    registry, _, _ = reference
    if torch.cuda.is_available():
        pytest.skip("checks the CPU-only behaviour")
    # The registry refuses a CUDA-only variant on a CPU-only box, as it does
    # for the reference's own Triton variants.
    with pytest.raises(RuntimeError, match="requires CUDA"):
        registry.resolve("w4a16_dense")
    # Called directly, the variant raises what the reference's validators
    # raise for CPU tensors (engine/kernels/w4a16_dense_gemv.py:171-197).
    fn = registry._REGISTRY["w4a16_dense"]["b200"].fn
    x = torch.zeros((1, 64), dtype=torch.bfloat16)
    packed = torch.zeros((8, 32), dtype=torch.uint8)
    scales = torch.ones((8, 2), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="requires CUDA"):
        fn(x, packed, scales)
    # Type errors come first, as in the reference.
    with pytest.raises(TypeError):
        fn(x.float(), packed, scales)
    kda = registry._REGISTRY["w4a16_grouped"]["b200"].fn
    with pytest.raises(ValueError):
        kda(x, torch.zeros((1, 9), dtype=torch.long), packed[None], scales[None])
