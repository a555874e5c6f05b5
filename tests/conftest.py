"""Shared test configuration.

Markers: ``gpu`` tests need a CUDA device (run on a B200 with ``-m gpu``);
everything else runs on the CPU.  GPU tests call the CUDA kernels through the
C ABI (``local_kimi_b200._lib``) via the torch-facing ``ops`` layer and check
them against the CPU oracle in ``oracle/``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_g32.pt"

# Tolerance of the north-star parity contract: an element passes when it is
# within 2e-2 relative OR 1e-3 absolute of the fp32-accumulated oracle.
REL_TOL = 2e-2
ABS_TOL = 1e-3


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden() -> dict:
    return torch.load(GOLDEN, weights_only=True)


@pytest.fixture(scope="session")
def cuda() -> torch.device:
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)


def bf16_spacing(magnitude: torch.Tensor) -> torch.Tensor:
    """Distance between adjacent bf16 values at ``magnitude`` (8 significant bits)."""
    m = magnitude.detach().float().cpu().abs().clamp_min(torch.finfo(torch.float32).tiny)
    return torch.exp2(torch.floor(torch.log2(m)) - 7)


def close_mask(actual: torch.Tensor, expected: torch.Tensor, rel: float = REL_TOL,
               abs_: float = ABS_TOL, allowance: torch.Tensor | None = None) -> torch.Tensor:
    """Elementwise pass mask: within ``rel`` relative OR ``abs_`` absolute.

    ``allowance`` (optional, per element) is the rounding uncertainty of the
    oracle's own bf16 intermediates where the result is formed by cancellation,
    e.g. out = bf16(routed) + shared in the MoE combine: one bf16 spacing of
    each rounded term it is built from (oracle.ops.combine_rounding_bound).
    Where no cancellation occurs the allowance is below the 2e-2 / 1e-3 test.
    """
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    diff = (a - e).abs()
    ok = (diff <= abs_) | (diff <= rel * e.abs()) | ((a == e) & torch.isfinite(e)) | (
        torch.isnan(a) & torch.isnan(e))
    if allowance is not None:
        ok |= diff <= allowance.detach().float().cpu() * 1.0001
    return ok


def assert_close(actual: torch.Tensor, expected: torch.Tensor, rel: float = REL_TOL,
                 abs_: float = ABS_TOL, what: str = "",
                 allowance: torch.Tensor | None = None) -> None:
    assert actual.shape == expected.shape, f"{what}: shape {tuple(actual.shape)} != {tuple(expected.shape)}"
    ok = close_mask(actual, expected, rel, abs_, allowance)
    if not bool(ok.all()):
        bad = (~ok).nonzero()
        first = tuple(bad[0].tolist())
        a = actual.detach().float().cpu()[first].item()
        e = expected.detach().float().cpu()[first].item()
        raise AssertionError(
            f"{what}: {int((~ok).sum())} of {ok.numel()} elements outside rel {rel} / abs {abs_}; "
            f"first at {first}: got {a}, expected {e}"
        )
