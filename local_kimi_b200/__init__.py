"""B200-native (sm_100a) quantized decode hot path for Kimi-Linear-48B-A3B.

The package is a drop-in for the kernel-registry operations of the reference
engine (engine/kernels): W4A16 dense / grouped / SwiGLU projections, the fused
down projection + routed combine, fused QKV, the sigmoid top-k router and the
KDA recurrent decode step.  Kernels are hand-written CUDA for sm_100a in
``csrc/``, compiled into ``libkimi_b200.so`` and called through the C ABI in
``include/kimi_b200.h``.

  from local_kimi_b200 import ops              # the operators
  from local_kimi_b200 import registry         # registry with the reference API
  from local_kimi_b200.kernels import install  # register into engine.kernels
"""

from __future__ import annotations

from . import ops, registry  # noqa: F401
from ._lib import KernelError, device_errors, pdl_enabled, set_pdl  # noqa: F401

__all__ = ["ops", "registry", "KernelError", "device_errors", "pdl_enabled", "set_pdl"]
__version__ = "0.1.0"
