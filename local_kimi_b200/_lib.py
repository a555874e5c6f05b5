"""ctypes binding of the C ABI in ``include/kimi_b200.h``.

The shared library ``libkimi_b200.so`` is built in-tree by
``local_kimi_b200.build``.  Loading it has no CUDA side effects; kernels run
only when an entry point is called.  Nothing here falls back to another
implementation: a missing library raises.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libkimi_b200.so")

# Status codes (kb_status in include/kimi_b200.h).
KB_OK = 0
STATUS_NAMES = {
    1: "KB_ERR_NULL_POINTER",
    2: "KB_ERR_BAD_SHAPE",
    3: "KB_ERR_BAD_GROUP",
    4: "KB_ERR_ALIGNMENT",
    5: "KB_ERR_WORKSPACE",
    6: "KB_ERR_UNSUPPORTED",
    7: "KB_ERR_LAUNCH",
    8: "KB_ERR_DEVICE",
}
MAX_DENSE_PROBLEMS = 8
MAX_ASSIGNMENTS = 4096


class DenseProblem(ctypes.Structure):
    """Mirror of ``kb_dense_problem``."""

    _fields_ = [
        ("x", c_void_p),
        ("x_stride", c_int64),
        ("M", c_int64),
        ("K", c_int64),
        ("packed", c_void_p),
        ("scales", c_void_p),
        ("N", c_int64),
        ("group", c_int64),
        ("y", c_void_p),
        ("y_stride", c_int64),
    ]


# name -> (restype, argtypes); every symbol declared in the header.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kb_version": (c_int, []),
    "kb_last_error": (ctypes.c_char_p, []),
    "kb_set_pdl": (None, [c_int]),
    "kb_get_pdl": (c_int, []),
    "kb_device_errors": (c_int, [c_void_p, ctypes.POINTER(c_uint32)]),
    "kb_w4a16_quantise": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "kb_w4a16_dense": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
         c_int64, c_void_p],
    ),
    "kb_w4a16_dense_multi": (c_int, [ctypes.POINTER(DenseProblem), c_int, c_void_p]),
    "kb_w4a16_grouped": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
         c_int64, c_int64, c_void_p, c_void_p],
    ),
    "kb_w4a16_swiglu": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    ),
    "kb_w4a16_dense_tc_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "kb_w4a16_dense_tc": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
         c_int64, c_void_p, c_size_t, c_void_p],
    ),
    "kb_w4a16_grouped_tc": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
         c_int64, c_int64, c_void_p, c_void_p],
    ),
    "kb_w4a16_swiglu_tc": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    ),
    "kb_w4a16_w2_combine_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "kb_w4a16_w2_combine": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
         c_int64, c_int64, c_int64, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "kb_moe_combine_routes": (
        c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    ),
    "kb_kda_prepare": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
         c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p],
    ),
    "kb_kda_prepare_step": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_float,
         c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_void_p,
         c_void_p, c_void_p],
    ),
    "kb_ep_dispatch": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    ),
    "kb_ep_combine": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64,
         c_void_p, c_int64, c_void_p],
    ),
    "kb_router_workspace_size": (c_size_t, [c_int64, c_int64]),
    "kb_router_topk": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int,
         c_float, c_void_p, c_int64, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "kb_router_static_scratch_bytes": (c_size_t, []),
    "kb_router_topk_static": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int,
         c_float, c_void_p, c_int64, c_void_p, c_void_p],
    ),
    "kb_step_create": (c_int, [c_int64, ctypes.POINTER(c_void_p)]),
    "kb_step_destroy": (None, [c_void_p]),
    "kb_step_add_dense": (
        c_int,
        [c_void_p, ctypes.POINTER(DenseProblem), c_int, c_void_p, c_int, ctypes.POINTER(c_int)],
    ),
    "kb_step_add_swiglu": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
         c_int64, c_void_p, c_int64, c_void_p, c_int, ctypes.POINTER(c_int)],
    ),
    "kb_step_add_router": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int,
         c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_int, ctypes.POINTER(c_int)],
    ),
    "kb_step_add_moe": (
        c_int,
        [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
         ctypes.POINTER(c_int)],
    ),
    "kb_step_add_kda": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p,
         c_int, ctypes.POINTER(c_int)],
    ),
    "kb_step_finalize": (c_int, [c_void_p]),
    "kb_step_launch": (c_int, [c_void_p, c_void_p]),
    "kb_step_info": (
        c_int,
        [c_void_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int),
         ctypes.POINTER(c_size_t)],
    ),
    "kb_step_set_trace": (c_int, [c_void_p, c_void_p, c_int64]),
    "kb_step_trace_entries": (c_int64, [c_void_p]),
    "kb_kda_decode_step": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int64, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p],
    ),
}

_LIB: ctypes.CDLL | None = None


class KernelError(RuntimeError):
    """A C ABI call returned a non-zero status."""

    def __init__(self, function: str, status: int, message: str) -> None:
        self.function = function
        self.status = status
        name = STATUS_NAMES.get(status, f"status {status}")
        super().__init__(f"{function} failed with {name}: {message}")


def lib() -> ctypes.CDLL:
    """Load the library once and declare every exported signature."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m local_kimi_b200.build` "
                "(needs nvcc). There is no fallback implementation."
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = handle
    return _LIB


def last_error() -> str:
    raw = lib().kb_last_error()
    return raw.decode("utf-8", "replace") if raw else ""


def check(function: str, status: int) -> None:
    """Raise :class:`KernelError` for a non-zero status."""
    if status != KB_OK:
        raise KernelError(function, status, last_error())


def call(function: str, *args: object) -> None:
    check(function, getattr(lib(), function)(*args))


def set_pdl(enabled: bool) -> None:
    lib().kb_set_pdl(1 if enabled else 0)


def pdl_enabled() -> bool:
    return bool(lib().kb_get_pdl())


def device_errors(stream: int | None = None) -> int:
    """Read and clear the device error word (synchronizes ``stream``)."""
    out = c_uint32(0)
    check("kb_device_errors", lib().kb_device_errors(c_void_p(stream or 0), ctypes.byref(out)))
    return int(out.value)
