"""The C-ABI library builds, loads and exports every declared symbol (CPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from local_kimi_b200 import _lib
from local_kimi_b200 import build as build_mod

HEADER = Path(__file__).resolve().parents[1] / "include" / "kimi_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def library() -> ctypes.CDLL:
    build_mod.build()
    return _lib.lib()


def test_header_declares_the_hot_path_entry_points():
    names = declared_functions()
    for required in ("kb_w4a16_dense", "kb_w4a16_grouped", "kb_w4a16_swiglu",
                     "kb_w4a16_w2_combine", "kb_router_topk", "kb_kda_decode_step",
                     "kb_w4a16_quantise", "kb_w4a16_dense_multi", "kb_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol(library):
    for name in declared_functions():
        assert hasattr(library, name), f"{name} declared in the header but not exported"


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_version_and_error_string_without_gpu(library):
    assert library.kb_version() >= 100
    assert _lib.last_error() == ""


def test_workspace_size_queries_are_pure(library):
    assert library.kb_w4a16_w2_combine_workspace_size(0, 9, 2304) == 0
    size = library.kb_w4a16_w2_combine_workspace_size(64, 9, 2304)
    assert size >= 64 * 9 * 2304 * 2 and size % 256 == 0
    assert library.kb_router_workspace_size(64, 256) >= 64 * 256 * 4


def test_invalid_arguments_return_status_without_launching(library):
    # A bad group size is rejected by validation before any CUDA call.
    status = library.kb_w4a16_dense(None, 64, 1, 64, None, None, 16, 48, None, 16, None)
    assert status == 3  # KB_ERR_BAD_GROUP
    assert "group" in _lib.last_error()
    status = library.kb_w4a16_dense(None, 64, 1, 48, None, None, 16, 32, None, 16, None)
    assert status == 2  # KB_ERR_BAD_SHAPE (K % 32)
    status = library.kb_w4a16_grouped(None, 64, 1, 64, None, 9, None, None, 4, 16, 32, None, None)
    assert status == 1  # KB_ERR_NULL_POINTER
    status = library.kb_kda_decode_step(None, 0, 0, 0, None, None, None, None, None, 1, 1, 300,
                                        8, 1.0, None, None, None)
    assert status == 6  # KB_ERR_UNSUPPORTED (Dk > 256)
    with pytest.raises(_lib.KernelError, match="KB_ERR_BAD_GROUP"):
        _lib.check("kb_w4a16_dense", 3)
    # Route combine: width not a multiple of 8, NULL routes, short weight rows.
    assert library.kb_moe_combine_routes(None, 1, 2, 7, None, 1, None, None) == 2
    assert library.kb_moe_combine_routes(None, 1, 2, 8, None, 1, None, None) == 1
    assert "NULL" in _lib.last_error()
    assert library.kb_moe_combine_routes(None, 0, 2, 8, None, 1, None, None) == 0


def test_step_program_validation_without_gpu(library):
    import ctypes

    handle = ctypes.c_void_p()
    assert library.kb_step_create(0, ctypes.byref(handle)) == 6  # KB_ERR_UNSUPPORTED
    assert library.kb_step_create(9, ctypes.byref(handle)) == 6
    assert library.kb_step_create(2, None) == 1  # KB_ERR_NULL_POINTER
    assert library.kb_step_create(2, ctypes.byref(handle)) == 0 and handle.value
    op = ctypes.c_int(-1)
    # No problems: rejected before any CUDA call; launching an unfinalized
    # program is refused.
    assert library.kb_step_add_dense(handle, None, 1, None, 0, ctypes.byref(op)) == 1
    assert library.kb_step_launch(handle, None) == 6
    library.kb_step_destroy(handle)
