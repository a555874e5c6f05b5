"""Torch-facing B200 operators with the reference kernel-registry signatures.

Every function here validates its arguments the way the reference entry point
does (``TypeError`` for rank/dtype, ``ValueError`` for shape/device), allocates
its outputs through the torch caching allocator, and launches the CUDA kernels
of ``libkimi_b200.so`` on ``torch.cuda.current_stream()``.  There is no CPU or
library fallback: CPU tensors raise ``ValueError`` and a missing library
raises ``RuntimeError``.  No call synchronizes the host, so the operators can
be captured in a CUDA graph after one warm-up call per shape (the warm-up
allocates the scratch buffers that the router and the down+combine kernels
keep between calls).

Reference entry points mirrored here:
  w4a16_dense       engine/kernels/w4a16_dense_gemv.py:312-336 (validation :171-197)
  w4a16_grouped     engine/kernels/w4a16_gemv.py:610-635 (validation :449-488)
  w4a16_swiglu      engine/kernels/w4a16_gemv.py:772-790, engine/kernels/__init__.py:182-197
  fused_w2_combine  engine/kernels/moe_combine.py:264-324 (validation :157-206)
  fused_qkv_w4a16   engine/kernels/w4a16_fused_qkv.py:342-389
  kda_decode_step   engine/kernels/kda_step.py:273-293 (validation :137-170)
  moe_router        engine/klinear/router.py:47-85
  quantise          engine/quant/w4a16.py:68-105 (group size as a parameter)
"""

from __future__ import annotations

from ctypes import c_float, c_int64, c_size_t, c_void_p

import torch

from . import _lib

REFERENCE_GROUP_SIZE = 32


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def _stream(device: torch.device) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _p(tensor: torch.Tensor | None) -> c_void_p:
    return c_void_p(0 if tensor is None else tensor.data_ptr())


def _require_cuda(tensor: torch.Tensor, what: str) -> None:
    if tensor.device.type != "cuda":
        raise ValueError(f"{what} requires CUDA")


def group_size_of(reduction: int, scale_columns: int) -> int:
    """Group size implied by a reduction width and the scale tensor's width."""
    if scale_columns <= 0 or reduction % scale_columns:
        raise ValueError(
            f"scales with {scale_columns} columns cannot cover a reduction width of {reduction}"
        )
    group = reduction // scale_columns
    if group < 32 or group % 32 or (group & (group - 1)):
        raise ValueError(f"group size {group} must be 32 times a power of two")
    return group


def _rows_16b(t: torch.Tensor) -> torch.Tensor:
    """Return ``t`` (2-D) with unit inner stride, 16-byte aligned rows."""
    if (
        t.stride(-1) != 1
        or t.stride(0) % 8
        or t.data_ptr() % 16
        or t.stride(0) < t.shape[-1]
    ):
        t = t.contiguous()
    return t


def _dense_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() and t.data_ptr() % 16 == 0 else t.contiguous()


_WORKSPACES: dict[tuple, torch.Tensor] = {}


def _workspace(kind: str, device: torch.device, nbytes: int, shape: tuple) -> torch.Tensor:
    """Zero-filled scratch kept per (kind, device, stream, problem shape).

    The router and down+combine kernels keep arrival counters in their scratch
    and leave them at zero after every call.  The counters' position depends on
    the problem shape, so a buffer is reused only for the same shape: a buffer
    shared between shapes could place one shape's counters on another shape's
    leftover data.
    """
    stream = torch.cuda.current_stream(device).cuda_stream
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (kind, index, stream, shape)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


# ---------------------------------------------------------------------------
# dense
# ---------------------------------------------------------------------------


def _validate_dense(
    activations: torch.Tensor, packed_weights: torch.Tensor, scales: torch.Tensor
) -> tuple[int, int, int, int]:
    if activations.ndim != 2 or activations.dtype != torch.bfloat16:
        raise TypeError("activations must be a BF16 [tokens, reduction] matrix")
    if packed_weights.ndim != 2 or packed_weights.dtype != torch.uint8:
        raise TypeError("packed weights must be a uint8 [output, reduction / 2] matrix")
    if scales.ndim != 2 or scales.dtype != torch.bfloat16:
        raise TypeError("scales must be a BF16 [output, reduction / group] matrix")
    _require_cuda(activations, "W4A16 dense GEMV")
    if not (activations.device == packed_weights.device == scales.device):
        raise ValueError("activations, packed weights, and scales must share a device")
    m, reduction = activations.shape
    output_size, packed_reduction = packed_weights.shape
    if output_size == 0 or reduction == 0:
        raise ValueError("W4A16 dense GEMV requires nonzero dimensions")
    if reduction % 32:
        raise ValueError("the reduction dimension must be divisible by group size 32")
    if packed_reduction * 2 != reduction:
        raise ValueError("packed weights have the wrong reduction width")
    if scales.shape[0] != output_size:
        raise ValueError("W4A16 scales have the wrong shape")
    group = group_size_of(reduction, scales.shape[1])
    return m, output_size, reduction, group


# Tensor-core (tcgen05) limits: K a multiple of 128, N of 8, at most 81 scale
# groups per row (the per-CTA scale buffers).
TC_MAX_GROUPS_PER_ROW = 81


def tc_supported(m: int, n: int, k: int, group: int) -> bool:
    return k % 128 == 0 and n % 8 == 0 and k // group <= TC_MAX_GROUPS_PER_ROW and m > 0


def prefer_tc(m: int, n: int, k: int, group: int) -> bool:
    """Whether the tensor-core path beats the projection engine for this shape.

    Measured on B200 (dense sweep over the decode shapes): the engine decodes
    each weight once per 16-token group, the tensor-core path once per 64
    tokens, so the tensor cores win from 64 tokens on every shape, from 32 on
    matrices of 16M+ weights and from 16 on the 9216-wide reduction.
    """
    if not tc_supported(m, n, k, group):
        return False
    if m >= 64:
        return True
    if m >= 32 and n * k >= 16 * 2**20:
        return True
    return m >= 16 and k >= 8192


def w4a16_dense(
    activations: torch.Tensor, packed_weights: torch.Tensor, scales: torch.Tensor
) -> torch.Tensor:
    """y[M,N] = activations[M,K] . dequant(W[N,K])^T, bf16 out (registry op w4a16_dense).

    Small token counts run on the projection engine, many tokens on the
    tcgen05 tensor-core path (``prefer_tc``); both keep the result contract.
    """
    m, n, k, group = _validate_dense(activations, packed_weights, scales)
    if prefer_tc(m, n, k, group):
        return w4a16_dense_tc(activations, packed_weights, scales)
    return w4a16_dense_engine(activations, packed_weights, scales)


def w4a16_dense_engine(
    activations: torch.Tensor, packed_weights: torch.Tensor, scales: torch.Tensor
) -> torch.Tensor:
    """w4a16_dense on the projection engine (kb_w4a16_dense), whatever the token count."""
    m, n, k, group = _validate_dense(activations, packed_weights, scales)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=activations.device)
    if m == 0:
        return out
    x = _rows_16b(activations)
    packed = _dense_contig(packed_weights)
    sc = _dense_contig(scales)
    _lib.call(
        "kb_w4a16_dense",
        _p(x), c_int64(x.stride(0)), c_int64(m), c_int64(k), _p(packed), _p(sc), c_int64(n),
        c_int64(group), _p(out), c_int64(out.stride(0)), _stream(x.device),
    )
    return out


def multi_prefers_tc(problems: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]) -> bool:
    """Whether ``w4a16_dense_multi`` runs these problems on the tensor-core path."""
    return bool(problems) and all(prefer_tc(*_validate_dense(*pr)) for pr in problems)


def w4a16_dense_multi(
    problems: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
) -> list[torch.Tensor]:
    """Several independent dense projections in one launch (one tensor-core
    launch each when ``prefer_tc`` picks that path for every problem)."""
    if len(problems) > _lib.MAX_DENSE_PROBLEMS:
        raise ValueError(f"at most {_lib.MAX_DENSE_PROBLEMS} problems per launch")
    if multi_prefers_tc(problems):
        return [w4a16_dense_tc(*pr) for pr in problems]
    arr = (_lib.DenseProblem * max(1, len(problems)))()
    outs: list[torch.Tensor] = []
    keep: list[torch.Tensor] = []
    device = None
    for i, (activations, packed_weights, scales) in enumerate(problems):
        m, n, k, group = _validate_dense(activations, packed_weights, scales)
        if device is None:
            device = activations.device
        elif activations.device != device:
            raise ValueError("all problems must share one device")
        out = torch.empty((m, n), dtype=torch.bfloat16, device=activations.device)
        outs.append(out)
        x = _rows_16b(activations) if m else activations
        packed = _dense_contig(packed_weights)
        sc = _dense_contig(scales)
        keep.extend((x, packed, sc))
        arr[i].x = x.data_ptr() if m else 0
        arr[i].x_stride = x.stride(0) if m else k
        arr[i].M = m
        arr[i].K = k
        arr[i].packed = packed.data_ptr()
        arr[i].scales = sc.data_ptr()
        arr[i].N = n
        arr[i].group = group
        arr[i].y = out.data_ptr()
        arr[i].y_stride = out.stride(0)
    if device is not None:
        _lib.call("kb_w4a16_dense_multi", arr, len(problems), _stream(device))
    return outs


def fused_qkv_w4a16(
    activations: torch.Tensor,
    q_packed: torch.Tensor,
    q_scales: torch.Tensor,
    k_packed: torch.Tensor,
    k_scales: torch.Tensor,
    v_packed: torch.Tensor,
    v_scales: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Q, K and V projections of one activation in one launch."""
    q, k, v = w4a16_dense_multi(
        [(activations, q_packed, q_scales), (activations, k_packed, k_scales),
         (activations, v_packed, v_scales)]
    )
    return q, k, v


def w4a16_dense_tc(
    activations: torch.Tensor, packed_weights: torch.Tensor, scales: torch.Tensor,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """w4a16_dense on the tcgen05 tensor-core path (many tokens); same result contract."""
    m, n, k, group = _validate_dense(activations, packed_weights, scales)
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=activations.device)
    if m == 0:
        return out
    x = _rows_16b(activations)
    packed = _dense_contig(packed_weights)
    sc = _dense_contig(scales)
    need = int(_lib.lib().kb_w4a16_dense_tc_workspace_size(m, k, n))
    ws = _workspace("dense_tc", x.device, need, (m, k, n)) if need else None
    _lib.call(
        "kb_w4a16_dense_tc",
        _p(x), c_int64(x.stride(0)), c_int64(m), c_int64(k), _p(packed), _p(sc), c_int64(n),
        c_int64(group), _p(out), c_int64(out.stride(0)), _p(ws),
        c_size_t(0 if ws is None else ws.numel()), _stream(x.device),
    )
    return out


# ---------------------------------------------------------------------------
# grouped
# ---------------------------------------------------------------------------


def _validate_grouped(
    activations: torch.Tensor,
    expert_indices: torch.Tensor,
    packed_weights: torch.Tensor,
    scales: torch.Tensor,
) -> tuple[int, int, int, int, int, int]:
    if activations.ndim != 2 or activations.dtype != torch.bfloat16:
        raise TypeError("activations must be a BF16 [tokens, reduction] matrix")
    if expert_indices.ndim != 2 or expert_indices.dtype != torch.long:
        raise TypeError("expert_indices must be an int64 [tokens, routes] matrix")
    if packed_weights.ndim != 3 or scales.ndim != 3:
        raise ValueError("grouped packed weights and scales must be rank three")
    if packed_weights.dtype != torch.uint8:
        raise TypeError("packed grouped weights must use torch.uint8 storage")
    if scales.dtype != torch.bfloat16:
        raise TypeError("grouped W4A16 scales must use torch.bfloat16 storage")
    _require_cuda(activations, "grouped W4A16 decode")
    if not (
        activations.device == expert_indices.device == packed_weights.device == scales.device
    ):
        raise ValueError("grouped W4A16 inputs must share one device")
    tokens, reduction = activations.shape
    route_tokens, routes = expert_indices.shape
    experts, output_size, packed_reduction = packed_weights.shape
    if route_tokens != tokens:
        raise ValueError("expert routing must have one row per token")
    if routes == 0 or experts == 0 or output_size == 0 or reduction == 0:
        raise ValueError("grouped W4A16 decode requires nonzero dimensions")
    if reduction % 32:
        raise ValueError("grouped W4A16 reduction width must be divisible by 32")
    if packed_reduction * 2 != reduction:
        raise ValueError("packed grouped weights have the wrong reduction width")
    if scales.shape[:2] != (experts, output_size):
        raise ValueError("grouped W4A16 scales have the wrong shape")
    group = group_size_of(reduction, scales.shape[2])
    if tokens * routes > _lib.MAX_ASSIGNMENTS:
        raise ValueError(
            f"tokens * routes = {tokens * routes} exceeds {_lib.MAX_ASSIGNMENTS} per call"
        )
    return tokens, routes, output_size, reduction, experts, group


def w4a16_grouped(
    activations: torch.Tensor,
    expert_indices: torch.Tensor,
    packed_weights: torch.Tensor,
    scales: torch.Tensor,
) -> torch.Tensor:
    """y[t,r] = x[t] . dequant(W[idx[t,r]])^T, bf16 [T,R,N] (registry op w4a16_grouped)."""
    t, r, n, k, e, group = _validate_grouped(activations, expert_indices, packed_weights, scales)
    out = torch.empty((t, r, n), dtype=torch.bfloat16, device=activations.device)
    if t == 0:
        return out
    x = _rows_16b(activations)
    idx = _dense_contig(expert_indices)
    packed = _dense_contig(packed_weights)
    sc = _dense_contig(scales)
    _lib.call(
        "kb_w4a16_grouped",
        _p(x), c_int64(x.stride(0)), c_int64(t), c_int64(k), _p(idx), c_int64(r), _p(packed),
        _p(sc), c_int64(e), c_int64(n), c_int64(group), _p(out), _stream(x.device),
    )
    return out


def w4a16_grouped_tc(
    activations: torch.Tensor,
    expert_indices: torch.Tensor,
    packed_weights: torch.Tensor,
    scales: torch.Tensor,
) -> torch.Tensor:
    """w4a16_grouped on the tcgen05 tensor-core path; same result contract."""
    t, r, n, k, e, group = _validate_grouped(activations, expert_indices, packed_weights, scales)
    out = torch.empty((t, r, n), dtype=torch.bfloat16, device=activations.device)
    if t == 0:
        return out
    x = _rows_16b(activations)
    idx = _dense_contig(expert_indices)
    packed = _dense_contig(packed_weights)
    sc = _dense_contig(scales)
    _lib.call(
        "kb_w4a16_grouped_tc",
        _p(x), c_int64(x.stride(0)), c_int64(t), c_int64(k), _p(idx), c_int64(r), _p(packed),
        _p(sc), c_int64(e), c_int64(n), c_int64(group), _p(out), _stream(x.device),
    )
    return out


def w4a16_swiglu_tc(
    activations: torch.Tensor,
    expert_indices: torch.Tensor,
    w1_packed: torch.Tensor,
    w1_scales: torch.Tensor,
    w3_packed: torch.Tensor,
    w3_scales: torch.Tensor,
) -> torch.Tensor:
    """w4a16_swiglu on the tcgen05 tensor-core path; same rounding contract."""
    dims = _validate_grouped(activations, expert_indices, w1_packed, w1_scales)
    if _validate_grouped(activations, expert_indices, w3_packed, w3_scales) != dims:
        raise ValueError("grouped W1 and W3 dimensions must match")
    if w3_packed.shape != w1_packed.shape or w3_scales.shape != w1_scales.shape:
        raise ValueError("grouped W1 and W3 shapes must match")
    t, r, n, k, e, group = dims
    out = torch.empty((t, r, n), dtype=torch.bfloat16, device=activations.device)
    if t == 0:
        return out
    x = _rows_16b(activations)
    idx = _dense_contig(expert_indices)
    p1, s1 = _dense_contig(w1_packed), _dense_contig(w1_scales)
    p3, s3 = _dense_contig(w3_packed), _dense_contig(w3_scales)
    _lib.call(
        "kb_w4a16_swiglu_tc",
        _p(x), c_int64(x.stride(0)), c_int64(t), c_int64(k), _p(idx), c_int64(r), _p(p1),
        _p(s1), _p(p3), _p(s3), c_int64(e), c_int64(n), c_int64(group), _p(out),
        _stream(x.device),
    )
    return out


def w4a16_swiglu(
    activations: torch.Tensor,
    expert_indices: torch.Tensor,
    w1_packed: torch.Tensor,
    w1_scales: torch.Tensor,
    w3_packed: torch.Tensor,
    w3_scales: torch.Tensor,
) -> torch.Tensor:
    """silu(x.W1[e]) * (x.W3[e]) with the bf16 rounding contract (registry op w4a16_swiglu)."""
    dims = _validate_grouped(activations, expert_indices, w1_packed, w1_scales)
    dims3 = _validate_grouped(activations, expert_indices, w3_packed, w3_scales)
    if dims3 != dims:
        raise ValueError("grouped W1 and W3 dimensions must match")
    if w3_packed.shape != w1_packed.shape:
        raise ValueError("grouped W1 and W3 packed shapes must match")
    if w3_scales.shape != w1_scales.shape:
        raise ValueError("grouped W1 and W3 scale shapes must match")
    t, r, n, k, e, group = dims
    out = torch.empty((t, r, n), dtype=torch.bfloat16, device=activations.device)
    if t == 0:
        return out
    x = _rows_16b(activations)
    idx = _dense_contig(expert_indices)
    p1, s1 = _dense_contig(w1_packed), _dense_contig(w1_scales)
    p3, s3 = _dense_contig(w3_packed), _dense_contig(w3_scales)
    _lib.call(
        "kb_w4a16_swiglu",
        _p(x), c_int64(x.stride(0)), c_int64(t), c_int64(k), _p(idx), c_int64(r), _p(p1),
        _p(s1), _p(p3), _p(s3), c_int64(e), c_int64(n), c_int64(group), _p(out),
        _stream(x.device),
    )
    return out


def _validate_combine(
    activated: torch.Tensor,
    expert_indices: torch.Tensor,
    combine_weights: torch.Tensor,
    w2_packed: torch.Tensor,
    w2_scales: torch.Tensor,
    weight_routes: int | None = None,
) -> tuple[int, int, int, int, int, int]:
    if activated.ndim != 3 or activated.dtype != torch.bfloat16:
        raise TypeError("activated must be a BF16 [tokens, routes, reduction] tensor")
    if expert_indices.ndim != 2 or expert_indices.dtype != torch.long:
        raise TypeError("expert_indices must be an int64 [tokens, routes] matrix")
    if combine_weights.ndim != 2 or combine_weights.dtype != torch.float32:
        raise TypeError("combine_weights must be a float32 [tokens, routes] matrix")
    if w2_packed.ndim != 3 or w2_scales.ndim != 3:
        raise ValueError("grouped W2 packed weights and scales must be rank three")
    if w2_packed.dtype != torch.uint8:
        raise TypeError("grouped W2 packed weights must use torch.uint8 storage")
    if w2_scales.dtype != torch.bfloat16:
        raise TypeError("grouped W2 scales must use torch.bfloat16 storage")
    _require_cuda(activated, "fused W2 combine")
    if not (
        activated.device
        == expert_indices.device
        == combine_weights.device
        == w2_packed.device
        == w2_scales.device
    ):
        raise ValueError("fused W2 combine inputs must share one device")
    tokens, routes, reduction = activated.shape
    experts, output_size, packed_reduction = w2_packed.shape
    if expert_indices.shape != (tokens, routes):
        raise ValueError("expert_indices must match the activated token-route shape")
    expected_w = routes if weight_routes is None else weight_routes
    if combine_weights.shape != (tokens, expected_w):
        raise ValueError("combine_weights must match the activated token-route shape")
    if routes == 0 or experts == 0 or output_size == 0 or reduction == 0:
        raise ValueError("fused W2 combine requires nonzero route and weight dimensions")
    if reduction % 32:
        raise ValueError("the grouped W2 reduction width must be divisible by 32")
    if packed_reduction * 2 != reduction:
        raise ValueError("grouped W2 packed weights have the wrong reduction width")
    if w2_scales.shape[:2] != (experts, output_size):
        raise ValueError("grouped W2 scales have the wrong shape")
    group = group_size_of(reduction, w2_scales.shape[2])
    if tokens * routes > _lib.MAX_ASSIGNMENTS:
        raise ValueError(
            f"tokens * routes = {tokens * routes} exceeds {_lib.MAX_ASSIGNMENTS} per call"
        )
    return tokens, routes, output_size, reduction, experts, group


def _down_combine(
    activated: torch.Tensor,
    expert_indices: torch.Tensor,
    combine_weights: torch.Tensor,
    w2_packed: torch.Tensor,
    w2_scales: torch.Tensor,
    dims: tuple[int, int, int, int, int, int],
) -> torch.Tensor:
    t, r, n, k, e, group = dims
    out = torch.empty((t, n), dtype=torch.bfloat16, device=activated.device)
    if t == 0:
        return out
    act = _dense_contig(activated)
    idx = _dense_contig(expert_indices)
    cw = combine_weights if combine_weights.stride(-1) == 1 else combine_weights.contiguous()
    p2, s2 = _dense_contig(w2_packed), _dense_contig(w2_scales)
    lib = _lib.lib()
    need = int(lib.kb_w4a16_w2_combine_workspace_size(t, r, n))
    ws = _workspace("w2_combine", act.device, need, (t, r, n))
    _lib.call(
        "kb_w4a16_w2_combine",
        _p(act), c_int64(t), c_int64(r), c_int64(k), _p(idx), _p(cw), c_int64(cw.stride(0)),
        _p(p2), _p(s2), c_int64(e), c_int64(n), c_int64(group), _p(out), _p(ws),
        c_size_t(ws.numel()), _stream(act.device),
    )
    return out


def fused_w2_combine(
    activated: torch.Tensor,
    expert_indices: torch.Tensor,
    combine_weights: torch.Tensor,
    w2_packed: torch.Tensor,
    w2_scales: torch.Tensor,
) -> torch.Tensor:
    """Down projection of every route plus the weighted combine, bf16 [T,N].

    The last route is the shared expert, added with weight exactly 1; its
    entry in ``combine_weights`` is ignored (moe_combine.py:209-261).
    """
    dims = _validate_combine(activated, expert_indices, combine_weights, w2_packed, w2_scales)
    return _down_combine(activated, expert_indices, combine_weights, w2_packed, w2_scales, dims)


def moe_down_combine(
    activated: torch.Tensor,
    stable_indices: torch.Tensor,
    expert_weights: torch.Tensor,
    w2_packed: torch.Tensor,
    w2_scales: torch.Tensor,
) -> torch.Tensor:
    """``fused_w2_combine`` taking the router's [T, R-1] weights directly.

    This is the form the MoE layer uses (engine/klinear/moe.py:317-334): the
    routed weights have one column per routed expert, the shared route last.
    """
    dims = _validate_combine(
        activated, stable_indices, expert_weights, w2_packed, w2_scales,
        weight_routes=activated.shape[1] - 1 if activated.ndim == 3 else None,
    )
    return _down_combine(activated, stable_indices, expert_weights, w2_packed, w2_scales, dims)


def moe_combine_routes(routes: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """bf16(sum_r float(routes[:, r]) * weights[:, r]) + routes[:, -1], bf16 [T, N].

    ``routes`` bf16 [T, R, N] holds the per-route expert outputs with the
    shared expert last; ``weights`` fp32 [T, >= R-1] the routing weights.  The
    combine half of fused_w2_combine, for outputs computed elsewhere (expert
    parallelism).
    """
    if routes.dtype != torch.bfloat16 or routes.ndim != 3:
        raise TypeError("routes must be BF16 [T, R, N]")
    if weights.dtype != torch.float32 or weights.ndim != 2:
        raise TypeError("weights must be FP32 [T, R-1]")
    t, r, n = routes.shape
    if weights.shape[0] != t or (r > 1 and weights.shape[1] < r - 1):
        raise ValueError("weights must have T rows and at least R-1 columns")
    if n % 8:
        raise ValueError("width must be a multiple of 8")
    _require_cuda(routes, "B200 combine")
    if weights.device != routes.device:
        raise ValueError("weights must be on the same CUDA device as routes")
    out = torch.empty((t, n), dtype=torch.bfloat16, device=routes.device)
    if t == 0:
        return out
    y = routes.contiguous()
    w = weights if weights.stride(1) == 1 else weights.contiguous()
    _lib.call("kb_moe_combine_routes", _p(y), c_int64(t), c_int64(r), c_int64(n), _p(w),
              c_int64(w.stride(0)), _p(out), _stream(y.device))
    return out


# ---------------------------------------------------------------------------
# expert-parallel data plane
# ---------------------------------------------------------------------------


def ep_dispatch(hidden: torch.Tensor, routed: torch.Tensor, per_rank: int, world: int,
                capacity: int, shared_id: int = -1) -> tuple[torch.Tensor, torch.Tensor]:
    """Pack each routed (token, route) pair's hidden row for its expert's rank.

    hidden bf16 [T, H]; routed int64 [T, k] global expert ids.  Returns
    (payload bf16 [world*capacity, H+8]: per slot the row, then the
    owner-local expert id as an int64 in the next four bf16 -- -1 for an
    unused slot; slots int32 [T*k]: the payload slot of each pair).
    capacity must be at least T*k.  With ``shared_id`` >= 0 the payload has T
    more rows after the slots: row world*capacity + t is hidden[t] with id
    ``shared_id`` (the rank's own rows for its shared expert, not exchanged).
    """
    if hidden.dtype != torch.bfloat16 or hidden.ndim != 2:
        raise TypeError("hidden must be BF16 [T, H]")
    if routed.dtype != torch.long or routed.ndim != 2 or routed.shape[0] != hidden.shape[0]:
        raise TypeError("routed must be int64 [T, k]")
    _require_cuda(hidden, "expert-parallel dispatch")
    if routed.device != hidden.device:
        raise ValueError("routed must be on the device of hidden")
    t, h = hidden.shape
    k = routed.shape[1]
    if capacity < t * k:
        raise ValueError("capacity must be at least tokens * top_k")
    extra = t if shared_id >= 0 else 0
    payload = torch.empty((world * capacity + extra, h + 8), dtype=torch.bfloat16,
                          device=hidden.device)
    slots = torch.empty((t * k,), dtype=torch.int32, device=hidden.device)
    if t == 0:
        payload_ids(payload[:world * capacity]).fill_(-1)
        return payload, slots
    x = _rows_16b(hidden)
    r = routed if routed.stride(1) == 1 else routed.contiguous()
    _lib.call("kb_ep_dispatch", _p(x), c_int64(x.stride(0)), c_int64(t), c_int64(h), _p(r),
              c_int64(r.stride(0)), c_int64(k), c_int64(per_rank), c_int64(world),
              c_int64(capacity), c_int64(shared_id), _p(payload), _p(slots), _stream(x.device))
    return payload, slots


def payload_ids(payload: torch.Tensor) -> torch.Tensor:
    """The int64 expert-id column of a dispatch payload, [n, 1] (a view)."""
    h = payload.shape[1] - 8
    return payload[:, h:h + 4].view(torch.long)


def ep_combine(y: torch.Tensor, slots: torch.Tensor, weights: torch.Tensor,
               shared: torch.Tensor) -> torch.Tensor:
    """bf16(sum_r float(y[slots[t,r]]) * weights[t,r]) + shared[t], bf16 [T, H]."""
    if y.dtype != torch.bfloat16 or shared.dtype != torch.bfloat16:
        raise TypeError("y and shared must be BF16")
    if weights.dtype != torch.float32 or slots.dtype != torch.int32:
        raise TypeError("weights must be FP32 and slots int32")
    _require_cuda(y, "expert-parallel combine")
    if not (slots.device == weights.device == shared.device == y.device):
        raise ValueError("combine inputs must share one device")
    t, h = shared.shape
    k = weights.shape[1]
    if slots.numel() != t * k or y.shape[1] != h:
        raise ValueError("slots must have T*k entries and y rows the width of shared")
    out = torch.empty((t, h), dtype=torch.bfloat16, device=y.device)
    if t == 0:
        return out
    yc = y.contiguous()
    sc = slots.contiguous()
    s = _rows_16b(shared)
    w = weights if weights.stride(1) == 1 else weights.contiguous()
    _lib.call("kb_ep_combine", _p(yc), _p(sc), c_int64(t), c_int64(k), c_int64(h), _p(w),
              c_int64(w.stride(0)), _p(s), c_int64(s.stride(0)), _p(out), c_int64(out.stride(0)),
              _stream(yc.device))
    return out


# ---------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------


def moe_router(
    hidden_states: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    top_k: int,
    *,
    renormalize: bool = True,
    routed_scaling_factor: float = 1.0,
    append_expert: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Sigmoid top-k routing of KLinearRouter.forward (router.py:47-85).

    Returns (indices int64 [T, top_k], weights fp32 [T, top_k]), ordered by
    (biased score desc, expert index asc).  With ``append_expert`` the indices
    are [T, top_k + 1] with that expert id as the last route, the
    shape-stable layout of engine/klinear/moe.py:23-36.
    """
    if hidden_states.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("router hidden states and weight must be BF16")
    if weight.ndim != 2:
        raise ValueError("router weight must have shape [experts, hidden]")
    _require_cuda(hidden_states, "B200 router")
    flat = hidden_states.reshape(-1, hidden_states.shape[-1])
    tokens, hidden = flat.shape
    experts = weight.shape[0]
    if weight.shape[1] != hidden:
        raise ValueError("router weight width does not match the hidden size")
    if not 0 < top_k <= experts:
        raise ValueError("top_k must be in the expert range")
    extra = 0 if append_expert is None else 1
    idx = torch.empty((tokens, top_k + extra), dtype=torch.long, device=flat.device)
    wts = torch.empty((tokens, top_k), dtype=torch.float32, device=flat.device)
    if tokens == 0:
        return idx, wts
    x = _rows_16b(flat)
    w = _dense_contig(weight)
    b = None
    if bias is not None:
        b = bias.detach()
        if b.dtype != torch.float32 or b.device != flat.device or not b.is_contiguous():
            b = b.to(device=flat.device, dtype=torch.float32).contiguous()
    lib = _lib.lib()
    need = int(lib.kb_router_workspace_size(tokens, experts))
    ws = _workspace("router", flat.device, need, (tokens, experts))
    _lib.call(
        "kb_router_topk",
        _p(x), c_int64(x.stride(0)), c_int64(tokens), c_int64(hidden), _p(w), _p(b),
        c_int64(experts), c_int64(top_k), 1 if renormalize else 0,
        c_float(float(routed_scaling_factor)), _p(idx),
        c_int64(-1 if append_expert is None else int(append_expert)), _p(wts), _p(ws),
        c_size_t(ws.numel()), _stream(flat.device),
    )
    return idx, wts


# ---------------------------------------------------------------------------
# KDA
# ---------------------------------------------------------------------------


def kda_decode_step(
    state: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    decay: torch.Tensor,
    beta: torch.Tensor,
    *,
    scale: float,
    out_bf16: torch.Tensor | None = None,
) -> torch.Tensor:
    """One KDA recurrent step; mutates ``state`` in place, returns fp32 [B,H,Dv]."""
    if state.ndim != 4:
        raise ValueError("state must have shape [batch, heads, d_k, d_v]")
    if any(t.dtype != torch.float32 for t in (state, q, k, v, decay, beta)):
        raise TypeError("KDA decode inputs must all use torch.float32")
    if not all(t.device == state.device for t in (q, k, v, decay, beta)):
        raise ValueError("KDA decode inputs must share one device")
    batch, heads, d_k, d_v = state.shape
    if batch == 0 or heads == 0 or d_k == 0 or d_v == 0:
        raise ValueError("KDA decode dimensions must be nonzero")
    if q.shape != (batch, heads, d_k):
        raise ValueError("q must have shape [batch, heads, d_k]")
    if k.shape != (batch, heads, d_k):
        raise ValueError("k must have shape [batch, heads, d_k]")
    if v.shape != (batch, heads, d_v):
        raise ValueError("v must have shape [batch, heads, d_v]")
    if decay.shape != (batch, heads, d_k):
        raise ValueError("decay must have shape [batch, heads, d_k]")
    if beta.shape != (batch, heads):
        raise ValueError("beta must have shape [batch, heads]")
    if state.device.type != "cuda":
        raise ValueError("fused KDA decode requires CUDA inputs")
    out = torch.empty((batch, heads, d_v), dtype=torch.float32, device=state.device)
    if out_bf16 is not None:
        if out_bf16.dtype != torch.bfloat16 or out_bf16.numel() != out.numel() or not (
            out_bf16.is_contiguous()
        ):
            raise ValueError("out_bf16 must be a contiguous BF16 tensor with B*H*Dv elements")
    work = state
    if state.stride(3) != 1 or state.stride(2) < d_v:
        work = state.contiguous()
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    dc, bc = decay.contiguous(), beta.contiguous()
    _lib.call(
        "kb_kda_decode_step",
        _p(work), c_int64(work.stride(0)), c_int64(work.stride(1)), c_int64(work.stride(2)),
        _p(qc), _p(kc), _p(vc), _p(dc), _p(bc), c_int64(batch), c_int64(heads), c_int64(d_k),
        c_int64(d_v), c_float(float(scale)), _p(out), _p(out_bf16), _stream(state.device),
    )
    if work is not state:
        state.copy_(work)
    return out


# ---------------------------------------------------------------------------
# codec
# ---------------------------------------------------------------------------


def kda_prepare(q_in: torch.Tensor, k_in: torch.Tensor, v_in: torch.Tensor,
                q_state: torch.Tensor, k_state: torch.Tensor, v_state: torch.Tensor,
                q_weight: torch.Tensor, k_weight: torch.Tensor, v_weight: torch.Tensor,
                raw_decay: torch.Tensor, dt_bias: torch.Tensor, a_log: torch.Tensor,
                raw_beta: torch.Tensor, *, num_heads: int, head_dim: int, eps: float = 1e-6):
    """KDA decode preparation (attention.py:192-230) in one launch: the three
    width-4 short convolutions (states [B, C, 4] updated in place), then the
    gates.  Returns fp32 (q, k, v, decay) [B, H, D] and beta [B, H]: the
    inputs of ``kda_decode_step``.  Projections, states, weights, raw_decay and
    raw_beta are bf16; dt_bias and a_log fp32 (a_log [H] or [1, 1, H, 1])."""
    batch = q_in.shape[0]
    x, weights, rd, rb, a, dt = _kda_prep_args(
        q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight, v_weight, raw_decay,
        dt_bias, a_log, raw_beta, num_heads, head_dim)
    outs = [torch.empty((batch, num_heads, head_dim), dtype=torch.float32, device=q_in.device)
            for _ in range(4)]
    beta = torch.empty((batch, num_heads), dtype=torch.float32, device=q_in.device)
    if batch == 0:
        return (*outs, beta)
    _lib.call("kb_kda_prepare", _p(x[0]), _p(x[1]), _p(x[2]), c_int64(x[0].stride(0)),
              _p(q_state), _p(k_state), _p(v_state), _p(weights[0]), _p(weights[1]),
              _p(weights[2]), _p(rd), c_int64(rd.stride(0)), _p(dt), _p(a), _p(rb),
              c_int64(rb.stride(0)), c_int64(batch), c_int64(num_heads), c_int64(head_dim),
              c_float(eps), _p(outs[0]), _p(outs[1]), _p(outs[2]), _p(outs[3]), _p(beta),
              _stream(q_in.device))
    return (*outs, beta)


def _kda_prep_args(q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight, v_weight,
                   raw_decay, dt_bias, a_log, raw_beta, num_heads, head_dim):
    """Validated, flattened preparation inputs: (q/k/v rows [B, C] sharing one
    row stride, weights [C, 4], raw_decay [B, C], raw_beta [B, H], a_log [H],
    dt_bias [C])."""
    batch = q_in.shape[0]
    c = num_heads * head_dim
    bf = (q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight, v_weight, raw_decay,
          raw_beta)
    if any(t.dtype != torch.bfloat16 for t in bf):
        raise TypeError("KDA prepare projections, states, weights and gate inputs must be BF16")
    if dt_bias.dtype != torch.float32 or a_log.dtype != torch.float32:
        raise TypeError("dt_bias and A_log must be FP32")
    _require_cuda(q_in, "KDA prepare")
    if any(t.device != q_in.device for t in bf + (dt_bias, a_log)):
        raise ValueError("KDA prepare tensors must share one device")
    x = [t.reshape(batch, c) for t in (q_in, k_in, v_in)]
    if any(t.stride(1) != 1 or t.stride(0) != x[0].stride(0) for t in x):
        x = [t.contiguous() for t in x]
    states = (q_state, k_state, v_state)
    if any(tuple(st.shape) != (batch, c, 4) or not st.is_contiguous() for st in states):
        raise ValueError("each short convolution state must be a contiguous [batch, channels, 4]")
    weights = [w.reshape(c, 4).contiguous() for w in (q_weight, k_weight, v_weight)]
    rd = raw_decay.reshape(batch, c).contiguous()
    rb = raw_beta.reshape(batch, num_heads).contiguous()
    a = a_log.reshape(num_heads).contiguous()
    dt = dt_bias.reshape(c).contiguous()
    return x, weights, rd, rb, a, dt


def kda_prepare_step_supported(state: torch.Tensor, head_dim: int) -> bool:
    """Whether ``kda_prepare_step`` takes this state: head_dim 128, fp32 CUDA
    state [B, H, 128, 128] with contiguous 16-byte aligned rows."""
    return (head_dim == 128 and state.is_cuda and state.dtype == torch.float32
            and state.ndim == 4 and state.shape[2] == 128 and state.shape[3] == 128
            and state.stride(3) == 1 and state.stride(2) == 128 and state.stride(1) % 4 == 0
            and state.stride(0) % 4 == 0 and state.data_ptr() % 16 == 0)


def kda_prepare_step(state: torch.Tensor, q_in: torch.Tensor, k_in: torch.Tensor,
                     v_in: torch.Tensor, q_state: torch.Tensor, k_state: torch.Tensor,
                     v_state: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                     v_weight: torch.Tensor, raw_decay: torch.Tensor, dt_bias: torch.Tensor,
                     a_log: torch.Tensor, raw_beta: torch.Tensor, *, num_heads: int,
                     head_dim: int, scale: float, eps: float = 1e-6,
                     out_bf16: torch.Tensor | None = None) -> torch.Tensor:
    """``kda_prepare`` then ``kda_decode_step`` in one launch (same results):
    the convolution states and the KDA state are updated in place; returns
    the fp32 output [B, H, D] (and fills ``out_bf16`` if given)."""
    if not kda_prepare_step_supported(state, head_dim):
        raise ValueError("kda_prepare_step needs head_dim 128 and a state with contiguous rows")
    batch = q_in.shape[0]
    if tuple(state.shape[:2]) != (batch, num_heads):
        raise ValueError("state must have shape [batch, heads, 128, 128]")
    x, weights, rd, rb, a, dt = _kda_prep_args(
        q_in, k_in, v_in, q_state, k_state, v_state, q_weight, k_weight, v_weight, raw_decay,
        dt_bias, a_log, raw_beta, num_heads, head_dim)
    if state.device != q_in.device:
        raise ValueError("the KDA state must be on the device of the inputs")
    out = torch.empty((batch, num_heads, head_dim), dtype=torch.float32, device=q_in.device)
    if out_bf16 is not None and (out_bf16.dtype != torch.bfloat16 or
                                 out_bf16.numel() != out.numel() or
                                 not out_bf16.is_contiguous()):
        raise ValueError("out_bf16 must be a contiguous BF16 tensor with B*H*D elements")
    if batch == 0:
        return out
    _lib.call("kb_kda_prepare_step", _p(x[0]), _p(x[1]), _p(x[2]), c_int64(x[0].stride(0)),
              _p(q_state), _p(k_state), _p(v_state), _p(weights[0]), _p(weights[1]),
              _p(weights[2]), _p(rd), c_int64(rd.stride(0)), _p(dt), _p(a), _p(rb),
              c_int64(rb.stride(0)), c_float(eps), _p(state), c_int64(state.stride(0)),
              c_int64(state.stride(1)), c_int64(state.stride(2)), c_int64(batch),
              c_int64(num_heads), c_int64(head_dim), c_float(float(scale)), _p(out),
              _p(out_bf16), _stream(q_in.device))
    return out


def quantise(weight: torch.Tensor, group_size: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """On-device quantise of a bf16 [N,K] matrix -> (packed uint8 [N,K/2], bf16 scales).

    Same arithmetic as engine/quant/w4a16.py:68-105 with the group size as a
    parameter.  Raises ValueError for non-finite weights (this check reads a
    flag back, so it synchronizes the stream).
    """
    if weight.ndim != 2:
        raise ValueError("weight must have shape [out_features, in_features]")
    if weight.dtype != torch.bfloat16:
        raise TypeError("weight must have dtype torch.bfloat16")
    _require_cuda(weight, "on-device quantise")
    n, k = weight.shape
    if k % group_size:
        raise ValueError(f"the reduction axis must be divisible by group size {group_size}")
    w = _rows_16b(weight)
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=weight.device)
    scales = torch.empty((n, k // group_size), dtype=torch.bfloat16, device=weight.device)
    flag = torch.zeros((1,), dtype=torch.int32, device=weight.device)
    _lib.call(
        "kb_w4a16_quantise",
        _p(w), c_int64(w.stride(0)), c_int64(n), c_int64(k), c_int64(group_size), _p(packed),
        _p(scales), _p(flag), _stream(weight.device),
    )
    if int(flag.item()):
        raise ValueError("weight must contain only finite values")
    return packed, scales
