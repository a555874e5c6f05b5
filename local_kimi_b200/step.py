"""Decode-step executor: a program of hot-path operations run in one launch.

``StepProgram`` wraps the ``kb_step_*`` C ABI (csrc/kb_step.cu).  Operations
are added with the device tensors they read and write (bound once, like the
static buffers of a captured CUDA graph) and the earlier operations they
depend on; ``launch()`` runs the whole program as one persistent kernel with
one CTA per SM.  It computes what the per-operation entry points of ``ops``
compute for the same inputs, up to fp32 summation order.

The reference runs one decode step as a captured graph of registry calls
(engine/klinear/generate.py:226-276); ``HotPathDecoder.build_program``
(local_kimi_b200/decode.py) builds the equivalent program for the hot path.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p

import torch

from . import _lib
from .ops import _p, _stream, group_size_of

MAX_TOKENS = 8
MAX_DEPS = 4


def _deps(deps) -> tuple[object, int]:
    deps = [int(d) for d in (deps or []) if d is not None]
    if len(deps) > MAX_DEPS:
        raise ValueError(f"at most {MAX_DEPS} dependencies per operation")
    if not deps:
        return None, 0
    arr = (c_int * len(deps))(*deps)
    return arr, len(deps)


def _group(packed: torch.Tensor, scales: torch.Tensor) -> int:
    return group_size_of(int(packed.shape[-1]) * 2, int(scales.shape[-1]))


def _require(t: torch.Tensor, dtype: torch.dtype, what: str) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{what} must be {dtype}")
    if t.device.type != "cuda":
        raise ValueError(f"{what} must be a CUDA tensor")


class StepProgram:
    """A finalized-once, launch-many program of hot-path operations."""

    def __init__(self, tokens: int) -> None:
        if not 1 <= tokens <= MAX_TOKENS:
            raise ValueError(f"the step executor supports 1 to {MAX_TOKENS} tokens")
        self.tokens = tokens
        self._keep: list[object] = []
        self.n_ops = 0
        handle = c_void_p()
        _lib.call("kb_step_create", c_int64(tokens), ctypes.byref(handle))
        self._h = handle
        self.finalized = False

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().kb_step_destroy(h)
            except Exception:
                pass
            self._h = None

    def _out(self) -> tuple[c_int, object]:
        o = c_int(-1)
        return o, ctypes.byref(o)

    def dense(self, problems, deps=None) -> int:
        """problems: up to three (x [T, K] bf16, packed, scales, y [T, N] bf16)."""
        arr = (_lib.DenseProblem * len(problems))()
        for i, (x, packed, scales, y) in enumerate(problems):
            _require(x, torch.bfloat16, "activations")
            _require(y, torch.bfloat16, "output")
            if x.stride(-1) != 1 or y.stride(-1) != 1:
                raise ValueError("activations and outputs need unit stride along K and N")
            n, k = int(packed.shape[0]), int(x.shape[-1])
            arr[i] = _lib.DenseProblem(_p(x), x.stride(0), x.shape[0], k, _p(packed),
                                       _p(scales), n, _group(packed, scales), _p(y),
                                       y.stride(0))
            self._keep += [x, packed, scales, y]
        d, nd = _deps(deps)
        o, ref = self._out()
        _lib.call("kb_step_add_dense", self._h, arr, len(problems), d, nd, ref)
        return o.value

    def swiglu(self, x, w1, w3, y, deps=None) -> int:
        """Dense gate/up pair: y = bf16(silu(bf16 x.w1^T)) * bf16(x.w3^T)."""
        (w1p, w1s), (w3p, w3s) = w1, w3
        _require(x, torch.bfloat16, "activations")
        _require(y, torch.bfloat16, "output")
        n, k = int(w1p.shape[-2]), int(x.shape[-1])
        self._keep += [x, w1p, w1s, w3p, w3s, y]
        d, nd = _deps(deps)
        o, ref = self._out()
        _lib.call("kb_step_add_swiglu", self._h, _p(x), c_int64(x.stride(0)), c_int64(k),
                  _p(w1p), _p(w1s), _p(w3p), _p(w3s), c_int64(n),
                  c_int64(_group(w1p, w1s)), _p(y), c_int64(y.stride(0)), d, nd, ref)
        return o.value

    def router(self, hidden, weight, bias, top_k, scaling, scratch, idx_out, w_out,
               renormalize=True, deps=None) -> int:
        """Router logits into ``scratch`` (16 * T * E bytes, contiguous, owned by
        the program: per launch parity and (token, expert) a 64-bit word with
        the choice key and the sigmoid score; one buffer per router, see
        ``router_scratch``); the selection runs in the expert block that uses
        this router and writes idx_out int64 [T, top_k+1] (shared id appended)
        and w_out."""
        _require(hidden, torch.bfloat16, "hidden states")
        _require(weight, torch.bfloat16, "router weight")
        if scratch.device.type != "cuda" or not scratch.is_contiguous():
            raise ValueError("router scratch must be a contiguous CUDA tensor")
        need = 16 * hidden.shape[0] * weight.shape[0]
        if scratch.numel() * scratch.element_size() < need:
            raise ValueError(f"router scratch needs {need} bytes")
        logits = scratch
        b = None
        if bias is not None:
            b = bias.to(torch.float32).contiguous()
        self._keep += [hidden, weight, b, logits, idx_out, w_out]
        d, nd = _deps(deps)
        o, ref = self._out()
        _lib.call("kb_step_add_router", self._h, _p(hidden), c_int64(hidden.stride(0)),
                  c_int64(hidden.shape[-1]), _p(weight), _p(b), c_int64(weight.shape[0]),
                  c_int64(top_k), 1 if renormalize else 0, c_float(float(scaling)), _p(logits),
                  _p(idx_out), _p(w_out), d, nd, ref)
        return o.value

    @staticmethod
    def router_scratch(tokens: int, experts: int, device=None) -> torch.Tensor:
        """A router scratch buffer for ``router``: [2, tokens, experts] int64."""
        return torch.empty((2, tokens, experts), dtype=torch.int64, device=device or "cuda")

    def moe(self, router_op, hidden, layer, activated, routed_out, out, deps=None) -> int:
        """Expert block of one MoE layer (MoELayerWeights); returns the index of
        its down/combine operation."""
        m = layer
        self._keep += [hidden, m.w1_packed, m.w1_scales, m.w3_packed, m.w3_scales, m.w2_packed,
                       m.w2_scales, activated, routed_out, out]
        d, nd = _deps(deps)
        o, ref = self._out()
        _lib.call("kb_step_add_moe", self._h, c_int(router_op), _p(hidden),
                  c_int64(hidden.stride(0)), c_int64(hidden.shape[-1]), _p(m.w1_packed),
                  _p(m.w1_scales), _p(m.w3_packed), _p(m.w3_scales), _p(m.w2_packed),
                  _p(m.w2_scales), c_int64(m.intermediate),
                  c_int64(_group(m.w1_packed, m.w1_scales)), _p(activated),
                  _p(routed_out), _p(out), d, nd, ref)
        return o.value

    def kda(self, state, q, k, v, decay, beta, scale, out=None, out_bf16=None, deps=None) -> int:
        B, H, Dk, Dv = state.shape
        self._keep += [state, q, k, v, decay, beta, out, out_bf16]
        d, nd = _deps(deps)
        o, ref = self._out()
        _lib.call("kb_step_add_kda", self._h, _p(state), c_int64(state.stride(0)),
                  c_int64(state.stride(1)), c_int64(state.stride(2)), _p(q), _p(k), _p(v),
                  _p(decay), _p(beta), c_int64(B), c_int64(H), c_int64(Dk), c_int64(Dv),
                  c_float(float(scale)), _p(out), _p(out_bf16), d, nd, ref)
        return o.value

    def finalize(self) -> "StepProgram":
        _lib.call("kb_step_finalize", self._h)
        n, st, sb, sm = c_int(0), c_int(0), c_int(0), c_size_t(0)
        _lib.call("kb_step_info", self._h, ctypes.byref(n), ctypes.byref(st), ctypes.byref(sb),
                  ctypes.byref(sm))
        self.n_ops, self.stages, self.stage_bytes, self.smem_bytes = (
            n.value, st.value, sb.value, sm.value)
        self.finalized = True
        return self

    def enable_trace(self) -> torch.Tensor:
        """Record a timeline on every launch; returns the int64 buffer
        [grid, n_ops, 8] (consumers start, inputs ready, routing built, end,
        producer done issuing, reducers done, shared-expert items done, spare;
        %globaltimer ns)."""
        n = int(_lib.lib().kb_step_trace_entries(self._h))
        buf = torch.zeros(n, dtype=torch.int64, device="cuda")
        _lib.call("kb_step_set_trace", self._h, _p(buf), c_int64(n))
        self._trace = buf
        return buf.view(-1, self.n_ops, 8)

    def launch(self, device: torch.device | None = None) -> None:
        """Run the whole program on the current stream."""
        dev = device or torch.device("cuda", torch.cuda.current_device())
        _lib.call("kb_step_launch", self._h, _stream(dev))
