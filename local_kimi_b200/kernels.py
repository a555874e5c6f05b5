"""Operation names, variant registration and the drop-in installer.

Importing this module registers the ``b200`` variant of every hot-path
operation in this package's registry (``local_kimi_b200.registry``) and makes
it the shipped default.  ``install()`` does the same inside the reference's
own registry (``engine.kernels.registry``), so that ``engine/klinear`` and
``engine/serve`` resolve the B200 kernels without any change to their code:

  * ``w4a16_dense``, ``w4a16_grouped``, ``w4a16_swiglu``: ``b200`` variants are
    registered next to the reference ones and set as the shipped default
    (engine/kernels/__init__.py:21-23, 26-218).  Callers resolve once and cache
    (engine/klinear/moe.py:269-270, engine/klinear/quantized.py:170-179), so
    install before the model prepares its banks.
  * ``kda_decode_step`` is imported by module path inside
    KDAAttention._step_kernel (engine/klinear/attention.py:153-165); the
    installer rebinds ``engine.kernels.kda_step.kda_decode_step``.
  * ``moe_combine`` and ``w4a16_qkv`` are unwired in the reference; they become
    registry ops whose reference variants are the reference's own
    ``fused_w2_combine_reference`` / ``fused_qkv_w4a16_reference`` and whose
    shipped default is ``b200``.

Variant selection after install still honours KIMI_KERNELS and
``registry.use``, e.g. ``KIMI_KERNELS=w4a16_dense=triton_gemv``.
"""

from __future__ import annotations

from types import ModuleType

from . import ops
from . import registry as _registry

VARIANT = "b200"

W4A16_DENSE = "w4a16_dense"
W4A16_GROUPED = "w4a16_grouped"
W4A16_SWIGLU = "w4a16_swiglu"
MOE_COMBINE = "moe_combine"
W4A16_QKV = "w4a16_qkv"
KDA_STEP = "kda_step"
MOE_ROUTER = "moe_router"

_DESCRIPTIONS = {
    W4A16_DENSE: "sm_100a W4A16 projection: HBM-streamed INT4 codes, bf16x2 decode in "
    "registers, tensor-core accumulate, deterministic split of the reduction.",
    W4A16_GROUPED: "sm_100a expert-grouped W4A16 projection; assignments that share an "
    "expert read its weights once.",
    W4A16_SWIGLU: "sm_100a fused gate/up projections + SwiGLU with the bf16 rounding "
    "contract of F.silu(gate) * up.",
    MOE_COMBINE: "sm_100a fused down projection + routing-weighted combine (last route = "
    "shared expert, weight 1).",
    W4A16_QKV: "sm_100a Q/K/V projections of one activation in one launch.",
    KDA_STEP: "sm_100a KDA decode step, state read and written once, in place.",
    MOE_ROUTER: "sm_100a sigmoid router: fp32 logits, top-k by (score desc, index asc), "
    "renormalised and scaled weights.",
}

_OPS = {
    W4A16_DENSE: ops.w4a16_dense,
    W4A16_GROUPED: ops.w4a16_grouped,
    W4A16_SWIGLU: ops.w4a16_swiglu,
    MOE_COMBINE: ops.fused_w2_combine,
    W4A16_QKV: ops.fused_qkv_w4a16,
    KDA_STEP: ops.kda_decode_step,
    MOE_ROUTER: ops.moe_router,
}


def _register_local() -> None:
    for op, fn in _OPS.items():
        if VARIANT not in _registry.variants(op):
            _registry.register(op, VARIANT, requires_cuda=True, description=_DESCRIPTIONS[op])(fn)
        _registry.set_default(op, VARIANT)


_register_local()


def install(
    reference_registry: ModuleType | None = None,
    *,
    kda_module: ModuleType | None = None,
    set_defaults: bool = True,
) -> ModuleType:
    """Register the B200 variants inside the reference's kernel registry.

    ``reference_registry`` defaults to ``engine.kernels.registry`` (importing
    ``engine.kernels`` first so its own variants exist).  Returns the registry
    module.  Safe to call more than once.
    """
    if reference_registry is None:
        import engine.kernels  # noqa: F401  (registers the reference variants)
        from engine.kernels import registry as reference_registry  # type: ignore[no-redef]

    reg = reference_registry
    for op in (W4A16_DENSE, W4A16_GROUPED, W4A16_SWIGLU):
        if VARIANT not in reg.variants(op):
            reg.register(op, VARIANT, requires_cuda=True, description=_DESCRIPTIONS[op])(_OPS[op])
        if set_defaults:
            reg.set_default(op, VARIANT)

    # Ops the reference ships but never registered: give them a registry entry
    # whose reference variant is the reference's own implementation.
    try:
        from engine.kernels import moe_combine as _mc  # type: ignore[import-not-found]

        if MOE_COMBINE not in _registry_ops(reg):
            reg.register(MOE_COMBINE, "reference", reference=True,
                         description="reference torch sequence")(_mc.fused_w2_combine_reference)
        if VARIANT not in reg.variants(MOE_COMBINE):
            reg.register(MOE_COMBINE, VARIANT, requires_cuda=True,
                         description=_DESCRIPTIONS[MOE_COMBINE])(_OPS[MOE_COMBINE])
        if set_defaults:
            reg.set_default(MOE_COMBINE, VARIANT)
    except ImportError:
        pass
    try:
        from engine.kernels import w4a16_fused_qkv as _qkv  # type: ignore[import-not-found]

        if W4A16_QKV not in _registry_ops(reg):
            reg.register(W4A16_QKV, "reference", reference=True, requires_cuda=True,
                         description="three dense calls")(_qkv.fused_qkv_w4a16_reference)
        if VARIANT not in reg.variants(W4A16_QKV):
            reg.register(W4A16_QKV, VARIANT, requires_cuda=True,
                         description=_DESCRIPTIONS[W4A16_QKV])(_OPS[W4A16_QKV])
        if set_defaults:
            reg.set_default(W4A16_QKV, VARIANT)
    except ImportError:
        pass

    if kda_module is None:
        try:
            import engine.kernels.kda_step as kda_module  # type: ignore[no-redef]
        except ImportError:
            kda_module = None
    if kda_module is not None:
        if not hasattr(kda_module, "_reference_kda_decode_step"):
            kda_module._reference_kda_decode_step = getattr(kda_module, "kda_decode_step", None)
        kda_module.kda_decode_step = ops.kda_decode_step
    return reg


def _registry_ops(reg: ModuleType) -> set[str]:
    table = getattr(reg, "_REGISTRY", None)
    if isinstance(table, dict):
        return set(table)
    names = set()
    for op in (MOE_COMBINE, W4A16_QKV):
        try:
            if reg.variants(op):
                names.add(op)
        except KeyError:
            pass
    return names
