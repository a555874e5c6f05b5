"""Named kernel variants per operation, with the reference registry's API.

Same public surface and selection rules as engine/kernels/registry.py:17-204,
so callers written against the reference registry work unchanged:

  register(op, variant, reference=, requires_cuda=, description=)  decorator
  reference_of(op) / variants(op) / set_default(op, variant) / default_of(op)
  resolve(op) / use(op, variant) / clear_override(op) / using(op, variant)
  active(op)

Selection order: programmatic override (use/using), then the KIMI_KERNELS
environment variable (``op=variant,op=variant``; unknown ops are ignored, an
unknown variant of a known op raises ValueError naming the available ones),
then the shipped default (set_default), then the op's reference variant.
``resolve`` refuses a ``requires_cuda`` variant when CUDA is unavailable
instead of falling back to something else.
"""

from __future__ import annotations

import os
from collections.abc import Callable, Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from typing import TypeVar

import torch

KernelFunction = Callable[..., object]
F = TypeVar("F", bound=KernelFunction)

ENV_VAR = "KIMI_KERNELS"


@dataclass(frozen=True)
class KernelVariant:
    name: str
    fn: KernelFunction
    is_reference: bool
    requires_cuda: bool
    description: str


class Registry:
    """One registry instance; the module-level functions use ``DEFAULT``."""

    def __init__(self) -> None:
        self._ops: dict[str, dict[str, KernelVariant]] = {}
        self._overrides: dict[str, str] = {}
        self._defaults: dict[str, str] = {}

    # -- registration -------------------------------------------------------
    def register(
        self,
        op: str,
        variant: str,
        *,
        reference: bool = False,
        requires_cuda: bool = False,
        description: str = "",
    ) -> Callable[[F], F]:
        def decorator(fn: F) -> F:
            table = self._ops.setdefault(op, {})
            if reference:
                for existing in table.values():
                    if existing.is_reference:
                        raise ValueError(
                            f"operation {op!r} already has reference variant "
                            f"{existing.name!r}; cannot register second reference "
                            f"variant {variant!r}"
                        )
            if variant in table:
                raise ValueError(f"variant {variant!r} is already registered for operation {op!r}")
            table[variant] = KernelVariant(variant, fn, reference, requires_cuda, description)
            return fn

        return decorator

    # -- queries --------------------------------------------------------------
    def reference_of(self, op: str) -> KernelVariant:
        for item in self._ops.get(op, {}).values():
            if item.is_reference:
                return item
        raise KeyError(f"operation {op!r} has no reference kernel variant")

    def variants(self, op: str) -> tuple[str, ...]:
        table = self._ops.get(op, {})
        refs = sorted(v.name for v in table.values() if v.is_reference)
        rest = sorted(v.name for v in table.values() if not v.is_reference)
        return tuple(refs + rest)

    def operations(self) -> tuple[str, ...]:
        return tuple(sorted(self._ops))

    def describe(self, op: str, variant: str) -> KernelVariant:
        return self._lookup(op, variant)

    def _lookup(self, op: str, variant: str) -> KernelVariant:
        table = self._ops.get(op)
        if table is None:
            raise KeyError(f"operation {op!r} has no registered kernel variants")
        if variant not in table:
            names = ", ".join(self.variants(op)) or "none"
            raise ValueError(
                f"unknown variant {variant!r} for operation {op!r}; available variants: {names}"
            )
        return table[variant]

    def _from_environment(self) -> dict[str, str]:
        chosen: dict[str, str] = {}
        for raw in os.getenv(ENV_VAR, "").split(","):
            entry = raw.strip()
            if not entry:
                continue
            op, sep, variant = (part.strip() for part in entry.partition("="))
            if not sep or not op:
                raise ValueError(f"invalid {ENV_VAR} entry {entry!r}; expected op=variant")
            if op not in self._ops:
                continue
            if not variant:
                names = ", ".join(self.variants(op)) or "none"
                raise ValueError(
                    f"unknown variant {variant!r} for operation {op!r}; available variants: {names}"
                )
            self._lookup(op, variant)
            chosen[op] = variant
        return chosen

    def _selected(self, op: str) -> KernelVariant:
        if op not in self._ops:
            raise KeyError(f"operation {op!r} has no registered kernel variants")
        if op in self._overrides:
            return self._lookup(op, self._overrides[op])
        env = self._from_environment().get(op)
        if env is not None:
            return self._lookup(op, env)
        if op in self._defaults:
            return self._lookup(op, self._defaults[op])
        return self.reference_of(op)

    # -- selection ------------------------------------------------------------
    def set_default(self, op: str, variant: str) -> None:
        self._lookup(op, variant)
        self._defaults[op] = variant

    def default_of(self, op: str) -> str:
        if op in self._defaults:
            return self._defaults[op]
        return self.reference_of(op).name

    def resolve(self, op: str) -> KernelFunction:
        chosen = self._selected(op)
        if chosen.requires_cuda and not torch.cuda.is_available():
            raise RuntimeError(
                f"kernel variant {chosen.name!r} for operation {op!r} requires CUDA, "
                "but torch.cuda.is_available() is False"
            )
        return chosen.fn

    def use(self, op: str, variant: str) -> None:
        self._lookup(op, variant)
        self._overrides[op] = variant

    def clear_override(self, op: str) -> None:
        self._overrides.pop(op, None)

    @contextmanager
    def using(self, op: str, variant: str) -> Iterator[None]:
        had = op in self._overrides
        previous = self._overrides.get(op)
        self.use(op, variant)
        try:
            yield
        finally:
            if had:
                self._overrides[op] = previous  # type: ignore[assignment]
            else:
                self._overrides.pop(op, None)

    def active(self, op: str) -> str:
        return self._selected(op).name


DEFAULT = Registry()

register = DEFAULT.register
reference_of = DEFAULT.reference_of
variants = DEFAULT.variants
operations = DEFAULT.operations
set_default = DEFAULT.set_default
default_of = DEFAULT.default_of
resolve = DEFAULT.resolve
use = DEFAULT.use
clear_override = DEFAULT.clear_override
using = DEFAULT.using
active = DEFAULT.active
