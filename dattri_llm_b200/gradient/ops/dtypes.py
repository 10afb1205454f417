"""Compute-dtype policy of the gradient operations.

One process-wide setting decides the dtype that dots, grams, projections and
materializations compute in:

* ``"auto"`` (the default): the promotion of the floating operands' dtypes, so bf16
  captures stay bf16 end to end and reach the tensor-core kernels as bf16, and mixed
  operands meet in the narrowest dtype that holds both;
* an explicit floating dtype (or one of its names, e.g. ``"bf16"``): every op computes
  in it.

Ops that need more range (covariances, eigendecompositions) pass ``minimum=`` and get
at least that dtype under either setting.  Integer operands (embedding token ids) never
take part in the promotion.  The setting is global rather than per thread because the
capture hooks run on autograd's worker threads, which must see the caller's choice.
Public names as in the reference's ``dattri_llm/gradient/ops/dtypes.py``.
"""

from __future__ import annotations

import functools
import threading
from collections.abc import Iterator
from contextlib import contextmanager

import torch

_FLOATING = (torch.float16, torch.bfloat16, torch.float32, torch.float64)
_ALIASES = {"fp16": torch.float16, "half": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32,
            "float": torch.float32, "fp64": torch.float64, "double": torch.float64}


class _Setting:
    """The active policy; writes go through a lock so that concurrent scopes stay consistent."""

    def __init__(self) -> None:
        self.policy: str | torch.dtype = "auto"
        self.lock = threading.Lock()

    def swap(self, policy: str | torch.dtype) -> str | torch.dtype:
        with self.lock:
            old, self.policy = self.policy, policy
        return old


_SETTING = _Setting()


def _parse(policy: str | torch.dtype) -> str | torch.dtype:
    if isinstance(policy, torch.dtype) or policy == "auto":
        return policy
    if isinstance(policy, str):
        dtype = _ALIASES.get(policy)
        if dtype is None:
            dtype = getattr(torch, policy, None)
        if dtype in _FLOATING:
            return dtype
    names = sorted({*_ALIASES, *(str(d).removeprefix("torch.") for d in _FLOATING)})
    raise ValueError(f"unknown compute dtype policy {policy!r}: expected 'auto', a torch.dtype or one of {names}")


def set_compute_dtype(policy: str | torch.dtype) -> str | torch.dtype:
    """Install *policy* for the whole process and hand back the one it replaces."""
    return _SETTING.swap(_parse(policy))


def get_compute_dtype() -> str | torch.dtype:
    """``"auto"`` or the forced :class:`torch.dtype`."""
    return _SETTING.policy


@contextmanager
def compute_dtype(policy: str | torch.dtype) -> Iterator[None]:
    """Run a block under *policy*, restoring the previous setting afterwards."""
    restore = set_compute_dtype(policy)
    try:
        yield
    finally:
        _SETTING.swap(restore)


def resolve(*tensors: torch.Tensor | None, minimum: torch.dtype | None = None) -> torch.dtype:
    """The dtype that an op on *tensors* computes in under the active policy."""
    policy = _SETTING.policy
    if policy == "auto":
        floats = [t.dtype for t in tensors if t is not None and t.is_floating_point()]
        chosen = functools.reduce(torch.promote_types, floats) if floats else torch.float32
    else:
        chosen = policy
    return chosen if minimum is None else torch.promote_types(chosen, minimum)


def align(*tensors: torch.Tensor | None, minimum: torch.dtype | None = None) -> tuple:
    """The floating operands cast to :func:`resolve`'s dtype; integers and ``None`` unchanged."""
    target = resolve(*tensors, minimum=minimum)
    return tuple(t.to(target) if t is not None and t.is_floating_point() and t.dtype != target else t
                 for t in tensors)


def as_float(*tensors: torch.Tensor | None, minimum: torch.dtype | None = None) -> tuple:
    """Every operand, integer ones included, cast to :func:`resolve`'s dtype (``None`` kept)."""
    target = resolve(*tensors, minimum=minimum)
    return tuple(t.to(target) if t is not None and t.dtype != target else t for t in tensors)
