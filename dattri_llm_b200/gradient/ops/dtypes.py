"""Compute-dtype policy of the gradient operations.

``"auto"`` (default) computes in the promoted dtype of the floating operands --
bf16 captures stay bf16 end to end, so the tensor-core kernels see bf16 -- while
covariance / eigendecomposition paths ask for an fp32 ``minimum``.  An explicit
dtype forces every op.  Parity: reference ``dattri_llm/gradient/ops/dtypes.py``.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager

import torch

_POLICY: str | torch.dtype = "auto"
_NAMED = {
    "auto": "auto", "float32": torch.float32, "fp32": torch.float32, "float64": torch.float64,
    "bfloat16": torch.bfloat16, "bf16": torch.bfloat16, "float16": torch.float16,
    "fp16": torch.float16,
}


def _as_policy(policy: str | torch.dtype) -> str | torch.dtype:
    if isinstance(policy, torch.dtype):
        return policy
    if isinstance(policy, str) and policy in _NAMED:
        return _NAMED[policy]
    raise ValueError(
        f"compute dtype policy must be 'auto', a torch.dtype, or one of "
        f"{sorted(k for k in _NAMED if k != 'auto')}; got {policy!r}",
    )


def set_compute_dtype(policy: str | torch.dtype) -> str | torch.dtype:
    """Set the process-wide compute dtype; returns the policy it replaces."""
    global _POLICY  # noqa: PLW0603
    previous, _POLICY = _POLICY, _as_policy(policy)
    return previous


def get_compute_dtype() -> str | torch.dtype:
    """The active policy -- ``"auto"`` or a :class:`torch.dtype`."""
    return _POLICY


@contextmanager
def compute_dtype(policy: str | torch.dtype) -> Iterator[None]:
    """Scope a compute-dtype policy to a block."""
    previous = set_compute_dtype(policy)
    try:
        yield
    finally:
        set_compute_dtype(previous)


def resolve(*tensors: torch.Tensor | None, minimum: torch.dtype | None = None) -> torch.dtype:
    """The dtype an op on *tensors* computes in under the active policy."""
    if _POLICY != "auto":
        dtype = _POLICY
    else:
        dtype = None
        for t in tensors:
            if t is None or not t.is_floating_point():
                continue
            dtype = t.dtype if dtype is None else torch.promote_types(dtype, t.dtype)
        if dtype is None:
            dtype = torch.float32
    if minimum is not None:
        dtype = torch.promote_types(dtype, minimum)
    return dtype


def align(*tensors: torch.Tensor | None, minimum: torch.dtype | None = None) -> tuple:
    """Cast the floating operands to the resolved dtype (integers pass through)."""
    dtype = resolve(*tensors, minimum=minimum)
    return tuple(
        t if (t is None or not t.is_floating_point() or t.dtype == dtype) else t.to(dtype)
        for t in tensors
    )


def as_float(*tensors: torch.Tensor | None, minimum: torch.dtype | None = None) -> tuple:
    """Like :func:`align`, but integer operands are converted too."""
    dtype = resolve(*tensors, minimum=minimum)
    return tuple(t if (t is None or t.dtype == dtype) else t.to(dtype) for t in tensors)
