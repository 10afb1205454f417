"""Installing and undoing an instance-level ``forward`` override.

A module may already carry a ``forward`` of its own on the instance (a model accelerator
such as ``dattri_llm_b200.models.mamba2.accelerate_mamba2`` installs one); undoing a capture
override must put that one back rather than fall through to the class's method.
"""

from __future__ import annotations

from collections.abc import Callable

from torch import nn


def swap_forward(module: nn.Module, forward: Callable) -> Callable[[], None]:
    """Set ``module.forward`` to *forward*; returns the undo, which restores the instance's
    previous ``forward`` attribute or removes the override when there was none."""
    previous = vars(module).get("forward")
    module.forward = forward

    def undo() -> None:
        if previous is None:
            vars(module).pop("forward", None)
        else:
            module.forward = previous

    return undo
