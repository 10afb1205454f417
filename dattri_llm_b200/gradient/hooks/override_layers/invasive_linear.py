"""``invasive_linear_io``: capture a linear layer without computing its weight gradient.

While collecting, the layer's forward is routed through
:class:`InvasiveLinearFunction`, whose backward returns only the input gradient:
the hooks still see the input activation and the output gradient, the
``dW = g^T a`` GEMM (the largest GEMM of a linear layer's backward) never runs,
and ``weight.grad`` is left untouched.  Parity: reference
``dattri_llm/gradient/hooks/override_layers/invasive_linear.py:35-163``.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import nn

from dattri_llm_b200.gradient.ops import canonical_class_name
from dattri_llm_b200.gradient.hooks.override_layers._forward_slot import swap_forward


def is_invasive_capable(module: nn.Module) -> bool:
    """Only ``nn.Linear`` layers can be captured invasively."""
    return isinstance(module, nn.Linear)


class InvasiveLinearFunction(torch.autograd.Function):
    """``y = x W^T + b`` whose backward produces only ``dx`` (no ``dW``, no ``db``)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        ctx.save_for_backward(weight)
        return nn.functional.linear(x, weight, bias)

    @staticmethod
    def backward(ctx, grad_out: torch.Tensor):
        (weight,) = ctx.saved_tensors
        dx = grad_out @ weight.to(grad_out.dtype) if ctx.needs_input_grad[0] else None
        return dx, None, None


def install_invasive_forward(model: nn.Module, layer_names: set[str],
                             should_intervene: Callable[[], bool]) -> list[Callable[[], None]]:
    """Override each named ``nn.Linear``'s forward while *should_intervene()*; returns reverts.

    Raises:
        ValueError: for a named layer that is not ``nn.Linear``.
    """
    root = getattr(model, "module", model)
    reverts: list[Callable[[], None]] = []
    for name, module in root.named_modules():
        if name not in layer_names:
            continue
        if not is_invasive_capable(module):
            raise ValueError(
                f"Layer '{name}' was assigned 'invasive_linear_io' but is "
                f"{canonical_class_name(module)}, not nn.Linear.",
            )
        original = module.forward

        def forward(x, *args, _mod=module, _orig=original, **kwargs):
            if should_intervene():
                return InvasiveLinearFunction.apply(x, _mod.weight, _mod.bias)
            return _orig(x, *args, **kwargs)

        reverts.append(swap_forward(module, forward))
    return reverts
