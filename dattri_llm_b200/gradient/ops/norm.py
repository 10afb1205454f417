"""Normalisation-layer factors: ``x_hat`` of LayerNorm / RMSNorm / GroupNorm and the
per-sample affine-parameter gradients.

Parity: reference ``dattri_llm/gradient/ops/norm.py:10-134``.  On an sm_100 device the
per-sample gradient of a LayerNorm / RMSNorm over the last axis is one fused kernel that
recomputes ``x_hat`` (``csrc/norm_grad.cu``); elsewhere it is ``sum_t x_hat * g``.
"""

from __future__ import annotations

import torch

from dattri_llm_b200.gradient.ops.preprocess import group_norm_x_hat, layer_norm_x_hat, rms_x_hat


def norm_per_sample_grad(x: torch.Tensor, g: torch.Tensor, layer_type: str, module_kwargs: dict,
                         include_bias: bool = True) -> torch.Tensor:
    """``(B, d)`` (or ``(B, 2d)`` with a bias) per-sample gradient of a norm layer's affine
    parameters from its raw input and output gradient."""
    from dattri_llm_b200.gradient.ops.materialize import materialize_factors

    return materialize_factors(x, g, layer_type, module_kwargs, include_bias)


__all__ = ["group_norm_x_hat", "layer_norm_x_hat", "norm_per_sample_grad", "rms_x_hat"]
