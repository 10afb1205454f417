"""Native per-sample norm-parameter gradients (``csrc/norm_grad.cu``)."""

from __future__ import annotations

import torch


def norm_per_sample_grad(x: torch.Tensor, g: torch.Tensor, *, eps: float, layer_norm: bool,
                         bias: bool) -> torch.Tensor:
    """``(B, d)`` per-sample ``dgamma`` of a LayerNorm / RMSNorm over the last axis (or
    ``(B, 2d)`` ``[dgamma | dbeta]`` with *bias*) from its raw input ``x`` and output
    gradient ``g``, both ``(B, T, d)`` bf16; ``x_hat`` is recomputed in the kernel (fp32)."""
    from dattri_llm_b200.ops import count_launch, native

    count_launch()
    return native().norm_per_sample_grad(x.contiguous(), g.contiguous(), float(eps), bool(layer_norm), bool(bias))
