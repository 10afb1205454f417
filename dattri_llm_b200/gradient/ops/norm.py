"""Per-sample gradients of normalisation layers' affine parameters.

For LayerNorm / RMSNorm / GroupNorm the weight gradient of one sample is
``sum_t x_hat[t] * g[t]`` (the bias part ``sum_t g[t]``), with ``x_hat`` the normalised
input recomputed from the raw input the capture kept.  ``per_token=True`` keeps the token
axis instead: ``(B, T*d)``.  Reference behaviour: ``dattri_llm/gradient/ops/norm.py``.

On an sm_100 device, LayerNorm / RMSNorm over the last axis in bf16 is one fused kernel
(``csrc/norm_grad.cu``) that recomputes ``x_hat`` per token in registers and reduces over
tokens, so neither ``x_hat`` nor the product is ever written to HBM.
"""

from __future__ import annotations

import torch

from dattri_llm_b200.gradient.ops import dtypes
from dattri_llm_b200.gradient.ops.preprocess import (
    group_norm_x_hat,
    layer_norm_x_hat,
    preprocess_factors,
    rms_x_hat,
    to_3d,
)

_FUSED_TYPES = ("nn.LayerNorm", "nn.RMSNorm")
_FUSED_MAX_WIDTH = 16384  # the kernel keeps one row of partial sums per CTA in shared memory


def _fused_width(x: torch.Tensor, g: torch.Tensor, layer_type: str, module_kwargs: dict | None) -> int | None:
    """The normalised width when the fused kernel applies, else ``None``."""
    if layer_type not in _FUSED_TYPES or module_kwargs is None:
        return None
    if x.dtype != torch.bfloat16 or g.dtype != torch.bfloat16 or x.shape != g.shape or x.ndim < 2:
        return None
    width = x.shape[-1]
    shape = tuple(module_kwargs.get("normalized_shape", (width,)))
    if shape != (width,) or width % 8 or width > _FUSED_MAX_WIDTH:
        return None
    from dattri_llm_b200 import ops as native_ops

    return width if native_ops.use_native(x, g) else None


def norm_per_sample_grad(x: torch.Tensor, g: torch.Tensor, layer_type: str, module_kwargs: dict | None,
                         include_bias: bool = True, per_token: bool = False) -> torch.Tensor:
    """``(B, d)`` -- ``(B, 2d)`` with a bias, ``(B, T*d)`` per token -- gradient of a norm
    layer's affine parameters from its raw input *x* and output gradient *g*."""
    width = None if per_token else _fused_width(x, g, layer_type, module_kwargs)
    if width is not None:
        from dattri_llm_b200 import ops as native_ops

        eps = module_kwargs.get("eps")
        eps = torch.finfo(x.dtype).eps if eps is None else eps
        bias = include_bias and bool(module_kwargs.get("has_bias", False))
        return native_ops.norm_per_sample_grad(x.reshape(x.shape[0], -1, width), g.reshape(g.shape[0], -1, width),
                                               eps=eps, layer_norm=layer_type == "nn.LayerNorm", bias=bias)
    x_hat, grad = dtypes.align(*preprocess_factors(x, g, layer_type, module_kwargs, include_bias))
    per_position = to_3d(x_hat) * to_3d(grad)
    return per_position.flatten(1) if per_token else per_position.sum(1)


__all__ = ["group_norm_x_hat", "layer_norm_x_hat", "norm_per_sample_grad", "rms_x_hat"]
