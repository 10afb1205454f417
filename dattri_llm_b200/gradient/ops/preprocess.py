"""Preprocessing of raw hook captures into contractable ``(a, g)`` factors.

Hooks store what autograd delivers -- the layer input and its output gradient.
Per layer type this module turns them into factors whose token-summed outer
product is the per-sample weight gradient (parity: reference
``dattri_llm/gradient/ops/preprocess.py:33-487`` and ``ops/norm.py:10-134``):

* Linear: a ones column appended to ``a`` carries the bias gradient.
* Conv: im2col of ``a`` to ``(N, L, C_in*prod(k))``; ``g`` to ``(N, L, C_out)``.
* ConvTranspose: roles reversed (``g`` unfolded), bias folded through one extra
  location and feature block.
* Grouped convolutions expose a group axis ``(N, L, G, .)`` that every kernel
  treats as an aligned batch axis (no cross-group products).
* LayerNorm / RMSNorm: ``a`` becomes ``x_hat``; with bias a ones block is appended
  and ``g`` duplicated, so ``a * g`` per position is ``[dgamma, dbeta]``.
* GroupNorm / InstanceNorm: per-group ``x_hat`` with spatial positions as tokens.
* Embedding: pad positions get zero ``g``; EmbeddingBag broadcasts each bag's
  gradient to its tokens (``1/T`` or ``1/#non-pad`` for ``mean``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from dattri_llm_b200.gradient.ops.types import CONV_TRANSPOSE_TYPES, CONV_TYPES, is_linear

# ---------------------------------------------------------------------------
# normalization statistics
# ---------------------------------------------------------------------------


def layer_norm_x_hat(x: torch.Tensor, normalized_shape: tuple, eps: float) -> torch.Tensor:
    """``(x - mean) / sqrt(var + eps)`` over the trailing *normalized_shape* axes."""
    dims = tuple(range(-len(normalized_shape), 0))
    mean = x.mean(dim=dims, keepdim=True)
    var = x.var(dim=dims, unbiased=False, keepdim=True)
    return (x - mean) / (var + eps).sqrt()


def rms_x_hat(x: torch.Tensor, normalized_shape: tuple, eps: float | None) -> torch.Tensor:
    """``x / sqrt(mean(x^2) + eps)``; ``eps=None`` is the dtype's machine epsilon."""
    dims = tuple(range(-len(normalized_shape), 0))
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    return x * torch.rsqrt(x.pow(2).mean(dim=dims, keepdim=True) + eps)


def group_norm_x_hat(x: torch.Tensor, num_groups: int, eps: float) -> torch.Tensor:
    """GroupNorm ``x_hat`` of ``(N, C, *spatial)``; ``num_groups == C`` is InstanceNorm."""
    n, c = x.shape[:2]
    grouped = x.reshape(n, num_groups, -1)
    mean = grouped.mean(dim=2, keepdim=True)
    var = grouped.var(dim=2, unbiased=False, keepdim=True)
    return ((grouped - mean) * torch.rsqrt(var + eps)).reshape(n, c, *x.shape[2:])


def _fold_positions(x_hat, g, normalized_shape):
    """Fold every axis between batch and the normalized axes into one position axis
    (e.g. a per-head QK-norm input ``(B, T, H, d)`` becomes ``(B, T*H, d)``)."""
    if x_hat.ndim <= 2 + len(normalized_shape):
        return x_hat, g
    d = math.prod(normalized_shape)
    return x_hat.reshape(x_hat.shape[0], -1, d), g.reshape(g.shape[0], -1, d)


def _bias_block(a: torch.Tensor, g: torch.Tensor, has_bias: bool):
    if not has_bias:
        return a, g
    return torch.cat([a, torch.ones_like(a)], dim=-1), torch.cat([g, g], dim=-1)


def _channels_as_tokens(x_hat, g, has_bias):
    n, c = x_hat.shape[:2]
    a = x_hat.reshape(n, c, -1).transpose(1, 2).contiguous()
    gg = g.reshape(n, c, -1).transpose(1, 2).contiguous()
    return _bias_block(a, gg, has_bias)


# ---------------------------------------------------------------------------
# convolution unfolding
# ---------------------------------------------------------------------------


def _unfold_nd(x: torch.Tensor, kw: dict, rank: int) -> torch.Tensor:
    """im2col of ``(N, C, *spatial)`` to ``(N, L, C*prod(k))`` (channel-major features)."""
    k, s, p, d = kw["kernel_size"], kw["stride"], kw["padding"], kw["dilation"]
    if rank == 2:
        return F.unfold(x, k, d, p, s).transpose(1, 2).contiguous()
    if any(pi > 0 for pi in p):
        pads = []
        for pi in reversed(p):
            pads += [pi, pi]
        x = F.pad(x, pads)
    n, c = x.shape[:2]
    # unfold each spatial axis in turn: (N, C, *out, *k)
    for axis in range(rank):
        x = x.unfold(2 + axis, d[axis] * (k[axis] - 1) + 1, s[axis])
        if d[axis] > 1:
            x = x[..., :: d[axis]]
    # x: (N, C, o_1..o_r, k_1..k_r) -> (N, L, C*prod(k))
    outs = x.shape[2 : 2 + rank]
    perm = [0, *range(2, 2 + rank), 1, *range(2 + rank, 2 + 2 * rank)]
    x = x.permute(*perm).contiguous()
    return x.reshape(n, math.prod(outs), c * math.prod(k))


def _conv_rank(layer_type: str) -> int:
    return int(layer_type[-2])


def _groups_axis(x: torch.Tensor, groups: int) -> torch.Tensor:
    if groups == 1:
        return x
    n, length, width = x.shape
    return x.reshape(n, length, groups, width // groups)


def _conv_transpose_factors(a, g, layer_type, kw, has_bias):
    rank = _conv_rank(layer_type)
    groups = kw.get("groups", 1)
    n, c_in = a.shape[:2]
    a_flat = a.reshape(n, c_in, -1).transpose(1, 2).contiguous()
    g_unf = _unfold_nd(g, kw, rank)
    a_flat, g_unf = _groups_axis(a_flat, groups), _groups_axis(g_unf, groups)
    if not has_bias:
        return a_flat, g_unf
    c_out = g.shape[1]
    c_out_g = c_out // groups
    db = g.reshape(n, c_out, -1).sum(dim=2)
    if groups > 1:
        db = db.reshape(n, groups, c_out_g)
    a_pad = torch.cat([a_flat, torch.zeros_like(a_flat[..., :1])], dim=-1)
    a_loc = torch.zeros_like(a_pad[:, :1])
    a_loc[..., -1] = 1.0
    g_pad = torch.cat([g_unf, torch.zeros_like(g_unf[..., :c_out_g])], dim=-1)
    g_loc = torch.zeros_like(g_pad[:, :1])
    g_loc[..., -c_out_g:] = db.unsqueeze(1)
    return torch.cat([a_pad, a_loc], dim=1), torch.cat([g_pad, g_loc], dim=1)


def _embedding_bag_factors(a, g, mode, padding_idx):
    if mode == "max":
        raise NotImplementedError("EmbeddingBag mode='max' is not supported for factorized gradients.")
    if a.ndim != 2:
        raise NotImplementedError("EmbeddingBag factorization supports only 2-D inputs (N, T) without offsets.")
    t = a.shape[1]
    g_tok = g.unsqueeze(1).expand(-1, t, -1).contiguous()
    if padding_idx is not None:
        pad = a == padding_idx
        g_tok = g_tok.masked_fill(pad.unsqueeze(-1), 0)
        if mode == "mean":
            g_tok = g_tok / (~pad).sum(dim=1).clamp_min(1).view(-1, 1, 1)
    elif mode == "mean":
        g_tok = g_tok / t
    return a, g_tok


# ---------------------------------------------------------------------------
# public API
# ---------------------------------------------------------------------------


def extract_module_kwargs(module: nn.Module, layer_type: str) -> dict:
    """The minimal serialisable hyperparameters :func:`preprocess_factors` needs.

    Raises:
        NotImplementedError: for embeddings with ``scale_grad_by_freq=True`` (a
            whole-batch statistic the per-sample factors cannot carry).
    """
    kw: dict = {"has_bias": getattr(module, "bias", None) is not None}
    if layer_type in ("nn.Embedding", "nn.EmbeddingBag") and getattr(module, "scale_grad_by_freq", False):
        raise NotImplementedError(
            f"{layer_type} with scale_grad_by_freq=True is not supported: the inverse-frequency "
            "scaling is a whole-batch statistic that per-sample factors do not model.",
        )
    if layer_type == "nn.Embedding":
        kw["num_embeddings"] = module.num_embeddings
        kw["padding_idx"] = module.padding_idx
    elif layer_type in CONV_TYPES or layer_type in CONV_TRANSPOSE_TYPES:
        kw.update(kernel_size=module.kernel_size, stride=module.stride, padding=module.padding,
                  dilation=module.dilation, groups=module.groups)
    elif layer_type in ("nn.LayerNorm", "nn.RMSNorm"):
        kw["normalized_shape"] = tuple(module.normalized_shape)
        kw["eps"] = module.eps
    elif layer_type == "nn.GroupNorm":
        kw.update(num_groups=module.num_groups, num_channels=module.num_channels, eps=module.eps)
    elif layer_type.startswith("nn.InstanceNorm"):
        kw.update(num_features=module.num_features, eps=module.eps)
    elif layer_type == "nn.EmbeddingBag":
        kw.update(num_embeddings=module.num_embeddings, mode=module.mode, padding_idx=module.padding_idx)
    return kw


def preprocess_factors(
    a: torch.Tensor,
    g: torch.Tensor,
    layer_type: str,
    module_kwargs: dict | None = None,
    include_bias: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Raw ``(input, grad_output)`` -> factors of the per-sample weight gradient.

    ``module_kwargs=None`` means the factors are already final (e.g. projected).
    """
    if module_kwargs is None:
        return a, g
    has_bias = bool(module_kwargs.get("has_bias", False)) and include_bias
    if layer_type in ("nn.LayerNorm", "nn.RMSNorm"):
        shape = tuple(module_kwargs.get("normalized_shape", (a.shape[-1],)))
        x_hat = (layer_norm_x_hat(a, shape, module_kwargs["eps"]) if layer_type == "nn.LayerNorm"
                 else rms_x_hat(a, shape, module_kwargs.get("eps")))
        x_hat, g = _fold_positions(x_hat, g, shape)
        return _bias_block(x_hat, g, has_bias)
    if layer_type == "nn.GroupNorm":
        x_hat = group_norm_x_hat(a, module_kwargs["num_groups"], module_kwargs["eps"])
        return _channels_as_tokens(x_hat, g, has_bias)
    if layer_type.startswith("nn.InstanceNorm"):
        x_hat = group_norm_x_hat(a, module_kwargs["num_features"], module_kwargs["eps"])
        return _channels_as_tokens(x_hat, g, has_bias)
    if layer_type == "nn.Embedding":
        pad = module_kwargs.get("padding_idx")
        if pad is not None:
            g = g.masked_fill((a == pad).unsqueeze(-1), 0)
        return a, g
    if layer_type == "nn.EmbeddingBag":
        return _embedding_bag_factors(a, g, module_kwargs["mode"], module_kwargs.get("padding_idx"))
    if layer_type in CONV_TYPES:
        rank = _conv_rank(layer_type)
        groups = module_kwargs.get("groups", 1)
        a_unf = _unfold_nd(a, module_kwargs, rank)
        n, c_out = g.shape[:2]
        g_out = g.reshape(n, c_out, -1).transpose(1, 2).contiguous()
        a_unf, g_out = _groups_axis(a_unf, groups), _groups_axis(g_out, groups)
        if has_bias:
            a_unf = torch.cat([a_unf, torch.ones_like(a_unf[..., :1])], dim=-1)
        return a_unf, g_out
    if layer_type in CONV_TRANSPOSE_TYPES:
        return _conv_transpose_factors(a, g, layer_type, module_kwargs, has_bias)
    if is_linear(layer_type) and has_bias:
        return torch.cat([a, torch.ones_like(a[..., :1])], dim=-1), g
    return a, g


def to_3d(x: torch.Tensor) -> torch.Tensor:
    """``(B, D) -> (B, 1, D)``; 3-D (and grouped 4-D) factors pass through."""
    return x.unsqueeze(1) if x.ndim == 2 else x


def preprocess_factorized(f, layer_type: str, include_bias: bool = True):
    """:func:`preprocess_factors` on a :class:`Factorized` (batch-first-safe)."""
    bf = f.as_batch_first()
    return preprocess_factors(bf.activation, bf.pre_activation_grad, layer_type,
                              bf.module_kwargs, include_bias)
