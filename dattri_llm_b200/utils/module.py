"""Builders of the per-layer ``module_kwargs`` dicts (layer hyperparameters).

A hooked layer's preprocessing reads its hyperparameters from this dict
(``ops.extract_module_kwargs`` builds it from the module itself).  These
builders are for layers whose class does not expose them in the standard
places -- e.g. Hugging Face ``LlamaRMSNorm`` keeps its epsilon in
``variance_epsilon``.  The keys are part of the on-disk record format and match
the reference's ``dattri_llm/utils/module.py:82-467``.
"""

from __future__ import annotations

from collections.abc import Sequence

_EMBEDDING_BAG_MODES = ("sum", "mean")


def _to_tuple(value: int | Sequence[int], rank: int, name: str) -> tuple[int, ...]:
    if isinstance(value, int):
        return (value,) * rank
    out = tuple(int(v) for v in value)
    if len(out) != rank:
        raise ValueError(f"{name} must be an int or a length-{rank} sequence, got {value!r}.")
    return out


def _conv(rank, kernel_size, stride, padding, dilation, has_bias, groups) -> dict:
    if groups < 1:
        raise ValueError(f"groups must be a positive int, got {groups!r}.")
    return {
        "has_bias": has_bias,
        "kernel_size": _to_tuple(kernel_size, rank, "kernel_size"),
        "stride": _to_tuple(stride, rank, "stride"),
        "padding": _to_tuple(padding, rank, "padding"),
        "dilation": _to_tuple(dilation, rank, "dilation"),
        "groups": int(groups),
    }


def linear_module_kwargs(*, has_bias: bool) -> dict:
    """``nn.Linear`` (and HF ``Conv1D``)."""
    return {"has_bias": has_bias}


def bilinear_module_kwargs(*, has_bias: bool) -> dict:
    """``nn.Bilinear``."""
    return {"has_bias": has_bias}


def embedding_module_kwargs(*, num_embeddings: int, padding_idx: int | None) -> dict:
    """``nn.Embedding``: vocab size (materialized width) and canonical padding index."""
    return {"has_bias": False, "num_embeddings": num_embeddings, "padding_idx": padding_idx}


def embedding_bag_module_kwargs(*, num_embeddings: int, mode: str, padding_idx: int | None) -> dict:
    """``nn.EmbeddingBag`` with a ``"sum"`` or ``"mean"`` bag reduction."""
    if mode not in _EMBEDDING_BAG_MODES:
        raise ValueError(f"mode must be one of {_EMBEDDING_BAG_MODES}, got {mode!r}.")
    return {"has_bias": False, "num_embeddings": num_embeddings, "mode": mode,
            "padding_idx": padding_idx}


def conv1d_module_kwargs(*, kernel_size, stride=1, padding=0, dilation=1, has_bias: bool,
                         groups: int = 1) -> dict:
    """``nn.Conv1d``."""
    return _conv(1, kernel_size, stride, padding, dilation, has_bias, groups)


def conv2d_module_kwargs(*, kernel_size, stride=1, padding=0, dilation=1, has_bias: bool,
                         groups: int = 1) -> dict:
    """``nn.Conv2d``."""
    return _conv(2, kernel_size, stride, padding, dilation, has_bias, groups)


def conv3d_module_kwargs(*, kernel_size, stride=1, padding=0, dilation=1, has_bias: bool,
                         groups: int = 1) -> dict:
    """``nn.Conv3d``."""
    return _conv(3, kernel_size, stride, padding, dilation, has_bias, groups)


def conv_transpose1d_module_kwargs(*, kernel_size, stride=1, padding=0, dilation=1,
                                   has_bias: bool, groups: int = 1) -> dict:
    """``nn.ConvTranspose1d`` (the unfold of its output gradient uses these)."""
    return _conv(1, kernel_size, stride, padding, dilation, has_bias, groups)


def conv_transpose2d_module_kwargs(*, kernel_size, stride=1, padding=0, dilation=1,
                                   has_bias: bool, groups: int = 1) -> dict:
    """``nn.ConvTranspose2d``."""
    return _conv(2, kernel_size, stride, padding, dilation, has_bias, groups)


def conv_transpose3d_module_kwargs(*, kernel_size, stride=1, padding=0, dilation=1,
                                   has_bias: bool, groups: int = 1) -> dict:
    """``nn.ConvTranspose3d``."""
    return _conv(3, kernel_size, stride, padding, dilation, has_bias, groups)


def layer_norm_module_kwargs(*, normalized_shape: int | Sequence[int], eps: float,
                             has_bias: bool) -> dict:
    """``nn.LayerNorm``."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    return {"has_bias": has_bias, "normalized_shape": tuple(normalized_shape), "eps": eps}


def rms_norm_module_kwargs(*, normalized_shape: int | Sequence[int], eps: float | None) -> dict:
    """``nn.RMSNorm`` and hand-rolled RMSNorms declared as such (HF ``LlamaRMSNorm``:
    pass its ``variance_epsilon``); ``eps=None`` means the dtype's machine epsilon."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    return {"has_bias": False, "normalized_shape": tuple(normalized_shape), "eps": eps}


def group_norm_module_kwargs(*, num_groups: int, num_channels: int, eps: float,
                             has_bias: bool) -> dict:
    """``nn.GroupNorm``."""
    return {"has_bias": has_bias, "num_groups": num_groups, "num_channels": num_channels,
            "eps": eps}


def _instance(num_features: int, eps: float, has_bias: bool) -> dict:
    return {"has_bias": has_bias, "num_features": num_features, "eps": eps}


def instance_norm1d_module_kwargs(*, num_features: int, eps: float = 1e-5,
                                  has_bias: bool = False) -> dict:
    """``nn.InstanceNorm1d`` (affine parameters, when present, are per channel)."""
    return _instance(num_features, eps, has_bias)


def instance_norm2d_module_kwargs(*, num_features: int, eps: float = 1e-5,
                                  has_bias: bool = False) -> dict:
    """``nn.InstanceNorm2d``."""
    return _instance(num_features, eps, has_bias)


def instance_norm3d_module_kwargs(*, num_features: int, eps: float = 1e-5,
                                  has_bias: bool = False) -> dict:
    """``nn.InstanceNorm3d``."""
    return _instance(num_features, eps, has_bias)
