"""Layer-type registry: string-typed layer families.

Layer types are canonical class-name strings (``"nn.Linear"``); they are stored
inside gradient records, so the vocabulary is the reference's
(``dattri_llm/gradient/ops/types.py:14-103``).
"""

from __future__ import annotations

from torch import nn

LINEAR_TYPES = frozenset(
    {"nn.Linear", "nn.Bilinear", "nn.NonDynamicallyQuantizableLinear",
     "transformers.pytorch_utils.Conv1D"},
)
CONV_TYPES = frozenset({"nn.Conv1d", "nn.Conv2d", "nn.Conv3d"})
CONV_TRANSPOSE_TYPES = frozenset({"nn.ConvTranspose1d", "nn.ConvTranspose2d", "nn.ConvTranspose3d"})
NORM_TYPES = frozenset(
    {"nn.LayerNorm", "nn.RMSNorm", "nn.GroupNorm", "nn.InstanceNorm1d", "nn.InstanceNorm2d",
     "nn.InstanceNorm3d"},
)
EMBEDDING_TYPES = frozenset({"nn.Embedding", "nn.EmbeddingBag"})
#: Layer-type marker of aggregated (batch-level) parameter gradients.
PARAM_GRAD_TYPES = "param_grad_layers"
#: Every layer type with per-sample (factorized) capture support.
ALL_LAYER_TYPES = LINEAR_TYPES | CONV_TYPES | CONV_TRANSPOSE_TYPES | NORM_TYPES | EMBEDDING_TYPES


def is_linear(layer_type: str) -> bool:
    """Linear family (incl. HF ``Conv1D``)."""
    return layer_type in LINEAR_TYPES


def is_conv(layer_type: str) -> bool:
    """Convolution layer."""
    return layer_type in CONV_TYPES


def is_conv_transpose(layer_type: str) -> bool:
    """Transposed convolution layer."""
    return layer_type in CONV_TRANSPOSE_TYPES


def is_norm(layer_type: str) -> bool:
    """Normalization layer."""
    return layer_type in NORM_TYPES


def is_embedding(layer_type: str) -> bool:
    """Embedding / EmbeddingBag."""
    return layer_type in EMBEDDING_TYPES


def is_kfac_eligible(layer_type: str) -> bool:
    """Layers whose gradient is an outer product, i.e. that carry K-FAC factors."""
    return is_linear(layer_type) or is_conv(layer_type) or is_conv_transpose(layer_type)


def canonical_class_name(module: nn.Module) -> str:
    """``"nn.<Class>"`` for torch.nn modules, else ``"<module>.<Class>"``.

    A class may declare the layer type it computes with a ``__bw_layer_type__``
    attribute (e.g. a fused-kernel subclass of ``nn.RMSNorm`` declares
    ``"nn.RMSNorm"``), which takes precedence.
    """
    declared = getattr(type(module), "__bw_layer_type__", None)
    if declared is not None:
        return declared
    cls = type(module)
    # FSDP2 (``fully_shard``) swaps a module's class for a generated ``FSDP<Class>`` subclass:
    # name the class it was made from.
    for c in cls.__mro__:
        if not c.__module__.startswith(("torch.distributed.fsdp", "torch.distributed._composable")):
            cls = c
            break
    mod, name = cls.__module__, cls.__name__
    return f"nn.{name}" if mod.startswith("torch.nn") else f"{mod}.{name}"
