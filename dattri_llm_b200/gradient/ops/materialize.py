"""Materialization of factorized captures into per-sample weight gradients.

Parity: reference ``dattri_llm/gradient/ops/materialize.py:22-146``.  Layouts
(part of the stored record format): linear / conv ``(B, D_out * K_in)`` row-major
``(out, in)``; conv-transpose ``(B, C_in * P)``; grouped conv per group
``(G, D_g, K_g)``; norm ``(B, d)`` (token-summed) or ``(B, T*d)`` per token;
embedding ``(B, vocab * E)``.

On an sm_100 device the linear/conv contraction ``g^T a`` over tokens runs on the
tensor cores (:func:`dattri_llm_b200.ops.per_sample_outer`), the norm reduction in
one fused pass, and the embedding scatter as one pass that writes every output row once
(the tokens sorted by sample and id, each row's tokens summed in fp32).
"""

from __future__ import annotations

import torch

from dattri_llm_b200.gradient.ops import dtypes
from dattri_llm_b200.gradient.ops.norm import norm_per_sample_grad
from dattri_llm_b200.gradient.ops.preprocess import preprocess_factors, to_3d
from dattri_llm_b200.gradient.ops.types import is_conv_transpose, is_embedding, is_norm


def _materialize_embedding(ids: torch.Tensor, g: torch.Tensor, vocab: int) -> torch.Tensor:
    """``(B, vocab * E)``: per sample, each token's gradient row added at its id."""
    (grad,) = dtypes.align(g)
    b, t = ids.shape
    e = grad.shape[-1]
    if ids.numel() and int(ids.max()) >= vocab:
        raise ValueError(
            f"Embedding token id {int(ids.max())} is out of range for num_embeddings={vocab}; "
            "the module_kwargs do not match the captured data.",
        )
    from dattri_llm_b200 import ops as native_ops

    if (native_ops.use_native(grad) and grad.dtype in (torch.bfloat16, torch.float32)
            and (e * grad.element_size()) % 16 == 0):
        return native_ops.embedding_dense_grad(ids, grad.reshape(b, t, e), vocab)
    flat = (ids.long() + torch.arange(b, device=ids.device)[:, None] * vocab).reshape(-1)
    out = torch.zeros(b * vocab, e, dtype=grad.dtype, device=grad.device)
    out.index_add_(0, flat, grad.reshape(-1, e))
    return out.reshape(b, vocab * e)


def _outer_over_tokens(left: torch.Tensor, right: torch.Tensor) -> torch.Tensor:
    """``(B, L, R) = sum_t left[b,t,:]^T right[b,t,:]`` (fp32 accumulate on the GPU)."""
    from dattri_llm_b200 import ops as native_ops

    if native_ops.use_native(left, right) and left.dtype == torch.bfloat16:
        return native_ops.per_sample_outer(left, right, out_dtype=left.dtype)
    return torch.bmm(left.transpose(1, 2), right)


def materialize_factors(
    a: torch.Tensor,
    g: torch.Tensor,
    layer_type: str,
    module_kwargs: dict | None = None,
    include_bias: bool = True,
    per_token: bool = False,
) -> torch.Tensor:
    """Per-sample weight gradient ``(B, d)`` of raw (or final) factors.

    Norm layers sum the token axis unless ``per_token=True`` (``(B, T*d)``).
    Embeddings need ``module_kwargs`` (the width is ``num_embeddings * E``).
    """
    if is_norm(layer_type):
        return norm_per_sample_grad(a, g, layer_type, module_kwargs, include_bias, per_token)
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    if is_embedding(layer_type):
        if module_kwargs is None:
            raise ValueError(
                "Materializing an embedding gradient requires module_kwargs with "
                "'num_embeddings' (the vocab size cannot be inferred from the factors).",
            )
        return _materialize_embedding(a, g, module_kwargs["num_embeddings"])
    a, g = dtypes.align(a, g)
    a_f, g_f = to_3d(a), to_3d(g)
    if a_f.ndim == 4:
        if is_conv_transpose(layer_type):
            return torch.einsum("btgc,btgp->bgcp", a_f, g_f).flatten(1)
        return torch.einsum("btgk,btgd->bgdk", a_f, g_f).flatten(1)
    if is_conv_transpose(layer_type):
        return _outer_over_tokens(a_f, g_f).flatten(1)
    return _outer_over_tokens(g_f, a_f).flatten(1)


def materialize(f, layer_type: str, include_bias: bool = True, per_token: bool = False) -> torch.Tensor:
    """Per-sample weight gradient ``(B, d)`` of one layer, whatever its form
    (a dense tensor is returned flattened to ``(B, d)``)."""
    if isinstance(f, torch.Tensor):
        return f.reshape(f.shape[0], -1)
    bf = f.as_batch_first()
    return materialize_factors(bf.activation, bf.pre_activation_grad, layer_type,
                               bf.module_kwargs, include_bias, per_token)
