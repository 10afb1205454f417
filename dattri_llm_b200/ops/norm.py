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


def embedding_dense_grad(ids: torch.Tensor, g: torch.Tensor, vocab: int) -> torch.Tensor:
    """``(B, vocab * E)`` per-sample embedding gradients: row ``v`` of sample ``b`` is the sum
    of ``g[b, t]`` over the tokens ``t`` with ``ids[b, t] == v``.  ``g`` is ``(B, T, E)`` bf16
    or fp32 (the result keeps its dtype); the tokens are sorted by ``b * vocab + id`` here
    (stable, so sums run in token order), each output row's first token is located by a
    search over the sorted keys, and the kernel writes every output row once."""
    from dattri_llm_b200.ops import count_launch, native

    b, t = ids.shape
    e = g.shape[-1]
    keys = (ids.long() + torch.arange(b, device=ids.device)[:, None] * vocab).reshape(-1)
    keys, order = torch.sort(keys, stable=True)
    starts = torch.searchsorted(keys, torch.arange(b * vocab + 1, device=ids.device))  # row r: [starts[r], starts[r+1])
    count_launch()
    out = native().embedding_dense_grad(starts, order.contiguous(), g.reshape(b * t, e).contiguous(), b * vocab)
    return out.reshape(b, vocab * e)
