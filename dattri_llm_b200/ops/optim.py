"""Native optimizer-geometry kernels (``csrc/rows.cu``)."""

from __future__ import annotations

import torch


def adam_direction(g: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, *, step: int,
                   beta1: float, beta2: float, eps: float) -> torch.Tensor:
    """Per-sample Adam update direction of ``g (..., p)`` (fp32): ``m_hat / (sqrt(v_hat) + eps)``
    with ``m = beta1 m0 + (1 - beta1) g`` and ``v = beta2 v0 + (1 - beta2) g^2`` for the
    optimizer's moments ``m0, v0`` (flattened to ``p``) -- one fused pass (the update
    ``torch.optim.Adam`` would take next if *g* were the whole batch's gradient).
    Reference: ``dattri_llm/gradient/ops/optimizer.py`` (Adam preconditioner)."""
    from dattri_llm_b200.ops import count_launch, native

    p = g.shape[-1]
    m0 = exp_avg.detach().reshape(-1).to(g.device, torch.float32).contiguous()
    v0 = exp_avg_sq.detach().reshape(-1).to(g.device, torch.float32).contiguous()
    if m0.numel() != p or v0.numel() != p:
        raise ValueError(f"optimizer moments have {m0.numel()} entries for a {p}-wide gradient")
    g32 = g.to(torch.float32).contiguous()
    if p % 4:
        raise ValueError("adam_direction: the width must be a multiple of 4")
    count_launch()
    return native().adam_direction(g32.reshape(-1, p), m0, v0, float(beta1), float(beta2), int(step),
                                   float(eps)).view(g.shape)
