"""Device-side generation of counter-based random projection matrices."""

from __future__ import annotations

import math

import torch

KINDS = {"rademacher": 0, "normal": 1, "gaussian": 1}


def projection_matrix_t(
    d_in: int,
    proj_dim: int,
    seed: int,
    *,
    kind: str = "rademacher",
    dtype: torch.dtype = torch.bfloat16,
    device: torch.device | str = "cuda",
) -> torch.Tensor:
    """The transposed ``(proj_dim, d_in)`` projection matrix, generated on the GPU.

    Bit-identical (Rademacher) to
    :func:`dattri_llm_b200.gradient.ops.projection.counter_projection_matrix`,
    the PyTorch statement of the same counter-based generator.
    """
    from dattri_llm_b200.ops import count_launch, native

    count_launch()
    if kind not in KINDS:
        raise ValueError(f"projection kind must be one of {sorted(KINDS)}, got {kind!r}")
    return native().projection_matrix_t(
        int(d_in), int(proj_dim), int(seed), KINDS[kind], 1.0 / math.sqrt(proj_dim), dtype,
        torch.device(device),
    )
