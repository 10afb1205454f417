"""Per-sample outer products and cross-grams on the tensor cores."""

from __future__ import annotations

import torch

from dattri_llm_b200.ops.gemm import STORE_BF16, STORE_F32, gemm_tn


def per_sample_outer(
    left: torch.Tensor,
    right: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.float32,
    left_t: torch.Tensor | None = None,
    right_t: torch.Tensor | None = None,
) -> torch.Tensor:
    """``out[b] = left[b]^T right[b]`` over the token axis: ``(B, T, L), (B, T, R) -> (B, L, R)``.

    The contraction runs over tokens, so the GEMM operands are the token-major
    transposes ``(B, L, T)`` / ``(B, R, T)``; callers that already hold them (the
    capture kernels write projected factors transposed) pass *left_t* / *right_t*.
    """
    from dattri_llm_b200.ops.gemm import transpose_last2

    lt = left_t if left_t is not None else transpose_last2(left)
    rt = right_t if right_t is not None else transpose_last2(right)
    if lt.dtype != torch.bfloat16:
        lt = lt.bfloat16()
    if rt.dtype != torch.bfloat16:
        rt = rt.bfloat16()
    b, l_dim, r_dim = lt.shape[0], lt.shape[1], rt.shape[1]
    out = torch.empty(b, l_dim, r_dim, dtype=out_dtype, device=lt.device)
    gemm_tn(lt, rt, out, mode=STORE_BF16 if out_dtype == torch.bfloat16 else STORE_F32)
    return out


def ghost_gram(a1: torch.Tensor, g1: torch.Tensor, a2: torch.Tensor, g2: torch.Tensor, *,
               diag_only: bool = False) -> torch.Tensor:
    """Fused factorized cross-gram ``(B1, B2)`` (fp32) of 3-D bf16 factors
    ``a (B, S, K)``, ``g (B, S, D)``; the token-pair products stay on chip.  With
    *diag_only* (``B1 == B2``) only the ``i == j`` entries are computed (the rest stay 0):
    per-sample dots / squared norms without the cross terms' work."""
    from dattri_llm_b200.ops import count_launch, error_word, native

    count_launch()
    b1, s1 = a1.shape[:2]
    b2, s2 = a2.shape[:2]
    out = torch.zeros(b1, b2, dtype=torch.float32, device=a1.device)
    if b1 == 0 or b2 == 0:
        return out

    def flat(x):
        x = x.reshape(-1, x.shape[-1])
        if x.shape[-1] % 8:
            x = torch.nn.functional.pad(x, (0, 8 - x.shape[-1] % 8))
        return x.contiguous().bfloat16()

    native().ghost_gram(flat(a1), flat(g1), flat(a2), flat(g2), s1, s2, out, error_word(a1.device), diag_only)
    return out


def ghost_dot(a1: torch.Tensor, g1: torch.Tensor, a2: torch.Tensor, g2: torch.Tensor) -> torch.Tensor:
    """``(B,)`` per-sample ``<dW1_i, dW2_i>`` of factorized gradients (``a2 is a1`` and
    ``g2 is g1`` give squared norms) in one fused launch: the diagonal sample blocks of the
    token-pair Gram only.  Reference: ``dattri_llm/gradient/ops/dot.py:307-411``."""
    return ghost_gram(a1, g1, a2, g2, diag_only=True).diagonal().clone()


def ghost_gram_tokens(tok1: torch.Tensor, g1: torch.Tensor, tok2: torch.Tensor, g2: torch.Tensor, *,
                      diag_only: bool = False) -> torch.Tensor:
    """Embedding-layer cross-gram ``(B1, B2)`` (fp32):
    ``K[i, j] = sum_{t, s} [tok1_it == tok2_js] <g1_it, g2_js>`` for token ids ``(B, S)``
    and output gradients ``(B, S, E)``.  One tcgen05 Gram of the gradients whose epilogue
    applies the token-equality mask and reduces per sample pair (no vocab-sized buffer and
    no token-pair matrix in HBM).  Reference: ``dattri_llm/gradient/ops/dot.py:58-74``."""
    from dattri_llm_b200.ops import count_launch, error_word, native

    count_launch()
    b1, s1 = tok1.shape
    b2, s2 = tok2.shape
    out = torch.zeros(b1, b2, dtype=torch.float32, device=g1.device)
    if b1 == 0 or b2 == 0 or s1 == 0 or s2 == 0:
        return out

    def flat(x):
        x = x.reshape(-1, x.shape[-1])
        if x.shape[-1] % 8:
            x = torch.nn.functional.pad(x, (0, 8 - x.shape[-1] % 8))
        return x.contiguous().bfloat16()

    native().ghost_gram_tokens(tok1.reshape(-1).long().contiguous(), flat(g1), tok2.reshape(-1).long().contiguous(),
                               flat(g2), s1, s2, out, error_word(g1.device), diag_only)
    return out


def mask_gather(rows_src: torch.Tensor, cols_src: torch.Tensor, rows: torch.Tensor, cols: torch.Tensor) -> torch.Tensor:
    """``(B, M)`` fp32 ``out[b, m] = sum_t rows_src[b, t, rows[m]] * cols_src[b, t, cols[m]]``:
    fixed coordinates of per-sample gradients ``rows_src_b^T cols_src_b`` gathered without
    forming them (the ``mask`` projection style)."""
    from dattri_llm_b200.ops import count_launch, error_word, native

    def prep(x):
        x = x.contiguous().bfloat16()
        if x.shape[-1] % 8:
            x = torch.nn.functional.pad(x, (0, 8 - x.shape[-1] % 8))
        return x

    r, c = prep(rows_src), prep(cols_src)
    out = torch.empty(r.shape[0], rows.numel(), dtype=torch.float32, device=r.device)
    count_launch()
    native().mask_gather(r, c, rows.to(device=r.device, dtype=torch.int32).contiguous(),
                         cols.to(device=r.device, dtype=torch.int32).contiguous(), out, error_word(r.device))
    return out
