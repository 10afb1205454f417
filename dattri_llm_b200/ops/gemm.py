"""Python entry points of the generic tcgen05 GEMM (``csrc/gemm_tc.cu``)."""

from __future__ import annotations

import torch

STORE_F32 = 0
STORE_BF16 = 1
STORE_ATOMIC_F32 = 2
STORE_BF16_T = 3
STORE_SQ_SUM_F32 = 8  # C += sum over the batch of (alpha * A_z B_z^T)^2

_SMS = 148


def _k_aligned(x: torch.Tensor) -> torch.Tensor:
    """Contiguous along K with K padded to a multiple of 8 (TMA's 16-byte rule)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    k = x.shape[-1]
    if k % 8:
        x = torch.nn.functional.pad(x, (0, 8 - k % 8))
    elif x.dim() >= 2 and x.shape[-2] > 1 and x.stride(-2) % 8:
        x = x.contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    return x


def transpose_last2(x: torch.Tensor) -> torch.Tensor:
    """``x.transpose(-1, -2).contiguous()``; bf16 CUDA tensors on sm_100 go through the library's
    tiled transpose kernel (16-byte vectors in and out through shared memory), others through torch."""
    from dattri_llm_b200.ops import count_launch, native, use_native

    if x.dtype == torch.bfloat16 and x.dim() >= 2 and use_native(x):
        count_launch()
        return native().transpose_last2(x)
    return x.transpose(-1, -2).contiguous()


_F32_MIN_WORK = 1 << 22  # below this M*N*K a torch matmul is cheaper than the split + launch


def matmul_f32(a: torch.Tensor, b: torch.Tensor, *, b_transposed: bool = False) -> torch.Tensor:
    """fp32 ``a @ b`` (``a @ b^T`` with *b_transposed*) on the tensor cores at fp32-class accuracy.

    For fp32 CUDA matrices on sm_100 (large enough to pay off) each operand is split as
    ``x = hi + lo`` with ``hi, lo`` bf16 and the three products ``hi_a hi_b + hi_a lo_b +
    lo_a hi_b`` run as ONE tcgen05 GEMM over the K-concatenated splits, accumulated in fp32
    (the bf16x3 method of Henry, Tang & Heinecke 2019: about 2^-16 relative error per
    product, against TF32's 2^-11).  Other inputs use ``torch.matmul``.
    """
    from dattri_llm_b200.ops import count_launch, native, use_native

    bt = b if b_transposed else b.t()  # (N, K) logical
    m, k = a.shape
    n = bt.shape[0]
    if not (a.dim() == 2 and bt.dim() == 2 and a.dtype == torch.float32 and bt.dtype == torch.float32
            and m * n * k >= _F32_MIN_WORK and use_native(a, bt)):
        return a @ bt.t()
    count_launch(3)
    a3 = native().split3_bf16(a, 0)
    b3 = native().split3_bf16(bt, 1)
    out = torch.empty(m, n, dtype=torch.float32, device=a.device)
    gemm_tn(a3, b3, out, mode=STORE_F32)
    return out


def gemm_tn(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    alpha: float = 1.0,
    mode: int = STORE_F32,
    splits: int = 1,
    accumulate: bool = False,
) -> torch.Tensor:
    """``out (op)= alpha * a @ b^T`` on the tensor cores (bf16 in, fp32 accumulate).

    *a* is ``(M, K)`` or ``(Z, M, K)``, *b* ``(N, K)`` (shared by every batch) or
    ``(Z, N, K)``; both bf16.  *mode* selects the store: fp32, bf16, fp32 atomic
    accumulation (``splits > 1`` spreads K over CTAs) or a transposed bf16 store
    into ``out`` shaped ``(Z, N, M)``.
    """
    from dattri_llm_b200.ops import count_launch, error_word, native

    count_launch()
    a = _k_aligned(a)
    b = _k_aligned(b)
    native().gemm_tn(a, b, out, float(alpha), int(mode), int(splits), bool(accumulate),
                     error_word(a.device))
    return out


def auto_splits(m: int, n: int, k: int, batch: int = 1, bn: int = 128) -> int:
    """Split-K factor that gives roughly one CTA per SM for a thin output."""
    tiles = -(-m // 128) * -(-n // bn) * batch
    kblocks = -(-k // 64)
    if tiles >= _SMS or kblocks < 8:
        return 1
    return max(1, min(kblocks // 4, _SMS // tiles))


def matmul_tn(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.float32,
    alpha: float = 1.0,
) -> torch.Tensor:
    """``alpha * a @ b^T`` with a freshly allocated output (split-K when thin)."""
    a2 = a if a.dim() >= 2 else a.unsqueeze(0)
    lead = a2.shape[:-2]
    batch = a2.shape[0] if a2.dim() == 3 else 1
    m, n, k = a2.shape[-2], b.shape[-2], a2.shape[-1]
    shape = (*lead, m, n)
    bn = 16 if n <= 16 else 32 if n <= 32 else 64 if n <= 64 else 128 if n <= 128 else 256
    splits = auto_splits(m, n, k, batch, bn)
    if out_dtype == torch.float32 and splits > 1:
        out = torch.zeros(shape, dtype=torch.float32, device=a.device)
        gemm_tn(a2, b, out, alpha=alpha, mode=STORE_ATOMIC_F32, splits=splits)
        return out
    out = torch.empty(shape, dtype=out_dtype, device=a.device)
    mode = STORE_BF16 if out_dtype == torch.bfloat16 else STORE_F32
    gemm_tn(a2, b, out, alpha=alpha, mode=mode)
    return out


def gemm_tn_seg(a: torch.Tensor, b: torch.Tensor, seg: int, *, alpha: float = 1.0,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``(a @ b^T)`` of ``a (S*seg, K)`` and ``b (N, K)`` stored per segment as a contiguous
    ``(S, N, seg)`` bf16 tensor -- the token-major ``(B, k, T)`` layout of a projected
    activation, each sample's ``(k, T)`` block contiguous."""
    from dattri_llm_b200.ops import count_launch, error_word, native

    a = _k_aligned(a)
    b = _k_aligned(b)
    s = a.shape[0] // seg
    if out is None:
        out = torch.empty(s, b.shape[0], seg, dtype=torch.bfloat16, device=a.device)
    count_launch()
    native().gemm_tn_seg(a, b, out, float(alpha), int(seg), error_word(a.device))
    return out


def gemm_grouped(a: list[torch.Tensor], b: list[torch.Tensor], out: list[torch.Tensor], *,
                 mode: int = STORE_BF16, alpha: float = 1.0) -> list[torch.Tensor]:
    """``out[i] = alpha * a[i] @ b[i]^T`` for every job ``i`` in ONE launch (each ``a[i]``
    ``(Z, M, K)``, ``b[i]`` ``(Z, N, K)`` or ``(N, K)``; every job the same shapes).  The job
    table lives on the device and is re-uploaded only when it changes; use one stream per
    device for these calls."""
    from dattri_llm_b200.ops import count_launch, error_word, native

    if not a:
        return out
    count_launch()
    native().gemm_grouped([_k_aligned(x) for x in a], [_k_aligned(x) for x in b], out, int(mode), float(alpha),
                          error_word(a[0].device))
    return out
