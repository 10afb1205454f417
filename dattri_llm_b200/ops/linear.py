"""Dense layers on the tcgen05 CTA-pair GEMM, with the capture projections riding along.

``linear(x, weight)`` is ``x @ weight^T`` whose forward and input-gradient GEMMs run on the
library's kernel (bf16 in, fp32 accumulate, bf16 out).  The input-gradient GEMM
``dy @ weight`` needs ``weight^T`` K-major; it is transposed once per weight version and
cached (frozen checkpoints are transposed once per run).

Capture fusion: the a-side LoGra projection of a layer is ``x @ P_a`` and its g-side
projection ``dy @ P_g``, where ``x`` and ``dy`` are exactly the A operands of the layer's
forward and input-gradient GEMMs.  With ``tail_t = P_a^T`` the forward appends ``P_a``'s
columns to the weight's as a narrow last column tile of the SAME launch and stores them
token-major ``(B, k, T)`` -- one read of ``x`` for both.  In the backward, a
:class:`CaptureSlot` whose ``grad_tail_t = P_g^T`` is set makes the input-gradient GEMM
emit ``(B, k, T)`` projected output gradients the same way, handed to ``slot.sink``.  The
capture hooks (``gradient/hooks/hooks.py``) fill the slot; without hooks the op is a plain
linear layer.  Reference hot sites replaced: ``dattri_llm/gradient/hooks/hooks.py:369-375``
(a-side ``addmm`` in the forward hook) and ``:631-634`` (g-side in the backward hook), plus
the cuBLAS GEMMs of the model itself.
"""

from __future__ import annotations

import weakref

import torch

_WT_CACHE: dict[int, tuple] = {}  # id(weight) -> (weak ref, version key, weight^T)
_FUSED_CAPTURE = [True]


def set_fused_capture(enabled: bool) -> bool:
    """Let fused-capture layers compute the capture projections inside their GEMMs
    (default) or leave them to the hooks' own projection launches; returns the old value."""
    old, _FUSED_CAPTURE[0] = _FUSED_CAPTURE[0], bool(enabled)
    return old


def fused_capture_enabled() -> bool:
    """Whether fused-capture layers project inside their GEMMs."""
    return _FUSED_CAPTURE[0]


def transposed(weight: torch.Tensor) -> torch.Tensor:
    """``weight^T`` contiguous (the K-major operand of ``dy @ weight``), cached per version.

    Keyed by the tensor's identity (checked through a weak reference, and dropped when the
    weight is freed); a new version, storage or shape recomputes it."""
    key = (weight._version, weight.data_ptr(), tuple(weight.shape), weight.dtype)
    hit = _WT_CACHE.get(id(weight))
    if hit is not None and hit[0]() is weight and hit[1] == key:
        return hit[2]
    from dattri_llm_b200.ops.gemm import transpose_last2

    wt = transpose_last2(weight.detach())
    if hit is None or hit[0]() is not weight:
        weakref.finalize(weight, _WT_CACHE.pop, id(weight), None)
    _WT_CACHE[id(weight)] = (weakref.ref(weight), key, wt)
    return wt


def supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether :func:`linear` runs natively: bf16 CUDA operands on sm_100, widths 8-aligned."""
    from dattri_llm_b200.ops import use_native

    return (x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0
            and weight.shape[0] % 8 == 0 and x.is_cuda and use_native(x, weight))


class CaptureSlot:
    """Per-call link between a fused linear's backward and the capture hooks.

    ``grad_tail_t``: ``P_g^T (k, d_out)`` to project the output gradient with inside the
    input-gradient GEMM (``None``: no g-side capture); ``sink(g_pt)``: receives the
    ``(B, k, T)`` token-major projected output gradient; ``seg``: tokens per sample."""

    __slots__ = ("grad_tail_t", "seg", "sink")

    def __init__(self, seg: int) -> None:
        self.grad_tail_t: torch.Tensor | None = None
        self.sink = None
        self.seg = seg


def _gemm_bf16(a2: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``out (M, N) = a2 @ b^T`` (bf16); *out* may be the 2-D view of a larger-rank buffer."""
    from dattri_llm_b200.ops.gemm import STORE_BF16, gemm_tn

    gemm_tn(a2, b, out, mode=STORE_BF16)
    return out


def gemm_with_tail(a2: torch.Tensor, b: torch.Tensor, tail_t: torch.Tensor, seg: int,
                   out: torch.Tensor | None = None):
    """``(a2 @ b^T, (a2 @ tail_t^T) token-major (M / seg, k, seg))`` -- one launch when ``b``'s
    rows are a multiple of 256, else the main GEMM and a segmented projection GEMM.  *out*
    (``(M, N)`` bf16, optional) receives the main product."""
    from dattri_llm_b200.ops import count_launch, error_word, native
    from dattri_llm_b200.ops.gemm import gemm_tn_seg

    m, n, k = a2.shape[0], b.shape[0], tail_t.shape[0]
    y = out if out is not None else torch.empty(m, n, dtype=torch.bfloat16, device=a2.device)
    if n % 256 == 0 and k <= 256 and m % seg == 0:
        t = torch.empty(m // seg, k, seg, dtype=torch.bfloat16, device=a2.device)
        count_launch()
        native().gemm_tn_tail(a2, b, tail_t, y, t, int(seg), error_word(a2.device))
        return y, t
    return _gemm_bf16(a2, b, y), gemm_tn_seg(a2, tail_t, seg)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, tail_t, slot):
        lead, d_in = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, d_in)
        if x2.stride(-1) != 1 or x2.stride(0) != d_in:
            x2 = x2.contiguous()
        y = torch.empty(*lead, weight.shape[0], dtype=torch.bfloat16, device=x.device)
        y2 = y.view(-1, weight.shape[0])
        a_pt = None
        if tail_t is not None:
            a_pt = gemm_with_tail(x2, weight, tail_t, slot.seg, out=y2)[1]
        else:
            _gemm_bf16(x2, weight, y2)
        ctx.save_for_backward(x2 if weight.requires_grad else None, weight)
        ctx.slot, ctx.lead, ctx.d_in = slot, lead, d_in
        if a_pt is not None:
            ctx.mark_non_differentiable(a_pt)
        return y, a_pt

    @staticmethod
    def backward(ctx, dy, _da):
        x2, weight = ctx.saved_tensors
        slot = ctx.slot
        n = weight.shape[0]
        dy2 = dy.reshape(-1, n)
        if dy2.stride(-1) != 1 or dy2.stride(0) != n:
            dy2 = dy2.contiguous()
        dx = dw = None
        tail = slot.grad_tail_t if slot is not None else None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(*ctx.lead, ctx.d_in, dtype=torch.bfloat16, device=dy.device)
            dx2 = dx.view(-1, ctx.d_in)
            if tail is not None:
                g_pt = gemm_with_tail(dy2, transposed(weight), tail, slot.seg, out=dx2)[1]
            else:
                _gemm_bf16(dy2, transposed(weight), dx2)
                g_pt = None
        elif tail is not None:
            from dattri_llm_b200.ops.gemm import gemm_tn_seg

            g_pt = gemm_tn_seg(dy2, tail, slot.seg)
        else:
            g_pt = None
        if g_pt is not None and slot.sink is not None:
            slot.sink(g_pt)
        if ctx.needs_input_grad[1]:
            dw = torch.mm(dy2.t(), x2)  # weight gradient (trajectory runs only; the frozen probe skips it)
        return dx, dw, None, None


def linear(x: torch.Tensor, weight: torch.Tensor, *, tail_t: torch.Tensor | None = None,
           slot: CaptureSlot | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``(x @ weight^T, projected x or None)``; see the module docstring.  *x* is
    ``(..., d_in)`` bf16; with *tail_t* ``(k, d_in)`` the second result is the
    ``(B, k, T)`` token-major ``x @ tail_t^T`` (*slot* gives T)."""
    if tail_t is not None and slot is None:
        raise ValueError("a projection tail needs a CaptureSlot (it carries the segment length)")
    return _Linear.apply(x, weight, tail_t, slot)
