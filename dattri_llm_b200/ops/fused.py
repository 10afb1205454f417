"""Autograd wrappers of the fused model-path kernels (``csrc/fused.cu``).

:func:`enabled` decides per call: bf16 CUDA tensors on sm_100 with 8-aligned
widths.  Each op is a ``torch.autograd.Function`` whose backward is the matching
fused kernel; parameter gradients (RMSNorm weight, LM-head weight) are computed
only when the parameter requires grad.
"""

from __future__ import annotations

import torch


def enabled(x: torch.Tensor) -> bool:
    """Whether the fused kernels apply to *x*."""
    from dattri_llm_b200.ops import use_native

    return x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0 and use_native(x)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()

        xc = x.contiguous()
        y, rstd = native().rmsnorm_fwd(xc, w.contiguous(), float(eps))
        ctx.save_for_backward(xc, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()

        x, w, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        dx = native().rmsnorm_bwd(dy, x, w.contiguous(), rstd) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            xhat = x.float() * rstd.view(*x.shape[:-1], 1)
            dw = (dy.float() * xhat).reshape(-1, x.shape[-1]).sum(0).to(w.dtype)
        return dx, dw, None


class _AddRMSNorm(torch.autograd.Function):
    """``h = x + delta`` (the bf16 residual stream) and ``y = rmsnorm(h) * w`` in one
    pass; the backward adds the residual gradient into the norm's input gradient, which
    both ``x`` and ``delta`` receive."""

    @staticmethod
    def forward(ctx, x, delta, w, eps):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()
        y, h, rstd = native().add_rmsnorm_fwd(x.contiguous(), delta.contiguous(), w.contiguous(), float(eps))
        ctx.save_for_backward(h, w, rstd)
        return y, h

    @staticmethod
    def backward(ctx, dy, dh):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()
        h, w, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dres = None if dh is None else dh.contiguous()
        dx = native().rmsnorm_bwd_acc(dy.contiguous(), h, w.contiguous(), rstd, dres)
        dw = None
        if ctx.needs_input_grad[2]:
            xhat = h.float() * rstd.view(*h.shape[:-1], 1)
            dw = (dy.float() * xhat).reshape(-1, h.shape[-1]).sum(0).to(w.dtype)
        return dx, dx, dw, None


class _RoPE(torch.autograd.Function):
    """Rotary position embedding of ``q (B, T, Hq, D)`` and ``k (B, T, Hk, D)`` with
    fp32 ``cos``/``sin`` tables ``(T, D/2)``; the backward rotates by ``-theta``."""

    @staticmethod
    def forward(ctx, q, k, cos, sin):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()
        ctx.save_for_backward(cos, sin)
        ctx.q_shape, ctx.k_shape = q.shape, k.shape
        qo, ko = native().rope(q, k, cos, sin, False)
        return qo, ko

    @staticmethod
    def backward(ctx, dq, dk):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()
        cos, sin = ctx.saved_tensors
        dq = torch.zeros(ctx.q_shape, dtype=torch.bfloat16, device=cos.device) if dq is None else dq
        dk = torch.zeros(ctx.k_shape, dtype=torch.bfloat16, device=cos.device) if dk is None else dk
        if dq.stride(-1) != 1:
            dq = dq.contiguous()
        if dk.stride(-1) != 1:
            dk = dk.contiguous()
        gq, gk = native().rope(dq, dk, cos, sin, True)
        return gq, gk, None, None


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()

        gc, uc = g.contiguous(), u.contiguous()
        ctx.save_for_backward(gc, uc)
        return native().swiglu_fwd(gc, uc)

    @staticmethod
    def backward(ctx, dh):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()

        g, u = ctx.saved_tensors
        dg, du = native().swiglu_bwd(dh.contiguous(), g, u)
        return dg, du


class _LinearCrossEntropy(torch.autograd.Function):
    """Sum over rows of CE(h W^T, target); bf16 logits kept for the backward, which
    rewrites them into dlogits in place (a second backward through the same graph is
    rejected).  Both GEMMs (logits and the input gradient ``dlogits @ W``) run on the
    tcgen05 CTA-pair kernel."""

    @staticmethod
    def forward(ctx, h, weight, target):
        from dattri_llm_b200.ops import count_launch, native
        from dattri_llm_b200.ops.gemm import STORE_BF16, gemm_tn

        count_launch()

        logits = torch.empty(h.shape[0], weight.shape[0], dtype=torch.bfloat16, device=h.device)
        gemm_tn(h, weight, logits, mode=STORE_BF16)
        loss, lse = native().ce_fwd(logits, target)
        ctx.logits = logits
        ctx.save_for_backward(h, weight, lse, target)
        return loss.sum()

    @staticmethod
    def backward(ctx, g):
        from dattri_llm_b200.ops import count_launch, native

        count_launch()

        h, weight, lse, target = ctx.saved_tensors
        logits = ctx.logits
        if logits is None:
            raise RuntimeError("the fused cross-entropy graph was already backpropagated "
                               "(it reuses its logits buffer in place)")
        ctx.logits = None
        native().ce_bwd_inplace(logits, lse, target, g.reshape(1).float().contiguous())
        dh = None
        if ctx.needs_input_grad[0]:
            from dattri_llm_b200.ops.gemm import STORE_BF16, gemm_tn
            from dattri_llm_b200.ops.linear import transposed

            dh = torch.empty(h.shape[0], weight.shape[1], dtype=torch.bfloat16, device=h.device)
            gemm_tn(logits, transposed(weight), dh, mode=STORE_BF16)
        dw = logits.t() @ h if ctx.needs_input_grad[1] else None
        return dh, dw, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float | None) -> torch.Tensor:
    """Fused RMSNorm over the last axis."""
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    return _RMSNorm.apply(x, weight, eps)


def add_rms_norm(x: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor,
                 eps: float | None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(rmsnorm(x + delta) * weight, x + delta)`` in one fused pass."""
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    return _AddRMSNorm.apply(x, delta, weight, eps)


def rope_enabled(q: torch.Tensor) -> bool:
    """Whether the fused RoPE kernel applies to ``q (B, T, H, D)``."""
    return (enabled(q) and q.dim() == 4 and q.shape[-1] % 16 == 0 and q.stride(-1) == 1
            and all(st % 8 == 0 for st in q.stride()[:3]) and q.data_ptr() % 16 == 0)


def rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Rotate ``q (B, T, Hq, D)``, ``k (B, T, Hk, D)`` by position (contiguous outputs)."""
    return _RoPE.apply(q, k, cos, sin)


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """Fused ``silu(g) * u``."""
    return _SwiGLU.apply(g, u)


def linear_cross_entropy(h: torch.Tensor, weight: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """``sum_i CE(h_i W^T, target_i)`` (targets ``-100`` ignored) without fp32 logits."""
    return _LinearCrossEntropy.apply(h.contiguous(), weight, target.contiguous().long())


class _GatedRMSNorm(torch.autograd.Function):
    """``bf16(w * rmsnorm(y * silu(g)))`` over the last axis (``csrc/gated_norm.cu``): y fp32,
    g bf16 (a column slice is fine), w bf16; the backward gives dy (fp32), dg (bf16) and dw."""

    @staticmethod
    def forward(ctx, y, g, w, eps):
        from dattri_llm_b200.ops import count_launch, native

        lead, d = y.shape[:-1], y.shape[-1]
        y2 = y.reshape(-1, d).contiguous()
        g2 = g.reshape(-1, d)
        if g2.stride(-1) != 1:
            g2 = g2.contiguous()
        count_launch()
        out, rstd = native().gated_rms_fwd(y2, g2, w.contiguous(), float(eps))
        ctx.save_for_backward(y2, g2, w, rstd)
        ctx.lead = lead
        return out.view(*lead, d)

    @staticmethod
    def backward(ctx, dout):
        from dattri_llm_b200.ops import count_launch, native

        y2, g2, w, rstd = ctx.saved_tensors
        d = y2.shape[-1]
        count_launch(2)
        dy, dg, dw = native().gated_rms_bwd(dout.reshape(-1, d).to(torch.bfloat16).contiguous(), y2, g2,
                                            w.contiguous(), rstd)
        return (dy.view(*ctx.lead, d), dg.view(*ctx.lead, d), dw.to(w.dtype) if ctx.needs_input_grad[2] else None,
                None)


def gated_rms_norm_enabled(y: torch.Tensor, g: torch.Tensor, w: torch.Tensor) -> bool:
    """Whether :func:`gated_rms_norm` applies: fp32 ``y``, bf16 ``g`` and ``w`` on sm_100,
    the width within the kernel's limit."""
    from dattri_llm_b200.ops import use_native

    return (y.dtype == torch.float32 and g.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and y.shape == g.shape and y.shape[-1] == w.numel() and y.shape[-1] <= 8192 and use_native(y, g, w))


def gated_rms_norm(y: torch.Tensor, g: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """``bf16(w * rmsnorm(y * silu(g)))``: the Mamba2 mixer's gated norm and its cast to the
    model dtype in one kernel each way."""
    return _GatedRMSNorm.apply(y, g, w, eps)


class _SSDIntra(torch.autograd.Function):
    """Intra-chunk SSD mixing (``csrc/ssd.cu``): ``y[b,c,s,h] = sum_{t<=s} cb[b,g,c,s,t]
    exp(cum[b,h,c,s] - cum[b,h,c,t]) x[b,c,t,h]`` with the decayed matrix never stored."""

    @staticmethod
    def forward(ctx, cb, cum, x):
        from dattri_llm_b200.ops import count_launch, native

        cb, cum, x = cb.contiguous(), cum.contiguous(), x.contiguous()
        count_launch()
        y = native().ssd_intra_fwd(cb, cum, x)
        ctx.save_for_backward(cb, cum, x)
        return y

    @staticmethod
    def backward(ctx, dy):
        from dattri_llm_b200.ops import count_launch, native

        cb, cum, x = ctx.saved_tensors
        count_launch(2)
        dcb, dcum, dx = native().ssd_intra_bwd(cb, cum, x, dy.contiguous().float())
        return dcb, dcum, dx


def ssd_intra_enabled(x: torch.Tensor, chunk: int) -> bool:
    """Whether :func:`ssd_intra` applies: fp32 CUDA on sm_100, head dim 64, chunk a multiple of 64."""
    from dattri_llm_b200.ops import use_native

    return x.dtype == torch.float32 and x.shape[-1] == 64 and chunk % 64 == 0 and use_native(x)


def ssd_intra(cb: torch.Tensor, cum: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Fused intra-chunk SSD: *cb* ``(B, G, C, S, S)`` group-level ``C_s . B_t``, *cum*
    ``(B, H, C, S)`` cumulative log-decay per chunk, *x* ``(B, C, S, H, P)``; returns ``y``
    like *x* (fp32)."""
    return _SSDIntra.apply(cb, cum, x)


class _CausalConvSiLU(torch.autograd.Function):
    """``silu(causal depthwise conv1d(x))`` over the token axis of a ``(B, L, C)`` bf16 tensor
    (``csrc/conv1d.cu``); weight ``(C, 1, 4)``, optional bias ``(C)``."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        from dattri_llm_b200.ops import count_launch, native

        w = weight.contiguous()
        count_launch()
        out = native().causal_conv_silu_fwd(x, w, bias)
        ctx.save_for_backward(x, w, bias)
        return out

    @staticmethod
    def backward(ctx, dout):
        from dattri_llm_b200.ops import count_launch, native

        x, w, bias = ctx.saved_tensors
        count_launch(3)
        dx, dw, db = native().causal_conv_silu_bwd(dout.to(torch.bfloat16).contiguous(), x, w, bias)
        dw = dw.view_as(w).to(w.dtype) if ctx.needs_input_grad[1] else None
        db = db.to(bias.dtype) if bias is not None and ctx.needs_input_grad[2] else None
        return dx, dw, db


def causal_conv_silu_enabled(x: torch.Tensor, conv) -> bool:
    """Whether :func:`causal_conv_silu` computes *conv* (an ``nn.Conv1d``) on ``x (B, L, C)``:
    depthwise, 4 taps, causal padding, bf16 on sm_100, even channel count and offsets."""
    from dattri_llm_b200.ops import use_native

    w = conv.weight
    return (x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 3 and x.stride(2) == 1
            and conv.groups == conv.in_channels == conv.out_channels == x.shape[2] and tuple(w.shape[1:]) == (1, 4)
            and tuple(conv.padding) == (3,) and tuple(conv.stride) == (1,) and tuple(conv.dilation) == (1,)
            and (conv.bias is None or conv.bias.dtype == torch.bfloat16) and x.shape[2] % 2 == 0
            and x.stride(1) % 2 == 0 and x.stride(0) % 2 == 0 and x.data_ptr() % 4 == 0 and use_native(x, w))


def causal_conv_silu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """``silu(conv1d(x^T, weight, bias, padding=3, groups=C)[..., :L])^T`` token-major, one kernel
    each way (the Mamba2 mixer's convolution and activation)."""
    return _CausalConvSiLU.apply(x, weight, bias)
