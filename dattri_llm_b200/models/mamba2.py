"""Mamba2 (state-space duality) forward for Hugging Face ``Mamba2`` models, memory-bounded.

The Hugging Face model falls back, without the ``mamba_ssm`` kernels, to a "naive" SSD
that broadcasts ``(batch, chunks, chunk, chunk, heads, head_dim)`` products before
reducing them -- 40 GB per layer for four 2,048-token sequences of the 2.7B architecture,
so training runs out of memory at any useful batch.  :func:`ssd_chunked` computes the same
chunked SSD (Dao & Gu 2024, "Transformers are SSMs", Listing 1) as batched matrix
products: per chunk, the causal ``(C B^T) . L`` mixing applied to ``x dt``, per-chunk end
states, the inter-chunk recurrence, and the states' contribution to each position.  The
products that involve only B and C are formed once per group (Mamba2-2.7B has one group for
its 80 heads), not once per head, and each head's intra-chunk decay is one exponential of
cumulative-sum differences.  Its largest intermediate is one ``(batch, heads, chunks, chunk,
chunk)`` fp32 tensor; above 2,048 tokens per call the scan is recomputed in the backward,
so only its inputs are kept per layer.

:func:`accelerate_mamba2` installs that forward on every ``Mamba2Mixer`` of a model (the
cache-free training / scoring call; decoding keeps the library's path) and moves the
model's bias-free linears onto the library's tcgen05 kernels (:func:`tc_linearize`).
Parameters, module names and hook points are unchanged: ``in_proj``, ``conv1d`` and
``out_proj`` are still called as modules, so capture hooks see them as before.
"""

from __future__ import annotations

import contextlib
import types

import torch
import torch.nn.functional as F
from torch import nn
from torch.utils.checkpoint import checkpoint

from dattri_llm_b200.models.layers import tc_linearize
from dattri_llm_b200.ops import fused


def _segment_sums(a: torch.Tensor) -> torch.Tensor:
    """``out[..., i, j] = a[..., j+1] + ... + a[..., i]`` for ``i >= j`` (``-inf`` above the
    diagonal): the log-decay from position ``j`` to ``i``.  Summed as a masked cumulative sum,
    so no large cumulative values are subtracted (used across chunks, where the totals grow)."""
    n = a.shape[-1]
    lower = torch.ones(n, n, dtype=torch.bool, device=a.device).tril(-1)
    spread = a[..., None].expand(*a.shape, n).masked_fill(~lower, 0)
    sums = spread.cumsum(dim=-2)
    return sums.masked_fill(~torch.ones(n, n, dtype=torch.bool, device=a.device).tril(), float("-inf"))


def _causal_decay(cum: torch.Tensor) -> torch.Tensor:
    """``exp(cum[..., i] - cum[..., j])`` for ``i >= j``, 0 above the diagonal: the decay from
    position ``j`` to ``i`` inside one chunk, from the chunk's cumulative log-decay (one pass;
    within a chunk the cumulative values stay small enough for the difference)."""
    n = cum.shape[-1]
    upper = torch.ones(n, n, dtype=torch.bool, device=cum.device).triu(1)
    return (cum[..., :, None] - cum[..., None, :]).masked_fill_(upper, float("-inf")).exp_()


@contextlib.contextmanager
def _tf32_products():
    """fp32 matrix products on TF32 tensor cores inside the block (fp32 accumulation; the
    precision the SSD chunk products of the reference Mamba2 kernels use), the previous
    setting restored after it."""
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous


def _swap(eq: str) -> tuple[str, str]:
    """For ``"A,B->C"`` with every index in two of the three terms: the equations of ``dA``
    (``"C,B->A"``) and ``dB`` (``"A,C->B"``)."""
    lhs, out = eq.split("->")
    a, b = lhs.split(",")
    return f"{out},{b}->{a}", f"{a},{out}->{b}"


class _TF32Product(torch.autograd.Function):
    """A two-operand fp32 einsum whose forward and backward products run on TF32 tensor
    cores (the chunk-state products of the SSD scan: batched GEMMs of 5,120 x 128 x 256 per
    chunk that fp32 CUDA-core kernels run an order of magnitude slower)."""

    @staticmethod
    def forward(ctx, eq, a, b):
        ctx.eq = eq
        ctx.save_for_backward(a, b)
        with _tf32_products():
            return torch.einsum(eq, a, b)

    @staticmethod
    def backward(ctx, dout):
        a, b = ctx.saved_tensors
        eq_a, eq_b = _swap(ctx.eq)
        with _tf32_products():
            da = torch.einsum(eq_a, dout, b) if ctx.needs_input_grad[1] else None
            db = torch.einsum(eq_b, a, dout) if ctx.needs_input_grad[2] else None
        return None, da, db


def _product(eq: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``einsum(eq, a, b)``, on TF32 tensor cores for fp32 CUDA operands."""
    if a.is_cuda and a.dtype == torch.float32 and b.dtype == torch.float32:
        return _TF32Product.apply(eq, a, b)
    return torch.einsum(eq, a, b)


def ssd_chunked(x: torch.Tensor, dt: torch.Tensor, a_head: torch.Tensor, b: torch.Tensor, c: torch.Tensor,
                chunk: int) -> torch.Tensor:
    """The SSD scan ``h_t = exp(dt_t A) h_{t-1} + dt_t B_t x_t^T``, ``y_t = h_t C_t`` (fp32).

    Args:
        x: ``(batch, length, heads, head_dim)``.
        dt: ``(batch, length, heads)``, already softplus'ed and clamped.
        a_head: ``(heads,)``, negative.
        b, c: ``(batch, length, groups, state)``; ``heads`` is a multiple of ``groups`` and
            head ``h`` reads group ``h // (heads // groups)``.  The group-level products
            (``C B^T``, ``C`` against the states) are formed once per group, not per head.
        chunk: chunk length.

    Returns:
        ``(batch, length, heads, head_dim)``.
    """
    bsz, length, heads, hd = x.shape
    groups = b.shape[2]
    rep = heads // groups
    pad = (-length) % chunk
    xdt = x * dt[..., None]
    log_a = a_head * dt  # (batch, length, heads)
    if pad:
        xdt, b, c = (F.pad(t, (0, 0, 0, 0, 0, pad)) for t in (xdt, b, c))
        log_a = F.pad(log_a, (0, 0, 0, pad))
    n_chunks = (length + pad) // chunk
    xdt = xdt.reshape(bsz, n_chunks, chunk, groups, rep, hd)
    b = b.reshape(bsz, n_chunks, chunk, groups, -1)
    c = c.reshape(bsz, n_chunks, chunk, groups, -1)
    cum = log_a.reshape(bsz, n_chunks, chunk, groups, rep).permute(0, 3, 4, 1, 2).cumsum(dim=-1)  # (b,g,r,c,s)
    # 1. within each chunk: (C B^T) per group, times each head's causal decay, applied to x dt
    cb = torch.einsum("bcsgn,bctgn->bgcst", c, b)
    if fused.ssd_intra_enabled(xdt, chunk):  # the decayed (chunk x chunk) matrices stay on chip
        y = fused.ssd_intra(cb, cum.reshape(bsz, heads, n_chunks, chunk),
                            xdt.reshape(bsz, n_chunks, chunk, heads, hd)).view(xdt.shape)
    else:
        mix = cb[:, :, None] * _causal_decay(cum)                      # (b, g, r, c, s, t)
        y = torch.einsum("bgrcst,bctgrp->bcsgrp", mix, xdt)
        del mix
    del cb
    # 2. each chunk's end state from its own inputs (the decay applied to x dt, not to B)
    to_end = torch.exp(cum[..., -1:] - cum)                            # (b, g, r, c, s)
    states = _product("bctgrp,bctgn->bcgrpn", xdt * to_end.permute(0, 3, 4, 1, 2)[..., None], b)
    # 3. carry states across chunk boundaries
    states = torch.cat([torch.zeros_like(states[:, :1]), states], dim=1)
    across = torch.exp(_segment_sums(F.pad(cum[..., -1], (1, 0))))    # (b, g, r, c+1, c+1)
    states = _product("bgrzc,bcgrpn->bzgrpn", across, states)[:, :-1]
    # 4. the incoming state's contribution to every position of the chunk
    from_start = torch.exp(cum).permute(0, 3, 4, 1, 2)[..., None]      # (b, c, s, g, r, 1)
    y = y + _product("bcsgn,bcgrpn->bcsgrp", c, states) * from_start
    y = y.reshape(bsz, n_chunks * chunk, heads, hd)
    return y[:, :length] if pad else y


def _scan_with_skip(x, dt, a_head, b_groups, c_groups, d_skip, chunk: int) -> torch.Tensor:
    """``ssd_chunked(...) + D x`` with B and C given per group ``(batch, length, groups, state)``."""
    return ssd_chunked(x, dt, a_head, b_groups, c_groups, chunk) + d_skip[:, None] * x


# A scan over more tokens than this keeps only its inputs and is recomputed in the backward;
# below it the (chunk x chunk) intermediates of all layers fit next to the model.
_RECOMPUTE_TOKENS = 2048


def _mixer_forward(self, hidden_states: torch.Tensor, cache_params=None, attention_mask=None, **kwargs):
    """``Mamba2Mixer.forward`` for the cache-free call, through :func:`ssd_chunked`."""
    masked = attention_mask is not None and not bool(attention_mask.all())
    if cache_params is not None or masked:
        return type(self).forward(self, hidden_states, cache_params=cache_params, attention_mask=attention_mask,
                                  **kwargs)
    bsz, length, _ = hidden_states.shape
    dtype = hidden_states.dtype
    projected = self.in_proj(hidden_states)
    groups_state = self.n_groups * self.ssm_state_size
    d_mlp = (projected.shape[-1] - 2 * self.intermediate_size - 2 * groups_state - self.num_heads) // 2
    _, _, gate, xbc, dt = projected.split([d_mlp, d_mlp, self.intermediate_size, self.conv_dim, self.num_heads],
                                          dim=-1)
    conv = self.conv1d
    if (self.activation in ("silu", "swish") and not (conv._forward_hooks or conv._forward_pre_hooks
                                                     or conv._backward_hooks)
            and fused.causal_conv_silu_enabled(xbc, conv)):
        xbc = fused.causal_conv_silu(xbc, conv.weight, conv.bias)  # nothing watches the convolution
    else:
        xbc = self.act(conv(xbc.transpose(1, 2))[..., :length].transpose(1, 2))
    x, b, c = xbc.split([self.intermediate_size, groups_state, groups_state], dim=-1)
    a_head = -torch.exp(self.A_log.float())
    dt = F.softplus(dt + self.dt_bias).clamp(self.time_step_limit[0], self.time_step_limit[1]).float()
    x = x.reshape(bsz, length, self.num_heads, self.head_dim).float()
    b = b.reshape(bsz, length, self.n_groups, self.ssm_state_size).float()
    c = c.reshape(bsz, length, self.n_groups, self.ssm_state_size).float()
    args = (x, dt, a_head, b, c, self.D, self.chunk_size)
    if torch.is_grad_enabled() and bsz * length > _RECOMPUTE_TOKENS:
        # the scan's (chunk x chunk) intermediates are rebuilt in the backward instead of
        # being kept for all layers at once: only the scan's inputs stay alive
        y = checkpoint(_scan_with_skip, *args, use_reentrant=False)
    else:
        y = _scan_with_skip(*args)
    y = y.reshape(bsz, length, -1)
    norm = self.norm
    if (dtype == torch.bfloat16 and not (norm._forward_hooks or norm._forward_pre_hooks or norm._backward_hooks)
            and fused.gated_rms_norm_enabled(y, gate, norm.weight)):
        scanned = fused.gated_rms_norm(y, gate, norm.weight, norm.variance_epsilon)  # nothing watches the norm
    else:
        scanned = norm(y, gate).to(dtype)
    return self.out_proj(scanned)


def accelerate_mamba2(model: nn.Module, *, linears: bool = True) -> int:
    """Install :func:`ssd_chunked` on every ``Mamba2Mixer`` of *model* (and, with *linears*,
    put its bias-free linears on the tcgen05 kernels).  Returns the number of mixers."""
    from transformers.models.mamba2.modeling_mamba2 import Mamba2Mixer

    mixers = [m for m in model.modules() if isinstance(m, Mamba2Mixer)]
    for mixer in mixers:
        mixer.forward = types.MethodType(_mixer_forward, mixer)
    if linears:
        tc_linearize(model)
    return len(mixers)
