"""Mamba2 (state-space duality) forward for Hugging Face ``Mamba2`` models, memory-bounded.

The Hugging Face model falls back, without the ``mamba_ssm`` kernels, to a "naive" SSD
that broadcasts ``(batch, chunks, chunk, chunk, heads, head_dim)`` products before
reducing them -- 40 GB per layer for four 2,048-token sequences of the 2.7B architecture,
so training runs out of memory at any useful batch.  :func:`ssd_chunked` computes the same
chunked SSD (Dao & Gu 2024, "Transformers are SSMs", Listing 1) as batched matrix
products: per chunk, the causal ``(C B^T) . L`` mixing applied to ``x dt``, per-chunk end
states, the inter-chunk recurrence, and the states' contribution to each position.  Its
largest intermediate is one ``(batch, heads, chunks, chunk, chunk)`` fp32 tensor, and in a
training step the scan is recomputed in the backward, so only its inputs are kept per
layer.

:func:`accelerate_mamba2` installs that forward on every ``Mamba2Mixer`` of a model (the
cache-free training / scoring call; decoding keeps the library's path) and moves the
model's bias-free linears onto the library's tcgen05 kernels (:func:`tc_linearize`).
Parameters, module names and hook points are unchanged: ``in_proj``, ``conv1d`` and
``out_proj`` are still called as modules, so capture hooks see them as before.
"""

from __future__ import annotations

import types

import torch
import torch.nn.functional as F
from torch import nn
from torch.utils.checkpoint import checkpoint

from dattri_llm_b200.models.layers import tc_linearize


def _segment_sums(a: torch.Tensor) -> torch.Tensor:
    """``out[..., i, j] = a[..., j+1] + ... + a[..., i]`` for ``i >= j`` (``-inf`` above the
    diagonal): the log-decay from position ``j`` to ``i`` of one chunk.  Summed as a masked
    cumulative sum, so no large cumulative values are subtracted."""
    n = a.shape[-1]
    lower = torch.ones(n, n, dtype=torch.bool, device=a.device).tril(-1)
    spread = a[..., None].expand(*a.shape, n).masked_fill(~lower, 0)
    sums = spread.cumsum(dim=-2)
    return sums.masked_fill(~torch.ones(n, n, dtype=torch.bool, device=a.device).tril(), float("-inf"))


def ssd_chunked(x: torch.Tensor, dt: torch.Tensor, a_head: torch.Tensor, b: torch.Tensor, c: torch.Tensor,
                chunk: int) -> torch.Tensor:
    """The SSD scan ``h_t = exp(dt_t A) h_{t-1} + dt_t B_t x_t^T``, ``y_t = h_t C_t`` (fp32).

    Args:
        x: ``(batch, length, heads, head_dim)``.
        dt: ``(batch, length, heads)``, already softplus'ed and clamped.
        a_head: ``(heads,)``, negative.
        b, c: ``(batch, length, heads, state)``.
        chunk: chunk length.

    Returns:
        ``(batch, length, heads, head_dim)``.
    """
    bsz, length, heads, _hd = x.shape
    pad = (-length) % chunk
    xdt = x * dt[..., None]
    log_a = a_head * dt  # (batch, length, heads)
    if pad:
        xdt, b, c = (F.pad(t, (0, 0, 0, 0, 0, pad)) for t in (xdt, b, c))
        log_a = F.pad(log_a, (0, 0, 0, pad))
    n_chunks = (length + pad) // chunk

    def chunked(t):  # (batch, length, ...) -> (batch, chunks, chunk, ...)
        return t.reshape(bsz, n_chunks, chunk, *t.shape[2:])

    xdt, b, c = chunked(xdt), chunked(b), chunked(c)
    log_a = chunked(log_a).permute(0, 3, 1, 2)          # (batch, heads, chunks, chunk)
    cum = log_a.cumsum(dim=-1)
    # 1. within each chunk: causal (C B^T) . decay, applied to x dt
    mix = torch.einsum("bcihn,bcjhn->bhcij", c, b) * torch.exp(_segment_sums(log_a))
    y = torch.einsum("bhcij,bcjhp->bcihp", mix, xdt)
    del mix
    # 2. each chunk's end state from its own inputs
    to_end = torch.exp(cum[..., -1:] - cum)              # (batch, heads, chunks, chunk)
    b_weighted = b * to_end.permute(0, 2, 3, 1)[..., None]
    states = torch.einsum("bcjhn,bcjhp->bchpn", b_weighted, xdt)
    # 3. carry states across chunk boundaries
    states = torch.cat([torch.zeros_like(states[:, :1]), states], dim=1)
    across = torch.exp(_segment_sums(F.pad(cum[..., -1], (1, 0))))  # (batch, heads, chunks+1, chunks+1)
    states = torch.einsum("bhzc,bchpn->bzhpn", across, states)[:, :-1]
    # 4. the incoming state's contribution to every position of the chunk
    from_start = torch.exp(cum).permute(0, 2, 3, 1)     # (batch, chunks, chunk, heads)
    y = y + torch.einsum("bcihn,bchpn->bcihp", c, states) * from_start[..., None]
    y = y.reshape(bsz, n_chunks * chunk, heads, -1)
    return y[:, :length] if pad else y


def _scan_with_skip(x, dt, a_head, b_groups, c_groups, d_skip, chunk: int) -> torch.Tensor:
    """``ssd_chunked(...) + D x`` with B and C given per group ``(batch, length, groups, state)``
    and widened to the heads here (recomputed in the backward, so never kept)."""
    heads = x.shape[2]
    b = b_groups.repeat_interleave(heads // b_groups.shape[2], dim=2)
    c = c_groups.repeat_interleave(heads // c_groups.shape[2], dim=2)
    return ssd_chunked(x, dt, a_head, b, c, chunk) + d_skip[:, None] * x


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
    xbc = self.act(self.conv1d(xbc.transpose(1, 2))[..., :length].transpose(1, 2))
    x, b, c = xbc.split([self.intermediate_size, groups_state, groups_state], dim=-1)
    a_head = -torch.exp(self.A_log.float())
    dt = F.softplus(dt + self.dt_bias).clamp(self.time_step_limit[0], self.time_step_limit[1]).float()
    x = x.reshape(bsz, length, self.num_heads, self.head_dim).float()
    b = b.reshape(bsz, length, self.n_groups, self.ssm_state_size).float()
    c = c.reshape(bsz, length, self.n_groups, self.ssm_state_size).float()
    args = (x, dt, a_head, b, c, self.D, self.chunk_size)
    if torch.is_grad_enabled():
        # the scan's (chunk x chunk) intermediates are rebuilt in the backward instead of
        # being kept for all layers at once: only the scan's inputs stay alive
        y = checkpoint(_scan_with_skip, *args, use_reentrant=False)
    else:
        y = _scan_with_skip(*args)
    scanned = self.norm(y.reshape(bsz, length, -1), gate)
    return self.out_proj(scanned.to(dtype))


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
