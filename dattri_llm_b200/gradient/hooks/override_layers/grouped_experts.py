"""Grouped capture of a fused-experts MoE block (sm_100a kernels on the GPU, PyTorch on the CPU).

The per-expert capture (:mod:`.fused_experts`) runs every routed expert through its own pair
of hookable proxies: ``2 E`` small GEMMs per block in the forward and as many in the
backward, each followed by row matching, a projection and a per-sample contraction -- for an
OLMoE-size model thousands of launches and host round trips per step, with the GPU idle
between them.  When every expert projection of a block is captured with one LoGra
projection and materialized (the ``auto`` / ``materialized`` capture styles at the block's
sequence length), the block runs instead as ONE autograd function:

forward   the (token, slot) rows sorted by expert with a stable device sort (no host
          synchronization), one ragged tcgen05 GEMM for every expert's gate/up projection,
          the model's own gate, one ragged down GEMM whose epilogue stores each row at its
          (token, slot) position, and the fp32-weighted combine;
capture   the gate/up input is projected once per token (``x P_a``) and gathered per slot;
          the down input and both output gradients are projected per slot row; every
          (expert, sample)'s ``sum_t g_p^T a_p`` comes from ONE batched GEMM over a
          token-indexed, zero-padded layout -- the contraction the per-expert path runs
          on its regrouped ``(B, T, k)`` factors;
backward  the combine's backward fused with placing the slot gradients in expert order
          (router-weight gradients from the same pass), two ragged GEMMs against the
          experts' transposed weights (built once per weight version), the gate's backward
          through autograd.

Each expert's ``(B, k_g * k_a)`` block reaches the capture manager under the per-expert
proxy names (``<experts>.dattri_experts.<e>.gate_up`` / ``.down``), so a store reads the
same whichever path wrote it; an expert no token of the step reached has zero rows.
Trainable expert weights, other projection styles, preconditioning, offload, callbacks
that watch individual layers, and recomputation inside a backward take the per-expert path.
The reference has no counterpart: it always loops over experts
(``dattri_llm/gradient/hooks/override_layers/fused_experts.py``).
"""

from __future__ import annotations

import torch

_ENABLED = [True]


def set_grouped_experts(enabled: bool) -> bool:
    """Allow (default) or forbid the grouped path; returns the previous setting."""
    previous = _ENABLED[0]
    _ENABLED[0] = bool(enabled)
    return previous


class _Plan:
    """Routing of one call: the (token, slot) rows in expert order and the ragged-GEMM tables."""

    def __init__(self, index: torch.Tensor, n_experts: int, batch: int, tokens: int) -> None:
        flat = index.reshape(-1)
        self.rows, self.k = flat.numel(), index.shape[1]
        experts_sorted, order = torch.sort(flat, stable=True)
        self.order = order                                   # slot row of sorted row r
        self.tok = torch.div(order, self.k, rounding_mode="floor")
        self.inverse = torch.empty_like(order)
        self.inverse[order] = torch.arange(self.rows, device=flat.device)
        counts = torch.bincount(flat, minlength=n_experts)[:n_experts]
        self.lens = counts.to(torch.int32)
        self.base = (torch.cumsum(counts, 0) - counts).to(torch.int32)
        tiles = torch.div(counts + 255, 256, rounding_mode="floor")
        self.prefix = torch.zeros(n_experts + 1, dtype=torch.int32, device=flat.device)
        self.prefix[1:] = torch.cumsum(tiles, 0)
        self.max_tiles = (self.rows + 255) // 256 + n_experts  # bound: each job rounds up once
        home = torch.zeros(self.rows, 2, dtype=torch.int32, device=flat.device)
        home[:, 1] = order
        self.home = home                                     # (rank 0, slot row) of sorted row r
        self.segment = experts_sorted * batch + torch.div(self.tok, tokens, rounding_mode="floor")
        self.position = self.tok % tokens
        self.n_experts, self.batch, self.tokens = n_experts, batch, tokens


class _NativeKernels:
    """The sm_100a kernels of the grouped path (bf16 CUDA tensors)."""

    @staticmethod
    def ragged(a, b3, plan, out=None, home_of=None):
        """``out[r] = a[r] @ b3[expert(r)]^T`` over the plan's expert segments; with
        *home_of* the epilogue stores row r at row ``order[r]`` of *home_of* instead."""
        from dattri_llm_b200 import ops

        ops.count_launch()
        err = ops.error_word(a.device)
        if home_of is None:
            ops.native().gemm_ragged(a, b3, out, plan.prefix, plan.base, plan.lens, plan.max_tiles, [], None, err)
            return out
        ops.native().gemm_ragged(a, b3, None, plan.prefix, plan.base, plan.lens, plan.max_tiles, [home_of],
                                 plan.home, err)
        return home_of

    @staticmethod
    def combine(slots, w32, out):
        """``out[t] = sum_j w32[t, j] slots[t * k + j]`` (fp32 sums)."""
        from dattri_llm_b200 import ops

        ops.count_launch()
        ops.native().moe_combine(slots, w32, out)
        return out

    @staticmethod
    def combine_backward(dy, slots, w32, plan):
        """``(g in expert order, dw)``: ``g[inverse[s]] = w32[s] dy[token(s)]`` and
        ``dw[s] = <dy[token(s)], slots[s]>``, from one pass over ``dy``."""
        from dattri_llm_b200 import ops

        g = dy.new_empty(plan.rows, dy.shape[1])
        dw = torch.empty_like(w32)
        origin = torch.empty(plan.rows, 2, dtype=torch.int32, device=dy.device)
        ops.count_launch()
        ops.native().moe_combine_bwd_dispatch(dy, slots, w32, dw, torch.zeros(plan.rows, dtype=torch.int32, device=dy.device),
                                              plan.inverse.to(torch.int32), [g], [origin], 0)
        return g, dw

    @staticmethod
    def outer(g_t, a_t):
        """``(S, k_g, k_a) = g_t @ a_t^T`` of token-major ``(S, k, T)`` factors (bf16 out)."""
        from dattri_llm_b200 import ops

        return ops.per_sample_outer(None, None, out_dtype=torch.bfloat16, left_t=g_t, right_t=a_t)

    @staticmethod
    def transpose(w):
        from dattri_llm_b200.ops import transpose_last2

        return transpose_last2(w)


class _TorchKernels:
    """The same steps in PyTorch (CPU tensors, any floating dtype)."""

    @staticmethod
    def ragged(a, b3, plan, out=None, home_of=None):
        res = a.new_empty(a.shape[0], b3.shape[1])
        for e, (start, n) in enumerate(zip(plan.base.tolist(), plan.lens.tolist(), strict=True)):
            if n:
                res[start:start + n] = a[start:start + n] @ b3[e].t()
        if home_of is None:
            out.copy_(res)
            return out
        home_of[plan.order] = res
        return home_of

    @staticmethod
    def combine(slots, w32, out):
        n, k = w32.shape
        out.copy_((slots[:n * k].view(n, k, -1).float() * w32[..., None]).sum(1))
        return out

    @staticmethod
    def combine_backward(dy, slots, w32, plan):
        n, k = w32.shape
        dyf = dy.float()[:, None, :]
        dw = (slots[:n * k].view(n, k, -1).float() * dyf).sum(-1)
        g_slots = (w32[..., None] * dyf).to(dy.dtype).reshape(n * k, -1)
        return g_slots.index_select(0, plan.order), dw

    @staticmethod
    def outer(g_t, a_t):
        return torch.bmm(g_t, a_t.transpose(1, 2))

    @staticmethod
    def transpose(w):
        return w.transpose(-1, -2).contiguous()


def _kernels(x: torch.Tensor):
    return _NativeKernels if x.is_cuda else _TorchKernels


def _per_sample_outer(g_rows, a_rows, plan, kernels) -> torch.Tensor:
    """``(E, B, k_g * k_a)``: per (expert, sample), ``sum_t g_p[t]^T a_p[t]`` over its rows."""
    segments = plan.n_experts * plan.batch
    padded = []
    for rows in (g_rows, a_rows):
        t_major = rows.new_zeros(segments, rows.shape[1], plan.tokens)
        t_major.permute(0, 2, 1)[plan.segment, plan.position] = rows  # (expert, sample, token) is unique
        padded.append(t_major)
    return kernels.outer(*padded).reshape(plan.n_experts, plan.batch, -1)


class _GroupedMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, plan, block):
        kern = _kernels(x)
        experts = block.experts
        w32 = weights.float().contiguous()
        xs = x.index_select(0, plan.tok)
        h1 = kern.ragged(xs, experts.gate_up_proj, plan, out=x.new_empty(plan.rows, experts.gate_up_proj.shape[1]))
        act = experts._apply_gate(h1).contiguous()
        slots = kern.ragged(act, experts.down_proj, plan, home_of=x.new_empty(plan.rows, x.shape[1]))
        y = kern.combine(slots, w32, x.new_empty(x.shape))
        pm = block.matrices
        a_up = pm["up_a"](x).index_select(0, plan.tok)
        a_down = pm["down_a"](act)
        ctx.save_for_backward(h1, slots, w32, a_up, a_down)
        ctx.plan, ctx.block, ctx.weights_dtype = plan, block, weights.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        h1, slots, w32, a_up, a_down = ctx.saved_tensors
        plan, block = ctx.plan, ctx.block
        kern = _kernels(h1)
        experts, pm = block.experts, block.matrices
        dy = dy.to(h1.dtype).contiguous()
        g_down, dw = kern.combine_backward(dy, slots, w32, plan)
        up_t, down_t = block.transposed(kern)
        d_act = kern.ragged(g_down, down_t, plan, out=dy.new_empty(plan.rows, down_t.shape[1]))
        with torch.enable_grad():
            h = h1.detach().requires_grad_(True)
            (g_up,) = torch.autograd.grad(experts._apply_gate(h), h, d_act)
        g_up = g_up.contiguous()
        dense_up = _per_sample_outer(pm["up_g"](g_up), a_up, plan, kern)
        dense_down = _per_sample_outer(pm["down_g"](g_down), a_down, plan, kern)
        block.deliver(dense_up, dense_down, dy.device)
        dx = None
        if ctx.needs_input_grad[0]:
            dx_slots = kern.ragged(g_up, up_t, plan, home_of=dy.new_empty(plan.rows, up_t.shape[1]))
            dx = kern.combine(dx_slots, torch.ones_like(w32), dy.new_empty(dy.shape))
        return dx, dw.to(ctx.weights_dtype), None, None


class GroupedExpertCapture:
    """The grouped path of one fused-experts block, bound to a capture manager.

    The manager (*host*) answers :meth:`grouped_matrices` (the four projections when the
    block's captures allow the grouped path, else ``None``), :meth:`routed_shape` (the
    block's ``(batch, tokens)``) and takes the results through :meth:`grouped_forward` /
    :meth:`grouped_backward`.
    """

    def __init__(self, host, experts_name: str, experts, proxy_root: str) -> None:
        self.host, self.name, self.experts = host, experts_name, experts
        n = experts.gate_up_proj.shape[0]
        self.up_names = [f"{experts_name}.{proxy_root}.{e}.gate_up" for e in range(n)]
        self.down_names = [f"{experts_name}.{proxy_root}.{e}.down" for e in range(n)]
        self.matrices: dict = {}
        self._transposed_key = None
        self._transposed = None

    def transposed(self, kernels) -> tuple[torch.Tensor, torch.Tensor]:
        """``(gate_up^T (E, H, 2I), down^T (E, I, H))``, rebuilt when the weights change."""
        up, down = self.experts.gate_up_proj, self.experts.down_proj
        key = (up.data_ptr(), up._version, down.data_ptr(), down._version)
        if key != self._transposed_key:
            self._transposed = (kernels.transpose(up.detach()), kernels.transpose(down.detach()))
            self._transposed_key = key
        return self._transposed

    def _static_ok(self, x: torch.Tensor) -> bool:
        from dattri_llm_b200 import ops

        up, down = getattr(self.experts, "gate_up_proj", None), getattr(self.experts, "down_proj", None)
        if not (isinstance(up, torch.Tensor) and isinstance(down, torch.Tensor)):
            return False
        if getattr(self.experts, "is_transposed", False) or getattr(self.experts, "has_bias", False):
            return False
        if not hasattr(self.experts, "_apply_gate") or up.requires_grad or down.requires_grad:
            return False
        if x.ndim != 2 or not x.is_floating_point() or any(t.dtype != x.dtype for t in (up, down)):
            return False
        if not x.is_cuda:
            return not (up.is_cuda or down.is_cuda)
        tensors_ok = x.dtype == torch.bfloat16 and up.is_contiguous() and down.is_contiguous()
        widths_ok = x.shape[1] % 8 == 0 and up.shape[1] % 16 == 0 and down.shape[2] % 8 == 0
        return tensors_ok and widths_ok and ops.use_native(x)

    def try_forward(self, x: torch.Tensor, index: torch.Tensor, weights: torch.Tensor) -> torch.Tensor | None:
        """The block's output through the grouped path, or ``None`` when it does not apply."""
        if not _ENABLED[0] or not torch.is_grad_enabled() or not self._static_ok(x):
            return None
        shape = self.host.routed_shape(x)
        if shape is None or index.ndim != 2 or index.shape[0] != x.shape[0]:
            return None
        batch, tokens = shape
        matrices = self.host.grouped_matrices(self, x, tokens)
        if matrices is None:
            return None
        self.matrices = matrices
        plan = _Plan(index, self.experts.gate_up_proj.shape[0], batch, tokens)
        self.host.grouped_forward(self)
        return _GroupedMoE.apply(x.contiguous(), weights, plan, self)

    def deliver(self, dense_up: torch.Tensor, dense_down: torch.Tensor, device: torch.device) -> None:
        """Hand the ``(E, B, k_g * k_a)`` results of one backward to the manager."""
        parts = dict(zip(self.up_names, dense_up.unbind(0)))
        parts.update(zip(self.down_names, dense_down.unbind(0)))
        self.host.grouped_backward(self, parts, device)
