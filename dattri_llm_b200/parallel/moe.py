"""Expert-parallel sparse MLP (OLMoE-style top-k routing) over NVLink peer memory.

Experts are sharded over the ranks (``n_experts / world`` each); the router is replicated.
One forward:

1. route: router GEMM, softmax, top-k (PyTorch; its backward reaches the router);
2. layout: per-expert row counts (``moe_count``) are exchanged (a tiny NCCL all-gather --
   the control plane); from them ``moe_place`` derives the receive layout (each owner's
   rows grouped by local expert, then by source rank) and this rank's ragged-GEMM tables;
3. dispatch: one kernel stores each (token, slot) row straight into its owner's receive
   buffer (16-byte peer stores, ``moe_dispatch``) with its origin;
4. experts: ONE ragged tcgen05 GEMM over all local experts' row segments (gate/up), a
   split SwiGLU, and ONE ragged down GEMM whose EPILOGUE stores every output row back into
   its source rank's combine buffer over NVLink (``kStoreBF16Scatter``) -- the combine
   all-to-all happens inside the GEMM;
5. combine: each source sums its k returned rows weighted by the router probabilities.

The backward mirrors it: slot gradients are dispatched to the owners, the experts'
input-gradient GEMM (against the transposed gate/up weights) returns its rows to the
sources from its epilogue, and the router weights get ``<dy, expert output>``.
Bounded cross-GPU barriers separate the phases.  The reference has no expert parallelism
(it captures MoE layers with replicated experts, ``dattri_llm/gradient/hooks/routing.py``).

Per-sample capture.  Every expert has two :class:`ExpertTap` stand-ins,
``experts.dattri_experts.<e>.gate_up`` and ``.down``, and the router's map is the
:class:`RouterTap` ``gate.dattri_router``: the layer names the replicated-expert proxies
of ``gradient/hooks/override_layers/fused_experts.py`` give a Hugging Face MoE block, so a
store written under expert parallelism reads like one written with replicated experts.
A capture manager hooks the taps like ``nn.Linear`` layers.  While a tap is hooked, the
layer runs the two-stage all-to-all form (:class:`_UpA2A`, :class:`_DownA2A`): the owner
returns each row's SwiGLU output to the source in the forward and its gate/up output
gradient in the backward, so
the source holds both factors of every expert projection for its own samples.  It feeds
them to the taps as ``(B, T, d)`` tensors, zero at the tokens not routed to the expert,
the layout the replicated path regroups its rows into.  Rows carry their slot index, so
no row fingerprinting is needed.  The same form runs on CPU over gloo, or whenever the
fused kernels do not apply (any dtype other than bf16).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from dattri_llm_b200.parallel.symm import PeerBarrier, SymmetricBuffer


class ExpertTap(nn.Module):
    """Capture stand-in for one expert projection ``(out_features, in_features)``.

    Its forward takes the projection's input at this rank's tokens (a ``(..., in)`` tensor,
    zero where the token was not routed to the expert) and returns a stride-0 zero tensor
    ``(..., out)`` whose gradient the expert-parallel backward sets to the projection's
    output gradient at those tokens.  The expert's weight lives on its owner rank, so the
    tap holds none; it is captured like a linear layer without bias, frozen or not.
    """

    __bw_layer_type__ = "nn.Linear"
    __bw_capture_tap__ = True
    __bw_capture_frozen__ = True
    bias = None

    def __init__(self, in_features: int, out_features: int) -> None:
        super().__init__()
        self.in_features, self.out_features = in_features, out_features

    def hooked(self) -> bool:
        """Whether a capture hook is installed on this tap."""
        return bool(self._forward_hooks or self._forward_pre_hooks)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        anchor = torch.zeros((), dtype=x.dtype, device=x.device, requires_grad=True)
        return _TapOut.apply(anchor, tuple(x.shape[:-1]) + (self.out_features,))


class RouterTap(nn.Module):
    """The router's linear map as a hookable layer: ``F.linear`` on the owning router's
    weight (no parameter of its own), captured like ``nn.Linear`` when that weight trains."""

    __bw_layer_type__ = "nn.Linear"
    __bw_capture_tap__ = True
    bias = None

    def __init__(self, router: nn.Module) -> None:
        super().__init__()
        object.__setattr__(self, "_router", router)  # not a submodule: no parameter duplication

    @property
    def weight(self) -> torch.Tensor:
        """The router's ``(E, H)`` weight."""
        return self._router.weight

    def proxied_parameters(self):
        """The router weight this tap reads."""
        yield self._router.weight

    def hooked(self) -> bool:
        """Whether a capture hook is installed on this tap."""
        return bool(self._forward_hooks or self._forward_pre_hooks)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self._router.weight)


class _Router(nn.Module):
    """Router weight ``(E, H)`` (state-dict key ``gate.weight``, as in Hugging Face MoE
    blocks) applied through its :class:`RouterTap` ``dattri_router``."""

    def __init__(self, hidden: int, n_experts: int, device, dtype) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(n_experts, hidden, device=device, dtype=dtype))
        self.dattri_router = RouterTap(self)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.dattri_router(x)


class _ExpertTaps(nn.Module):
    """Container of the experts' taps, so their names are ``experts.dattri_experts.<e>.*``:
    the names the replicated-expert capture gives the same projections."""

    def __init__(self, n_experts: int, hidden: int, intermediate: int) -> None:
        super().__init__()
        self.dattri_experts = nn.ModuleList([nn.ModuleDict({
            "gate_up": ExpertTap(hidden, 2 * intermediate),
            "down": ExpertTap(intermediate, hidden),
        }) for _ in range(n_experts)])


class _TapOut(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, shape):
        return anchor.new_zeros(()).expand(shape)

    @staticmethod
    def backward(ctx, grad):
        return None, None


class _A2APlan:
    """Routing of one layer call for the all-to-all form: slots sorted by owner rank,
    per-rank row counts both ways (one small all-to-all), received rows grouped by local
    expert, and this rank's slots grouped by global expert.  All counts reach the host in
    one read, so the per-expert loops below slice instead of synchronizing."""

    def __init__(self, topi: torch.Tensor, mod: ExpertParallelMoE) -> None:
        self.t, self.k = topi.shape
        self.group, self.world = mod.group, mod.world
        e_l = mod.experts_per_rank
        n_exp = mod.n_experts
        flat = topi.reshape(-1)
        owner = torch.div(flat, e_l, rounding_mode="floor")
        self.order = torch.argsort(owner, stable=True)
        send = torch.bincount(owner, minlength=self.world)
        recv = send.clone()
        if self.world > 1:
            dist.all_to_all_single(recv, send, group=self.group)
        self.send, self.recv = send.tolist(), recv.tolist()
        local_expert = self.to_owner((flat[self.order] % e_l).contiguous())
        # received rows grouped by local expert; this rank's slots grouped by global expert
        self.by_expert = torch.argsort(local_expert, stable=True)
        self.slots_by_expert = torch.argsort(flat, stable=True)
        counts = torch.cat([torch.bincount(local_expert, minlength=e_l), torch.bincount(flat, minlength=n_exp)])
        counts = counts.tolist()
        self.rows_per_expert, self.slots_per_expert = counts[:e_l], counts[e_l:]
        offs = [0]
        for c in self.slots_per_expert:
            offs.append(offs[-1] + c)
        self.slot_offsets = offs

    def to_owner(self, rows: torch.Tensor) -> torch.Tensor:
        """Rows in this rank's send order -> the rows every source sent to this rank."""
        if self.world == 1:
            return rows
        out = rows.new_empty((sum(self.recv),) + tuple(rows.shape[1:]))
        dist.all_to_all_single(out, rows.contiguous(), self.recv, self.send, group=self.group)
        return out

    def to_source(self, rows: torch.Tensor) -> torch.Tensor:
        """Owner rows back to their sources, in each source's send order."""
        if self.world == 1:
            return rows
        out = rows.new_empty((sum(self.send),) + tuple(rows.shape[1:]))
        dist.all_to_all_single(out, rows.contiguous(), self.send, self.recv, group=self.group)
        return out

    def to_slots(self, rows: torch.Tensor) -> torch.Tensor:
        """Rows in send order -> ``(t*k, ...)`` in slot order."""
        out = torch.empty_like(rows)
        out[self.order] = rows
        return out

    def hit(self) -> list[int]:
        """Global experts that received at least one of this rank's slots."""
        return [e for e, c in enumerate(self.slots_per_expert) if c]

    def expert_slots(self, e: int) -> torch.Tensor:
        """Slot indices of this rank routed to global expert *e* (ascending)."""
        return self.slots_by_expert[self.slot_offsets[e]:self.slot_offsets[e + 1]]

    def expert_mm(self, x: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """``x[r] @ weights[local_expert[r]].T`` for every received row."""
        parts = x[self.by_expert].split(self.rows_per_expert)
        y = torch.cat([part @ weights[e].t() for e, part in enumerate(parts)]) if parts else x.new_empty(0)
        out = x.new_empty(x.shape[0], weights.shape[1])
        out[self.by_expert] = y.view(x.shape[0], weights.shape[1])
        return out

    def tap_grads(self, hit: list[int], slot_rows: torch.Tensor, lead: tuple[int, ...]) -> list[torch.Tensor]:
        """Per hit expert, *slot_rows* at its tokens scattered into a zero ``(*lead, d)``."""
        out = []
        for e in hit:
            sel = self.expert_slots(e)
            g = slot_rows.new_zeros(self.t, slot_rows.shape[1])
            g[torch.div(sel, self.k, rounding_mode="floor")] = slot_rows[sel]
            out.append(g.view(*lead, slot_rows.shape[1]))
        return out


def _swiglu(h: torch.Tensor) -> torch.Tensor:
    g, u = h.float().chunk(2, -1)
    return (F.silu(g) * u).to(h.dtype)


def _swiglu_bwd(da: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    g, u = h.float().chunk(2, -1)
    d = da.float()
    s = torch.sigmoid(g)
    return torch.cat([d * u * s * (1 + g * (1 - s)), d * g * s], -1).to(h.dtype)


class _UpA2A(torch.autograd.Function):
    """Dispatch, gate/up projection and SwiGLU at the owners; returns every slot's SwiGLU
    output to its source: ``(t*k, I)`` in slot order."""

    @staticmethod
    def forward(ctx, x2, plan, mod, hit, lead, *taps):
        rows = plan.to_owner(x2[torch.div(plan.order, plan.k, rounding_mode="floor")])
        h = plan.expert_mm(rows, mod.gate_up)
        act = plan.to_slots(plan.to_source(_swiglu(h)))
        ctx.plan, ctx.mod, ctx.hit, ctx.lead = plan, mod, hit, lead
        ctx.save_for_backward(h)
        return act

    @staticmethod
    def backward(ctx, d_act):
        plan, mod = ctx.plan, ctx.mod
        (h,) = ctx.saved_tensors
        d_rows = plan.to_owner(d_act.to(h.dtype)[plan.order])
        dh = _swiglu_bwd(d_rows, h)
        d_in = plan.expert_mm(dh, mod.gate_up_t)
        hidden = d_in.shape[1]
        back = plan.to_slots(plan.to_source(torch.cat([d_in, dh], 1) if ctx.hit else d_in))
        dx2 = back[:, :hidden].reshape(plan.t, plan.k, hidden).sum(1)
        taps = plan.tap_grads(ctx.hit, back[:, hidden:], ctx.lead) if ctx.hit else []
        return (dx2, None, None, None, None, *taps)


class _DownA2A(torch.autograd.Function):
    """Down projection at the owners, rows returned to their sources and combined with
    the router weights: ``y (t, H)``."""

    @staticmethod
    def forward(ctx, act, topv, plan, mod, hit, lead, *taps):
        out = plan.to_slots(plan.to_source(plan.expert_mm(plan.to_owner(act[plan.order]), mod.down)))
        w = topv.float()
        y = (out.view(plan.t, plan.k, -1).float() * w[..., None]).sum(1).to(act.dtype)
        ctx.plan, ctx.mod, ctx.hit, ctx.lead = plan, mod, hit, lead
        ctx.save_for_backward(out, w)
        return y

    @staticmethod
    def backward(ctx, dy):
        plan, mod = ctx.plan, ctx.mod
        out, w = ctx.saved_tensors
        dyf = dy.float()
        d_slot = (dyf[:, None, :] * w[..., None]).reshape(plan.t * plan.k, -1).to(out.dtype)
        d_topv = (out.view(plan.t, plan.k, -1).float() * dyf[:, None, :]).sum(-1)
        d_act = plan.to_slots(plan.to_source(plan.expert_mm(plan.to_owner(d_slot[plan.order]), mod.down_t)))
        taps = plan.tap_grads(ctx.hit, d_slot, ctx.lead) if ctx.hit else []
        return (d_act, d_topv, None, None, None, None, *taps)


class _Routed:
    """One fused call's routing: the receive layout, this rank's owner-side ragged-GEMM tables
    and the rows it received (read once on the host, to size the expert buffers)."""

    def __init__(self, mod: ExpertParallelMoE, x2: torch.Tensor, topi: torch.Tensor) -> None:
        from dattri_llm_b200 import ops

        t, k = topi.shape
        world, rank, e_l = mod.world, mod.rank, mod.experts_per_rank
        dev = x2.device
        if t > mod.max_tokens:
            raise ValueError(f"{t} tokens exceed this layer's capacity of {mod.max_tokens} per rank")
        n_exp = world * e_l
        topi = topi.reshape(-1).contiguous()
        rows = topi.numel()
        # int32 scratch: [counts | cursor | tile_prefix | base | len | total]
        work = torch.zeros(2 * n_exp + 3 * e_l + 2, dtype=torch.int32, device=dev)
        counts, cursor = work[:n_exp], work[n_exp:2 * n_exp]
        self.prefix = work[2 * n_exp:2 * n_exp + e_l + 1]
        self.base = work[2 * n_exp + e_l + 1:2 * n_exp + 2 * e_l + 1]
        self.lens = work[2 * n_exp + 2 * e_l + 1:2 * n_exp + 3 * e_l + 1]
        self.rows_dev = work[2 * n_exp + 3 * e_l + 1:]
        ops.count_launch()
        ops.native().moe_count(topi, counts)
        all_counts = torch.empty(world, n_exp, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(all_counts, counts, group=mod.group)  # the control plane
        self.dest = torch.empty(rows, dtype=torch.int32, device=dev)
        self.row = torch.empty(rows, dtype=torch.int32, device=dev)
        ops.count_launch()
        ops.native().moe_place(topi, all_counts, rank, e_l, cursor, self.dest, self.row, self.prefix, self.base,
                               self.lens, self.rows_dev)
        mod.barrier.wait()  # every rank is done with the previous use of the receive buffers
        ops.count_launch()
        ops.native().moe_dispatch(x2, k, self.dest, self.row, mod.recv_x.peers, mod.recv_meta.peers, rank)
        mod.barrier.wait()  # every row has landed
        # One host read per layer (it sizes the expert buffers exactly); the dispatch above is
        # already queued, so the GPU stays busy while the host waits.
        self.total_in = int(self.rows_dev.item())
        self.max_tiles = (self.total_in + 255) // 256 + e_l  # 256-row blocks of the ragged GEMM
        self.t, self.k = t, k

    def owners_forward(self, mod: ExpertParallelMoE) -> tuple[torch.Tensor, torch.Tensor]:
        """Experts' gate/up (``h``), SwiGLU (``a``) and down projection of the received rows; the
        down GEMM's epilogue stores every output row into its source's combine buffer."""
        from dattri_llm_b200 import ops

        dev = mod.recv_x.local.device
        n = self.total_in
        err = ops.error_word(dev)
        h = torch.empty(max(n, 1), 2 * mod.intermediate, dtype=torch.bfloat16, device=dev)
        a = torch.empty(max(n, 1), mod.intermediate, dtype=torch.bfloat16, device=dev)
        if n:
            ops.count_launch(3)
            ops.native().gemm_ragged(mod.recv_x.local[:n], mod.gate_up, h, self.prefix, self.base, self.lens,
                                     self.max_tiles, [], None, err)
            ops.native().swiglu_split(h, a, self.rows_dev)
            ops.native().gemm_ragged(a[:n], mod.down, None, self.prefix, self.base, self.lens, self.max_tiles,
                                     mod.combine.peers, mod.recv_meta.local[:n], err)
        return h, a

    def dispatch_grads(self, mod: ExpertParallelMoE, dy: torch.Tensor, slots: torch.Tensor,
                       w: torch.Tensor) -> torch.Tensor:
        """Backward of the combine: router-weight gradients, and every slot's gradient stored
        into its owner's receive buffer (one kernel); returns ``d topv`` (fp32)."""
        from dattri_llm_b200 import ops

        dtopv = torch.empty(self.t, self.k, dtype=torch.float32, device=dy.device)
        mod.barrier.wait()
        ops.count_launch()
        ops.native().moe_combine_bwd_dispatch(dy, slots, w, dtopv, self.dest, self.row, mod.recv_x.peers,
                                              mod.recv_meta.peers, mod.rank)
        mod.barrier.wait()
        return dtopv

    def owners_backward(self, mod: ExpertParallelMoE, h: torch.Tensor) -> torch.Tensor | None:
        """Owner side of the backward: the experts' input gradient of the received slot
        gradients, returned to the sources' ``dx_slots`` from the GEMM epilogue; returns the
        gate/up output gradient ``dh`` of the received rows (``None`` with no rows)."""
        from dattri_llm_b200 import ops

        n = self.total_in
        if not n:
            return None
        err = ops.error_word(h.device)
        dout = mod.recv_x.local[:n]
        da = torch.empty(n, mod.intermediate, dtype=torch.bfloat16, device=h.device)
        dh = torch.empty_like(h[:n])
        ops.count_launch(3)
        ops.native().gemm_ragged(dout, mod.down_t, da, self.prefix, self.base, self.lens, self.max_tiles, [], None,
                                 err)
        ops.native().swiglu_split_bwd(da, h[:n].contiguous(), dh, self.rows_dev)
        ops.native().gemm_ragged(dh, mod.gate_up_t, None, self.prefix, self.base, self.lens, self.max_tiles,
                                 mod.dx_slots.peers, mod.recv_meta.local[:n], err)
        return dh

    def return_rows(self, mod: ExpertParallelMoE, rows: torch.Tensor, buf) -> None:
        """Store received row r of *rows* into its source rank's symmetric *buf* at its slot
        (the origin the dispatch recorded), 16-byte peer stores."""
        from dattri_llm_b200 import ops

        n = self.total_in
        if not n:
            return
        meta = mod.recv_meta.local[:n]
        ops.count_launch()
        ops.native().moe_dispatch(rows.contiguous(), 1, meta[:, 0].contiguous(), meta[:, 1].contiguous(), buf.peers,
                                  [], mod.rank)

    def combine_dx(self, mod: ExpertParallelMoE, w: torch.Tensor) -> torch.Tensor:
        """``dx[t] = sum_j dx_slots[t * k + j]`` once every row is home."""
        from dattri_llm_b200 import ops

        dx = torch.empty(self.t, mod.hidden, dtype=torch.bfloat16, device=w.device)
        ops.count_launch()
        ops.native().moe_combine(mod.dx_slots.local[:self.t * self.k], torch.ones_like(w), dx)
        return dx


def _combine(mod: ExpertParallelMoE, topv: torch.Tensor, t: int, k: int, keep: bool):
    """``y`` from the combine buffer (router-weighted sum of the k returned rows) plus the fp32
    weights and the slot rows (a copy when *keep*: the buffer is reused by the next layer)."""
    from dattri_llm_b200 import ops

    w = topv.float().contiguous()
    slots = mod.combine.local[:t * k]
    if keep:
        slots = slots.clone()
    y = torch.empty(t, mod.hidden, dtype=torch.bfloat16, device=w.device)
    ops.count_launch()
    ops.native().moe_combine(slots, w, y)
    return y, w, slots


class _EPMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, topv, topi, mod):
        rt = _Routed(mod, x2, topi)
        h, _a = rt.owners_forward(mod)
        mod.barrier.wait()  # every output row is home
        y, w, slots = _combine(mod, topv, rt.t, rt.k, ctx.needs_input_grad[0] or ctx.needs_input_grad[1])
        ctx.mod, ctx.rt, ctx.topv_dtype = mod, rt, topv.dtype
        ctx.save_for_backward(w, slots, h)
        return y

    @staticmethod
    def backward(ctx, dy):
        mod, rt = ctx.mod, ctx.rt
        w, slots, h = ctx.saved_tensors
        dtopv = rt.dispatch_grads(mod, dy.to(torch.bfloat16).contiguous(), slots, w)
        rt.owners_backward(mod, h)
        mod.barrier.wait()
        return rt.combine_dx(mod, w), dtopv.to(ctx.topv_dtype), None, None


class _EPGroupedMoE(torch.autograd.Function):
    """The fused expert-parallel block with the grouped capture of every expert projection.

    Per-sample capture needs four factors per routed row: the gate/up input (the token's own
    hidden state) and the down projection's output gradient (``w * dy`` of the slot) are on the
    source rank already and are projected there; the down input (the SwiGLU output) and the
    gate/up output gradient exist only at the expert's owner, which projects them and stores
    the ``k``-wide rows back into the source's symmetric buffer at their slot (the origin the
    dispatch recorded), so only ``k`` columns per row cross NVLink.  Each source then forms
    every (expert, sample)'s ``sum_t g_p^T a_p`` over its own slots in one batched GEMM and
    hands the ``(E, B, k_g * k_a)`` blocks to the capture manager under the taps' names."""

    @staticmethod
    def forward(ctx, x2, topv, topi, mod, block, batch, tokens):
        pm = block.matrices
        rt = _Routed(mod, x2, topi)
        h, a = rt.owners_forward(mod)
        a_buf = mod.capture_rows(pm["down_a"].proj_dim)
        if rt.total_in:
            rt.return_rows(mod, pm["down_a"](a[:rt.total_in]), a_buf)
        mod.barrier.wait()  # every output row and projected down input is home
        y, w, slots = _combine(mod, topv, rt.t, rt.k, True)
        n = rt.t * rt.k
        a_down = a_buf.local[:n].clone()
        slot_tok = torch.div(torch.arange(n, device=x2.device), rt.k, rounding_mode="floor")
        a_up = pm["up_a"](x2).index_select(0, slot_tok)
        ctx.mod, ctx.rt, ctx.block, ctx.topv_dtype = mod, rt, block, topv.dtype
        ctx.shape = (batch, tokens)
        ctx.save_for_backward(w, slots, h, a_up, a_down, topi.reshape(-1), slot_tok)
        return y

    @staticmethod
    def backward(ctx, dy):
        from dattri_llm_b200.gradient.hooks.override_layers.grouped_experts import _NativeKernels, _per_sample_outer

        mod, rt, block = ctx.mod, ctx.rt, ctx.block
        w, slots, h, a_up, a_down, experts, slot_tok = ctx.saved_tensors
        pm = block.matrices
        dy = dy.to(torch.bfloat16).contiguous()
        dtopv = rt.dispatch_grads(mod, dy, slots, w)
        dh = rt.owners_backward(mod, h)
        g_buf = mod.capture_rows(pm["up_g"].proj_dim)
        if dh is not None:
            rt.return_rows(mod, pm["up_g"](dh), g_buf)
        mod.barrier.wait()  # every input-gradient row and projected gate/up gradient is home
        dx = rt.combine_dx(mod, w)
        n = rt.t * rt.k
        g_up = g_buf.local[:n].clone()
        g_slots = (w[..., None] * dy.float()[:, None, :]).to(torch.bfloat16).reshape(n, -1)
        g_down = pm["down_g"](g_slots)
        batch, tokens = ctx.shape
        plan = _SlotPlan(experts, slot_tok, mod.n_experts, batch, tokens)
        dense_up = _per_sample_outer(g_up, a_up, plan, _NativeKernels)
        dense_down = _per_sample_outer(g_down, a_down, plan, _NativeKernels)
        block.deliver(dense_up, dense_down, dy.device)
        return dx, dtopv.to(ctx.topv_dtype), None, None, None, None, None


class _SlotPlan:
    """Where each of this rank's slot rows sits in the token-major per-(expert, sample)
    layout of the batched outer product: segment ``expert * batch + sample``, position the
    token within its sample (unique: a token's k slots go to k different experts)."""

    def __init__(self, experts: torch.Tensor, slot_tok: torch.Tensor, n_experts: int, batch: int,
                 tokens: int) -> None:
        self.n_experts, self.batch, self.tokens = n_experts, batch, tokens
        self.segment = experts * batch + torch.div(slot_tok, tokens, rounding_mode="floor")
        self.position = slot_tok % tokens


class EPGroupedCapture:
    """Binds one :class:`ExpertParallelMoE` to a capture manager (*host*) for the grouped
    capture: the manager answers :meth:`grouped_matrices` for the block's expert taps and
    takes each backward's per-expert blocks through :meth:`grouped_backward`, as for a
    replicated fused-experts block (``gradient/hooks/override_layers/grouped_experts.py``)."""

    def __init__(self, host, name: str, mod: ExpertParallelMoE) -> None:
        self.host, self.name, self.mod = host, name, mod
        prefix = f"{name}.experts.dattri_experts" if name else "experts.dattri_experts"
        self.up_names = [f"{prefix}.{e}.gate_up" for e in range(mod.n_experts)]
        self.down_names = [f"{prefix}.{e}.down" for e in range(mod.n_experts)]
        self.experts = _ExpertShapes(mod)
        self.matrices: dict = {}

    def try_forward(self, x: torch.Tensor, x2: torch.Tensor, topv: torch.Tensor,
                    topi: torch.Tensor) -> torch.Tensor | None:
        """The block's output through the grouped path, or ``None`` when the captures do not
        allow it (the caller then runs the all-to-all form)."""
        if x.ndim != 3 or x2.dtype != torch.bfloat16 or not x2.is_cuda:
            return None
        batch, tokens = int(x.shape[0]), int(x.shape[1])
        matrices = self.host.grouped_matrices(self, x2, tokens)
        if matrices is None or any(m.proj_dim % 8 for m in matrices.values()):
            return None
        self.matrices = matrices
        self.host.grouped_forward(self)
        return _EPGroupedMoE.apply(x2, topv, topi, self.mod, self, batch, tokens)

    def deliver(self, dense_up: torch.Tensor, dense_down: torch.Tensor, device: torch.device) -> None:
        """Hand the ``(E, B, k_g * k_a)`` results of one backward to the manager."""
        parts = dict(zip(self.up_names, dense_up.unbind(0)))
        parts.update(zip(self.down_names, dense_down.unbind(0)))
        self.host.grouped_backward(self, parts, device)


class _ExpertShapes:
    """The expert weight shapes the manager's checks read (``gate_up_proj (E, 2I, H)``,
    ``down_proj (E, H, I)``; the leading axis is this rank's share)."""

    def __init__(self, mod: ExpertParallelMoE) -> None:
        self.gate_up_proj, self.down_proj = mod.gate_up, mod.down


class _Buffers:
    """Symmetric receive / combine buffers and the barrier, shared by every EP layer of one
    shape on a device (the layers run one after another on one stream)."""

    _pool: dict = {}

    def __init__(self, capacity: int, slots: int, hidden: int, dev: torch.device, group) -> None:
        self.recv_x = SymmetricBuffer((capacity, hidden), torch.bfloat16, dev, group)
        self.recv_meta = SymmetricBuffer((capacity, 2), torch.int32, dev, group)
        self.combine = SymmetricBuffer((slots, hidden), torch.bfloat16, dev, group)
        self.dx_slots = SymmetricBuffer((slots, hidden), torch.bfloat16, dev, group)
        self.barrier = PeerBarrier(dev, group)
        self.slots, self.dev, self.group = slots, dev, group
        self.capture: dict[int, SymmetricBuffer] = {}

    def capture_rows(self, width: int) -> SymmetricBuffer:
        """A ``(slots, width)`` bf16 symmetric buffer for projected rows returned to their
        sources; created on first use (every rank reaches the same layer call, so the
        allocation is collective)."""
        buf = self.capture.get(width)
        if buf is None:
            buf = self.capture[width] = SymmetricBuffer((self.slots, width), torch.bfloat16, self.dev, self.group)
        return buf

    @classmethod
    def get(cls, capacity: int, slots: int, hidden: int, dev: torch.device, group) -> _Buffers:
        key = (capacity, slots, hidden, dev, id(group))
        if key not in cls._pool:
            cls._pool[key] = cls(capacity, slots, hidden, dev, group)
        return cls._pool[key]


class ExpertParallelMoE(nn.Module):
    """Top-k MoE MLP with experts sharded over the process group (frozen experts: the
    attribution probe's case; the router may train).  Build collectively.

    On CUDA in bf16 the forward is the fused peer-memory path above.  While its
    ``experts.dattri_experts`` taps are hooked by a capture manager that allows the grouped
    capture (one LoGra projection per side, materialized), it is the same fused path with the
    captures taken inside it (:class:`_EPGroupedMoE`); under other captures, and on other
    devices or dtypes, it is the two-stage all-to-all form (``torch.distributed`` all-to-all,
    any backend)."""

    def __init__(self, hidden: int, intermediate: int, n_experts: int, top_k: int, *, max_tokens: int,
                 norm_topk_prob: bool = False, group=None, device: torch.device | None = None,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        if hidden % 8 or intermediate % 8:
            raise ValueError("hidden and intermediate sizes must be multiples of 8")
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = torch.device(dev)
        self.hidden, self.intermediate, self.n_experts, self.top_k = hidden, intermediate, n_experts, top_k
        self.experts_per_rank = n_experts // self.world
        self.norm_topk_prob = norm_topk_prob
        self.max_tokens = max_tokens
        self.capacity = self.world * max_tokens * top_k
        self.dtype = dtype
        self.fused = dev.type == "cuda" and dtype == torch.bfloat16
        self.gate = _Router(hidden, n_experts, dev, dtype)
        e_l = self.experts_per_rank
        self.register_buffer("gate_up", torch.zeros(e_l, 2 * intermediate, hidden, device=dev, dtype=dtype))
        self.register_buffer("down", torch.zeros(e_l, hidden, intermediate, device=dev, dtype=dtype))
        self.register_buffer("gate_up_t", torch.zeros(e_l, hidden, 2 * intermediate, device=dev, dtype=dtype))
        self.register_buffer("down_t", torch.zeros(e_l, intermediate, hidden, device=dev, dtype=dtype))
        self.experts = _ExpertTaps(n_experts, hidden, intermediate)
        self._taps = [t for pair in self.experts.dattri_experts for t in pair.values()]
        if self.fused:
            bufs = _Buffers.get(self.capacity, max_tokens * top_k, hidden, dev, group)
            self.recv_x, self.recv_meta = bufs.recv_x, bufs.recv_meta
            self.combine, self.dx_slots, self.barrier = bufs.combine, bufs.dx_slots, bufs.barrier
            self.capture_rows = bufs.capture_rows
        self.grouped_capture: EPGroupedCapture | None = None  # set by a capture manager

    @property
    def dattri_experts(self) -> nn.ModuleList:
        """The per-expert ``{"gate_up", "down"}`` taps."""
        return self.experts.dattri_experts

    @torch.no_grad()
    def load_experts(self, gate_up_all: torch.Tensor, down_all: torch.Tensor, router: torch.Tensor) -> None:
        """Take this rank's slice of the full ``(E, 2I, H)`` / ``(E, H, I)`` expert weights and
        the ``(E, H)`` router weight (identical on every rank)."""
        e_l, r = self.experts_per_rank, self.rank
        gu = gate_up_all[r * e_l:(r + 1) * e_l].to(self.gate_up.device, self.dtype)
        dn = down_all[r * e_l:(r + 1) * e_l].to(self.down.device, self.dtype)
        self.gate_up.copy_(gu)
        self.down.copy_(dn)
        self.gate_up_t.copy_(gu.transpose(1, 2))
        self.down_t.copy_(dn.transpose(1, 2))
        self.gate.weight.copy_(router.to(self.gate.weight.device, self.dtype))

    def route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``(top-k probabilities, top-k expert ids)`` of every token, flattened to ``(t, k)``.

        The router runs on *x* in its own shape, so a capture hook on ``gate`` sees the
        ``(B, T, H)`` layout of the samples."""
        probs = torch.softmax(self.gate(x).float().reshape(-1, self.n_experts), dim=-1)
        topv, topi = probs.topk(self.top_k, dim=-1)
        if self.norm_topk_prob:
            topv = topv / topv.sum(-1, keepdim=True)
        return topv, topi

    def capturing(self) -> bool:
        """Whether a gradient will be captured through the expert taps on this call."""
        return torch.is_grad_enabled() and any(t._forward_hooks for t in self._taps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        xd = x.to(self.dtype)
        topv, topi = self.route(xd)
        x2 = xd.reshape(-1, self.hidden).contiguous()
        y = None
        if self.fused and not self.capturing():
            y = _EPMoE.apply(x2, topv, topi, self)
        elif self.fused and self.grouped_capture is not None and torch.is_grad_enabled():
            y = self.grouped_capture.try_forward(xd, x2, topv, topi)
        if y is None:
            y = self._all_to_all(x2, topv, topi, tuple(shape[:-1]))
        return y.view(*shape[:-1], self.hidden)

    def _all_to_all(self, x2, topv, topi, lead):
        plan = _A2APlan(topi, self)
        hit = plan.hit() if self.capturing() else []
        # The taps run under grad mode (their hooks record only then); their inputs do not
        # require grad.
        up_taps = [self.dattri_experts[e]["gate_up"](self._tap_input(x2, plan, e, lead)) for e in hit]
        act = _UpA2A.apply(x2, plan, self, hit, lead, *up_taps)
        down_taps = [self.dattri_experts[e]["down"](self._tap_input(act, plan, e, lead, slots=True)) for e in hit]
        return _DownA2A.apply(act, topv, plan, self, hit, lead, *down_taps)

    @staticmethod
    @torch.no_grad()
    def _tap_input(rows_src, plan, e, lead, slots=False):
        """Expert *e*'s projection input at this rank's tokens, zero elsewhere: from token
        rows (``slots=False``) or from slot rows."""
        sel = plan.expert_slots(e)
        tok = torch.div(sel, plan.k, rounding_mode="floor")
        out = rows_src.new_zeros(plan.t, rows_src.shape[1])
        out[tok] = rows_src[sel if slots else tok]
        return out.view(*lead, rows_src.shape[1])


def _is_silu(act: object) -> bool:
    return isinstance(act, nn.SiLU) or "silu" in type(act).__name__.lower()


def expert_parallelize(model: nn.Module, *, max_tokens: int, group=None, device: torch.device | None = None,
                       dtype: torch.dtype | None = None) -> list[str]:
    """Replace every Hugging Face fused-experts MoE block of *model* (a ``gate`` router with an
    ``(E, H)`` weight next to ``experts`` holding ``gate_up_proj (E, 2I, H)`` /
    ``down_proj (E, H, I)`` with a SiLU gate, e.g. OLMoE's sparse MoE block) by an
    :class:`ExpertParallelMoE` holding this rank's experts.  Call collectively, with the
    same weights on every rank.  Returns the replaced blocks' names.

    Raises:
        ValueError: for a block whose experts are transposed, carry biases or use another
            activation, or a router without ``top_k``.
    """
    from dattri_llm_b200.gradient.hooks.override_layers.fused_experts import DOWN, GATE_UP, is_fused_experts

    replaced = []
    for name, block in list(model.named_modules()):
        experts, router = getattr(block, "experts", None), getattr(block, "gate", None)
        if experts is None or router is None or not is_fused_experts(experts):
            continue
        gu, dn = getattr(experts, GATE_UP), getattr(experts, DOWN)
        n_exp, two_i, hidden = gu.shape
        w = getattr(router, "weight", None)
        if not isinstance(w, torch.Tensor) or tuple(w.shape) != (n_exp, hidden):
            continue
        if getattr(experts, "is_transposed", False) or getattr(experts, "has_bias", False):
            raise ValueError(f"{name}: transposed or biased experts are not supported under expert parallelism")
        if not _is_silu(getattr(experts, "act_fn", None)):
            raise ValueError(f"{name}: expert parallelism implements the SiLU-gated (SwiGLU) experts only")
        top_k = getattr(router, "top_k", None)
        if top_k is None:
            raise ValueError(f"{name}: the router does not say its top_k")
        ep = ExpertParallelMoE(hidden, two_i // 2, n_exp, int(top_k), max_tokens=max_tokens,
                               norm_topk_prob=bool(getattr(router, "norm_topk_prob", False)), group=group,
                               device=device if device is not None else gu.device,
                               dtype=dtype if dtype is not None else gu.dtype)
        ep.load_experts(gu.detach(), dn.detach(), w.detach())
        ep.gate.weight.requires_grad_(w.requires_grad)
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else None
        if parent is None:
            raise ValueError("the model itself is an MoE block; wrap it in a parent module")
        setattr(parent, child, ep)
        replaced.append(name)
    return replaced


def expert_parallel_buffers(model: nn.Module) -> list[str]:
    """Fully qualified names of the per-rank expert shards of every
    :class:`ExpertParallelMoE` in *model*: buffers that differ by rank by design, which a
    data-parallel wrapper must neither broadcast nor check for equality."""
    out = []
    for name, m in model.named_modules():
        if isinstance(m, ExpertParallelMoE):
            out += [f"{name}.{b}" if name else b for b, _ in m.named_buffers(recurse=False)]
    return out
