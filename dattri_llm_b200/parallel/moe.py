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
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from dattri_llm_b200.parallel.symm import PeerBarrier, SymmetricBuffer


class _EPMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, topv, topi, mod):
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
        prefix = work[2 * n_exp:2 * n_exp + e_l + 1]
        base = work[2 * n_exp + e_l + 1:2 * n_exp + 2 * e_l + 1]
        lens = work[2 * n_exp + 2 * e_l + 1:2 * n_exp + 3 * e_l + 1]
        rows_dev = work[2 * n_exp + 3 * e_l + 1:]
        ops.count_launch()
        ops.native().moe_count(topi, counts)
        all_counts = torch.empty(world, n_exp, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(all_counts, counts, group=mod.group)  # the control plane
        dest32 = torch.empty(rows, dtype=torch.int32, device=dev)
        row32 = torch.empty(rows, dtype=torch.int32, device=dev)
        ops.count_launch()
        ops.native().moe_place(topi, all_counts, rank, e_l, cursor, dest32, row32, prefix, base, lens, rows_dev)

        mod.barrier.wait()  # every rank is done with the previous use of the receive buffers
        ops.count_launch()
        ops.native().moe_dispatch(x2, k, dest32, row32, mod.recv_x.peers, mod.recv_meta.peers, rank)
        mod.barrier.wait()  # every row has landed
        # One host read per layer (it sizes the expert buffers exactly); the dispatch above is
        # already queued, so the GPU stays busy while the host waits.
        total_in = int(rows_dev.item())
        max_tiles = (total_in + 255) // 256 + e_l  # 256-row blocks of the ragged GEMM

        err = ops.error_word(dev)
        h = torch.empty(max(total_in, 1), 2 * mod.intermediate, dtype=torch.bfloat16, device=dev)
        a = torch.empty(max(total_in, 1), mod.intermediate, dtype=torch.bfloat16, device=dev)
        if total_in:
            xin = mod.recv_x.local[:total_in]
            ops.count_launch(3)
            ops.native().gemm_ragged(xin, mod.gate_up, h, prefix, base, lens, max_tiles, [], None, err)
            ops.native().swiglu_split(h, a, rows_dev)
            # The down GEMM stores every output row back into its source rank's combine buffer.
            ops.native().gemm_ragged(a[:total_in], mod.down, None, prefix, base, lens, max_tiles,
                                     mod.combine.peers, mod.recv_meta.local[:total_in], err)
        mod.barrier.wait()  # every output row is home
        w = topv.float().contiguous()
        slots = mod.combine.local[:t * k]
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            slots = slots.clone()  # the combine buffer is reused by the next layer
        y = torch.empty(t, mod.hidden, dtype=torch.bfloat16, device=dev)
        ops.count_launch()
        ops.native().moe_combine(slots, w, y)
        ctx.mod = mod
        ctx.save_for_backward(w, slots, dest32, row32, h, prefix, base, lens, rows_dev)
        ctx.total_in, ctx.max_tiles, ctx.topv_dtype = total_in, max_tiles, topv.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        from dattri_llm_b200 import ops

        mod = ctx.mod
        w, slots, dest32, row32, h, prefix, base, lens, rows_dev = ctx.saved_tensors
        t, k = w.shape
        dev = dy.device
        dy = dy.to(torch.bfloat16).contiguous()
        dtopv = torch.empty(t, k, dtype=torch.float32, device=dev)
        mod.barrier.wait()
        ops.count_launch()
        # router-weight gradient and the slot gradients' dispatch to the owners in one kernel
        ops.native().moe_combine_bwd_dispatch(dy, slots, w, dtopv, dest32, row32, mod.recv_x.peers,
                                              mod.recv_meta.peers, mod.rank)
        mod.barrier.wait()
        total_in = ctx.total_in
        if total_in:
            err = ops.error_word(dev)
            dout = mod.recv_x.local[:total_in]
            da = torch.empty(total_in, mod.intermediate, dtype=torch.bfloat16, device=dev)
            dh = torch.empty_like(h[:total_in])
            ops.count_launch(3)
            ops.native().gemm_ragged(dout, mod.down_t, da, prefix, base, lens, ctx.max_tiles, [], None, err)
            ops.native().swiglu_split_bwd(da, h[:total_in].contiguous(), dh, rows_dev)
            # The input-gradient GEMM returns every row to its source rank.
            ops.native().gemm_ragged(dh, mod.gate_up_t, None, prefix, base, lens, ctx.max_tiles,
                                     mod.dx_slots.peers, mod.recv_meta.local[:total_in], err)
        mod.barrier.wait()
        dx = torch.empty(t, mod.hidden, dtype=torch.bfloat16, device=dev)
        ops.count_launch()
        ops.native().moe_combine(mod.dx_slots.local[:t * k], torch.ones_like(w), dx)  # sum of the k slots
        return dx, dtopv.to(ctx.topv_dtype), None, None


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

    @classmethod
    def get(cls, capacity: int, slots: int, hidden: int, dev: torch.device, group) -> _Buffers:
        key = (capacity, slots, hidden, dev, id(group))
        if key not in cls._pool:
            cls._pool[key] = cls(capacity, slots, hidden, dev, group)
        return cls._pool[key]


class ExpertParallelMoE(nn.Module):
    """Top-k MoE MLP with experts sharded over the process group (frozen experts: the
    attribution probe's case; the router may train).  Build collectively."""

    def __init__(self, hidden: int, intermediate: int, n_experts: int, top_k: int, *, max_tokens: int,
                 norm_topk_prob: bool = False, group=None, device: torch.device | None = None) -> None:
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        if hidden % 8 or intermediate % 8:
            raise ValueError("hidden and intermediate sizes must be multiples of 8")
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.hidden, self.intermediate, self.n_experts, self.top_k = hidden, intermediate, n_experts, top_k
        self.experts_per_rank = n_experts // self.world
        self.norm_topk_prob = norm_topk_prob
        self.max_tokens = max_tokens
        self.capacity = self.world * max_tokens * top_k
        self.gate = nn.Linear(hidden, n_experts, bias=False, device=dev, dtype=torch.bfloat16)
        e_l = self.experts_per_rank
        self.register_buffer("gate_up", torch.zeros(e_l, 2 * intermediate, hidden, device=dev, dtype=torch.bfloat16))
        self.register_buffer("down", torch.zeros(e_l, hidden, intermediate, device=dev, dtype=torch.bfloat16))
        self.register_buffer("gate_up_t", torch.zeros(e_l, hidden, 2 * intermediate, device=dev, dtype=torch.bfloat16))
        self.register_buffer("down_t", torch.zeros(e_l, intermediate, hidden, device=dev, dtype=torch.bfloat16))
        bufs = _Buffers.get(self.capacity, max_tokens * top_k, hidden, dev, group)
        self.recv_x, self.recv_meta = bufs.recv_x, bufs.recv_meta
        self.combine, self.dx_slots, self.barrier = bufs.combine, bufs.dx_slots, bufs.barrier

    @torch.no_grad()
    def load_experts(self, gate_up_all: torch.Tensor, down_all: torch.Tensor, router: torch.Tensor) -> None:
        """Take this rank's slice of the full ``(E, 2I, H)`` / ``(E, H, I)`` expert weights and
        the ``(E, H)`` router weight (identical on every rank)."""
        e_l, r = self.experts_per_rank, self.rank
        gu = gate_up_all[r * e_l:(r + 1) * e_l].to(self.gate_up.device, torch.bfloat16)
        dn = down_all[r * e_l:(r + 1) * e_l].to(self.down.device, torch.bfloat16)
        self.gate_up.copy_(gu)
        self.down.copy_(dn)
        self.gate_up_t.copy_(gu.transpose(1, 2))
        self.down_t.copy_(dn.transpose(1, 2))
        self.gate.weight.copy_(router.to(self.gate.weight.device, torch.bfloat16))

    def route(self, x2: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``(top-k probabilities, top-k expert ids)`` of every token."""
        probs = torch.softmax(self.gate(x2).float(), dim=-1)
        topv, topi = probs.topk(self.top_k, dim=-1)
        if self.norm_topk_prob:
            topv = topv / topv.sum(-1, keepdim=True)
        return topv, topi

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.hidden).to(torch.bfloat16).contiguous()
        topv, topi = self.route(x2)
        y = _EPMoE.apply(x2, topv, topi, self)
        return y.view(*shape[:-1], self.hidden)
