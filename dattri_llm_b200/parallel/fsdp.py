"""Row-sharded linear layers whose collectives live inside their GEMMs (FSDP-style).

:class:`ShardedLinear` keeps ``1/world`` of its weight rows on each rank, in symmetric
memory, plus the transposed shard.  Nothing is all-gathered into HBM:

* forward   ``y = x W^T``: ONE launch (``gemm_tn_staged`` mode 0) whose first CTAs pull
  the remote shards over NVLink into a local staging matrix -- every remote byte once --
  while every CTA's GEMM tile starts on its own shard's rows or waits (bounded) on the
  flag of the owner whose rows it needs;
* backward  ``dx = dy W``: the same over the peers' transposed shards, gated per K range
  (mode 1);
* weight gradient (when the weight trains): ``dW = dy^T x`` reduce-scattered INSIDE its
  GEMM -- the epilogue stores every fp32 element with 16-byte NVLink stores into its
  owner rank's slot for this rank (``gemm_tn_rs``); after a bounded cross-GPU barrier each
  owner adds its ``world`` slots into its gradient shard (``slot_reduce``, local memory).

The capture hooks see an ``nn.Linear`` (same module boundary, full-width input and
output), so per-sample capture is unchanged.  The reference reaches the same math through
FSDP's NCCL all-gather / reduce-scatter around cuBLAS GEMMs
(``dattri_llm/gradient/streaming.py:1175-1203``).
"""

from __future__ import annotations

import functools

import torch
import torch.distributed as dist
from torch import nn

from dattri_llm_b200.parallel.symm import PeerBarrier, SymmetricBuffer


class _Staging:
    """A local staging matrix for one gathered weight shape and staging mode, with its copy
    flags and the launch counter that gates them (shared by every layer of that shape and
    mode: launches on one stream use it one after another).  A flag counts the pieces of its
    owner copied so far and a launch waits for ``epoch x pieces per owner``; the two modes
    cut their shards into different numbers of pieces, so they never share a counter."""

    _pool: dict = {}

    def __init__(self, rows: int, cols: int, world: int, device: torch.device) -> None:
        self.buf = torch.empty(rows, cols, dtype=torch.bfloat16, device=device)
        self.flags = torch.zeros(world, dtype=torch.int32, device=device)
        self.epoch = 0

    @classmethod
    def get(cls, rows: int, cols: int, world: int, device: torch.device, mode: int) -> _Staging:
        key = (rows, cols, world, device, mode)
        st = cls._pool.get(key)
        if st is None:
            st = cls._pool[key] = cls(rows, cols, world, device)
        return st

    def launch(self, a: torch.Tensor, peers, out: torch.Tensor, mode: int, self_rank: int) -> None:
        from dattri_llm_b200 import ops

        self.epoch += 1
        ops.count_launch()
        ops.native().gemm_tn_staged(a, peers, self.buf, out, self.flags, self.epoch, mode, self_rank,
                                    ops.STORE_BF16, 1.0, ops.error_word(a.device))


class _SlotRing:
    """Two symmetric slot buffers (``world`` fp32 slots of one weight shard each) shared by
    every sharded layer of one shape.  Consecutive weight-gradient reductions alternate
    between them: a source writes buffer ``i`` again only after the barrier that follows
    the next reduction, which every owner reaches after summing buffer ``i``."""

    _pool: dict = {}

    def __init__(self, shard_elems: int, device: torch.device, group) -> None:
        world = dist.get_world_size(group)
        self.bufs = [SymmetricBuffer((world * shard_elems,), torch.float32, device, group) for _ in range(2)]
        self.ptrs = [torch.tensor([int(p.data_ptr()) for p in b.peers], dtype=torch.int64, device=device)
                     for b in self.bufs]
        self.turn = 0

    @classmethod
    def get(cls, shard_elems: int, device: torch.device, group) -> _SlotRing:
        key = (shard_elems, device, id(group))
        ring = cls._pool.get(key)
        if ring is None:
            ring = cls._pool[key] = cls(shard_elems, device, group)
        return ring

    def next(self) -> tuple[SymmetricBuffer, torch.Tensor]:
        i = self.turn
        self.turn ^= 1
        return self.bufs[i], self.ptrs[i]


class _AGLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight_shard, layer):
        from dattri_llm_b200 import ops

        k = layer.in_features
        x2 = x.reshape(-1, k)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = torch.empty(x2.shape[0], layer.out_features, dtype=torch.bfloat16, device=x.device)
        _Staging.get(layer.out_features, k, layer.world, x.device, 0).launch(x2, layer._w.peers, y, 0, layer.rank)
        ctx.layer = layer
        ctx.save_for_backward(x2 if weight_shard.requires_grad else x2.new_empty(0))
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], layer.out_features)

    @staticmethod
    def backward(ctx, dy):
        from dattri_llm_b200 import ops

        layer = ctx.layer
        dy2 = dy.reshape(-1, layer.out_features)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(dy2.shape[0], layer.in_features, dtype=torch.bfloat16, device=dy.device)
            _Staging.get(layer.in_features, layer.out_features, layer.world, dy.device, 1).launch(
                dy2, layer._wt.peers, dx, 1, layer.rank)
            dx = dx.view(ctx.in_shape)
        if ctx.needs_input_grad[1]:
            (x2,) = ctx.saved_tensors
            layer._reduce_scatter_wgrad(dy2, x2)
        return dx, None, None


class ShardedLinear(nn.Linear):
    """A bias-free ``nn.Linear`` whose weight rows are sharded over the process group."""

    def __init__(self, linear: nn.Linear, group=None) -> None:
        nn.Module.__init__(self)
        if linear.bias is not None:
            raise ValueError("ShardedLinear shards bias-free linears")
        w = linear.weight.detach()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if self.out_features % (world * 64) or self.in_features % 8:
            raise ValueError(f"out_features ({self.out_features}) must split into 64-row multiples over "
                             f"{world} ranks and in_features must be a multiple of 8")
        rows = self.out_features // world
        dev = w.device
        self._w = SymmetricBuffer((rows, self.in_features), torch.bfloat16, dev, group)
        self._wt = SymmetricBuffer((self.in_features, rows), torch.bfloat16, dev, group)
        shard = w[rank * rows:(rank + 1) * rows].to(torch.bfloat16)
        self._w.local.copy_(shard)
        self._wt.local.copy_(shard.t())
        self.rows, self.rank, self.world = rows, rank, world
        self.weight = nn.Parameter(self._w.local, requires_grad=linear.weight.requires_grad)
        self.register_parameter("bias", None)
        self._group = group
        self._grad = None
        self._barrier = None
        if self.weight.requires_grad:
            # Created here, collectively, not lazily in the backward (autograd's thread).
            shard_elems = rows * self.in_features
            self._grad = torch.zeros(shard_elems, dtype=torch.float32, device=dev)
            self._slots = _SlotRing.get(shard_elems, dev, group)
            self._barrier = PeerBarrier(dev, group)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        return _AGLinear.apply(x, self.weight, self)

    # -- training: weight gradient reduce-scattered inside its GEMM ----------------------
    def _reduce_scatter_wgrad(self, dy2: torch.Tensor, x2: torch.Tensor) -> None:
        from dattri_llm_b200 import ops

        if self._grad is None:
            raise RuntimeError("this ShardedLinear was built with a frozen weight; it keeps no gradient")
        dyt = ops.gemm.transpose_last2(dy2)  # (N, M): tokens contiguous
        xt = ops.gemm.transpose_last2(x2)    # (K, M)
        shard = self.rows * self.in_features
        slots, ptrs = self._slots.next()
        ops.count_launch(2)
        ops.native().gemm_tn_rs(dyt, xt, ptrs, self.world, shard // 4, self.out_features, self.in_features,
                                self.in_features, 1.0, ops.error_word(dy2.device), self.rank)
        self._barrier.wait()  # every source's slot for this rank has landed
        ops.native().slot_reduce(slots.local, self.world, shard, self._grad, shard, True)

    def grad_shard(self) -> torch.Tensor | None:
        """This rank's ``(rows, in_features)`` fp32 weight-gradient shard (after
        :func:`sync_sharded_grads`)."""
        return None if self._grad is None else self._grad.view(self.rows, self.in_features)

    def zero_grad_shard(self) -> None:
        """Zero this rank's gradient shard (collectively, before the next backward)."""
        if self._grad is not None:
            self._grad.zero_()


def sync_sharded_grads(model: nn.Module) -> None:
    """Barrier across the ranks of the sharded layers.  Every :class:`ShardedLinear`
    gradient shard already holds its sum over ranks in stream order once the backward has
    run (each reduction ends in the owner's slot sum); this only lines the ranks up."""
    for m in model.modules():
        if isinstance(m, ShardedLinear) and m._barrier is not None:
            m._barrier.wait()
            return


class _FrozenShard:
    """The sharded state of a frozen linear converted in place (:func:`shard_frozen_linears`):
    the same fields :class:`_AGLinear` reads from a :class:`ShardedLinear`."""

    def __init__(self, module: nn.Linear, group) -> None:
        w = module.weight.detach()
        self.in_features, self.out_features = module.in_features, module.out_features
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.rows = self.out_features // self.world
        dev = w.device
        self._w = SymmetricBuffer((self.rows, self.in_features), torch.bfloat16, dev, group)
        self._wt = SymmetricBuffer((self.in_features, self.rows), torch.bfloat16, dev, group)
        shard = w[self.rank * self.rows:(self.rank + 1) * self.rows].to(torch.bfloat16)
        self._w.local.copy_(shard)
        self._wt.local.copy_(shard.t())

    def _reduce_scatter_wgrad(self, dy2, x2) -> None:  # pragma: no cover - frozen weights only
        raise RuntimeError("a frozen sharded linear has no weight gradient")


def _sharded_forward(module: nn.Module, x: torch.Tensor) -> torch.Tensor:
    state = module._bw_frozen_shard
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    return _AGLinear.apply(x, module.weight, state)


def can_shard_frozen(module: nn.Module, world: int) -> bool:
    """Whether :func:`shard_frozen_linears` converts *module*: a bias-free ``nn.Linear``
    (or subclass) with a frozen bf16-castable weight whose rows split into 64-row multiples
    over *world* ranks and whose input width is a multiple of 8."""
    return (isinstance(module, nn.Linear) and module.bias is None and not module.weight.requires_grad
            and module.out_features % (world * 64) == 0 and module.in_features % 8 == 0
            and module.weight.is_cuda)


def shard_frozen_linears(model: nn.Module, group=None) -> list[str]:
    """Shard every eligible frozen linear of *model* over *group*, in place (collective).

    Each converted module keeps its identity -- and so every hook already registered on it
    -- but its full weight is replaced by this rank's row shard, its forward by the fused
    all-gather GEMM (``gemm_tn_staged`` mode 0) and its input gradient by the fused
    transposed-shard GEMM (mode 1); ``module.in_features`` / ``out_features`` are
    unchanged, so the capture engine still sees the full layer.  This is the FSDP
    FULL_SHARD layout of an attribution probe (frozen weights: no gradient reduce-scatter)
    with the parameter all-gather inside the GEMMs instead of NCCL around cuBLAS.  Returns
    the converted names.
    """
    world = dist.get_world_size(group)
    # Weights used outside their module's forward stay whole: tied weights, and the output
    # embedding (a fused LM-head loss reads it directly).
    uses: dict[int, int] = {}
    for _n, p in model.named_parameters(remove_duplicate=False):
        uses[id(p)] = uses.get(id(p), 0) + 1
    out_emb = model.get_output_embeddings() if hasattr(model, "get_output_embeddings") else None
    converted = []
    for name, module in model.named_modules():
        if getattr(module, "_bw_frozen_shard", None) is not None or not can_shard_frozen(module, world):
            continue
        if module is out_emb or uses.get(id(module.weight), 0) > 1:
            continue
        state = _FrozenShard(module, group)
        module._bw_frozen_shard = state
        module.weight = nn.Parameter(state._w.local, requires_grad=False)
        module.forward = functools.partial(_sharded_forward, module)
        converted.append(name)
    if converted:
        torch.cuda.synchronize(next(iter(model.parameters())).device)
    dist.barrier(group=group)
    return converted


def shard_linears(model: nn.Module, names: list[str] | None = None, group=None) -> list[str]:
    """Replace bias-free ``nn.Linear`` children (all, or those named) by :class:`ShardedLinear`
    in place, collectively; returns the replaced names."""
    replaced = []
    for name, mod in list(model.named_modules()):
        for child_name, child in list(mod.named_children()):
            full = f"{name}.{child_name}" if name else child_name
            if type(child) is not nn.Linear or child.bias is not None:
                continue
            if names is not None and full not in names:
                continue
            setattr(mod, child_name, ShardedLinear(child, group))
            replaced.append(full)
    return replaced
