"""Online data selection inside the training step.

At every step end the per-sample gradients of the batch are scored against a
target (``"batch"``: the batch itself; ``"fixed"``: a given gradient;
``"val_loader"``: the gradient of the next validation batch, captured by a
secondary backward through the same hooks), samples are selected for removal
(``hard`` threshold, ``bottom_fraction`` or ``negative_bottom_fraction``; summed
over layers or ``layer_wise``) and their contributions are subtracted from the
parameters' ``.grad`` before the optimizer step:

* single device: subtract the dropped samples' per-sample gradients;
* DDP: after DDP's averaged write-back (queued behind the backward's final
  callbacks), one count all-reduce then one packed all-reduce of every hooked
  parameter's dropped contribution, divided by the world size;
* FSDP (``use_orig_params``): the same packed reduction, each rank subtracting
  only the slice of the flat parameter it owns.

Every rank runs the same collectives in the same order each step, even when it
drops nothing.  Scores are ghost cross-grams (:meth:`Gradient.similarity`), which
run on the fused tcgen05 kernels.  Parity: reference
``dattri_llm/gradient/callbacks/data_selection_callback.py:94-1348``.
"""

from __future__ import annotations

import math
import warnings
from collections.abc import Callable, Iterable, Mapping
from typing import Any, NamedTuple

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord, base_layer_name
from dattri_llm_b200.utils.autograd import queue_after_backward_finalization
from dattri_llm_b200.utils.distributed import dist_world_size, is_dist_initialized

_THRESHOLD_MODES = frozenset({"hard", "bottom_fraction", "negative_bottom_fraction"})
_SCORE_MODES = frozenset({"ghost", "materialized"})
_TARGET_MODES = frozenset({"batch", "fixed", "val_loader"})
_CHANNELS_FIRST = frozenset({"nn.GroupNorm", "nn.InstanceNorm1d", "nn.InstanceNorm2d", "nn.InstanceNorm3d"})


class _Shard(NamedTuple):
    shape: tuple[int, ...]
    in_shard: bool
    start: int | None
    end: int | None


def _concat_batches(batches: list) -> object:
    """Concatenate validation batches (tensors, mappings or sequences of them)."""
    first = batches[0]
    if torch.is_tensor(first):
        if len({tuple(b.shape[1:]) for b in batches}) != 1:
            raise ValueError("val_targets_per_pass > 1 needs val batches whose non-batch dimensions "
                             "agree; pad in the loader's collate_fn, or set val_targets_per_pass=1.")
        return torch.cat(list(batches), dim=0)
    if isinstance(first, Mapping):
        if {frozenset(b.keys()) for b in batches} != {frozenset(first.keys())}:
            raise ValueError("val_targets_per_pass > 1 needs every val batch to carry the same keys.")
        return type(first)({k: _concat_batches([b[k] for b in batches]) for k in first})
    if isinstance(first, (list, tuple)):
        if len({len(b) for b in batches}) != 1:
            raise ValueError("val_targets_per_pass > 1 needs every val batch to have the same length.")
        return type(first)(_concat_batches([b[i] for b in batches]) for i in range(len(first)))
    raise TypeError(f"Cannot concatenate val batches of type {type(first).__name__}.")


def _token_contraction(g: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    """``(out, in) = g^T a`` over the token rows of ``g (N, out)`` and ``a (N, in)``, fp32."""
    from dattri_llm_b200 import ops as native_ops

    aligned = g.shape[0] % 8 == 0 and g.shape[1] % 8 == 0 and a.shape[1] % 8 == 0
    if aligned and g.dtype == a.dtype == torch.bfloat16 and native_ops.use_native(g, a):
        return native_ops.per_sample_outer(g[None], a[None], out_dtype=torch.float32)[0]
    return g.float().T @ a.float()



def _sum_over_ranks(buf: torch.Tensor, world: int) -> None:
    """In-place sum of the packed dropped contributions over ranks: the NVLink peer all-reduce
    kernels when the group is the whole NCCL world on sm_100 GPUs (every rank packs the same
    layout, so the call is collective), else ``torch.distributed.all_reduce``."""
    import torch.distributed as dist

    from dattri_llm_b200.parallel import symm

    if world == dist.get_world_size() and symm.all_reduce_sum_(buf):
        return
    dist.all_reduce(buf)

class DataSelectionCallback(HookManagerCallback):
    """Score every sample of each step and remove the selected ones' gradient contributions.

    Args:
        model: The trained model (or its DDP/FSDP wrapper).
        target: ``"batch"``, ``"fixed"`` or ``"val_loader"``.
        target_gradient: The fixed target (``target="fixed"``).
        val_loader / val_loss_fn: Source and loss of the validation target.
        renormalize: Rescale the kept samples so the update keeps the batch mean's scale.
        val_targets_per_pass: Validation batches captured per secondary backward.
        scoring_kwargs: ``{"score_mode": "ghost" | "materialized"}``.
        selection_kwargs: ``{"threshold", "threshold_mode", "layer_wise"}``.
    """

    _SCORING_KEYS = frozenset({"score_mode"})
    _SELECTION_KEYS = frozenset({"threshold", "threshold_mode", "layer_wise"})

    def __init__(self, model: nn.Module, target: str = "batch", target_gradient: Gradient | None = None,
                 val_loader: Iterable | None = None, val_loss_fn: Callable | None = None,
                 renormalize: bool = False, val_targets_per_pass: int = 1, *,
                 scoring_kwargs: dict[str, Any] | None = None,
                 selection_kwargs: dict[str, Any] | None = None) -> None:
        scoring_kwargs = dict(scoring_kwargs or {})
        selection_kwargs = dict(selection_kwargs or {})
        for given, allowed, what in ((scoring_kwargs, self._SCORING_KEYS, "scoring_kwargs"),
                                     (selection_kwargs, self._SELECTION_KEYS, "selection_kwargs")):
            unknown = set(given) - allowed
            if unknown:
                raise ValueError(f"Unknown {what} keys: {sorted(unknown)}; allowed: {sorted(allowed)}.")
        scoring_kwargs.setdefault("score_mode", "ghost")
        selection_kwargs.setdefault("threshold", 0.0)
        selection_kwargs.setdefault("threshold_mode", "hard")
        selection_kwargs.setdefault("layer_wise", False)
        t_mode, thr = selection_kwargs["threshold_mode"], selection_kwargs["threshold"]
        if t_mode not in _THRESHOLD_MODES:
            raise ValueError(f"threshold_mode must be one of {sorted(_THRESHOLD_MODES)}, got {t_mode!r}.")
        if t_mode != "hard" and not 0.0 <= thr < 1.0:
            raise ValueError(f"threshold must be in [0, 1) for threshold_mode={t_mode!r}, got {thr}.")
        if scoring_kwargs["score_mode"] not in _SCORE_MODES:
            raise ValueError(f"score_mode must be one of {sorted(_SCORE_MODES)}, got "
                             f"{scoring_kwargs['score_mode']!r}.")
        if target not in _TARGET_MODES:
            raise ValueError(f"target must be one of {sorted(_TARGET_MODES)}, got {target!r}.")
        if target == "fixed" and target_gradient is None:
            raise ValueError("target='fixed' requires target_gradient to be a Gradient object.")
        if target == "val_loader" and val_loader is None:
            raise ValueError("target='val_loader' requires val_loader.")
        if target == "val_loader" and val_loss_fn is None:
            raise ValueError("target='val_loader' requires val_loss_fn.")
        if val_targets_per_pass < 1:
            raise ValueError(f"val_targets_per_pass must be >= 1, got {val_targets_per_pass}.")
        if val_targets_per_pass > 1 and t_mode == "hard":
            warnings.warn(
                "val_targets_per_pass > 1 with threshold_mode='hard': batching the val targets rescales "
                "the scores by a per-step constant when the val loss averages over its batch, so an "
                "absolute threshold no longer means what it did at val_targets_per_pass=1.",
                stacklevel=2,
            )
        self._scoring_kwargs, self._selection_kwargs = scoring_kwargs, selection_kwargs
        self._root = getattr(model, "module", model)
        self._model = model
        self._shards: dict[int, _Shard] | None = None
        self._fsdp_world = 1
        self._target, self._target_gradient = target, target_gradient
        self._val_per_pass = val_targets_per_pass
        self._val_targets: list[Gradient] = []
        self._val_loader, self._val_loss_fn = val_loader, val_loss_fn
        self._val_iter = iter(val_loader) if val_loader is not None else None
        self._renormalize = renormalize
        self._manager = None
        self._in_val_pass = False
        self._pending_val: Gradient | None = None
        self.last_scores: torch.Tensor | None = None
        self.last_dropped: list[int] = []

    def on_register(self, hook_manager) -> None:
        """Remember the manager (its hooks capture the validation target)."""
        self._manager = hook_manager

    # ------------------------------------------------------------ step
    def on_step_end(self, record: GradientRecord) -> None:
        """Score, select and remove contributions for *record*'s step."""
        if self._in_val_pass:
            self._pending_val = record.gradient
            return
        if self._target == "val_loader":
            self._collect_val_gradient()
        target = self._resolve_target()
        layer_scores = self.compute_scores(record.gradient, target, scoring_kwargs=self._scoring_kwargs)
        dropped = self._select(layer_scores)
        summed = self._sum(layer_scores)
        self.last_scores = None if summed is None else summed.detach().cpu()
        union: set[int] = set()
        for idx in dropped.values():
            union.update(idx)
        self.last_dropped = sorted(union)
        self._ensure_shard_map()
        if self._shards:
            self._remove_fsdp(record, self._global_drops(dropped))
        elif is_dist_initialized() and dist_world_size() > 1:
            self._remove_ddp(record, self._global_drops(dropped))
        elif union:
            self.remove_contributions(record, dropped, self._root, renormalize=self._renormalize)

    @staticmethod
    def _sum(layer_scores: dict[str, torch.Tensor]) -> torch.Tensor | None:
        total = None
        for s in layer_scores.values():
            total = s.clone() if total is None else total + s
        return total

    def _select(self, layer_scores: dict[str, torch.Tensor]) -> dict[str, list[int]]:
        if self._selection_kwargs.get("layer_wise", False):
            return {n: self.select_samples(s, selection_kwargs=self._selection_kwargs)
                    for n, s in layer_scores.items()}
        summed = self._sum(layer_scores)
        shared = [] if summed is None else self.select_samples(summed, selection_kwargs=self._selection_kwargs)
        return {n: list(shared) for n in layer_scores}

    def _global_drops(self, dropped: dict[str, list[int]]) -> list[int]:
        if self._selection_kwargs.get("layer_wise", False):
            raise NotImplementedError("selection_kwargs['layer_wise'] is not supported under FSDP/DDP; "
                                      "use single-device training for per-layer selection.")
        return next((list(v) for v in dropped.values()), [])

    def _resolve_target(self) -> Gradient | None:
        if self._target == "batch":
            return None
        if self._target == "fixed":
            return self._target_gradient
        return self._pending_val

    def _next_val_batch(self):
        try:
            return next(self._val_iter)
        except StopIteration:
            self._val_iter = iter(self._val_loader)
            return next(self._val_iter)

    def _collect_val_gradient(self) -> None:
        if self._manager is None:
            raise RuntimeError("target='val_loader' requires this callback to be attached to a "
                               "HookManager: the val gradient is captured through the manager's hooks.")
        if self._val_targets:
            self._pending_val = self._val_targets.pop(0)
            return
        batches = [self._next_val_batch() for _ in range(self._val_per_pass)]
        batch = batches[0] if len(batches) == 1 else _concat_batches(batches)
        saved = {n: (p.grad.detach().clone() if p.grad is not None else None)
                 for n, p in self._root.named_parameters()}
        state = self._manager.save_state()
        self._manager.clear_state()
        self._pending_val = None
        self._in_val_pass = True
        try:
            with torch.enable_grad():
                self._root.zero_grad()
                self._val_loss_fn(self._root, batch).backward()
        finally:
            self._in_val_pass = False
            self._manager.load_state(state)
            for n, p in self._root.named_parameters():
                p.grad = saved[n]
        if self._pending_val is not None and self._val_per_pass > 1:
            captured = self._pending_val
            self._val_targets = [captured.slice("batch", [i]) for i in range(1, captured.batch_size)]
            self._pending_val = captured.slice("batch", [0])
        if self._pending_val is None:
            raise RuntimeError("The val backward did not complete a capture step, so no val target was "
                               "collected: val_loss_fn must run the model so that the backward reaches "
                               "every hooked layer.")

    @staticmethod
    def select_samples(scores: torch.Tensor, *, selection_kwargs: dict[str, Any] | None = None) -> list[int]:
        """Indices to drop: ``hard`` (score < threshold), ``bottom_fraction`` (lowest
        ``round(B * threshold)``) or ``negative_bottom_fraction`` (those of them below 0)."""
        kw = selection_kwargs or {}
        thr, mode = kw.get("threshold", 0.0), kw.get("threshold_mode", "hard")
        if mode == "hard":
            return (scores < thr).nonzero(as_tuple=True)[0].tolist()
        n = round(scores.shape[0] * thr)
        if n == 0:
            return []
        bottom = scores.argsort()[:n].tolist()
        return bottom if mode == "bottom_fraction" else [i for i in bottom if scores[i] < 0]

    @staticmethod
    def compute_scores(gradient: Gradient, target: Gradient | None = None, *,
                       scoring_kwargs: dict[str, Any] | None = None) -> dict[str, torch.Tensor]:
        """``{layer: (B,)}`` alignment of each sample with the target (row sums of the
        per-layer cross-gram; the batch itself when *target* is ``None``)."""
        mode = "materialized" if (scoring_kwargs or {}).get("score_mode", "ghost") == "materialized" else "auto"
        if target is not None and target.device != gradient.device:
            target = target.to(gradient.device)
        scorable = [n for n in gradient.layer_names if gradient.layer_types.get(n) != ops.PARAM_GRAD_TYPES]
        other = gradient if target is None else target
        if len(scorable) < len(gradient.layer_names):
            gradient = gradient.select_layers(scorable)
            other = gradient if target is None else other.select_layers([n for n in scorable if n in other.layer_names])
        b = gradient.batch_size
        out = {}
        for name, m in gradient.similarity(other, mode=mode).items():
            s = m.sum(1)
            out[name] = s.expand(b) if s.shape[0] < b else s
        return out

    # ------------------------------------------------------------ removal (single device)
    @staticmethod
    def remove_contributions(record: GradientRecord, dropped: dict[str, list[int]], root: nn.Module, *,
                             renormalize: bool = False) -> None:
        """Subtract the dropped samples' gradients from ``.grad`` of every factorized layer."""
        b = record.gradient.batch_size
        for name, val in record.gradient.data.items():
            drop = dropped.get(name, [])
            if not isinstance(val, Factorized) or not drop:
                continue
            bf = val.as_batch_first()
            if bf.pre_activation_grad.shape[0] < b:
                continue
            try:
                module = root.get_submodule(base_layer_name(name))
            except AttributeError:
                continue
            lt = record.gradient.layer_types[name]
            if renormalize and 0 < len(drop) < b:
                a_d, g_d = DataSelectionCallback._reweighted(bf, drop)
            else:
                a_d, g_d = bf.activation[drop], bf.pre_activation_grad[drop]
            weight = getattr(module, "weight", None)
            if weight is not None and weight.grad is not None:
                contrib = DataSelectionCallback._weight_contribution(lt, bf.module_kwargs, a_d, g_d,
                                                                      tuple(weight.shape))
                if ops.is_embedding(lt):
                    vocab = contrib.numel() // weight.shape[1]
                    weight.grad[:vocab] -= contrib.reshape(vocab, -1).to(weight.grad.device, weight.grad.dtype)
                else:
                    weight.grad -= contrib.reshape_as(weight.grad).to(weight.grad.device, weight.grad.dtype)
            bias = getattr(module, "bias", None)
            if bias is not None and bias.grad is not None:
                bias.grad -= DataSelectionCallback._bias_contribution(lt, g_d, bias.shape[0]).to(
                    bias.grad.device, bias.grad.dtype)

    @staticmethod
    def _reweighted(bf: Factorized, drop: list[int]):
        """Factors whose token-summed gradient is the dropped samples' sum minus the kept
        samples' scaled by ``k / (B - k)`` (keeps the mean's scale after removal)."""
        g = bf.pre_activation_grad
        b, k = g.shape[0], len(drop)
        w = torch.full((b,), -k / (b - k), dtype=torch.float32, device=g.device)
        w[drop] = 1.0
        return bf.activation, g * w.view(-1, *([1] * (g.dim() - 1)))

    @staticmethod
    def _weight_contribution(lt: str, mk: dict | None, a_d, g_d, shape: tuple[int, ...]) -> torch.Tensor:
        """Sum of the dropped samples' weight gradients, flat in the parameter's layout.  For a
        linear layer that is ONE contraction over every dropped token, ``G^T A`` (a tcgen05
        GEMM with fp32 accumulation for bf16 factors on sm_100), instead of one ``(out, in)``
        gradient per sample summed afterwards."""
        if lt == "nn.Linear" and a_d.is_floating_point() and a_d.dim() == g_d.dim() >= 2:
            return _token_contraction(g_d.reshape(-1, g_d.shape[-1]), a_d.reshape(-1, a_d.shape[-1])).reshape(-1)
        contrib = ops.materialize(Factorized(a_d, g_d, mk), lt, include_bias=False).sum(0)
        if ops.is_embedding(lt):
            return contrib
        if ops.is_norm(lt):
            return contrib.reshape(-1, math.prod(shape)).sum(0)
        if lt == "transformers.pytorch_utils.Conv1D":
            return contrib.reshape(shape[1], shape[0]).T.reshape(-1)
        return contrib.reshape(-1)

    @staticmethod
    def _bias_contribution(lt: str, g_d: torch.Tensor, channels: int) -> torch.Tensor:
        (g,) = ops.dtypes.align(g_d, minimum=torch.float32)
        if ops.is_conv(lt) or ops.is_conv_transpose(lt) or lt in _CHANNELS_FIRST:
            return g.movedim(1, -1).reshape(-1, channels).sum(0)
        return g.reshape(-1, channels).sum(0)

    # ------------------------------------------------------------ removal (DDP / FSDP)
    def _ensure_shard_map(self) -> None:
        if self._shards is not None:
            return
        shards: dict[int, _Shard] = {}
        for m in self._model.modules():
            flat = getattr(m, "_flat_param", None)
            infos = getattr(flat, "_shard_param_infos", None) if flat is not None else None
            params = getattr(flat, "_params", None) if flat is not None else None
            shapes = getattr(flat, "_shapes", None) if flat is not None else None
            if infos is None or params is None or shapes is None:
                continue
            for p, info, shape in zip(params, infos, shapes, strict=True):
                shards[id(p)] = _Shard(tuple(shape), bool(info.in_shard), info.intra_param_start_idx,
                                       info.intra_param_end_idx)
        self._shards = shards
        if shards:
            self._fsdp_world = dist_world_size()

    @staticmethod
    def _coll_device() -> torch.device:
        import torch.distributed as dist

        if "nccl" in str(dist.get_backend()).lower():
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")

    def _contributions(self, record, dropped, shape_of) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """``[(param, flat fp32 contribution in the full parameter's layout)]``; zeros on a
        rank that drops nothing, so every rank packs the same buffer."""
        b = record.gradient.batch_size
        renorm = self._renormalize and 0 < len(dropped) < b
        out = []
        for name, val in sorted(record.gradient.data.items()):
            if not isinstance(val, Factorized):
                continue
            bf = val.as_batch_first()
            if bf.pre_activation_grad.shape[0] < b:
                continue
            try:
                module = self._root.get_submodule(base_layer_name(name))
            except AttributeError:
                continue
            lt = record.gradient.layer_types[name]
            if renorm:
                a_d, g_d = self._reweighted(bf, dropped)
            elif dropped:
                a_d, g_d = bf.activation[dropped], bf.pre_activation_grad[dropped]
            else:
                a_d = g_d = None
            dev = record.gradient.device
            weight = getattr(module, "weight", None)
            wshape = shape_of(weight) if weight is not None else None
            if wshape is not None:
                flat = torch.zeros(math.prod(wshape), dtype=torch.float32, device=dev)
                if dropped:
                    c = self._weight_contribution(lt, bf.module_kwargs, a_d, g_d, wshape)
                    flat[: c.numel()] = c.float()
                out.append((weight, flat))
            bias = getattr(module, "bias", None)
            bshape = shape_of(bias) if bias is not None else None
            if bshape is not None:
                ch = math.prod(bshape)
                flat = (self._bias_contribution(lt, g_d, ch).float() if dropped
                        else torch.zeros(ch, dtype=torch.float32, device=dev))
                out.append((bias, flat))
        return out

    def _remove_fsdp(self, record: GradientRecord, dropped: list[int]) -> None:
        import torch.distributed as dist

        world = self._fsdp_world
        use_dist = world > 1 and is_dist_initialized()
        if use_dist:
            dev = self._coll_device()
            count = torch.tensor([len(dropped)], dtype=torch.long, device=dev)
            dist.all_reduce(count)
            if not int(count.item()):
                return
        elif not dropped:
            return
        entries = self._contributions(record, dropped, lambda p: self._shards[id(p)].shape
                                      if id(p) in self._shards else None)
        if not entries:
            return
        if use_dist:
            buf = torch.cat([f for _, f in entries]).to(dev)
            _sum_over_ranks(buf, world)
            buf /= world
            off = 0
            for p, f in entries:
                self._subtract_slice(p, buf[off: off + f.numel()])
                off += f.numel()
        else:
            for p, f in entries:
                self._subtract_slice(p, f)

    def _subtract_slice(self, param: torch.Tensor, full: torch.Tensor) -> None:
        spec = self._shards[id(param)]
        if not spec.in_shard or param.grad is None:
            return
        seg = full.reshape(-1)[spec.start: spec.end + 1]
        param.grad -= seg.to(param.grad.device, param.grad.dtype)

    def _remove_ddp(self, record: GradientRecord, dropped: list[int]) -> None:
        def apply() -> None:
            import torch.distributed as dist

            world = dist_world_size()
            dev = self._coll_device()
            count = torch.tensor([len(dropped)], dtype=torch.long, device=dev)
            dist.all_reduce(count)
            if not int(count.item()):
                return
            entries = self._contributions(record, dropped, lambda p: tuple(p.shape))
            if not entries:
                return
            buf = torch.cat([f for _, f in entries]).to(dev)
            _sum_over_ranks(buf, world)
            buf /= world
            off = 0
            for p, f in entries:
                n = f.numel()
                if p.grad is not None:
                    p.grad -= buf[off: off + n].reshape(p.grad.shape).to(p.grad.device, p.grad.dtype)
                off += n

        if not queue_after_backward_finalization(apply):
            apply()
