"""Optimizer state of a hooked layer, laid out like the layer's per-sample gradient.

A captured layer's per-sample gradient is a flat row-major ``(out, in[+1])`` block for
linear and conv layers (the bias as the last column of each row) and weight-then-bias for
norms and embeddings.  :class:`OptimizerSnapshot` returns optimizer state tensors
(``exp_avg``, ``exp_avg_sq``, ...) in exactly that layout, optionally only at a set of flat
coordinates (the ``mask`` projection), wherever the parameters live:

* a plain module, or one under DDP: the parameters the optimizer holds;
* FSDP2 (``fully_shard``): DTensor state, gathered with ``full_tensor()``;
* FSDP1 with ``use_orig_params=True``: each rank holds a contiguous slice of every original
  parameter's flattened storage; the slice is placed into a zero tensor of the full shape
  and the ranks' pieces are summed (one packed all-reduce for several state keys).  The
  slice can only be located while FSDP exposes the original parameters as views of its
  flat parameter, i.e. inside the layer's backward -- :meth:`OptimizerSnapshot.bind`.

:class:`GradientPreconditioner` applies the optimizer's update rule to per-sample gradient
rows during capture (LESS-style Adam-preconditioned gradients).  Public names as in the
reference's ``dattri_llm/gradient/optimizer_state.py``.
"""

from __future__ import annotations

import math
import weakref
from collections.abc import Callable, Iterable
from dataclasses import dataclass, field

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.gradient import base_layer_name
from dattri_llm_b200.gradient.ops.types import canonical_class_name, is_conv, is_embedding, is_linear, is_norm
from dattri_llm_b200.utils.distributed import dist_world_size, is_dist_initialized

HF_CONV1D = "transformers.pytorch_utils.Conv1D"
_FLAT_PARAMS_MSG = ("this optimizer steps FSDP flat parameters, whose per-layer layout cannot be recovered; "
                    "wrap the model with FullyShardedDataParallel(use_orig_params=True).")


def optimizer_type(optimizer: torch.optim.Optimizer) -> str:
    """Name of the ``torch.optim`` class whose update rule *optimizer* follows (its own class
    or the nearest base class with a known rule).

    Raises:
        NotImplementedError: no known rule (non-coordinate-wise optimizers and the like).
    """
    known = ops.OPTIMIZER_STATE_KEYS
    name = next((cls.__name__ for cls in type(optimizer).__mro__ if cls.__name__ in known), None)
    if name is None:
        raise NotImplementedError(f"no per-coordinate update rule is known for {type(optimizer).__name__}; "
                                  f"supported optimizers: {sorted(known)}.")
    return name


def hf_trainer_param_names(model: nn.Module) -> list[str]:
    """Trainable parameter names in the order a Hugging Face ``Trainer`` puts them into its
    optimizer: the weight-decayed group (everything but biases and norm weights) first."""
    from transformers.trainer_pt_utils import get_parameter_names

    norm_types = [nn.LayerNorm]
    if hasattr(nn, "RMSNorm"):
        norm_types.append(nn.RMSNorm)
    decayed = set(get_parameter_names(model, norm_types))
    names = [name for name, p in model.named_parameters() if p.requires_grad]
    first = [name for name in names if name in decayed and "bias" not in name]
    taken = set(first)
    return first + [name for name in names if name not in taken]


def optimizer_from_state_dict(model: nn.Module, state_dict: dict, param_names: Iterable[str] | None = None,
                              *, optimizer_cls: type = torch.optim.AdamW) -> torch.optim.Optimizer:
    """An *optimizer_cls* over *model* restored from a saved ``state_dict``; saved parameter
    indices are mapped to *model*'s parameters through *param_names* (default: the
    Hugging Face Trainer order)."""
    by_name = dict(model.named_parameters())
    order = list(param_names) if param_names is not None else hf_trainer_param_names(model)
    groups = [{**{k: v for k, v in saved.items() if k != "params"},
               "params": [by_name[order[i]] for i in saved["params"]]} for saved in state_dict["param_groups"]]
    restored = optimizer_cls(groups)
    restored.load_state_dict(state_dict)
    return restored


def _is_dtensor(t: object) -> bool:
    try:
        from torch.distributed.tensor import DTensor
    except ImportError:  # pragma: no cover - builds without distributed tensors
        return False
    return isinstance(t, DTensor)


def _all_reduce_sum(t: torch.Tensor) -> None:
    if is_dist_initialized() and dist_world_size() > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.SUM)


# ---------------------------------------------------------------------------------- sources
@dataclass(frozen=True)
class _Local:
    """A parameter the optimizer holds whole (plain module or DDP)."""

    param: nn.Parameter

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.param.shape)

    def read(self, optimizer, key):
        return optimizer.state.get(self.param, {}).get(key)


@dataclass(frozen=True)
class _DTensorParam:
    """An FSDP2 parameter: its state is a DTensor, gathered on read."""

    param: nn.Parameter

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.param.shape)

    def read(self, optimizer, key):
        val = optimizer.state.get(self.param, {}).get(key)
        return val.full_tensor() if _is_dtensor(val) else val


@dataclass(frozen=True)
class _FlatSlice:
    """An FSDP1 original parameter: this rank's view ``param`` covers flat elements
    ``[lo, hi]`` (inclusive) of the full parameter, or nothing (``lo is None``)."""

    param: nn.Parameter
    full_shape: tuple[int, ...]
    lo: int | None
    hi: int | None

    @property
    def shape(self) -> tuple[int, ...]:
        return self.full_shape

    def read(self, optimizer, key):
        return optimizer.state.get(self.param, {}).get(key)

    def on_zeros(self, local: torch.Tensor | None, like: torch.Tensor) -> torch.Tensor:
        """This rank's piece of the full tensor, zeros elsewhere (summed over ranks later)."""
        full = torch.zeros(math.prod(self.full_shape), dtype=like.dtype, device=like.device)
        if self.lo is not None and local is not None and local.numel() > 0:
            full[self.lo:self.hi + 1] = local.reshape(-1).to(full.dtype)
        return full.view(self.full_shape)


@dataclass
class _Layer:
    """A hooked layer's parameters (``{"weight": source, "bias": source}``) as the optimizer
    sees them, filled in by :meth:`OptimizerSnapshot.bind`."""

    module: nn.Module
    layer_type: str
    sources: dict[str, object] = field(default_factory=dict)

    @property
    def sharded(self) -> bool:
        return isinstance(self.sources.get("weight"), _FlatSlice)


def _fsdp1_slice(module: nn.Module, role: str, t: torch.Tensor) -> _FlatSlice | None:
    """Locate an FSDP1 original parameter inside its flat parameter (only while FSDP exposes
    the original parameters as views, i.e. in forward / backward)."""
    flat = getattr(t, "_base", None)
    infos = getattr(flat, "_shard_param_infos", None)
    if infos is None:
        return None
    if flat._params is None:
        raise NotImplementedError(_FLAT_PARAMS_MSG)
    for param, shard, shape, where in zip(flat._params, infos, flat._shapes, flat._param_infos, strict=True):
        if where.module is module and where.param_name == role:
            inside = shard.in_shard
            return _FlatSlice(param, tuple(shape), shard.intra_param_start_idx if inside else None,
                              shard.intra_param_end_idx if inside else None)
    return None


def _fsdp2_param(root: nn.Module, module: nn.Module, role: str) -> nn.Parameter | None:
    """The sharded (DTensor) parameter FSDP2 registered for ``module.<role>``, if any."""
    for unit in root.modules():
        state_of = getattr(unit, "_get_fsdp_state", None)
        if state_of is None:
            continue
        group = getattr(state_of(), "_fsdp_param_group", None)
        for fsdp_param in getattr(group, "fsdp_params", ()):
            owner = fsdp_param._module_info
            if owner.module is module and owner.param_name == role:
                return fsdp_param.sharded_param
    return None


_IDX_ON_DEVICE: dict[tuple[int, str], tuple] = {}  # (id(idx), device) -> (weak ref, copy)


def _on_device(idx: torch.Tensor, device: torch.device) -> torch.Tensor:
    """*idx* on *device*, copied once per index tensor and device (coordinates are fixed per
    layer; a host-to-device copy per read would stall the host every time)."""
    if idx.device == device:
        return idx
    key = (id(idx), str(device))
    hit = _IDX_ON_DEVICE.get(key)
    if hit is not None and hit[0]() is idx:
        return hit[1]
    moved = idx.to(device)
    weakref.finalize(idx, _IDX_ON_DEVICE.pop, key, None)
    _IDX_ON_DEVICE[key] = (weakref.ref(idx), moved)
    return moved


class OptimizerSnapshot:
    """Per-layer optimizer state in each hooked layer's gradient layout (see the module
    docstring).  *model* may be wrapped (DDP / FSDP); layer names are resolved inside."""

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer) -> None:
        self._root = getattr(model, "module", model)
        self._optimizer = optimizer
        self.optimizer_type = optimizer_type(optimizer)
        if any(getattr(p, "_is_flat_param", False) for g in optimizer.param_groups for p in g["params"]):
            raise NotImplementedError(_FLAT_PARAMS_MSG)
        self._group_of = {id(p): g for g in optimizer.param_groups for p in g["params"]}
        self._layers: dict[str, _Layer] = {}
        self._host_steps: dict[int, int] = {}  # id(param) -> updates, for counts kept on the GPU
        self._step_hook = None

    @property
    def optimizer(self) -> torch.optim.Optimizer:
        """The optimizer being read."""
        return self._optimizer

    def module(self, layer_name: str) -> nn.Module:
        """The module behind *layer_name* (a virtual ``name@k`` invocation maps to ``name``)."""
        return self._root.get_submodule(base_layer_name(layer_name))

    # ------------------------------------------------------------------ binding
    def _layer(self, layer_name: str) -> _Layer:
        layer = self._layers.get(layer_name)
        if layer is None:
            module = self.module(layer_name)
            lt = canonical_class_name(module)
            if getattr(module, "weight", None) is None:
                raise ValueError(f"layer {layer_name!r} ({lt}) has no weight parameter.")
            if not (is_linear(lt) or is_conv(lt) or is_norm(lt) or is_embedding(lt)):
                raise NotImplementedError(f"no gradient layout for optimizer state of {lt} layers "
                                          f"({layer_name!r}); linear, conv, norm and embedding layers have one.")
            layer = self._layers[layer_name] = _Layer(module, lt)
        return layer

    def bind(self, layer_name: str) -> None:
        """Work out where the optimizer keeps the layer's parameters.  Under FSDP1 call this
        while the layer's parameters are exposed (its backward); elsewhere any time.

        Raises:
            RuntimeError: an FSDP1 layer read before it was ever bound.
            NotImplementedError: FSDP1 without ``use_orig_params``.
        """
        layer = self._layer(layer_name)
        for role in ("weight", "bias"):
            t = getattr(layer.module, role, None)
            if t is None or role in layer.sources:
                continue
            if _is_dtensor(t):
                layer.sources[role] = _DTensorParam(t)
                continue
            sharded = _fsdp2_param(self._root, layer.module, role)
            if sharded is not None:
                layer.sources[role] = _DTensorParam(sharded)
                continue
            piece = _fsdp1_slice(layer.module, role, t)
            if piece is not None:
                layer.sources[role] = piece
            elif getattr(t, "_fsdp_flattened", False):
                raise RuntimeError(f"{layer_name!r} is FSDP-sharded and has not been bound: call "
                                   "OptimizerSnapshot.bind() for it during its backward before reading its state.")
            else:
                layer.sources[role] = _Local(t)

    def parameters(self, layer_name: str, include_bias: bool = True) -> list[tuple[str, nn.Parameter]]:
        """``[(role, parameter)]`` for ``weight`` (and ``bias``) as the optimizer holds them."""
        self.bind(layer_name)
        sources = self._layers[layer_name].sources
        roles = ("weight", "bias") if include_bias else ("weight",)
        return [(role, sources[role].param) for role in roles if role in sources]

    def _sources(self, layer_name: str, include_bias: bool) -> dict[str, object]:
        self.bind(layer_name)
        sources = self._layers[layer_name].sources
        return {role: src for role, src in sources.items() if include_bias or role == "weight"}

    # ------------------------------------------------------------------ layout
    def width(self, layer_name: str, include_bias: bool = True) -> int:
        """Length of the layer's flattened gradient."""
        return sum(math.prod(src.shape) for src in self._sources(layer_name, include_bias).values())

    def flatten(self, layer_name: str, tensors: dict[str, torch.Tensor],
                idx: torch.Tensor | None = None) -> torch.Tensor:
        """``{"weight"[, "bias"]}`` tensors in the layer's flat gradient layout (the entries at
        flat coordinates *idx* when given)."""
        layer = self._layer(layer_name)
        weight, bias = tensors["weight"], tensors.get("bias")
        if layer.layer_type == HF_CONV1D:  # stores (in, out)
            weight = weight.t()
        per_row = is_linear(layer.layer_type) or is_conv(layer.layer_type)
        if per_row:
            weight = weight.reshape(weight.shape[0], -1)
            if bias is not None:
                weight = torch.cat([weight, bias.reshape(-1, 1).to(weight.dtype)], dim=1)
            flat = weight.reshape(-1)
        else:
            parts = [weight.reshape(-1)] + ([] if bias is None else [bias.reshape(-1).to(weight.dtype)])
            flat = torch.cat(parts)
        return flat if idx is None else flat[_on_device(idx, flat.device)]

    # ------------------------------------------------------------------ hyperparameters
    def group(self, layer_name: str) -> dict:
        """The optimizer parameter group that holds the layer's weight.

        Raises:
            ValueError: the weight is not optimized by this optimizer.
        """
        weight = self._sources(layer_name, False)["weight"].param
        group = self._group_of.get(id(weight))
        if group is None:
            raise ValueError(f"the optimizer does not hold {layer_name!r}'s weight.")
        return group

    def hyperparameters(self, layer_name: str) -> dict:
        """The optimizer's defaults with the layer's group settings on top."""
        merged = dict(self._optimizer.defaults)
        merged.update((k, v) for k, v in self.group(layer_name).items() if k != "params")
        return merged

    def step_count(self, layer_name: str) -> int:
        """How many updates the layer's weight has had (0 before the first)."""
        src = self._sources(layer_name, False)["weight"]
        step = src.read(self._optimizer, "step")
        if step is None and isinstance(src, _FlatSlice):  # no piece of it on this rank
            steps = [st["step"] for st in self._optimizer.state.values() if "step" in st]
            step = max(steps, default=0)
        if isinstance(step, torch.Tensor):
            step = self._device_step(src.param, step) if step.is_cuda else step.item()
        return int(step or 0)

    def _device_step(self, param: torch.Tensor, step: torch.Tensor) -> int:
        """The update count of *param* when the optimizer keeps it in a GPU tensor (fused or
        capturable AdamW): read once, then counted on the host by a post-step hook, since a
        read per call would wait for every kernel queued before it."""
        key = id(param)
        if key not in self._host_steps:
            self._host_steps[key] = int(step.item())
            if self._step_hook is None:
                self._step_hook = self._optimizer.register_step_post_hook(self._count_step)
        return self._host_steps[key]

    def _count_step(self, optimizer, args, kwargs) -> None:
        """Post-step hook: a parameter with a gradient has just been updated once more."""
        for group in optimizer.param_groups:
            for p in group["params"]:
                if p.grad is not None and id(p) in self._host_steps:
                    self._host_steps[id(p)] += 1

    # ------------------------------------------------------------------ state tensors
    def _assemble(self, layer_name: str, key: str, idx, include_bias: bool, reduce: bool):
        sources = self._sources(layer_name, include_bias)
        values = {role: src.read(self._optimizer, key) for role, src in sources.items()}
        sharded = self._layers[layer_name].sharded
        if sharded:
            # every rank must take part in the sum, also one that holds none of this layer
            like = next((v for v in values.values() if v is not None), None)
            if like is None:
                like = next((st[key] for st in self._optimizer.state.values() if key in st), None)
            if like is None:
                return None
            if like.ndim == 0:
                return next((v for v in values.values() if v is not None), like)
            full = {role: src.on_zeros(values[role], like) for role, src in sources.items()}
            out = self.flatten(layer_name, full, idx)
            if reduce:
                _all_reduce_sum(out)
            return out
        present = [v for v in values.values() if v is not None]
        if not present:
            return None
        if present[0].ndim == 0:
            return present[0]
        ref = present[0]
        full = {role: values[role] if values[role] is not None
                else torch.zeros(src.shape, dtype=ref.dtype, device=ref.device) for role, src in sources.items()}
        return self.flatten(layer_name, full, idx)

    def state(self, layer_name: str, key: str, idx: torch.Tensor | None = None,
              include_bias: bool = True) -> torch.Tensor | None:
        """State *key* of the layer in its gradient layout (at *idx*); a scalar state (e.g.
        ``step``) as stored; ``None`` before the optimizer created it."""
        return self._assemble(layer_name, key, idx, include_bias, reduce=True)

    def states(self, layer_name: str, idx: torch.Tensor | None = None,
               include_bias: bool = True) -> dict[str, torch.Tensor | None]:
        """Every state the optimizer's update rule reads, ``{key: tensor}``; under FSDP1 the
        vector states travel in one packed all-reduce."""
        keys = ops.OPTIMIZER_STATE_KEYS[self.optimizer_type]
        self.bind(layer_name)
        if not self._layers[layer_name].sharded:
            return {key: self._assemble(layer_name, key, idx, include_bias, reduce=True) for key in keys}
        found = {key: self._assemble(layer_name, key, idx, include_bias, reduce=False) for key in keys}
        vectors = [key for key, val in found.items() if val is not None and val.ndim > 0]
        if vectors:
            packed = torch.cat([found[key].reshape(-1) for key in vectors])
            _all_reduce_sum(packed)
            offset = 0
            for key in vectors:
                n = found[key].numel()
                found[key] = packed[offset:offset + n].view(found[key].shape)
                offset += n
        return found

    def precondition(self, layer_name: str, entries: torch.Tensor, idx: torch.Tensor | None = None,
                     include_bias: bool = True) -> torch.Tensor:
        """The update direction the optimizer would take for each row of *entries*
        ``(B, width)`` (per-sample gradients in the layer's layout, or at *idx*)."""
        current = self.states(layer_name, idx, include_bias)
        moved = {key: None if val is None else val.to(entries.device) for key, val in current.items()}
        return ops.precondition(entries, moved, optimizer_type=self.optimizer_type,
                                step=self.step_count(layer_name) + 1, **self.hyperparameters(layer_name))


class GradientPreconditioner:
    """``(layer_name, entries, proj_kw) -> directions``: the optimizer geometry the capture
    hooks apply to per-sample gradient rows.  The snapshot may be given lazily (a callable)."""

    def __init__(self, snapshot: OptimizerSnapshot | Callable[[], OptimizerSnapshot],
                 projector: ops.DattriProjector | None = None) -> None:
        self._make = snapshot if not isinstance(snapshot, OptimizerSnapshot) else None
        self._snapshot = snapshot if isinstance(snapshot, OptimizerSnapshot) else None
        self.projector = projector
        self.enabled = True

    @property
    def snapshot(self) -> OptimizerSnapshot:
        """The optimizer snapshot (created on first use when given lazily)."""
        if self._snapshot is None:
            self._snapshot = self._make()
        return self._snapshot

    def __call__(self, layer_name: str, entries: torch.Tensor, proj_kw: dict | None = None) -> torch.Tensor:
        with_bias = True if proj_kw is None else bool(proj_kw.get("include_bias", True))
        coords = None
        if proj_kw is not None and proj_kw.get("style", "logra") == "mask":
            width = self.snapshot.width(layer_name, with_bias)
            coords = ops.mask_coordinates({layer_name: proj_kw}, layer_name, width, self.projector,
                                          device=entries.device)
        return self.snapshot.precondition(layer_name, entries, coords, with_bias)
