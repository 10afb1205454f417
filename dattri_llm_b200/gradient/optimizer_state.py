"""Read an optimizer's per-parameter state in a hooked layer's materialized layout.

A layer's per-sample gradient is laid out ``(out, in[+bias])`` row-major (bias as
the last column of each row for linear/conv, appended after the weight for
norms/embeddings).  :class:`OptimizerSnapshot` reads the optimizer moments of the
layer's parameters in that same layout (optionally only at ``mask`` coordinates),
under a single device, DDP, FSDP1 (``use_orig_params=True``: this rank's slice of
the flat parameter laid on zeros, then one packed SUM all-reduce) or FSDP2
(``DTensor.full_tensor()``).  :class:`GradientPreconditioner` maps a layer's
per-sample gradient block through the optimizer's update rule
(:func:`ops.precondition`).  Parity: reference
``dattri_llm/gradient/optimizer_state.py:62-590``.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable
from typing import NamedTuple

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.gradient import base_layer_name
from dattri_llm_b200.gradient.ops.types import canonical_class_name, is_conv, is_embedding, is_linear, is_norm
from dattri_llm_b200.utils.distributed import dist_world_size, is_dist_initialized

HF_CONV1D = "transformers.pytorch_utils.Conv1D"
_UNSUPPORTED = ("the optimizer holds flat parameters this reader cannot lay out: "
                "FullyShardedDataParallel needs use_orig_params=True.")


class _Slice(NamedTuple):
    """This rank's share of an FSDP1 original parameter: the local view, the full
    shape, and the element range ``[start, end]`` (``None``: nothing local)."""

    param: nn.Parameter
    shape: tuple[int, ...]
    start: int | None
    end: int | None


def optimizer_type(optimizer: torch.optim.Optimizer) -> str:
    """The ``torch.optim`` class name whose update rule applies (searched along the MRO).

    Raises:
        NotImplementedError: for optimizers without a coordinate-wise rule.
    """
    for cls in type(optimizer).__mro__:
        if cls.__name__ in ops.OPTIMIZER_STATE_KEYS:
            return cls.__name__
    raise NotImplementedError(
        f"{type(optimizer).__name__} is not a supported optimizer: its update is not "
        f"coordinate-wise, or its state is not a per-parameter tensor. Supported: "
        f"{sorted(ops.OPTIMIZER_STATE_KEYS)}.",
    )


def hf_trainer_param_names(model: nn.Module) -> list[str]:
    """Trainable parameter names in the order the HF Trainer builds its optimizer groups
    (weight-decayed first, then the rest)."""
    from transformers.trainer_pt_utils import get_parameter_names

    norms = tuple(t for t in (nn.LayerNorm, getattr(nn, "RMSNorm", None)) if t is not None)
    decay = {n for n in get_parameter_names(model, norms) if "bias" not in n}
    trainable = [n for n, p in model.named_parameters() if p.requires_grad]
    return [n for n in trainable if n in decay] + [n for n in trainable if n not in decay]


def optimizer_from_state_dict(model: nn.Module, state_dict: dict, param_names: Iterable[str] | None = None,
                              *, optimizer_cls: type = torch.optim.AdamW) -> torch.optim.Optimizer:
    """Rebuild an optimizer over *model* from a saved state dict (indices mapped through
    *param_names*, default the HF Trainer order)."""
    params = dict(model.named_parameters())
    names = list(hf_trainer_param_names(model) if param_names is None else param_names)
    groups = []
    for saved in state_dict["param_groups"]:
        g = {k: v for k, v in saved.items() if k != "params"}
        g["params"] = [params[names[i]] for i in saved["params"]]
        groups.append(g)
    opt = optimizer_cls(groups)
    opt.load_state_dict(state_dict)
    return opt


def _is_dtensor(t: object) -> bool:
    try:
        from torch.distributed.tensor import DTensor
    except ImportError:  # pragma: no cover
        return False
    return isinstance(t, DTensor)


def _sum_over_ranks(t: torch.Tensor) -> None:
    if is_dist_initialized() and dist_world_size() > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.SUM)


class OptimizerSnapshot:
    """Optimizer state of each hooked layer, in the layer's materialized layout."""

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer) -> None:
        self._model = getattr(model, "module", model)
        self._optimizer = optimizer
        self.optimizer_type = optimizer_type(optimizer)
        self._groups: dict[int, dict] = {}
        for group in optimizer.param_groups:
            for p in group["params"]:
                self._groups[id(p)] = group
                if getattr(p, "_is_flat_param", False):
                    raise NotImplementedError(_UNSUPPORTED)
        self._slices: dict[tuple[str, str], _Slice] = {}
        self._dtensors: dict[tuple[str, str], nn.Parameter] = {}

    @property
    def optimizer(self) -> torch.optim.Optimizer:
        """The wrapped optimizer."""
        return self._optimizer

    def module(self, layer_name: str) -> nn.Module:
        """The module of *layer_name* (virtual ``@k`` suffixes stripped)."""
        return self._model.get_submodule(base_layer_name(layer_name))

    def parameters(self, layer_name: str, include_bias: bool = True) -> list[tuple[str, nn.Parameter]]:
        """``[("weight", p), ("bias", p)]`` as the optimizer holds them.

        Raises:
            ValueError / NotImplementedError: for layers without weight or of an unsupported type.
        """
        module = self.module(layer_name)
        lt = canonical_class_name(module)
        weight = getattr(module, "weight", None)
        if weight is None:
            raise ValueError(f"layer {layer_name!r} ({lt}) has no weight parameter.")
        if not (is_linear(lt) or is_conv(lt) or is_norm(lt) or is_embedding(lt)):
            raise NotImplementedError(
                f"optimizer-state layout is not defined for layer type {lt} (layer {layer_name!r}); "
                "supported: linear, conv, norm, embedding.",
            )
        roles = [("weight", weight)]
        bias = getattr(module, "bias", None) if include_bias else None
        if bias is not None:
            roles.append(("bias", bias))
        self.bind(layer_name)
        out = []
        for role, p in roles:
            if (layer_name, role) in self._slices:
                p = self._slices[layer_name, role].param
            else:
                p = self._dtensors.get((layer_name, role), p)
            out.append((role, p))
        return out

    def bind(self, layer_name: str) -> None:
        """Resolve how the layer's parameters are sharded (call inside the layer's backward
        under FSDP1, where the original parameters are views of the flat parameter).

        Raises:
            RuntimeError / NotImplementedError: for unbound or unsupported FSDP layouts.
        """
        module = self.module(layer_name)
        for role in ("weight", "bias"):
            t = getattr(module, role, None)
            if t is None or (layer_name, role) in self._slices or (layer_name, role) in self._dtensors:
                continue
            if _is_dtensor(t):
                self._dtensors[layer_name, role] = t
                continue
            sharded = self._fsdp2_param(module, role)
            if sharded is not None:
                self._dtensors[layer_name, role] = sharded
                continue
            flat = getattr(t, "_base", None)
            infos = getattr(flat, "_shard_param_infos", None)
            if infos is None:
                if getattr(t, "_fsdp_flattened", False):
                    raise RuntimeError(
                        f"layer {layer_name!r} is sharded by FSDP and its optimizer state was read "
                        "before the layer was bound: call OptimizerSnapshot.bind(layer_name) from "
                        "inside the layer's backward first.",
                    )
                continue
            if flat._params is None:
                raise NotImplementedError(_UNSUPPORTED)
            for param, info, shape, where in zip(flat._params, infos, flat._shapes, flat._param_infos,
                                                 strict=True):
                if where.module is module and where.param_name == role:
                    self._slices[layer_name, role] = _Slice(
                        param, tuple(shape), info.intra_param_start_idx if info.in_shard else None,
                        info.intra_param_end_idx if info.in_shard else None)

    def _fsdp2_param(self, module: nn.Module, role: str) -> nn.Parameter | None:
        for unit in self._model.modules():
            get_state = getattr(unit, "_get_fsdp_state", None)
            group = getattr(get_state(), "_fsdp_param_group", None) if get_state else None
            for fp in getattr(group, "fsdp_params", ()):
                info = fp._module_info
                if info.module is module and info.param_name == role:
                    return fp.sharded_param
        return None

    def _laid_on_zeros(self, layer_name: str, role: str, local: torch.Tensor | None):
        sl = self._slices.get((layer_name, role))
        if sl is None:
            return local
        dtype = torch.float32 if local is None else local.dtype
        device = "cpu" if local is None else local.device
        full = torch.zeros(math.prod(sl.shape), dtype=dtype, device=device)
        if sl.start is not None and local is not None and local.numel():
            full[sl.start : sl.end + 1] = local.reshape(-1)
        return full.reshape(sl.shape)

    def _sharded(self, layer_name: str) -> bool:
        return (layer_name, "weight") in self._slices

    def width(self, layer_name: str, include_bias: bool = True) -> int:
        """Number of entries of the layer's flattened gradient."""
        return sum(math.prod(self._slices[layer_name, r].shape) if (layer_name, r) in self._slices
                   else p.numel() for r, p in self.parameters(layer_name, include_bias))

    def _row_layout(self, layer_name: str) -> bool:
        lt = canonical_class_name(self.module(layer_name))
        return is_linear(lt) or is_conv(lt)

    def flatten(self, layer_name: str, tensors: dict[str, torch.Tensor],
                idx: torch.Tensor | None = None) -> torch.Tensor:
        """Flatten ``{"weight", "bias"}`` tensors into the materialized layout (entries at *idx*)."""
        w = tensors["weight"]
        if canonical_class_name(self.module(layer_name)) == HF_CONV1D:
            w = w.transpose(0, 1)
        b = tensors.get("bias")
        rows = w.shape[0] if self._row_layout(layer_name) else 1
        w_rows = w.reshape(rows, -1)
        if idx is None:
            if b is None:
                return w.reshape(-1)
            if rows > 1:
                return torch.cat([w_rows, b.reshape(-1, 1)], dim=1).reshape(-1)
            return torch.cat([w.reshape(-1), b.reshape(-1)])
        idx = idx.to(w.device)
        d_in = w_rows.shape[1]
        if b is None:
            return w.reshape(-1)[idx]
        if rows > 1:
            o, i = idx // (d_in + 1), idx % (d_in + 1)
            return torch.where(i == d_in, b.reshape(-1)[o], w_rows[o, i.clamp(max=d_in - 1)])
        return torch.where(idx >= d_in, b.reshape(-1)[(idx - d_in).clamp(min=0)],
                           w.reshape(-1)[idx.clamp(max=d_in - 1)])

    def group(self, layer_name: str) -> dict:
        """The optimizer param group of the layer's weight.

        Raises:
            ValueError: when the weight is not in the optimizer.
        """
        _, weight = self.parameters(layer_name)[0]
        try:
            return self._groups[id(weight)]
        except KeyError:
            raise ValueError(f"layer {layer_name!r}'s weight is not in the optimizer.") from None

    def hyperparameters(self, layer_name: str) -> dict:
        """The optimizer defaults overridden by the layer's group."""
        out = dict(self._optimizer.defaults)
        out.update({k: v for k, v in self.group(layer_name).items() if k != "params"})
        return out

    def step_count(self, layer_name: str) -> int:
        """Updates the layer's weight has received (0 before the first)."""
        _, weight = self.parameters(layer_name)[0]
        step = self._optimizer.state.get(weight, {}).get("step")
        if step is None and self._sharded(layer_name):
            step = max((st["step"] for st in self._optimizer.state.values() if "step" in st), default=0)
        step = 0 if step is None else step
        return int(step.item() if isinstance(step, torch.Tensor) else step)

    def state(self, layer_name: str, key: str, idx: torch.Tensor | None = None,
              include_bias: bool = True) -> torch.Tensor | None:
        """One state tensor (``exp_avg`` ...) in the layer's layout; scalars returned as is."""
        params = self.parameters(layer_name, include_bias)
        values = {r: self._optimizer.state.get(p, {}).get(key) for r, p in params}
        if self._sharded(layer_name):
            return self._sharded_state(layer_name, key, values, idx)
        values = {r: v.full_tensor() if _is_dtensor(v) else v for r, v in values.items()}
        if all(v is None for v in values.values()):
            return None
        first = next(v for v in values.values() if v is not None)
        if first.ndim == 0:
            return first
        tensors = {r: (torch.zeros(tuple(p.shape), dtype=first.dtype, device=first.device)
                       if values[r] is None else values[r]) for r, p in params}
        return self.flatten(layer_name, tensors, idx)

    def _sharded_state(self, layer_name, key, values, idx, reduce: bool = True):
        states = [st[key] for st in self._optimizer.state.values() if key in st]
        if not states:
            return None
        if states[0].ndim == 0:
            return next((v for v in values.values() if v is not None), states[0])
        device, dtype = states[0].device, states[0].dtype
        tensors = {r: self._laid_on_zeros(layer_name, r, v).to(device=device, dtype=dtype)
                   for r, v in values.items()}
        out = self.flatten(layer_name, tensors, idx)
        if reduce:
            _sum_over_ranks(out)
        return out

    def states(self, layer_name: str, idx: torch.Tensor | None = None,
               include_bias: bool = True) -> dict[str, torch.Tensor | None]:
        """Every state key the optimizer's rule reads (one packed all-reduce under FSDP1)."""
        keys = ops.OPTIMIZER_STATE_KEYS[self.optimizer_type]
        self.bind(layer_name)
        if not self._sharded(layer_name):
            return {k: self.state(layer_name, k, idx, include_bias) for k in keys}
        params = self.parameters(layer_name, include_bias)
        out = {}
        for k in keys:
            values = {r: self._optimizer.state.get(p, {}).get(k) for r, p in params}
            out[k] = self._sharded_state(layer_name, k, values, idx, reduce=False)
        packed = [k for k, v in out.items() if v is not None and v.ndim > 0]
        if packed:
            buf = torch.cat([out[k].reshape(-1) for k in packed])
            _sum_over_ranks(buf)
            for k, part in zip(packed, buf.split([out[k].numel() for k in packed]), strict=True):
                out[k] = part.reshape(out[k].shape)
        return out

    def precondition(self, layer_name: str, entries: torch.Tensor, idx: torch.Tensor | None = None,
                     include_bias: bool = True) -> torch.Tensor:
        """The update direction of per-sample gradient rows *entries* ``(B, width)``."""
        state = {k: None if v is None else v.to(entries.device)
                 for k, v in self.states(layer_name, idx, include_bias).items()}
        return ops.precondition(entries, state, optimizer_type=self.optimizer_type,
                                step=self.step_count(layer_name) + 1, **self.hyperparameters(layer_name))


class GradientPreconditioner:
    """Callable ``(layer_name, entries, proj_kw) -> directions`` the capture hooks apply."""

    def __init__(self, snapshot: OptimizerSnapshot | Callable[[], OptimizerSnapshot],
                 projector: ops.DattriProjector | None = None) -> None:
        self._source = snapshot
        self._snapshot = snapshot if isinstance(snapshot, OptimizerSnapshot) else None
        self.projector = projector
        self.enabled = True

    @property
    def snapshot(self) -> OptimizerSnapshot:
        """The snapshot (built on first use)."""
        if self._snapshot is None:
            self._snapshot = self._source()
        return self._snapshot

    def __call__(self, layer_name: str, entries: torch.Tensor, proj_kw: dict | None = None) -> torch.Tensor:
        include_bias = True if proj_kw is None else bool(proj_kw.get("include_bias", True))
        idx = None
        if proj_kw is not None and proj_kw.get("style", "logra") == "mask":
            idx = ops.mask_coordinates({layer_name: proj_kw}, layer_name,
                                       self.snapshot.width(layer_name, include_bias), self.projector,
                                       device=entries.device)
        return self.snapshot.precondition(layer_name, entries, idx, include_bias)
