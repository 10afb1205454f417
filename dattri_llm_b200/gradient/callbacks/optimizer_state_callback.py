"""Record an Adam-family optimizer's moments on every captured layer, around each update.

AdamW-influence needs, for every training step, the first and second moments of each
attributed layer just before and just after the optimizer's update, plus the step count
and hyperparameters.  This callback reads them:

* at the end of each capture step (:meth:`on_step_end`, before the user calls
  ``optimizer.step()``): the "pre" record of the layers captured in that step;
* when told the update happened (:meth:`record_post`): the "post" record of the same layers.

A layer under the ``mask`` projection is recorded only at its mask coordinates (the
coordinates its captured gradient lives on).  Records stay in memory, or go to a
:class:`TrajectorySnapshots` directory as ``dynamics_<s>_{pre,post}.pt`` when one is given.
:meth:`dynamics` assembles ``{step: {"pre", "post", "step", "lr", "betas", "eps",
"weight_decay"}}`` -- the layout the reference writes (its
``dattri_llm/gradient/callbacks/optimizer_state_callback.py``), so dynamics files are
interchangeable.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Mapping

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.optimizer_state import OptimizerSnapshot
from dattri_llm_b200.gradient.snapshots import LazyDynamics, TrajectorySnapshots

_ADAM_FAMILY = ("Adam", "AdamW")
_HYPERPARAMETERS = ("lr", "betas", "eps", "weight_decay")


def assemble_dynamics(pre: dict, post: dict) -> dict:
    """The dynamics entry of one step from its "pre" and "post" records."""
    entry = {"pre": pre["layers"], "post": post["layers"], "step": post["step"]}
    entry.update({key: pre[key] for key in _HYPERPARAMETERS})
    entry["betas"] = tuple(entry["betas"])
    return entry


class _MemoryRecords:
    """Records kept in dictionaries (``pre`` / ``post``: ``{step: record}``)."""

    def __init__(self) -> None:
        self.pre: dict[int, dict] = {}
        self.post: dict[int, dict] = {}

    def put(self, step: int, side: str, record: dict) -> None:
        getattr(self, side)[step] = record

    def layers_of(self, step: int) -> list[str] | None:
        rec = self.pre.get(step)
        return None if rec is None else list(rec["layers"])

    def assembled(self) -> Mapping[int, dict]:
        return {step: assemble_dynamics(rec, self.post[step]) for step, rec in self.pre.items() if step in self.post}


class _DiskRecords:
    """Records written into a snapshot directory; the layer list of each pending step is
    remembered so that its "post" record covers the same layers."""

    def __init__(self, store: TrajectorySnapshots) -> None:
        self.store = store
        self.pending: dict[int, list[str]] = {}
        self.pre: dict[int, dict] = {}   # empty: records live on disk
        self.post: dict[int, dict] = {}

    def put(self, step: int, side: str, record: dict) -> None:
        self.store.save_dynamics(step, side, record)
        if side == "pre":
            self.pending[step] = list(record["layers"])

    def layers_of(self, step: int) -> list[str] | None:
        return self.pending.get(step)

    def assembled(self) -> Mapping[int, dict]:
        return LazyDynamics(self.store, assemble_dynamics)


class OptimizerStateCallback(HookManagerCallback):
    """Adam moments of the captured layers before and after every optimizer update.

    Args:
        model: the model whose optimizer is read (hooked names resolve in it).
        optimizer: the optimizer, or a zero-argument callable returning it (resolved on
            first use, for optimizers created after the callback).
        projection_kwargs: the capture's projection settings (mask coordinates).
        layers: record only these layers (default: every captured layer).
        snapshots: write the records into this snapshot directory instead of memory.
    """

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer | Callable[[], torch.optim.Optimizer],
                 *, projection_kwargs: dict[str, dict] | None = None, layers: Iterable[str] | None = None,
                 snapshots: TrajectorySnapshots | None = None) -> None:
        self._model = model
        self._optimizer = optimizer
        self._reader: OptimizerSnapshot | None = None
        self._projection = projection_kwargs
        self._only = None if layers is None else frozenset(layers)
        self._projector = ops.DattriProjector()
        self._coords: dict[str, torch.Tensor | None] = {}
        self._records = _DiskRecords(snapshots) if snapshots is not None else _MemoryRecords()

    @property
    def pre(self) -> dict[int, dict]:
        """In-memory "pre" records, ``{step: record}`` (empty when writing to disk)."""
        return self._records.pre

    @property
    def post(self) -> dict[int, dict]:
        """In-memory "post" records, ``{step: record}`` (empty when writing to disk)."""
        return self._records.post

    @property
    def snapshot(self) -> OptimizerSnapshot:
        """The optimizer-state reader, made on first use.

        Raises:
            NotImplementedError: the optimizer is not Adam or AdamW.
        """
        if self._reader is None:
            opt = self._optimizer() if callable(self._optimizer) else self._optimizer
            reader = OptimizerSnapshot(self._model, opt)
            if reader.optimizer_type not in _ADAM_FAMILY:
                raise NotImplementedError(f"only Adam-family moments can be recorded; the optimizer is a "
                                          f"{reader.optimizer_type}.")
            self._reader = reader
        return self._reader

    def coordinates(self, layer_name: str) -> torch.Tensor | None:
        """The flat coordinates recorded for *layer_name* (``None``: all of them)."""
        if layer_name not in self._coords:
            width = self.snapshot.width(layer_name)
            self._coords[layer_name] = ops.mask_coordinates(self._projection, layer_name, width, self._projector)
        return self._coords[layer_name]

    def _wanted(self, layer_name: str) -> bool:
        return self._only is None or layer_name in self._only

    def _moments(self, names: list[str]) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """fp32 host copies of (exp_avg, exp_avg_sq) at each layer's coordinates; zeros for a
        parameter the optimizer has not stepped yet.  The layers' device values travel to the
        host in one copy per device (one synchronization per record, not one per tensor)."""
        reader = self.snapshot
        slots: list[tuple[str, int, torch.Tensor | int]] = []  # (layer, moment, device value or size)
        for name in names:
            idx = self.coordinates(name)
            size = reader.width(name) if idx is None else idx.numel()
            for m, key in enumerate(("exp_avg", "exp_avg_sq")):
                val = reader.state(name, key, idx)
                slots.append((name, m, size if val is None else val.detach().reshape(-1)))
        by_device: dict[torch.device, list[torch.Tensor]] = {}
        for _name, _m, v in slots:
            if isinstance(v, torch.Tensor):
                by_device.setdefault(v.device, []).append(v)
        host: dict[int, torch.Tensor] = {}
        for vals in by_device.values():
            flat = torch.cat([v.float() for v in vals]).to("cpu")
            for v, part in zip(vals, flat.split([v.numel() for v in vals]), strict=True):
                host[id(v)] = part.clone()  # each record owns its storage
        out: dict[str, list[torch.Tensor]] = {name: [None, None] for name in names}
        for name, m, v in slots:
            out[name][m] = host[id(v)] if isinstance(v, torch.Tensor) else torch.zeros(v)
        return {name: (pair[0], pair[1]) for name, pair in out.items()}

    def _record(self, layer_names: Iterable[str]) -> dict:
        names = [n for n in layer_names if self._wanted(n)]
        record: dict = {"layers": self._moments(names)}
        if names:
            hyper = self.snapshot.hyperparameters(names[0])
            record["step"] = self.snapshot.step_count(names[0])
            record.update({key: hyper[key] for key in _HYPERPARAMETERS})
        return record

    def on_layer_backward(self, layer_name, grad_output, layer_type, module_kwargs=None) -> None:
        """Under FSDP1 a layer's flat-parameter slice can only be located while its unsharded
        views exist, i.e. during its backward: bind it then."""
        if self._wanted(layer_name):
            self.snapshot.bind(layer_name)

    def on_step_end(self, record) -> None:
        """The "pre" record of the step's layers (the update has not run yet)."""
        self._records.put(record.step, "pre", self._record(record.gradient.data.keys()))

    def record_post(self, step: int) -> None:
        """The "post" record of *step*; call right after ``optimizer.step()``.

        Raises:
            KeyError: *step* has no "pre" record.
        """
        layers = self._records.layers_of(step)
        if layers is None:
            raise KeyError(f"record_post({step}): this callback saw no capture step {step} before the update.")
        self._records.put(step, "post", self._record(layers))

    def dynamics(self) -> Mapping[int, dict]:
        """``{step: dynamics entry}`` for every step with both records (read lazily from disk
        when writing to a snapshot directory)."""
        return self._records.assembled()
