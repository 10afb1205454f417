"""Snapshot an Adam-family optimizer's moments on each captured layer's coordinates.

``on_step_end`` records ``(exp_avg, exp_avg_sq)`` of every layer of the step (at its
``mask`` coordinates when the layer is mask-projected) *before* the update;
``record_post(step)``, called after ``optimizer.step()``, records them after.
``dynamics()`` assembles ``{step: {"pre", "post", "step", "lr", "betas", "eps",
"weight_decay"}}`` for AdamW-influence.  With ``snapshots`` the entries go to disk.
Parity: reference ``dattri_llm/gradient/callbacks/optimizer_state_callback.py``.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Mapping

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.optimizer_state import OptimizerSnapshot
from dattri_llm_b200.gradient.snapshots import LazyDynamics, TrajectorySnapshots


def _host_f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", torch.float32, copy=True)


def assemble_dynamics(pre: dict, post: dict) -> dict:
    """One step's dynamics entry from its pre- and post-update records."""
    return {"pre": pre["layers"], "post": post["layers"], "step": post["step"], "lr": pre["lr"],
            "betas": tuple(pre["betas"]), "eps": pre["eps"], "weight_decay": pre["weight_decay"]}


class OptimizerStateCallback(HookManagerCallback):
    """Adam moments before/after every update, per captured layer."""

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer | Callable[[], torch.optim.Optimizer],
                 *, projection_kwargs: dict[str, dict] | None = None, layers: Iterable[str] | None = None,
                 snapshots: TrajectorySnapshots | None = None) -> None:
        self._model = model
        self._opt_src = optimizer
        self._snapshot: OptimizerSnapshot | None = None
        self._projection = projection_kwargs
        self._layers = None if layers is None else set(layers)
        self._projector = ops.DattriProjector()
        self._coords: dict[str, torch.Tensor | None] = {}
        self._store = snapshots
        self._layers_at: dict[int, list[str]] = {}
        self.pre: dict[int, dict] = {}
        self.post: dict[int, dict] = {}

    @property
    def snapshot(self) -> OptimizerSnapshot:
        """The optimizer snapshot (built on first use).

        Raises:
            NotImplementedError: for a non-Adam optimizer.
        """
        if self._snapshot is None:
            src = self._opt_src
            snap = OptimizerSnapshot(self._model, src() if callable(src) else src)
            if snap.optimizer_type not in ("Adam", "AdamW"):
                raise NotImplementedError("OptimizerStateCallback records Adam-family moments; got a "
                                          f"{snap.optimizer_type} optimizer.")
            self._snapshot = snap
        return self._snapshot

    def coordinates(self, layer_name: str) -> torch.Tensor | None:
        """The layer's recorded coordinates (``None``: every entry)."""
        if layer_name not in self._coords:
            self._coords[layer_name] = ops.mask_coordinates(
                self._projection, layer_name, self.snapshot.width(layer_name), self._projector)
        return self._coords[layer_name]

    def _read(self, layers: Iterable[str]) -> dict:
        snap = self.snapshot
        out: dict = {"layers": {}}
        for name in layers:
            if self._layers is not None and name not in self._layers:
                continue
            idx = self.coordinates(name)
            m, v = snap.state(name, "exp_avg", idx), snap.state(name, "exp_avg_sq", idx)
            zeros = torch.zeros(snap.width(name) if idx is None else idx.numel())
            out["layers"][name] = (zeros if m is None else _host_f32(m),
                                   zeros.clone() if v is None else _host_f32(v))
            if "step" not in out:
                out["step"] = snap.step_count(name)
                hp = snap.hyperparameters(name)
                out.update({k: hp[k] for k in ("lr", "betas", "eps", "weight_decay")})
        return out

    def on_layer_backward(self, layer_name, grad_output, layer_type, module_kwargs=None) -> None:
        """Bind FSDP1 parameter slices while the layer's views are live."""
        if self._layers is None or layer_name in self._layers:
            self.snapshot.bind(layer_name)

    def on_step_end(self, record) -> None:
        """Record the pre-update moments of the step's layers."""
        entry = self._read(record.gradient.data.keys())
        if self._store is not None:
            self._store.save_dynamics(record.step, "pre", entry)
            self._layers_at[record.step] = list(entry["layers"])
        else:
            self.pre[record.step] = entry

    def record_post(self, step: int) -> None:
        """Record the post-update moments of *step* (call after ``optimizer.step()``).

        Raises:
            KeyError: when *step* has no pre-update record.
        """
        if self._store is not None:
            layers = self._layers_at.get(step)
            if layers is None:
                raise KeyError(f"no pre-step snapshot recorded for step {step}.")
            self._store.save_dynamics(step, "post", self._read(layers))
            return
        if step not in self.pre:
            raise KeyError(f"no pre-step snapshot recorded for step {step}.")
        self.post[step] = self._read(self.pre[step]["layers"].keys())

    def dynamics(self) -> Mapping[int, dict]:
        """``{step: dynamics}`` of every step with both records."""
        if self._store is not None:
            return LazyDynamics(self._store, assemble_dynamics)
        return {s: assemble_dynamics(pre, self.post[s]) for s, pre in self.pre.items() if s in self.post}
