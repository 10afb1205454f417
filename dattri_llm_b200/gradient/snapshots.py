"""Per-step parameters, batches and optimizer moments of a training trajectory.

Trajectory methods (DVEmb, AdamW-influence, LESS replays) revisit every training step.
Instead of storing per-step gradients they can store what regenerates them: the trainable
parameters before the step, the step's batch and, for Adam-family optimizers, the moments
before and after the update.  One directory holds one trajectory:

    snapshots.json              marker file ({"format": 1}); identifies the directory
    theta_<s>.pt                {parameter name: tensor} of the trainable parameters
    theta_<s>.ref               the text "<t>": step s had the same parameters as step t
    batch_<s>.pt                the batch of step s (tensors on the host)
    dynamics_<s>_pre.pt         optimizer moments before step s's update
    dynamics_<s>_post.pt        ... and after it

The names and contents are the reference's (``dattri_llm/gradient/snapshots.py``), so a
trajectory recorded by either framework replays in the other.  Files are written to a
temporary name and renamed into place, so a reader never sees a half-written snapshot.
"""

from __future__ import annotations

import json
import os
import pathlib
import re
from collections.abc import Callable, Iterator, Mapping

import torch
from torch import nn

MANIFEST_FILE = "snapshots.json"
_ENTRY = re.compile(r"^(theta|batch|dynamics)_(\d+)(?:_(pre|post))?\.(pt|ref)$")


def _host_copy(obj: object) -> object:
    """*obj* with every tensor detached and moved to the host (containers rebuilt)."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu()
    if isinstance(obj, dict):
        return {key: _host_copy(val) for key, val in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(map(_host_copy, obj))
    return obj


def _write_atomic(path: pathlib.Path, write: Callable[[pathlib.Path], None]) -> None:
    tmp = path.with_name(f".{path.name}.tmp{os.getpid()}")
    write(tmp)
    os.replace(tmp, path)


class TrajectorySnapshots:
    """A snapshot directory (created, with its marker file, when missing)."""

    def __init__(self, root: str | pathlib.Path) -> None:
        self.root = pathlib.Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        marker = self.root / MANIFEST_FILE
        if not marker.exists():
            _write_atomic(marker, lambda p: p.write_text(json.dumps({"format": 1})))

    @staticmethod
    def is_snapshot_dir(path: object) -> bool:
        """Whether *path* names a snapshot directory (it holds the marker file)."""
        if not isinstance(path, (str, pathlib.Path)):
            return False
        return (pathlib.Path(path) / MANIFEST_FILE).is_file()

    def __repr__(self) -> str:
        return f"TrajectorySnapshots({str(self.root)!r}, steps={len(self.steps())})"

    # ------------------------------------------------------------------ directory scan
    def _index(self) -> dict[str, set[int]]:
        """Steps present per kind: ``theta`` (file or reference), ``batch``, ``pre``, ``post``."""
        found: dict[str, set[int]] = {"theta": set(), "batch": set(), "pre": set(), "post": set()}
        for entry in os.scandir(self.root):
            m = _ENTRY.match(entry.name)
            if m is None:
                continue
            kind, step, side, ext = m.group(1), int(m.group(2)), m.group(3), m.group(4)
            if kind == "dynamics" and side is not None and ext == "pt":
                found[side].add(step)
            elif kind == "theta" or (kind == "batch" and ext == "pt"):
                found[kind].add(step)
        return found

    def steps(self) -> list[int]:
        """Steps that can be replayed: parameters (or a reference to them) and a batch."""
        idx = self._index()
        return sorted(idx["theta"] & idx["batch"])

    def dynamics_steps(self) -> list[int]:
        """Steps with optimizer moments from both sides of the update."""
        idx = self._index()
        return sorted(idx["pre"] & idx["post"])

    # ------------------------------------------------------------------ parameters
    def save_parameters(self, step: int, model: nn.Module, *, same_as: int | None = None) -> None:
        """Record the trainable parameters before *step*; with *same_as*, only note that they
        equal the ones recorded for that step (no tensor file)."""
        if same_as is not None:
            _write_atomic(self.root / f"theta_{step}.ref", lambda p: p.write_text(str(int(same_as))))
            return
        state = {name: t.detach().cpu() for name, t in model.named_parameters() if t.requires_grad}
        _write_atomic(self.root / f"theta_{step}.pt", lambda p: torch.save(state, p))

    def _resolve_parameters(self, step: int) -> pathlib.Path:
        """Follow ``.ref`` links from *step* to the tensor file they end at."""
        seen: list[int] = []
        while True:
            link = self.root / f"theta_{step}.ref"
            if not link.exists():
                break
            if step in seen:
                raise KeyError(f"parameter references loop through steps {seen + [step]} in {self.root}")
            seen.append(step)
            step = int(link.read_text().strip())
        target = self.root / f"theta_{step}.pt"
        if not target.exists():
            via = f" (reached through {seen})" if seen else ""
            raise KeyError(f"step {step} has no recorded parameters in {self.root}{via}")
        return target

    def load_parameters(self, step: int, model: nn.Module) -> None:
        """Write the parameters recorded for *step* into *model*'s trainable parameters.

        Raises:
            KeyError: the step, or one of the model's trainable parameters, was not recorded.
        """
        state = torch.load(self._resolve_parameters(step), weights_only=True)
        trainable = [(name, t) for name, t in model.named_parameters() if t.requires_grad]
        absent = [name for name, _ in trainable if name not in state]
        if absent:
            raise KeyError(f"the snapshot of step {step} lacks trainable parameter(s) {absent[:4]}")
        with torch.no_grad():
            for name, t in trainable:
                t.copy_(state[name].to(device=t.device, dtype=t.dtype))

    # ------------------------------------------------------------------ batches
    def save_batch(self, step: int, batch: object) -> None:
        """Record the batch of *step* (tensors copied to the host)."""
        host = _host_copy(batch)
        _write_atomic(self.root / f"batch_{step}.pt", lambda p: torch.save(host, p))

    def load_batch(self, step: int) -> object:
        """The batch recorded for *step*.

        Raises:
            KeyError: none was recorded.
        """
        path = self.root / f"batch_{step}.pt"
        if not path.is_file():
            raise KeyError(f"step {step} has no recorded batch in {self.root}")
        return torch.load(path, weights_only=False)

    # ------------------------------------------------------------------ optimizer moments
    def save_dynamics(self, step: int, side: str, entry: dict) -> None:
        """Record optimizer moments of *step*: *side* ``"pre"`` (before its update) or
        ``"post"`` (after it)."""
        if side not in ("pre", "post"):
            raise ValueError(f"dynamics side is 'pre' or 'post', not {side!r}.")
        host = _host_copy(entry)
        _write_atomic(self.root / f"dynamics_{step}_{side}.pt", lambda p: torch.save(host, p))

    def load_dynamics(self, step: int, side: str) -> dict | None:
        """The moments recorded for *step* and *side*, or ``None`` when absent."""
        path = self.root / f"dynamics_{step}_{side}.pt"
        if not path.is_file():
            return None
        return torch.load(path, weights_only=False)


class LazyDynamics(Mapping):
    """Read-only ``{step: assemble(pre, post)}`` over a snapshot directory's moments,
    loaded from disk when a step is looked up (the step list is fixed at construction)."""

    def __init__(self, snapshots: TrajectorySnapshots, assemble: Callable[[dict, dict], dict]) -> None:
        self._source = snapshots
        self._assemble = assemble
        self._available = tuple(snapshots.dynamics_steps())

    def __getitem__(self, step: int) -> dict:
        if step not in self._available:
            raise KeyError(step)
        pre, post = self._source.load_dynamics(step, "pre"), self._source.load_dynamics(step, "post")
        if pre is None or post is None:
            raise KeyError(step)
        return self._assemble(pre, post)

    def __iter__(self) -> Iterator[int]:
        return iter(self._available)

    def __len__(self) -> int:
        return len(self._available)

    def __contains__(self, step: object) -> bool:
        return step in self._available
