"""Per-step parameters, batches and optimizer moments of a training trajectory.

File layout (shared with the reference, ``dattri_llm/gradient/snapshots.py``):
``theta_<s>.pt`` (trainable parameters; ``theta_<s>.ref`` holds the step whose
file to reuse), ``batch_<s>.pt``, ``dynamics_<s>_{pre,post}.pt`` and the manifest
``snapshots.json``.  A trajectory method replays any step from these files
instead of storing its gradients.
"""

from __future__ import annotations

import json
import pathlib
from collections.abc import Iterator, Mapping

import torch
from torch import nn

MANIFEST_FILE = "snapshots.json"


def _to_cpu(obj: object) -> object:
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu")
    if isinstance(obj, dict):
        return {k: _to_cpu(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_cpu(v) for v in obj)
    return obj


def _steps_of(root: pathlib.Path, pattern: str) -> set[int]:
    return {int(p.stem.split("_")[1]) for p in root.glob(pattern)}


class TrajectorySnapshots:
    """A directory of per-step snapshots."""

    def __init__(self, root: str | pathlib.Path) -> None:
        self.root = pathlib.Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        manifest = self.root / MANIFEST_FILE
        if not manifest.exists():
            manifest.write_text(json.dumps({"format": 1}))

    @staticmethod
    def is_snapshot_dir(path: object) -> bool:
        """Whether *path* is a snapshot directory (has the manifest)."""
        return isinstance(path, (str, pathlib.Path)) and (pathlib.Path(path) / MANIFEST_FILE).is_file()

    def __repr__(self) -> str:
        return f"TrajectorySnapshots({str(self.root)!r}, steps={len(self.steps())})"

    def save_parameters(self, step: int, model: nn.Module, *, same_as: int | None = None) -> None:
        """Save the trainable parameters at *step* (or a reference to step *same_as*)."""
        if same_as is not None:
            (self.root / f"theta_{step}.ref").write_text(str(int(same_as)))
            return
        torch.save({n: p.detach().to("cpu") for n, p in model.named_parameters() if p.requires_grad},
                   self.root / f"theta_{step}.pt")

    def _parameter_file(self, step: int) -> pathlib.Path:
        ref = self.root / f"theta_{step}.ref"
        if ref.exists():
            return self._parameter_file(int(ref.read_text()))
        path = self.root / f"theta_{step}.pt"
        if not path.exists():
            raise KeyError(f"no parameter snapshot for step {step} in {self.root}.")
        return path

    def load_parameters(self, step: int, model: nn.Module) -> None:
        """Copy step *step*'s parameters into *model*.

        Raises:
            KeyError: for a missing snapshot or parameter.
        """
        state = torch.load(self._parameter_file(step), weights_only=True)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if not p.requires_grad:
                    continue
                if name not in state:
                    raise KeyError(f"parameter {name!r} has no snapshot at step {step}.")
                p.copy_(state[name].to(p.device, p.dtype))

    def save_batch(self, step: int, batch: object) -> None:
        """Save the batch of *step* (moved to host)."""
        torch.save(_to_cpu(batch), self.root / f"batch_{step}.pt")

    def load_batch(self, step: int) -> object:
        """The batch of *step*."""
        path = self.root / f"batch_{step}.pt"
        if not path.exists():
            raise KeyError(f"no batch snapshot for step {step} in {self.root}.")
        return torch.load(path, weights_only=False)

    def save_dynamics(self, step: int, side: str, entry: dict) -> None:
        """Save optimizer moments before (``"pre"``) or after (``"post"``) *step*'s update."""
        if side not in ("pre", "post"):
            raise ValueError(f"side must be 'pre' or 'post', got {side!r}.")
        torch.save(_to_cpu(entry), self.root / f"dynamics_{step}_{side}.pt")

    def load_dynamics(self, step: int, side: str) -> dict | None:
        """The saved moments, or ``None``."""
        path = self.root / f"dynamics_{step}_{side}.pt"
        return torch.load(path, weights_only=False) if path.exists() else None

    def dynamics_steps(self) -> list[int]:
        """Steps with both pre and post moments."""
        return sorted(_steps_of(self.root, "dynamics_*_pre.pt") & _steps_of(self.root, "dynamics_*_post.pt"))

    def steps(self) -> list[int]:
        """Steps with both parameters and a batch."""
        params = _steps_of(self.root, "theta_*.pt") | _steps_of(self.root, "theta_*.ref")
        return sorted(params & _steps_of(self.root, "batch_*.pt"))


class LazyDynamics(Mapping):
    """``{step: assembled dynamics}`` read from a snapshot directory on access."""

    def __init__(self, snapshots: TrajectorySnapshots, assemble) -> None:
        self._snapshots = snapshots
        self._assemble = assemble
        self._steps = snapshots.dynamics_steps()

    def __getitem__(self, step: int) -> dict:
        pre = self._snapshots.load_dynamics(step, "pre")
        post = self._snapshots.load_dynamics(step, "post")
        if pre is None or post is None:
            raise KeyError(step)
        return self._assemble(pre, post)

    def __iter__(self) -> Iterator[int]:
        return iter(self._steps)

    def __len__(self) -> int:
        return len(self._steps)

    def __contains__(self, step: object) -> bool:
        return step in self._steps
