"""Store the trainable parameters at every capture step (for trajectory replay)."""

from __future__ import annotations

from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback


class ParameterSnapshotCallback(HookManagerCallback):
    """Calls ``snapshots.save_parameters(record.step, model)`` after every step."""

    def __init__(self, model, snapshots) -> None:
        self._model = model
        self.snapshots = snapshots

    def on_step_end(self, record) -> None:
        """Save the parameters of *record*'s step."""
        self.snapshots.save_parameters(record.step, self._model)
