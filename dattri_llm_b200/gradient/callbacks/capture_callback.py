"""Holds the most recent step's :class:`GradientRecord` in memory (used by the streamer)."""

from __future__ import annotations

from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback


class CaptureCallback(HookManagerCallback):
    """Keeps ``record``: the last completed step's record (``None`` before the first)."""

    def __init__(self) -> None:
        self.record = None

    def on_step_end(self, record) -> None:
        """Keep *record*."""
        self.record = record
