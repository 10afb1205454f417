"""Periodic persistence of captured records into a :class:`GradientStorageManager`.

Records are held in an outbox keyed by step and written every ``offload_interval``
distinct steps (and at context end), whole or sliced into one record per sample.  Under
gradient accumulation the backwards of one optimizer update are first joined into one
record.  With ``async_write`` the outbox goes through :class:`AsyncGradientWriter`
(device-to-host copies on a side stream into pinned buffers, disk IO on a background
thread).  Parity: reference ``dattri_llm/gradient/callbacks/offload_callback.py``.
"""

from __future__ import annotations

import itertools

from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.gradient import GradientRecord


def _hashes(record: GradientRecord) -> list:
    h = record.input_hash
    return h if isinstance(h, list) else [h]


class _UpdateWindow:
    """The backwards of one optimizer update, joined along the batch into one record
    numbered by update."""

    def __init__(self, backwards: int) -> None:
        self.backwards, self.parts, self.updates = backwards, [], 0

    def add(self, record: GradientRecord) -> GradientRecord | None:
        """The joined record once *record* completes a window (*record* itself without
        accumulation), else ``None``."""
        if self.backwards == 1:
            return record
        self.parts.append(record)
        return self.close() if len(self.parts) == self.backwards else None

    def close(self) -> GradientRecord | None:
        """Join whatever the window holds (a short last window included)."""
        if not self.parts:
            return None
        parts, self.parts = self.parts, []
        gradient = parts[0].gradient
        for part in parts[1:]:
            gradient = gradient.concatenate(part.gradient, dim="batch")
        ids = list(itertools.chain.from_iterable(_hashes(p) for p in parts))
        joined = GradientRecord(self.updates, ids, gradient, parts[0].sample_id_key)
        self.updates += 1
        return joined


def _one_per_sample(record: GradientRecord) -> list[GradientRecord]:
    ids = _hashes(record)
    return [GradientRecord(record.step, ids[i], record.gradient.slice(dim="batch", index=i), record.sample_id_key)
            for i in range(record.gradient.batch_size)]


class OffloadCallback(HookManagerCallback):
    """Save records every *offload_interval* steps.

    Args:
        offload_interval: Distinct steps held before a write.
        file_manager: The destination store.
        recording_type: ``"per_batch"`` (one record per step) or ``"per_sample"``.
        gradient_accumulation_steps: Backwards per optimizer update (joined into one record).
        async_write: Write through an :class:`AsyncGradientWriter`.
        max_pending_writes: Queue depth of the async writer (back-pressure).
    """

    def __init__(self, offload_interval: int, file_manager, recording_type: str = "per_batch",
                 gradient_accumulation_steps: int = 1, async_write: bool = False,
                 max_pending_writes: int = 2) -> None:
        if recording_type not in ("per_batch", "per_sample"):
            raise ValueError(f"unknown recording_type {recording_type!r}: expected 'per_batch' or 'per_sample'.")
        if gradient_accumulation_steps < 1:
            raise ValueError(f"gradient_accumulation_steps is {gradient_accumulation_steps}; it must be at least 1.")
        self.file_manager = file_manager
        self._every = offload_interval
        self._split = recording_type == "per_sample"
        self._async, self._queue_depth = async_write, max_pending_writes
        self._writer = None
        self._window = _UpdateWindow(gradient_accumulation_steps)
        self._outbox: dict[int, list[GradientRecord]] = {}  # step -> records, in arrival order
        file_manager.declare_gradient_accumulation_steps(gradient_accumulation_steps)

    def on_step_end(self, record: GradientRecord) -> None:
        """Hold *record* (joined with its update's other backwards first)."""
        ready = self._window.add(record)
        if ready is not None:
            self._hold(ready)

    def on_context_end(self) -> None:
        """Write everything held and close the async writer."""
        tail = self._window.close()
        if tail is not None:
            self._hold(tail)
        self._write()
        writer, self._writer = self._writer, None
        if writer is not None:
            writer.close()

    @property
    def staged(self) -> list[GradientRecord]:
        """Records waiting for the next write."""
        return [r for rows in self._outbox.values() for r in rows]

    def _hold(self, record: GradientRecord) -> None:
        if record.step not in self._outbox and len(self._outbox) >= self._every:
            self._write()
        rows = _one_per_sample(record) if self._split else [record]
        self._outbox.setdefault(record.step, []).extend(rows)

    def _write(self) -> None:
        batch = self.staged
        self._outbox = {}
        if not batch:
            return
        if not self._async:
            self.file_manager.save_bulk(batch)
            return
        if self._writer is None:
            from dattri_llm_b200.gradient.async_writer import AsyncGradientWriter

            self._writer = AsyncGradientWriter(self.file_manager, max_pending=self._queue_depth)
        self._writer.submit(batch)
