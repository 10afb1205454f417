"""Periodic persistence of captured records into a :class:`GradientStorageManager`.

Records are staged and flushed every ``offload_interval`` distinct steps (and at
context end), per batch or sliced per sample; gradient-accumulation windows are
merged into one record per optimizer update.  With ``async_write`` the flush goes
through :class:`AsyncGradientWriter` (device-to-host copies on a side stream into
pinned buffers, disk IO on a background thread).  Parity: reference
``dattri_llm/gradient/callbacks/offload_callback.py``.
"""

from __future__ import annotations

from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.gradient import GradientRecord


class OffloadCallback(HookManagerCallback):
    """Save records every *offload_interval* steps.

    Args:
        offload_interval: Distinct steps staged per flush.
        file_manager: The destination store.
        recording_type: ``"per_batch"`` (one record per step) or ``"per_sample"``.
        gradient_accumulation_steps: Backwards per optimizer update (merged into one record).
        async_write: Flush through an :class:`AsyncGradientWriter`.
        max_pending_writes: Queue depth of the async writer (back-pressure).
    """

    def __init__(self, offload_interval: int, file_manager, recording_type: str = "per_batch",
                 gradient_accumulation_steps: int = 1, async_write: bool = False,
                 max_pending_writes: int = 2) -> None:
        if recording_type not in ("per_sample", "per_batch"):
            raise ValueError(f"recording_type must be 'per_sample' or 'per_batch', got {recording_type!r}.")
        if gradient_accumulation_steps < 1:
            raise ValueError(f"gradient_accumulation_steps must be >= 1, got {gradient_accumulation_steps}.")
        self._interval = offload_interval
        self.file_manager = file_manager
        self._recording = recording_type
        self._accum = gradient_accumulation_steps
        self._async = async_write
        self._max_pending = max_pending_writes
        self._writer = None
        file_manager.declare_gradient_accumulation_steps(gradient_accumulation_steps)
        self._window: list[GradientRecord] = []
        self._update_step = 0
        self._staged: list[GradientRecord] = []
        self._staged_steps: set = set()

    def on_step_end(self, record: GradientRecord) -> None:
        """Stage *record* (after merging a full accumulation window)."""
        if self._accum > 1:
            self._window.append(record)
            if len(self._window) < self._accum:
                return
            record = self._merge_window()
        self._stage(record)

    def _merge_window(self) -> GradientRecord:
        window, self._window = self._window, []
        grad = window[0].gradient
        for rec in window[1:]:
            grad = grad.concatenate(rec.gradient, dim="batch")
        hashes = [h for rec in window
                  for h in (rec.input_hash if isinstance(rec.input_hash, list) else [rec.input_hash])]
        merged = GradientRecord(self._update_step, hashes, grad, window[0].sample_id_key)
        self._update_step += 1
        return merged

    def _stage(self, record: GradientRecord) -> None:
        records = self._expand(record)
        if record.step not in self._staged_steps and len(self._staged_steps) >= self._interval:
            self._flush()
        self._staged.extend(records)
        self._staged_steps.add(record.step)

    def _expand(self, record: GradientRecord) -> list[GradientRecord]:
        if self._recording != "per_sample":
            return [record]
        hashes = record.input_hash if isinstance(record.input_hash, list) else [record.input_hash]
        return [GradientRecord(record.step, hashes[i], record.gradient.slice(dim="batch", index=i),
                               record.sample_id_key) for i in range(record.gradient.batch_size)]

    def on_context_end(self) -> None:
        """Flush everything staged and close the async writer."""
        if self._window:
            self._stage(self._merge_window())
        self._flush()
        if self._writer is not None:
            writer, self._writer = self._writer, None
            writer.close()

    def _flush(self) -> None:
        if not self._staged:
            return
        if self._async:
            if self._writer is None:
                from dattri_llm_b200.gradient.async_writer import AsyncGradientWriter

                self._writer = AsyncGradientWriter(self.file_manager, max_pending=self._max_pending)
            self._writer.submit(self._staged)
        else:
            self.file_manager.save_bulk(self._staged)
        self._staged = []
        self._staged_steps = set()

    @property
    def staged(self) -> list[GradientRecord]:
        """Records waiting for the next flush."""
        return list(self._staged)
