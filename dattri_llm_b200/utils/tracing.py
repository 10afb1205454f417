"""Tracing and structured metrics: NVTX ranges, device timers, JSONL metric rows.

The reference library has no tracing of its own (its benchmarks time phases with
``torch.cuda.synchronize`` plus a wall clock, ``experiments/benchmark/utils/log.py:89-181``).
This module adds the three pieces a GPU deployment needs:

* :func:`trace_range` — an NVTX push/pop around a named phase (one batch of the
  streamer, one capture step, one store write, one score block), so a timeline
  profiler shows where a step spends its time.  Off by default; turned on by
  :func:`set_tracing` or the ``DATTRI_B200_NVTX=1`` environment variable.  When off,
  or on a host without CUDA, it costs one boolean test.
* :class:`DeviceTimer` — CUDA-event timing of a region on the current stream, with the
  elapsed time reduced by MAX over the ranks of the process group (the slowest rank
  sets a collective step's time).  On a CPU-only host it falls back to
  ``time.perf_counter`` so the same code runs in tests.
* :class:`MetricsLogger` — appends one JSON object per record to a ``.jsonl`` file, on
  rank 0 only, each stamped with the time and the world size.
"""

from __future__ import annotations

import contextlib
import json
import os
import time
from collections.abc import Iterator

import torch

from dattri_llm_b200.utils.distributed import all_reduce_max, dist_rank, dist_world_size

_ENV = "DATTRI_B200_NVTX"
_enabled: bool | None = None


def tracing_enabled() -> bool:
    """Whether :func:`trace_range` emits NVTX ranges."""
    global _enabled
    if _enabled is None:
        _enabled = os.environ.get(_ENV, "0").lower() not in ("", "0", "false", "no")
    return _enabled


def set_tracing(enabled: bool) -> None:
    """Turn NVTX ranges on or off for this process (overrides ``DATTRI_B200_NVTX``)."""
    global _enabled
    _enabled = bool(enabled)


def _nvtx_available() -> bool:
    return torch.cuda.is_available()


@contextlib.contextmanager
def trace_range(name: str) -> Iterator[None]:
    """NVTX range *name* around the body when tracing is on; a no-op otherwise.

    The range is popped even if the body raises, so a failing step leaves the NVTX
    stack balanced for the next one.
    """
    if not (tracing_enabled() and _nvtx_available()):
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class DeviceTimer:
    """Time a region on the device; the reported time is the MAX over ranks.

    Usage::

        timer = DeviceTimer()
        with timer:
            step()
        ms = timer.elapsed_ms()    # synchronizes, then reduces over ranks

    Repeated ``with`` blocks accumulate.  On CUDA the events are recorded on the
    current stream at entry and exit, so the time is the device time of the work
    queued between them; ``elapsed_ms`` synchronizes the exit events before reading
    them.  Without CUDA the host clock is used.
    """

    def __init__(self, device: torch.device | str | None = None) -> None:
        if device is not None:
            dev = torch.device(device)
        elif torch.cuda.is_available():
            dev = torch.device("cuda", torch.cuda.current_device())
        else:
            dev = torch.device("cpu")
        self.device = dev
        self._cuda = dev.type == "cuda"
        self._pairs: list[tuple[object, object]] = []
        self._host_ms = 0.0
        self._t0: object = None

    def __enter__(self) -> DeviceTimer:
        if self._cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self._t0 = ev
        else:
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc: object) -> None:
        if self._t0 is None:
            return
        if self._cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self._pairs.append((self._t0, ev))
        else:
            self._host_ms += (time.perf_counter() - float(self._t0)) * 1e3
        self._t0 = None

    def local_ms(self) -> float:
        """This rank's accumulated time in milliseconds (synchronizes on CUDA)."""
        total = self._host_ms
        for a, b in self._pairs:
            b.synchronize()
            total += a.elapsed_time(b)
        return total

    def elapsed_ms(self) -> float:
        """Accumulated time, MAX over the ranks of the process group.

        A collective: inside a process group every rank must call it, in the same order
        as its other collectives.
        """
        t = torch.tensor([self.local_ms()], dtype=torch.float64)
        if dist_world_size() > 1:
            all_reduce_max(t)
        return float(t.item())

    def reset(self) -> None:
        """Drop the accumulated time."""
        self._pairs.clear()
        self._host_ms = 0.0
        self._t0 = None


class MetricsLogger:
    """Append structured metric rows to a JSON-lines file, from rank 0 only.

    Each :meth:`log` writes one line: the given fields plus ``time`` (seconds since the
    epoch) and ``world_size``.  Values that are tensors are converted with ``.tolist()``.
    Other ranks accept the call and write nothing, so callers need no rank test.
    """

    def __init__(self, path: str | os.PathLike, *, all_ranks: bool = False) -> None:
        self.path = os.fspath(path)
        rank = dist_rank() or 0
        self.active = all_ranks or rank == 0
        if all_ranks and rank:
            root, ext = os.path.splitext(self.path)
            self.path = f"{root}.rank{rank}{ext or '.jsonl'}"
        if self.active:
            parent = os.path.dirname(self.path)
            if parent:
                os.makedirs(parent, exist_ok=True)

    @staticmethod
    def _plain(v: object) -> object:
        if isinstance(v, torch.Tensor):
            return v.detach().cpu().tolist()
        if isinstance(v, dict):
            return {str(k): MetricsLogger._plain(x) for k, x in v.items()}
        if isinstance(v, (list, tuple)):
            return [MetricsLogger._plain(x) for x in v]
        return v

    def log(self, **fields: object) -> None:
        """Write one row with *fields* (rank 0 only)."""
        if not self.active:
            return
        row = {k: self._plain(v) for k, v in fields.items()}
        row.setdefault("time", time.time())
        row.setdefault("world_size", dist_world_size())
        with open(self.path, "a", encoding="utf-8") as f:
            f.write(json.dumps(row, sort_keys=True) + "\n")

    def read(self) -> list[dict]:
        """All rows written so far (empty on an inactive rank or before the first row)."""
        if not os.path.exists(self.path):
            return []
        with open(self.path, encoding="utf-8") as f:
            return [json.loads(line) for line in f if line.strip()]


def throughput_row(name: str, items: float, ms: float, *, unit: str = "items/s", peak: float | None = None,
                   **extra: object) -> dict:
    """A metric row for *items* processed in *ms* milliseconds.

    With *peak* (same unit as the rate) the row also carries ``fraction_of_peak``.
    """
    rate = items / (ms / 1e3) if ms > 0 else float("inf")
    row: dict = {"name": name, "value": rate, "unit": unit, "ms": ms, "items": items}
    if peak:
        row["fraction_of_peak"] = rate / peak
    row.update(extra)
    return row
