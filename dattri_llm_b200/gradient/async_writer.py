"""Write gradient record groups to a store from a background thread.

``submit`` enqueues the D2H copy of a group's device tensors on a per-device side
stream, into pinned host buffers from a small reusable pool, after an event on the
producing stream -- so the copy overlaps the next training step -- and hands the
group to one writer thread that waits for the copy's event and performs the store
write.  Back-pressure: at most ``max_pending`` groups are in flight.  An error of
the writer thread is re-raised at the next ``submit``/``flush``/``close``.
Parity: reference ``dattri_llm/gradient/async_writer.py:46-207``.

Thread safety: while the writer is open the store belongs to the writer thread;
read from it only after :meth:`flush` or :meth:`close`.
"""

from __future__ import annotations

import queue
import threading

import torch

from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord

_STOP = object()


class _PinnedPool:
    """Reusable pinned host buffers keyed by byte size (returned when a group is written)."""

    def __init__(self) -> None:
        self._free: dict[int, list[torch.Tensor]] = {}
        self._lock = threading.Lock()

    def take(self, nbytes: int) -> torch.Tensor:
        with self._lock:
            lst = self._free.get(nbytes)
            if lst:
                return lst.pop()
        return torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)

    def give(self, buf: torch.Tensor) -> None:
        with self._lock:
            self._free.setdefault(buf.numel(), []).append(buf)


class AsyncGradientWriter:
    """Background writer of record groups into a :class:`GradientStorageManager`.

    Args:
        file_manager: Destination store.
        max_pending: Groups allowed in flight before :meth:`submit` blocks (``>= 1``).
    """

    def __init__(self, file_manager, max_pending: int = 2) -> None:
        if max_pending < 1:
            raise ValueError(f"max_pending must be >= 1, got {max_pending}.")
        self._fm = file_manager
        self._queue: queue.Queue = queue.Queue(maxsize=max_pending)
        self._error: BaseException | None = None
        self._closed = False
        self._streams: dict[int, torch.cuda.Stream] = {}
        self._pool = _PinnedPool()
        self._thread = threading.Thread(target=self._run, name="bw-gradient-writer", daemon=True)
        self._thread.start()

    def submit(self, records: list[GradientRecord]) -> None:
        """Enqueue one group (blocks while ``max_pending`` are in flight); re-raises a
        previous write error."""
        self._check_error()
        if self._closed:
            raise RuntimeError("AsyncGradientWriter is closed.")
        staged, events, buffers = self._stage_host(records)
        self._queue.put((staged, events, buffers))

    def flush(self) -> None:
        """Wait until every submitted group is written."""
        self._queue.join()
        self._check_error()

    def close(self) -> None:
        """Flush, stop the thread and re-raise a pending error."""
        if self._closed:
            return
        self._queue.join()
        self._closed = True
        self._queue.put(_STOP)
        self._thread.join()
        self._check_error(consume=True)

    def __enter__(self) -> AsyncGradientWriter:
        return self

    def __exit__(self, *exc) -> bool:
        if exc[0] is None:
            self.close()
        else:
            try:
                self.close()
            except Exception:  # noqa: BLE001 - keep the original exception
                pass
        return False

    def _check_error(self, consume: bool = False) -> None:
        err = self._error
        if err is not None:
            if consume:
                self._error = None
            raise RuntimeError("asynchronous gradient write failed") from err

    def _stream(self, device: torch.device) -> torch.cuda.Stream:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        s = self._streams.get(idx)
        if s is None:
            s = self._streams[idx] = torch.cuda.Stream(device=idx)
        return s

    def _to_host(self, t: torch.Tensor, events: list, buffers: list) -> torch.Tensor:
        if t.device.type != "cuda":
            return t
        src = t.detach()
        nbytes = src.numel() * src.element_size()
        buf = self._pool.take(nbytes)
        buffers.append(buf)
        host = buf.view(src.dtype).view(src.shape) if nbytes else torch.empty(src.shape, dtype=src.dtype)
        stream = self._stream(src.device)
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(src.device))
        with torch.cuda.stream(stream):
            stream.wait_event(ready)
            if nbytes:
                host.copy_(src.contiguous(), non_blocking=True)
            src.record_stream(stream)
            done = torch.cuda.Event()
            done.record(stream)
        events.append(done)
        return host

    def _stage_host(self, records: list[GradientRecord]):
        events: list = []
        buffers: list = []
        out = []
        for r in records:
            g = r.gradient
            data = {}
            for n, v in g.data.items():
                if isinstance(v, Factorized):
                    data[n] = Factorized(self._to_host(v.activation, events, buffers),
                                         self._to_host(v.pre_activation_grad, events, buffers),
                                         module_kwargs=v.module_kwargs, batch_first=v.batch_first)
                else:
                    data[n] = self._to_host(v, events, buffers)
            grad = Gradient(dict(g.representation), data, dict(g.layer_types), dict(g.indexing),
                            validate_on_init=False)
            out.append(GradientRecord(r.step, r.input_hash, grad, getattr(r, "sample_id_key", None)))
        return out, events, buffers

    def _run(self) -> None:
        while True:
            item = self._queue.get()
            try:
                if item is _STOP:
                    return
                records, events, buffers = item
                for e in events:
                    e.synchronize()
                if self._error is None:
                    try:
                        self._fm.save_bulk(records)
                    except BaseException as exc:  # noqa: BLE001 - surfaced on the caller's thread
                        self._error = exc
                del records
                if getattr(self._fm, "residency", "disk") == "disk":
                    # a disk store copied the bytes out; a memory store keeps them
                    for b in buffers:
                        self._pool.give(b)
            finally:
                self._queue.task_done()
