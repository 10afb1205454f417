"""A keyed tensor cache with a byte budget and three residencies.

Entries are tensors or nested containers of tensors (dicts, lists, tuples, objects with an
integer ``nbytes``).  Residency decides where an entry lives:

``memory``  entries stay in memory; an insert that would exceed the budget is refused
            (``put`` returns ``False``) so that the caller can fall back;
``disk``    every entry is written to a spill directory at once and read back per lookup;
``tiered``  entries stay in memory while the budget allows; to make room, the entries
            inserted earliest move to disk, and an entry larger than the whole budget
            goes straight to disk.

A budget is a fixed byte count or a fraction of the memory that is free *when asked*
(the device's free memory for CUDA, the host's available memory otherwise), so that a
long run adapts to what the rest of the job holds.  The cache holds projection matrices,
the dense per-layer gradients that the scoring loop reuses, and the in-memory gradient
stores.  Public names and options as in the reference's ``dattri_llm/utils/cache.py``.
"""

from __future__ import annotations

import contextlib
import os
import shutil
import tempfile
from collections import OrderedDict
from collections.abc import Callable, Hashable
from dataclasses import dataclass
from pathlib import Path

import torch

from dattri_llm_b200.options import CacheResidency  # noqa: F401  (re-exported option type)

CACHE_RESIDENCIES = ("disk", "memory", "tiered")
DEFAULT_CACHE_FRACTION = 0.35
_HOST_FALLBACK_BYTES = 16 << 30


def tensor_nbytes(value: object) -> int:
    """Bytes of the tensors inside *value* (tensors, ``nbytes`` objects, nested containers)."""
    total, pending = 0, [value]
    while pending:
        item = pending.pop()
        if isinstance(item, torch.Tensor):
            total += item.element_size() * item.numel()
        elif isinstance(item, dict):
            pending.extend(item.values())
        elif isinstance(item, (list, tuple)):
            pending.extend(item)
        else:
            size = getattr(item, "nbytes", None)
            if isinstance(size, int):
                total += size
    return total


def available_host_bytes() -> int:
    """Host memory available to new allocations (a 16 GiB guess when unknown)."""
    try:
        import psutil

        return int(psutil.virtual_memory().available)
    except Exception:  # noqa: BLE001 - psutil missing or unreadable: ask the OS directly
        pass
    try:
        return os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    except (ValueError, OSError, AttributeError):
        return _HOST_FALLBACK_BYTES


class CacheBudget:
    """How many bytes a cache may hold: *limit_bytes*, or *fraction* of the memory free
    on *device* (the host's available memory when *device* is ``None`` or a CPU)."""

    def __init__(self, device: torch.device | str | None = None, *, fraction: float = DEFAULT_CACHE_FRACTION,
                 limit_bytes: int | None = None) -> None:
        self.device = None if device is None else torch.device(device)
        self.fraction = float(fraction)
        self.limit_bytes = None if limit_bytes is None else int(limit_bytes)

    def total(self) -> int:
        """The budget now, in bytes."""
        if self.limit_bytes is not None:
            return self.limit_bytes
        on_gpu = self.device is not None and self.device.type == "cuda"
        free = torch.cuda.mem_get_info(self.device)[0] if on_gpu else available_host_bytes()
        return int(self.fraction * free)

    def fits(self, nbytes: int, held: int = 0) -> bool:
        """Whether *nbytes* more fit beside the *held* bytes already charged."""
        return nbytes + held <= self.total()


@dataclass
class _Entry:
    value: object = None      # the object, while it is in memory
    path: Path | None = None  # its file, once it is on disk
    nbytes: int = 0           # bytes charged to the budget while in memory


def _default_write(path: Path, value: object) -> None:
    torch.save(value, path)


def _default_read(path: Path) -> object:
    return torch.load(path, map_location="cpu", weights_only=False)


class TensorCache:
    """Keyed cache of tensors (or tensor containers) under a :class:`CacheBudget`.

    *writer* / *reader* replace ``torch.save`` / ``torch.load`` for spilled entries (the
    writer may return the path it actually wrote); *on_spill* is told where each spilled
    key went; *nbytes_fn* replaces :func:`tensor_nbytes`.  *spill_dir* is a directory, a
    callable that makes one on first use, or ``None`` for a private temporary directory
    (deleted by :meth:`close`, as is one made by the callable).
    """

    def __init__(self, residency: str = "memory", *, budget: CacheBudget | int | None = None,
                 spill_dir: str | Path | Callable[[], Path] | None = None,
                 writer: Callable[[Path, object], Path | None] | None = None,
                 reader: Callable[[Path], object] | None = None,
                 on_spill: Callable[[Hashable, Path], None] | None = None,
                 nbytes_fn: Callable[[object], int] | None = None) -> None:
        if residency not in CACHE_RESIDENCIES:
            raise ValueError(f"unknown cache residency {residency!r}; choose from {list(CACHE_RESIDENCIES)}.")
        self._mode = residency
        self._budget = CacheBudget(limit_bytes=budget) if isinstance(budget, int) else budget
        self._dir_source = spill_dir
        self._dir: Path | None = None if spill_dir is None or callable(spill_dir) else Path(spill_dir)
        self._dir_is_private = spill_dir is None or callable(spill_dir)
        self._write = writer or _default_write
        self._read = reader or _default_read
        self._on_spill = on_spill
        self._size_of = nbytes_fn or tensor_nbytes
        self._entries: OrderedDict[Hashable, _Entry] = OrderedDict()  # insertion order = spill order
        self._in_memory = 0
        self._files_written = 0
        self._open = True

    # ------------------------------------------------------------------ inspection
    @property
    def residency(self) -> str:
        """``memory``, ``disk`` or ``tiered``."""
        return self._mode

    @property
    def nbytes(self) -> int:
        """Bytes of the entries currently in memory."""
        return self._in_memory

    @property
    def spill_dir(self) -> Path | None:
        """Where spilled entries are written (``None`` until the first spill of a private one)."""
        return self._dir

    def __len__(self) -> int:
        return len(self._entries)

    def __contains__(self, key: Hashable) -> bool:
        return key in self._entries

    def keys(self) -> list[Hashable]:
        """Every key: those in memory first, then those on disk, each in insertion order."""
        return ([k for k, e in self._entries.items() if e.path is None]
                + [k for k, e in self._entries.items() if e.path is not None])

    def location(self, key: Hashable) -> Path | None:
        """The file of a spilled entry; ``None`` for an entry in memory or a missing key."""
        entry = self._entries.get(key)
        return None if entry is None else entry.path

    # ------------------------------------------------------------------ access
    def get(self, key: Hashable, default: object = None) -> object:
        """The entry for *key* (read back from its file when spilled), else *default*."""
        entry = self._entries.get(key)
        if entry is None:
            return default
        return self._read(entry.path) if entry.path is not None else entry.value

    def put(self, key: Hashable, value: object) -> bool:
        """Store *value* under *key*, replacing any previous entry.  Returns ``False`` only
        when a ``memory`` cache has no room for it (nothing is stored then)."""
        if not self._open:
            raise RuntimeError("TensorCache is closed.")
        self.discard(key)
        if self._mode == "disk":
            self._entries[key] = self._to_disk(key, value)
            return True
        size = self._size_of(value)
        if not self._room_for(size):
            if self._mode == "memory":
                return False
            self._make_room(size)
            if not self._room_for(size):
                self._entries[key] = self._to_disk(key, value)
                return True
        self._entries[key] = _Entry(value=value, nbytes=size)
        self._in_memory += size
        return True

    def get_or_compute(self, key: Hashable, compute: Callable[[], object]) -> object:
        """The entry for *key*; on a miss, ``compute()`` is stored (if it fits) and returned."""
        if key in self._entries:
            return self.get(key)
        value = compute()
        self.put(key, value)
        return value

    def discard(self, key: Hashable) -> None:
        """Forget *key*, deleting its file if it was spilled."""
        entry = self._entries.pop(key, None)
        if entry is None:
            return
        if entry.path is None:
            self._in_memory -= entry.nbytes
        else:
            self._delete_files(entry.path)

    def clear(self) -> None:
        """Forget every entry."""
        for key in list(self._entries):
            self.discard(key)

    def close(self) -> None:
        """Drop every entry and delete a private spill directory; idempotent."""
        if not self._open:
            return
        self._open = False
        self._entries.clear()
        self._in_memory = 0
        if self._dir_is_private and self._dir is not None:
            shutil.rmtree(self._dir, ignore_errors=True)
            self._dir = None

    def __enter__(self) -> TensorCache:
        return self

    def __exit__(self, *_exc: object) -> bool:
        self.close()
        return False

    def __del__(self) -> None:
        with contextlib.suppress(Exception):
            self.close()

    # ------------------------------------------------------------------ internals
    def _room_for(self, size: int) -> bool:
        return self._budget is None or self._budget.fits(size, self._in_memory)

    def _make_room(self, size: int) -> None:
        """Tiered: move the earliest in-memory entries to disk until *size* fits."""
        for key in [k for k, e in self._entries.items() if e.path is None]:
            if self._room_for(size):
                return
            entry = self._entries[key]
            self._in_memory -= entry.nbytes
            self._entries[key] = self._to_disk(key, entry.value)

    def _to_disk(self, key: Hashable, value: object) -> _Entry:
        if self._dir is None:
            made = self._dir_source() if callable(self._dir_source) else tempfile.mkdtemp(prefix="bw_cache_")
            self._dir = Path(made)
        self._dir.mkdir(parents=True, exist_ok=True)
        target = self._dir / f"entry_{self._files_written:08d}.pt"
        self._files_written += 1
        written = self._write(target, value)
        path = target if written is None else Path(written)
        if self._on_spill is not None:
            self._on_spill(key, path)
        return _Entry(path=path)

    @staticmethod
    def _delete_files(path: Path) -> None:
        """A spilled entry may span several files sharing its stem (e.g. data + metadata)."""
        folder = path.parent
        if not folder.is_dir():
            return
        for f in folder.glob(f"{path.stem}*"):
            f.unlink(missing_ok=True)
