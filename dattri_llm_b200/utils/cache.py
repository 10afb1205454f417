"""Budgeted, residency-aware tensor cache.

Parity: reference ``dattri_llm/utils/cache.py:55-372`` (``CacheBudget``,
``TensorCache``; residencies ``memory`` / ``disk`` / ``tiered``).  Used for
projection matrices, dense-materialization reuse in the scoring loop and the
memory/tiered gradient stores.  ``memory`` refuses entries beyond the budget,
``disk`` spills every entry, ``tiered`` spills least-recently-inserted entries
to make room.
"""

from __future__ import annotations

from dattri_llm_b200.options import CacheResidency  # noqa: F401  (re-exported option types)
import contextlib
import shutil
import tempfile
from collections import OrderedDict
from collections.abc import Callable, Hashable
from pathlib import Path

import torch

CACHE_RESIDENCIES = ("disk", "memory", "tiered")
DEFAULT_CACHE_FRACTION = 0.35


def tensor_nbytes(value: object) -> int:
    """Bytes held by a tensor, an object with an int ``nbytes``, or a dict/list/tuple of those."""
    if isinstance(value, torch.Tensor):
        return value.numel() * value.element_size()
    nbytes = getattr(value, "nbytes", None)
    if isinstance(nbytes, int):
        return nbytes
    if isinstance(value, dict):
        return sum(tensor_nbytes(v) for v in value.values())
    if isinstance(value, (list, tuple)):
        return sum(tensor_nbytes(v) for v in value)
    return 0


def available_host_bytes() -> int:
    """``MemAvailable`` of the host (16 GiB when it cannot be read)."""
    try:
        with Path("/proc/meminfo").open(encoding="utf-8") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except (OSError, ValueError, IndexError):
        pass
    return 16 * 2**30


class CacheBudget:
    """Byte budget a cache may occupy on a device: a fixed limit, or a fraction
    of the device's currently free memory (host ``MemAvailable`` for CPU)."""

    def __init__(
        self,
        device: torch.device | str | None = None,
        *,
        fraction: float = DEFAULT_CACHE_FRACTION,
        limit_bytes: int | None = None,
    ) -> None:
        self._device = torch.device(device) if device is not None else None
        self._fraction = float(fraction)
        self._limit = limit_bytes

    @property
    def device(self) -> torch.device | None:
        """The device whose memory the budget is a fraction of."""
        return self._device

    def total(self) -> int:
        """The budget in bytes, evaluated now."""
        if self._limit is not None:
            return int(self._limit)
        if self._device is not None and self._device.type == "cuda":
            free, _ = torch.cuda.mem_get_info(self._device)
            return int(free * self._fraction)
        return int(available_host_bytes() * self._fraction)

    def fits(self, nbytes: int, held: int = 0) -> bool:
        """Whether *nbytes* more fit next to *held* bytes."""
        return held + nbytes <= self.total()


def _torch_save(path: Path, value: object) -> None:
    torch.save(value, path)


def _torch_load(path: Path) -> object:
    return torch.load(path, map_location="cpu", weights_only=False)


class TensorCache:
    """Keyed, budgeted, residency-aware cache of tensors (or tensor containers)."""

    def __init__(
        self,
        residency: str = "memory",
        *,
        budget: CacheBudget | int | None = None,
        spill_dir: str | Path | Callable[[], Path] | None = None,
        writer: Callable[[Path, object], Path | None] | None = None,
        reader: Callable[[Path], object] | None = None,
        on_spill: Callable[[Hashable, Path], None] | None = None,
        nbytes_fn: Callable[[object], int] | None = None,
    ) -> None:
        if residency not in CACHE_RESIDENCIES:
            raise ValueError(
                f"residency must be one of {list(CACHE_RESIDENCIES)}, got {residency!r}.",
            )
        self._residency = residency
        self._budget = CacheBudget(limit_bytes=budget) if isinstance(budget, int) else budget
        self._spill_factory = spill_dir if callable(spill_dir) else None
        self._spill_dir = Path(spill_dir) if spill_dir is not None and not callable(spill_dir) else None
        self._owns_spill_dir = spill_dir is None or callable(spill_dir)
        self._writer = writer or _torch_save
        self._reader = reader or _torch_load
        self._on_spill = on_spill
        self._nbytes = nbytes_fn or tensor_nbytes
        self._memory: OrderedDict[Hashable, object] = OrderedDict()
        self._sizes: dict[Hashable, int] = {}
        self._held = 0
        self._disk: dict[Hashable, Path] = {}
        self._seq = 0
        self._closed = False

    residency = property(lambda self: self._residency, doc="The cache's residency.")
    nbytes = property(lambda self: self._held, doc="Bytes held in memory.")
    spill_dir = property(lambda self: self._spill_dir, doc="Directory of spilled entries.")

    def __len__(self) -> int:
        return len(self._memory) + len(self._disk)

    def __contains__(self, key: Hashable) -> bool:
        return key in self._memory or key in self._disk

    def keys(self) -> list[Hashable]:
        """Every key, in-memory first."""
        return [*self._memory.keys(), *self._disk.keys()]

    def location(self, key: Hashable) -> Path | None:
        """The file a spilled entry lives in (``None`` if in memory or absent)."""
        return self._disk.get(key)

    def get(self, key: Hashable, default: object = None) -> object:
        """The entry for *key* (read back from disk when spilled), else *default*."""
        if key in self._memory:
            return self._memory[key]
        path = self._disk.get(key)
        return default if path is None else self._reader(path)

    def put(self, key: Hashable, value: object) -> bool:
        """Insert *value*; ``False`` when a ``memory`` cache has no room for it."""
        if self._closed:
            raise RuntimeError("TensorCache is closed.")
        self.discard(key)
        if self._residency == "disk":
            self._spill(key, value)
            return True
        nbytes = self._nbytes(value)
        if self._budget is not None and not self._budget.fits(nbytes, self._held):
            if self._residency == "memory":
                return False
            while self._memory and not self._budget.fits(nbytes, self._held):
                oldest = next(iter(self._memory))
                self._spill(oldest, self._memory.pop(oldest))
                self._held -= self._sizes.pop(oldest)
            if not self._budget.fits(nbytes, self._held):
                self._spill(key, value)
                return True
        self._memory[key] = value
        self._sizes[key] = nbytes
        self._held += nbytes
        return True

    def get_or_compute(self, key: Hashable, compute: Callable[[], object]) -> object:
        """Cached value for *key*, computing and inserting it on a miss."""
        if key in self:
            return self.get(key)
        value = compute()
        self.put(key, value)
        return value

    def discard(self, key: Hashable) -> None:
        """Drop *key* from memory and disk."""
        if key in self._memory:
            del self._memory[key]
            self._held -= self._sizes.pop(key)
        path = self._disk.pop(key, None)
        if path is not None and path.parent.exists():
            for p in path.parent.iterdir():
                if p.name.startswith(path.stem):
                    p.unlink(missing_ok=True)

    def clear(self) -> None:
        """Drop every entry."""
        for key in self.keys():
            self.discard(key)

    def close(self) -> None:
        """Release memory and delete an owned spill directory."""
        if self._closed:
            return
        self._closed = True
        self._memory.clear()
        self._sizes.clear()
        self._held = 0
        self._disk.clear()
        if self._owns_spill_dir and self._spill_dir is not None:
            shutil.rmtree(self._spill_dir, ignore_errors=True)
            self._spill_dir = None

    def __enter__(self) -> TensorCache:
        return self

    def __exit__(self, *_exc: object) -> bool:
        self.close()
        return False

    def __del__(self) -> None:
        with contextlib.suppress(Exception):
            self.close()

    def _spill(self, key: Hashable, value: object) -> None:
        if self._spill_dir is None:
            self._spill_dir = (
                Path(self._spill_factory()) if self._spill_factory is not None
                else Path(tempfile.mkdtemp(prefix="bw_cache_"))
            )
        self._spill_dir.mkdir(parents=True, exist_ok=True)
        path = self._spill_dir / f"entry_{self._seq:08d}.pt"
        self._seq += 1
        written = self._writer(path, value)
        path = Path(written) if written is not None else path
        self._disk[key] = path
        if self._on_spill is not None:
            self._on_spill(key, path)
