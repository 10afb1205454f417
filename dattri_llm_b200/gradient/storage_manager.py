"""The gradient store: residency-managed persistence of :class:`GradientRecord` groups.

On-disk format (identical to the reference's, ``dattri_llm/gradient/storage_manager.py``,
so stores are interchangeable):

* one directory per rank under distributed execution (``rank_<r>/``);
* ``index.jsonl``: an append-only log, one JSON line per written group
  ``{"file": <rel path>, "records": [{"idx", "step", "hashes": [...]}, ...]}``;
  a line cut off by a crash mid-write is ignored on read, and the next append starts
  on a new line;
* ``index_meta.json``: ``{"format": 2, "sample_id_key", "gradient_accumulation_steps"}``;
* groups ``batch_<n>.mmap.bin`` (raw tensor bytes, each part 8-byte aligned) +
  ``batch_<n>.mmap.meta`` (``torch.save`` of ``{"format": 2, "records": [...]}`` with
  per-part ``byte_off / nbytes / shape / dtype``), read back zero-copy through
  ``torch.from_file``; or pickled ``.pt`` groups.

Residencies: ``disk``; ``memory`` (groups held in a budgeted in-memory cache,
``MemoryError`` when full); ``tiered`` (least-recent groups spill to disk files in the
same format).  Re-opening a directory merges every rank's index, so a store written
by N ranks is read as one; an interrupted collection resumes by appending (batch
ids continue after the highest existing one).
"""

from __future__ import annotations

from dattri_llm_b200.options import CacheResidency, DiskFormat  # noqa: F401  (re-exported option types)
import contextlib
import io
import json
import operator
import pickle
import tempfile
import warnings
import zipfile
from collections.abc import Iterable
from pathlib import Path

import numpy as np
import torch

from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
from dattri_llm_b200.utils.cache import CACHE_RESIDENCIES, TensorCache, available_host_bytes
from dattri_llm_b200.utils.distributed import dist_rank
from dattri_llm_b200.utils.hashing import hash_sample
from dattri_llm_b200.utils.tracing import trace_range

DISK_FORMATS = ("pickle", "memmap")
MEMMAP_FORMAT = 2
_ALIGN = 8
_DTYPES = {str(v).removeprefix("torch."): v for v in vars(torch).values() if isinstance(v, torch.dtype)}


def _dtype_name(dtype: torch.dtype) -> str:
    return str(dtype).removeprefix("torch.")


def _dtype_from_name(name: str) -> torch.dtype:
    try:
        return _DTYPES[name]
    except KeyError:
        raise ValueError(f"Unknown tensor dtype {name!r} in memmap metadata.") from None


def _records_nbytes(records: list[GradientRecord]) -> int:
    return sum(r.gradient.nbytes for r in records)


def _host_record(record: GradientRecord) -> GradientRecord:
    """*record* with every payload on the host.  The dense layers of one device and dtype
    travel in one copy (a record holds one tensor per captured layer -- hundreds -- and a
    blocking copy each would stall the host once per layer); factorized payloads move as
    they are."""
    g = record.gradient
    if g.device.type == "cpu":
        return record
    groups: dict[tuple, list[str]] = {}
    for name, v in g.data.items():
        if isinstance(v, torch.Tensor) and v.is_cuda:
            groups.setdefault((v.device, v.dtype), []).append(name)
    data = dict(g.data)
    for names in groups.values():
        flat = torch.cat([g.data[n].reshape(-1) for n in names]).to("cpu")
        for n, piece in zip(names, flat.split([g.data[n].numel() for n in names]), strict=True):
            data[n] = piece.view(g.data[n].shape)
    for name, v in data.items():
        if isinstance(v, Factorized):
            data[name] = v.to(device="cpu")
        elif v.is_cuda:
            data[name] = v.to("cpu")
    host = Gradient(dict(g.representation), data, dict(g.layer_types), dict(g.indexing))
    return GradientRecord(record.step, record.input_hash, host, getattr(record, "sample_id_key", None))


def _memmappable(records: list[GradientRecord]) -> bool:
    return all(isinstance(v, (torch.Tensor, Factorized)) for r in records for v in r.gradient.data.values())


class _PlainPickle:
    """A ``pickle_module`` for ``torch.save`` of tensor-free objects: its pickler is the C one,
    with no per-object ``persistent_id`` hook (it would find no tensor or storage to record)."""

    class Pickler:
        def __init__(self, file, protocol=2) -> None:
            self._file, self._protocol = file, protocol

        def dump(self, obj) -> None:
            pickle.dump(obj, self._file, protocol=self._protocol)


class _NoGlobals(pickle.Unpickler):
    """Unpickler of plain data (dicts, lists, strings, numbers): any class or function
    reference, or any tensor record, is refused."""

    def find_class(self, module, name):
        raise pickle.UnpicklingError(f"{module}.{name} is not plain data")


def _load_meta(path: Path) -> object:
    """A memmap group's metadata.  Plain-data archives are read by the C unpickler with every
    global refused (as safe as ``weights_only``, much faster for large metadata); anything
    else goes through ``torch.load(weights_only=True)``."""
    try:
        with zipfile.ZipFile(path) as zf:
            member = next(n for n in zf.namelist() if n.endswith("/data.pkl"))
            return _NoGlobals(io.BytesIO(zf.read(member))).load()
    except (zipfile.BadZipFile, StopIteration, pickle.UnpicklingError, EOFError, ValueError):
        return torch.load(path, weights_only=True)


def write_memmap_group(records: list[GradientRecord], handle_path: Path) -> None:
    """Write *records* as ``<handle>.bin`` + ``<handle>.meta`` (memmap format 2)."""
    chunks: list[np.ndarray] = []
    offset = 0

    def part(t: torch.Tensor) -> dict:
        nonlocal offset
        dense = t.detach().to("cpu").contiguous()
        raw = dense.reshape(-1).view(torch.uint8).numpy() if dense.numel() else np.empty(0, np.uint8)
        spec = {"byte_off": offset, "nbytes": int(raw.nbytes), "shape": list(dense.shape),
                "dtype": _dtype_name(dense.dtype)}
        chunks.append(raw)
        offset += raw.nbytes
        pad = (-offset) % _ALIGN
        if pad:
            chunks.append(np.zeros(pad, np.uint8))
            offset += pad
        return spec

    metas = []
    for rec in records:
        layers = {}
        for name, v in rec.gradient.data.items():
            if isinstance(v, Factorized):
                layers[name] = {"kind": "factorized",
                                "parts": {"activation": part(v.activation),
                                          "pre_activation_grad": part(v.pre_activation_grad)},
                                "module_kwargs": v.module_kwargs, "batch_first": v.batch_first}
            else:
                layers[name] = {"kind": "dense", "parts": {"data": part(v)}}
        g = rec.gradient
        metas.append({"step": rec.step, "input_hash": rec.input_hash,
                      "sample_id_key": getattr(rec, "sample_id_key", None),
                      "representation": dict(g.representation), "layer_types": dict(g.layer_types),
                      "indexing": dict(g.indexing), "layers": layers})
    with Path(f"{handle_path}.bin").open("wb") as f:
        for c in chunks:
            f.write(memoryview(c))
    # the metadata holds no tensors: the C pickler writes it (torch.save's own pickler calls a
    # Python hook per object, an order of magnitude slower for hundreds of layers per record);
    # the file is the same torch zip archive, so any torch.load reads it
    torch.save({"format": MEMMAP_FORMAT, "records": metas}, Path(f"{handle_path}.meta"), pickle_module=_PlainPickle)


def read_memmap_group(handle_path: Path) -> list[GradientRecord]:
    """Read a memmap group; tensors are views of one ``torch.from_file`` buffer.

    Raises:
        ValueError: for another memmap format version.
    """
    payload = _load_meta(Path(f"{handle_path}.meta"))
    if not isinstance(payload, dict) or payload.get("format") != MEMMAP_FORMAT:
        found = payload.get("format") if isinstance(payload, dict) else "pre-v2"
        raise ValueError(
            f"{Path(handle_path).name} was written in memmap format {found!r}, but this version "
            f"reads format {MEMMAP_FORMAT}. Re-collect the store; the byte offsets are not compatible.",
        )
    bin_path = Path(f"{handle_path}.bin")
    total = bin_path.stat().st_size
    buf = (torch.from_file(str(bin_path), shared=False, size=total, dtype=torch.uint8) if total
           else torch.empty(0, dtype=torch.uint8))

    def view(spec: dict) -> torch.Tensor:
        dtype, shape = _dtype_from_name(spec["dtype"]), tuple(spec["shape"])
        if spec["nbytes"] == 0:
            return torch.empty(shape, dtype=dtype)
        return buf[spec["byte_off"]: spec["byte_off"] + spec["nbytes"]].view(dtype).reshape(shape)

    out = []
    for meta in payload["records"]:
        data = {}
        for name, layer in meta["layers"].items():
            p = layer["parts"]
            if layer["kind"] == "factorized":
                data[name] = Factorized(view(p["activation"]), view(p["pre_activation_grad"]),
                                        module_kwargs=layer["module_kwargs"], batch_first=layer["batch_first"])
            else:
                data[name] = view(p["data"])
        grad = Gradient(meta["representation"], data, meta["layer_types"], meta["indexing"],
                        validate_on_init=False)
        out.append(GradientRecord(meta["step"], meta["input_hash"], grad, meta["sample_id_key"]))
    return out


def _expand_log_line(payload: dict) -> dict[str, list[dict]]:
    out: dict[str, list[dict]] = {}
    for rec in payload["records"]:
        for pos, h in enumerate(rec["hashes"]):
            out.setdefault(h, []).append({"file": payload["file"], "idx": rec["idx"], "step": rec["step"],
                                          "sample_idx": pos})
    return out


def _merge_index(dst: dict, src: dict) -> None:
    for h, entries in src.items():
        have = dst.setdefault(h, [])
        for e in entries:
            if e not in have:
                have.append(e)


class GradientStorageManager:
    """Residency-managed storage and retrieval of :class:`GradientRecord` objects.

    Args:
        save_dir: Store root (per-rank subdirectories under distributed execution).
        residency: ``"disk"`` (default), ``"memory"`` or ``"tiered"``.
        budget_bytes: Memory budget of ``memory``/``tiered`` (default for tiered: half the host's).
        disk_format: ``"memmap"`` (default) or ``"pickle"``.
    """

    _INDEX_LOG_FILE = "index.jsonl"
    _INDEX_META_FILE = "index_meta.json"
    _INDEX_FORMAT = 2

    def __init__(self, save_dir: str, *, residency: str = "disk", budget_bytes: int | None = None,
                 disk_format: str = "memmap") -> None:
        if residency not in CACHE_RESIDENCIES:
            raise ValueError(f"residency must be one of {list(CACHE_RESIDENCIES)}, got {residency!r}.")
        if disk_format not in DISK_FORMATS:
            raise ValueError(f"disk_format must be one of {list(DISK_FORMATS)}, got {disk_format!r}.")
        self._root = Path(save_dir)
        self._residency = residency
        self._disk_format = disk_format
        self._budget = budget_bytes if budget_bytes is not None else (
            available_host_bytes() // 2 if residency == "tiered" else None)
        self._seq = 0
        self._groups = TensorCache(residency if residency != "disk" else "memory", budget=self._budget,
                                   spill_dir=self._spill_dir, writer=self._write_spilled,
                                   reader=self._read_spilled, on_spill=self._on_spilled,
                                   nbytes_fn=_records_nbytes)
        self._group_entries: dict[str, list[dict]] = {}
        self._closed = False
        self._meta_written: dict | None = None
        self._save_dir: Path | None = None
        self._prefix = ""
        self._next_batch = 0
        self._sample_id_key = None
        self._id_key_known = False
        self._accum: int | None = None
        self._index: dict[str, list[dict]] = self._read_all_indexes() if residency == "disk" else {}

    # ------------------------------------------------------------ identity
    def _ensure_save_dir(self) -> Path:
        if self._save_dir is None:
            rank = dist_rank()
            if rank is not None:
                self._save_dir, self._prefix = self._root / f"rank_{rank}", f"rank_{rank}/"
            else:
                self._save_dir = self._root
            self._next_batch = self._compute_next_batch_id()
        return self._save_dir

    @property
    def save_dir(self) -> Path:
        """The store root."""
        return self._root

    @property
    def sample_id_key(self):
        """The identifier scheme of the records (``None``: content hashes)."""
        return self._sample_id_key

    def _adopt_sample_id_key(self, key) -> None:
        if self._id_key_known:
            if key != self._sample_id_key:
                raise ValueError(
                    f"Record was captured with sample_id_key={key!r} but this store uses "
                    f"sample_id_key={self._sample_id_key!r}; one store cannot mix identifier schemes.",
                )
            return
        self._sample_id_key, self._id_key_known = key, True

    @property
    def gradient_accumulation_steps(self) -> int:
        """Backwards per stored step."""
        return self._accum if self._accum is not None else 1

    def declare_gradient_accumulation_steps(self, n: int) -> None:
        """Declare the step convention of this store.

        Raises:
            ValueError: for ``n < 1`` or a conflicting earlier declaration.
        """
        if n < 1:
            raise ValueError(f"gradient_accumulation_steps must be >= 1, got {n}.")
        if self._accum is not None and self._accum != n:
            raise ValueError(
                f"This store was collected with gradient_accumulation_steps={self._accum}; cannot mix "
                f"with {n} -- one store cannot hold two step conventions.",
            )
        self._accum = n

    # ------------------------------------------------------------ writing
    def save(self, record: GradientRecord) -> str:
        """Save one single-hash record as its own group; returns its location."""
        if isinstance(record.input_hash, list):
            raise TypeError("save() takes a single-hash record; this record carries a per-batch hash "
                            "list -- use save_bulk([record]) instead.")
        record = _host_record(record)
        loc = self._write_group([record], f"step_{record.step:06d}_{record.input_hash}")
        self._index_entry(record, loc, 0)
        self._persist_index([record], loc)
        self._commit_group(loc, [record])
        return loc

    def save_bulk(self, records: list[GradientRecord]) -> str:
        """Save *records* as one group (one file pair, one index line)."""
        with trace_range("dattri.store.write"):
            records = [_host_record(r) for r in records]
            loc = self._write_group(records, None)
        for i, r in enumerate(records):
            self._index_entry(r, loc, i)
        self._persist_index(records, loc)
        self._commit_group(loc, records)
        return loc

    @property
    def residency(self) -> str:
        """The residency."""
        return self._residency

    @property
    def disk_format(self) -> str:
        """The on-disk format."""
        return self._disk_format

    @property
    def budget_bytes(self) -> int | None:
        """Memory budget of memory/tiered residency."""
        return self._budget

    @property
    def resident_bytes(self) -> int:
        """Bytes of groups held in memory."""
        return self._groups.nbytes

    def _write_group(self, records, base_name) -> str:
        if self._residency in ("memory", "tiered"):
            loc = f"mem_{self._seq:08d}"
            self._seq += 1
            return loc
        d = self._ensure_save_dir()
        d.mkdir(parents=True, exist_ok=True)
        if base_name is None:
            base_name = f"batch_{self._next_batch:06d}"
            self._next_batch += 1
        return self._prefix + self._serialize(records, d, base_name)

    def _serialize(self, records, directory: Path, base_name: str) -> str:
        if self._disk_format == "memmap" and _memmappable(records):
            handle = f"{base_name}.mmap"
            write_memmap_group(records, directory / handle)
        else:
            handle = f"{base_name}.pt"
            torch.save(records, directory / handle)
        return handle

    def _commit_group(self, loc: str, records) -> None:
        if self._residency in ("memory", "tiered") and not self._groups.put(loc, records):
            self._group_entries.pop(loc, None)
            for h in list(self._index):
                self._index[h] = [e for e in self._index[h] if e["file"] != loc]
                if not self._index[h]:
                    del self._index[h]
            raise MemoryError(
                f"memory store budget_bytes={self._budget} cannot hold another record group "
                f"({_records_nbytes(records)} bytes); use residency='tiered' to spill to disk, or a "
                "larger budget.",
            )

    def _resident(self, loc: str):
        if loc in self._groups and self._groups.location(loc) is None:
            return self._groups.get(loc)
        return None

    def _spill_dir(self) -> Path:
        self._root.mkdir(parents=True, exist_ok=True)
        return Path(tempfile.mkdtemp(prefix="tiered_spill_", dir=self._root))

    def _write_spilled(self, path: Path, records) -> Path:
        return path.parent / self._serialize(records, path.parent, path.stem)

    def _read_spilled(self, path: Path):
        return self.load_records(str(path.relative_to(self._root)))

    def _on_spilled(self, loc: str, path: Path) -> None:
        disk = str(path.relative_to(self._root))
        for e in self._group_entries.get(loc, []):
            e["file"] = disk
        if loc in self._group_entries:
            self._group_entries[disk] = self._group_entries.pop(loc)

    def close(self) -> None:
        """Release in-memory groups and spill files."""
        if not self._closed:
            self._closed = True
            self._groups.close()

    def __enter__(self) -> GradientStorageManager:
        return self

    def __exit__(self, *_exc) -> bool:
        self.close()
        return False

    def __del__(self) -> None:
        with contextlib.suppress(Exception):
            self.close()

    # ------------------------------------------------------------ index
    def _index_entry(self, record: GradientRecord, filename: str, idx: int) -> None:
        self._adopt_sample_id_key(getattr(record, "sample_id_key", None))
        hashes = record.input_hash if isinstance(record.input_hash, list) else [record.input_hash]
        if isinstance(record.input_hash, list):
            b = record.gradient.batch_size
            if len(hashes) != b:
                raise ValueError(
                    f"Record at step {record.step} carries {len(hashes)} sample hashes but its "
                    f"gradient batch size is {b}; the indexed sample_idx positions would not match.",
                )
        for pos, h in enumerate(hashes):
            entry = {"file": filename, "idx": idx, "step": record.step, "sample_idx": pos}
            entries = self._index.setdefault(str(h), [])
            if entry not in entries:
                entries.append(entry)
                self._group_entries.setdefault(filename, []).append(entry)

    def _identifier_for(self, inputs: dict) -> str:
        key = self._sample_id_key
        if key is None:
            return hash_sample(inputs)
        if isinstance(key, int) and isinstance(inputs, (list, tuple)):
            value = inputs[key]
        else:
            fld = f"_arg{key}" if isinstance(key, int) else key
            if fld not in inputs:
                raise KeyError(f"This store identifies samples by sample_id_key={key!r}, but the "
                               f"provided inputs carry no {fld!r} field (keys: {sorted(inputs)}).")
            value = inputs[fld]
        if isinstance(value, torch.Tensor):
            value = value.item()
        return str(value)

    def lookup(self, inputs: dict) -> list[tuple[int, int]]:
        """``[(step, sample_idx)]`` where the sample of *inputs* is stored."""
        return self.lookup_by_hash(self._identifier_for(inputs))

    def lookup_by_hash(self, input_hash: str) -> list[tuple[int, int]]:
        """``[(step, sample_idx)]`` of an identifier.

        Raises:
            KeyError: for an unknown identifier.
        """
        input_hash = str(input_hash)
        if input_hash not in self._index:
            raise KeyError(f"Hash {input_hash[:16]}... not in index. Has the collect() context "
                           "closed, and is save_dir correct?")
        return sorted((e["step"], e["sample_idx"]) for e in self._index[input_hash])

    def load_sample(self, inputs: dict, step: int, sample_idx: int) -> Gradient:
        """The stored gradient of one sample at one step."""
        return self.load_sample_by_hash(self._identifier_for(inputs), step, sample_idx)

    def load_sample_by_hash(self, input_hash: str, step: int, sample_idx: int) -> Gradient:
        """The stored gradient of an identifier at ``(step, sample_idx)``.

        Raises:
            KeyError: when nothing is stored there.
        """
        input_hash = str(input_hash)
        for e in self._index.get(input_hash, []):
            if e["step"] == step and e["sample_idx"] == sample_idx:
                return self._load_entry(e).gradient.slice(dim="batch", index=sample_idx)
        pairs = self.lookup_by_hash(input_hash) if input_hash in self._index else []
        raise KeyError(f"No record for hash {input_hash[:16]}... at (step={step}, sample_idx={sample_idx}). "
                       f"Available (step, sample_idx) pairs: {pairs}.")

    def load_all(self, inputs: dict) -> list[GradientRecord]:
        """Every record holding the sample of *inputs*, by step."""
        return self.load_all_by_hash(self._identifier_for(inputs))

    def load_all_by_hash(self, input_hash: str) -> list[GradientRecord]:
        """Every record holding an identifier, by step."""
        input_hash = str(input_hash)
        if input_hash not in self._index:
            raise KeyError(f"Hash {input_hash[:16]}... not in index. Has the collect() context "
                           "closed, and is save_dir correct?")
        return [self._load_entry(e) for e in sorted(self._index[input_hash], key=operator.itemgetter("step"))]

    def available_steps(self) -> list[int]:
        """Every stored step."""
        return sorted({e["step"] for es in self._index.values() for e in es})

    def iter_steps(self, steps: int | Iterable[int]) -> list[tuple[str, dict[int, list[int]]]]:
        """``[(file, {step: [record idx]})]`` of the groups holding *steps* (files sorted)."""
        wanted = {steps} if isinstance(steps, int) else set(steps)
        by_file: dict[str, dict[int, set[int]]] = {}
        for es in self._index.values():
            for e in es:
                if e["step"] in wanted:
                    by_file.setdefault(e["file"], {}).setdefault(e["step"], set()).add(e["idx"])
        return [(f, {s: sorted(i) for s, i in sorted(by_file[f].items())}) for f in sorted(by_file)]

    def load_records(self, file_relpath: str) -> list[GradientRecord]:
        """Every record of one group."""
        res = self._resident(file_relpath)
        if res is not None:
            return res
        if file_relpath.endswith(".mmap"):
            return read_memmap_group(self._root / file_relpath)
        obj = torch.load(self._root / file_relpath, weights_only=False)
        return obj if isinstance(obj, list) else [obj]

    def _load_entry(self, entry: dict) -> GradientRecord:
        res = self._resident(entry["file"])
        if res is not None:
            return res[entry["idx"]]
        return self.load_records(entry["file"])[entry["idx"]]

    @property
    def index(self) -> dict[str, list[dict]]:
        """``{identifier: [{"file", "idx", "step", "sample_idx"}]}``."""
        return self._index

    def own_records(self) -> list[tuple[int, list[str]]]:
        """``(step, hashes)`` of every record in this process's own directory (``rank_<r>/``
        under distributed execution), in the order they were written.  A group counts only
        once its index line is complete, so after a crash this lists whole groups."""
        log = self._ensure_save_dir() / self._INDEX_LOG_FILE
        out: list[tuple[int, list[str]]] = []
        if not log.exists():
            return out
        with log.open(encoding="utf-8") as f:
            for line in f:
                line = line.strip()
                if not line:
                    continue
                try:
                    payload = json.loads(line)
                except json.JSONDecodeError:
                    continue  # cut off by a crash mid-write
                out += [(int(r["step"]), [str(h) for h in r["hashes"]]) for r in payload["records"]]
        return out

    def _read_all_indexes(self) -> dict[str, list[dict]]:
        merged: dict[str, list[dict]] = {}
        for d in [self._root] + [d for d in sorted(self._root.glob("rank_*")) if d.is_dir()]:
            self._read_index_dir(d, merged)
        return merged

    def _read_index_dir(self, directory: Path, merged: dict) -> None:
        log = directory / self._INDEX_LOG_FILE
        if not log.exists():
            return
        meta_path = directory / self._INDEX_META_FILE
        if meta_path.exists():
            meta = json.loads(meta_path.read_text(encoding="utf-8"))
            self._adopt_sample_id_key(meta["sample_id_key"])
            self.declare_gradient_accumulation_steps(meta.get("gradient_accumulation_steps", 1))
        with log.open(encoding="utf-8") as f:
            for line in f:
                line = line.strip()
                if not line:
                    continue
                try:
                    payload = json.loads(line)
                except json.JSONDecodeError:
                    # a line cut off by a crash mid-write (the next append starts a new line)
                    warnings.warn(f"Ignoring a truncated line in {log} -- the records it "
                                  "described are not indexed.", stacklevel=2)
                    continue
                _merge_index(merged, _expand_log_line(payload))

    def _persist_index(self, records, loc: str) -> None:
        if self._residency == "disk":
            self._append_index(records, loc)

    def _write_index_meta(self, d: Path) -> None:
        meta = {"format": self._INDEX_FORMAT, "sample_id_key": self._sample_id_key,
                "gradient_accumulation_steps": self.gradient_accumulation_steps}
        if meta == self._meta_written:
            return
        tmp = d / (self._INDEX_META_FILE + ".tmp")
        tmp.write_text(json.dumps(meta), encoding="utf-8")
        tmp.replace(d / self._INDEX_META_FILE)
        self._meta_written = meta

    def _append_index(self, records, loc: str) -> None:
        d = self._ensure_save_dir()
        d.mkdir(parents=True, exist_ok=True)
        self._write_index_meta(d)
        line = {"file": loc, "records": [
            {"idx": i, "step": r.step,
             "hashes": [str(h) for h in (r.input_hash if isinstance(r.input_hash, list) else [r.input_hash])]}
            for i, r in enumerate(records)]}
        log = d / self._INDEX_LOG_FILE
        torn = False
        if log.exists() and log.stat().st_size:
            with log.open("rb") as f:
                f.seek(-1, 2)
                torn = f.read(1) != b"\n"  # a line cut off by a crash: end it first
        with log.open("a", encoding="utf-8") as f:
            f.write(("\n" if torn else "") + json.dumps(line, separators=(",", ":")) + "\n")
            f.flush()

    def _compute_next_batch_id(self) -> int:
        if not self._save_dir.exists():
            return 0
        ids = [int(p.name[6:].split(".")[0]) for p in self._save_dir.glob("batch_*")
               if p.name[6:].split(".")[0].isdigit()]
        return max(ids) + 1 if ids else 0
