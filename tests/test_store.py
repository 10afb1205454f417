"""Gradient store (the on-disk cache format) and the async writer, on CPU."""

from __future__ import annotations

import json

import pytest
import torch

from dattri_llm_b200.gradient.async_writer import AsyncGradientWriter
from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager


def _block(b: int, seed: int, *, factorized: bool = False) -> Gradient:
    g = torch.Generator().manual_seed(seed)
    if factorized:
        data = {"l0": Factorized(torch.randn(b, 3, 4, generator=g), torch.randn(b, 3, 5, generator=g))}
        return Gradient({"l0": "factorized"}, data, {"l0": "nn.Linear"}, {"l0": "batch_token"})
    data = {"l0": torch.randn(b, 12, generator=g), "l1": torch.randn(b, 7, generator=g).bfloat16()}
    return Gradient(dict.fromkeys(data, "materialized"), data, dict.fromkeys(data, "nn.Linear"))


def _ids(prefix: str, n: int) -> list[str]:
    return [f"{prefix}{i:04d}" for i in range(n)]


def _same(a: Gradient, b: Gradient) -> None:
    assert set(a.data) == set(b.data)
    for n in a.data:
        x, y = a.data[n], b.data[n]
        if isinstance(x, Factorized):
            torch.testing.assert_close(x.activation, y.activation)
            torch.testing.assert_close(x.pre_activation_grad, y.pre_activation_grad)
        else:
            assert x.dtype == y.dtype
            torch.testing.assert_close(x, y)


@pytest.mark.parametrize("disk_format", ["memmap", "pickle"])
@pytest.mark.parametrize("residency", ["disk", "memory", "tiered"])
def test_roundtrip(tmp_path, disk_format, residency):
    store = GradientStorageManager(str(tmp_path / "s"), residency=residency, disk_format=disk_format)
    blocks = {0: _block(4, 0), 1: _block(4, 1), 2: _block(3, 2, factorized=True)}
    for step, blk in blocks.items():
        store.save_bulk([GradientRecord(step, _ids(f"s{step}_", blk.batch_size), blk)])
    assert store.available_steps() == [0, 1, 2]
    for step, blk in blocks.items():
        loaded = []
        for f, by_step in store.iter_steps(step):
            recs = store.load_records(f)
            loaded.extend(recs[i] for i in by_step[step])
        assert len(loaded) == 1
        assert loaded[0].input_hash == _ids(f"s{step}_", blk.batch_size)
        _same(loaded[0].gradient, blk)
    store.close()


def test_reopen_from_disk_and_lookup(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    blk = _block(4, 3)
    store.save_bulk([GradientRecord(5, _ids("x", 4), blk), GradientRecord(6, _ids("y", 4), _block(4, 4))])
    store.close()
    again = GradientStorageManager(str(tmp_path / "s"))
    assert again.available_steps() == [5, 6]
    hits = again.lookup_by_hash("x0002")
    assert hits and hits[0][0] == 5
    one = again.load_sample_by_hash("x0002", 5, hits[0][1])
    torch.testing.assert_close(one.data["l0"][0], blk.data["l0"][2])


def test_index_files_are_written(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    store.save_bulk([GradientRecord(0, _ids("a", 2), _block(2, 5))])
    store.close()
    files = {p.name for p in (tmp_path / "s").rglob("*") if p.is_file()}
    assert any(n.endswith(".jsonl") for n in files), files
    metas = list((tmp_path / "s").rglob("index_meta.json"))
    assert metas and json.loads(metas[0].read_text()).get("format") is not None


def test_async_writer_matches_sync(tmp_path):
    sync = GradientStorageManager(str(tmp_path / "sync"))
    asyn = GradientStorageManager(str(tmp_path / "async"))
    writer = AsyncGradientWriter(asyn, max_pending=2)
    for step in range(5):
        rec = GradientRecord(step, _ids(f"s{step}_", 3), _block(3, 10 + step))
        sync.save_bulk([rec])
        writer.submit([rec])
    writer.close()
    for step in range(5):
        a = [r for f, by in sync.iter_steps(step) for r in (sync.load_records(f)[i] for i in by[step])]
        b = [r for f, by in asyn.iter_steps(step) for r in (asyn.load_records(f)[i] for i in by[step])]
        assert len(a) == len(b) == 1
        _same(a[0].gradient, b[0].gradient)


def test_rejects_unknown_options(tmp_path):
    with pytest.raises(ValueError):
        GradientStorageManager(str(tmp_path / "s"), residency="gpu")
    with pytest.raises(ValueError):
        GradientStorageManager(str(tmp_path / "s"), disk_format="hdf5")


def test_memmap_metadata_reads_back_through_torch_load_and_refuses_globals(tmp_path):
    """The metadata is written by the C pickler into torch's zip archive: ``torch.load`` reads
    it as written, and the fast reader refuses anything that is not plain data (a file holding
    a tensor falls back to ``torch.load(weights_only=True)``)."""
    import pickle

    from dattri_llm_b200.gradient import storage_manager as sm

    meta = {"format": 2, "records": [{"step": 3, "input_hash": ["h"], "sample_id_key": None,
                                      "layers": {"l": {"kind": "dense", "parts": {"data": {
                                          "byte_off": 0, "nbytes": 8, "shape": [1, 2], "dtype": "float32"}}}}}]}
    path = tmp_path / "g.mmap.meta"
    torch.save(meta, path, pickle_module=sm._PlainPickle)
    assert torch.load(path, weights_only=True) == meta
    assert sm._load_meta(path) == meta
    other = tmp_path / "t.meta"
    torch.save({"t": torch.arange(3)}, other)
    assert torch.equal(sm._load_meta(other)["t"], torch.arange(3))

    class Evil:
        def __reduce__(self):
            return (print, ("executed",))

    bad = tmp_path / "bad.meta"
    torch.save({"x": 1}, bad)
    import zipfile

    with zipfile.ZipFile(bad) as zf:
        names = zf.namelist()
    member = next(n for n in names if n.endswith("/data.pkl"))
    with pytest.raises(pickle.UnpicklingError):
        sm._NoGlobals(__import__("io").BytesIO(pickle.dumps(Evil()))).load()
    assert member.endswith("data.pkl")
