"""Gradient-store guard rails and multi-writer layout (CPU): one store never mixes sample
identifier schemes or step conventions, a memmap group of another format version is
refused with a clear message, a record whose hash count differs from its batch is refused,
and two ranks writing ``rank_N/`` directories are read back as one store."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dattri_llm_b200.gradient.gradient import Gradient, GradientRecord
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager


def _record(step: int, ids: list[str], *, key=None, seed: int = 0) -> GradientRecord:
    g = torch.Generator().manual_seed(seed)
    grad = Gradient({"w": "materialized"}, {"w": torch.randn(len(ids), 6, generator=g)}, {"w": "nn.Linear"},
                    {"w": "batch"})
    return GradientRecord(step=step, input_hash=list(ids), gradient=grad, sample_id_key=key)


def test_identifier_schemes_do_not_mix(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    store.save_bulk([_record(0, ["a", "b"])])
    with pytest.raises(ValueError, match="identifier"):
        store.save_bulk([_record(1, ["1", "2"], key="idx")])
    store.close()


def test_step_conventions_do_not_mix(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    store.declare_gradient_accumulation_steps(2)
    store.declare_gradient_accumulation_steps(2)
    with pytest.raises(ValueError):
        store.declare_gradient_accumulation_steps(3)
    with pytest.raises(ValueError):
        store.declare_gradient_accumulation_steps(0)
    store.close()


def test_hash_count_must_match_the_batch(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    rec = _record(0, ["a", "b", "c"])
    rec.input_hash = ["a", "b"]
    with pytest.raises(ValueError, match="batch size"):
        store.save_bulk([rec])
    store.close()


def test_other_memmap_format_version_is_refused(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    store.save_bulk([_record(0, ["a", "b"])])
    store.close()
    metas = list((tmp_path / "s").rglob("*.mmap.meta"))
    assert metas
    payload = torch.load(metas[0], weights_only=True)
    payload["format"] = 1
    torch.save(payload, metas[0])
    reopened = GradientStorageManager(str(tmp_path / "s"))
    ((f, _by),) = reopened.iter_steps(0)
    with pytest.raises(ValueError, match="format"):
        reopened.load_records(f)
    reopened.close()


def test_lookup_by_inputs_and_by_id_key(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    store.save_bulk([_record(3, ["10", "11"], key="idx", seed=1)])
    store.close()
    reopened = GradientStorageManager(str(tmp_path / "s"))
    assert reopened.sample_id_key == "idx"
    assert reopened.lookup({"idx": torch.tensor(11)}) == [(3, 1)]
    with pytest.raises(KeyError):
        reopened.lookup({"x": torch.zeros(2)})
    got = reopened.load_sample({"idx": 10}, 3, 0)
    want = _record(3, ["10", "11"], key="idx", seed=1).gradient.data["w"][0:1]
    torch.testing.assert_close(got.data["w"], want)
    reopened.close()


def _writer(rank, world, port, root):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        store = GradientStorageManager(root)
        for step in range(2):
            store.save_bulk([_record(step, [f"r{rank}s{step}i{i}" for i in range(2)], seed=10 * rank + step)])
        store.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_per_rank_directories_read_back_as_one_store(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    root = str(tmp_path / "shared")
    mp.spawn(_writer, args=(2, port, root), nprocs=2, join=True)
    assert (tmp_path / "shared" / "rank_0").is_dir() and (tmp_path / "shared" / "rank_1").is_dir()
    reader = GradientStorageManager(root)
    assert reader.available_steps() == [0, 1]
    for rank in range(2):
        for step in range(2):
            for i in range(2):
                h = f"r{rank}s{step}i{i}"
                assert reader.lookup_by_hash(h) == [(step, i)]
                got = reader.load_sample_by_hash(h, step, i).data["w"]
                want = _record(step, ["x", "y"], seed=10 * rank + step).gradient.data["w"][i : i + 1]
                torch.testing.assert_close(got, want)
    reader.close()
