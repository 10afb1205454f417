"""Persistence callbacks on CPU:

* ``OffloadCallback`` stages ``offload_interval`` distinct steps per flush; under gradient
  accumulation it merges each window's backwards into one record (the update step), a
  ragged last window included; ``per_sample`` recording stores one record per sample;
* the stored records equal the captured ones, whether written synchronously or through
  ``AsyncGradientWriter``;
* a write error in the background thread is re-raised by the next ``submit`` / ``flush`` /
  ``close`` instead of being lost.
"""

from __future__ import annotations

import pytest
import torch

from dattri_llm_b200.gradient.async_writer import AsyncGradientWriter
from dattri_llm_b200.gradient.callbacks import OffloadCallback
from dattri_llm_b200.gradient.gradient import Gradient, GradientRecord
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager


def _rec(step, n=2, seed=0):
    g = torch.Generator().manual_seed(seed * 100 + step)
    grad = Gradient({"w": "materialized"}, {"w": torch.randn(n, 4, generator=g)}, {"w": "nn.Linear"}, {"w": "batch"})
    return GradientRecord(step, [f"s{step}_{i}_{seed}" for i in range(n)], grad)


def _stored(store, step):
    out = []
    for f, by in store.iter_steps(step):
        recs = store.load_records(f)
        out.extend(recs[i] for i in by[step])
    return out


@pytest.mark.parametrize("async_write", [False, True])
def test_interval_flushes_and_contents(tmp_path, async_write):
    store = GradientStorageManager(str(tmp_path / "s"))
    cb = OffloadCallback(offload_interval=2, file_manager=store, async_write=async_write)
    recs = [_rec(s) for s in range(5)]
    for r in recs[:2]:
        cb.on_step_end(r)
    assert len(cb.staged) == 2  # interval not exceeded yet
    cb.on_step_end(recs[2])  # a third distinct step flushes the first two
    assert [r.step for r in cb.staged] == [2]
    for r in recs[3:]:
        cb.on_step_end(r)
    cb.on_context_end()
    store.close()
    reader = GradientStorageManager(str(tmp_path / "s"))
    assert reader.available_steps() == [0, 1, 2, 3, 4]
    for r in recs:
        (got,) = _stored(reader, r.step)
        assert list(got.input_hash) == list(r.input_hash)
        torch.testing.assert_close(got.gradient.data["w"], r.gradient.data["w"])
    reader.close()


def test_accumulation_windows_merge_into_update_steps(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    cb = OffloadCallback(offload_interval=10, file_manager=store, gradient_accumulation_steps=3)
    recs = [_rec(s, seed=1) for s in range(7)]  # windows: 0-2, 3-5, ragged 6
    for r in recs:
        cb.on_step_end(r)
    cb.on_context_end()
    store.close()
    reader = GradientStorageManager(str(tmp_path / "s"))
    assert reader.gradient_accumulation_steps == 3  # the step convention is part of the store
    assert reader.available_steps() == [0, 1, 2]
    for update, window in enumerate([recs[0:3], recs[3:6], recs[6:7]]):
        (got,) = _stored(reader, update)
        want = torch.cat([r.gradient.data["w"] for r in window])
        torch.testing.assert_close(got.gradient.data["w"], want)
        assert list(got.input_hash) == [h for r in window for h in r.input_hash]
    reader.close()


def test_per_sample_recording_stores_one_record_per_sample(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    cb = OffloadCallback(offload_interval=1, file_manager=store, recording_type="per_sample")
    r = _rec(0, n=3, seed=2)
    cb.on_step_end(r)
    cb.on_context_end()
    store.close()
    reader = GradientStorageManager(str(tmp_path / "s"))
    got = _stored(reader, 0)
    assert len(got) == 3
    for i, rec in enumerate(sorted(got, key=lambda x: x.input_hash)):
        assert rec.input_hash == r.input_hash[i]
        torch.testing.assert_close(rec.gradient.data["w"], r.gradient.data["w"][i : i + 1])
    reader.close()


def test_bad_options_are_rejected(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    with pytest.raises(ValueError):
        OffloadCallback(offload_interval=1, file_manager=store, recording_type="per_token")
    with pytest.raises(ValueError):
        OffloadCallback(offload_interval=1, file_manager=store, gradient_accumulation_steps=0)
    with pytest.raises(ValueError):
        AsyncGradientWriter(store, max_pending=0)
    store.close()


class _FailingStore:
    """A store whose writes fail (a full disk, say)."""

    def save_bulk(self, records):
        raise OSError("no space left on device")


def test_background_write_error_is_reraised():
    writer = AsyncGradientWriter(_FailingStore(), max_pending=1)
    writer.submit([_rec(0)])
    with pytest.raises(RuntimeError, match="asynchronous gradient write failed") as info:
        writer.flush()
    assert isinstance(info.value.__cause__, OSError)
    with pytest.raises(RuntimeError):
        writer.close()


def test_reopened_store_refuses_another_step_convention(tmp_path):
    store = GradientStorageManager(str(tmp_path / "s"))
    cb = OffloadCallback(offload_interval=1, file_manager=store, gradient_accumulation_steps=2)
    for s in range(2):
        cb.on_step_end(_rec(s))
    cb.on_context_end()
    store.close()
    reopened = GradientStorageManager(str(tmp_path / "s"))
    with pytest.raises(ValueError, match="gradient_accumulation_steps"):
        OffloadCallback(offload_interval=1, file_manager=reopened, gradient_accumulation_steps=1)
    reopened.close()
