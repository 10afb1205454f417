"""Trajectory snapshots and store readers on CPU:

* ``TrajectorySnapshots`` round-trips trainable parameters (frozen ones are not stored,
  ``same_as`` references resolve through chains), batches and optimizer dynamics, lists
  only steps with both parameters and a batch, and names the missing step or parameter;
* ``iter_gradient_blocks`` yields every stored block of the requested steps exactly once,
  with and without loader workers and with a layer filter; ``resolve_steps`` keeps the
  stored subset and refuses an empty one.
"""

from __future__ import annotations

import tempfile

import pytest
import torch
from torch import nn

import dattri_llm_b200 as bw
from dattri_llm_b200.gradient.datasets import iter_gradient_blocks, resolve_steps
from dattri_llm_b200.gradient.gradient import Gradient, GradientRecord
from dattri_llm_b200.gradient.snapshots import LazyDynamics, TrajectorySnapshots
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager


def _model(seed):
    torch.manual_seed(seed)
    m = nn.Sequential(nn.Linear(3, 4), nn.Linear(4, 2))
    m[1].bias.requires_grad_(False)
    return m


def test_parameter_batch_and_dynamics_roundtrip(tmp_path):
    snaps = TrajectorySnapshots(tmp_path / "traj")
    assert TrajectorySnapshots.is_snapshot_dir(tmp_path / "traj")
    a = _model(0)
    snaps.save_parameters(0, a)
    snaps.save_parameters(1, a, same_as=0)
    snaps.save_parameters(2, a, same_as=1)  # a chain of references
    for s in range(3):
        snaps.save_batch(s, {"x": torch.full((2, 3), float(s))})
    snaps.save_parameters(3, _model(1))  # no batch: not a complete step
    assert snaps.steps() == [0, 1, 2]
    b = _model(5)
    frozen_before = b[1].bias.detach().clone()
    snaps.load_parameters(2, b)
    torch.testing.assert_close(b[0].weight, a[0].weight)
    torch.testing.assert_close(b[1].bias, frozen_before)  # frozen parameters are not part of a snapshot
    torch.testing.assert_close(snaps.load_batch(1)["x"], torch.full((2, 3), 1.0))
    with pytest.raises(KeyError):
        snaps.load_parameters(7, b)
    with pytest.raises(KeyError):
        snaps.load_batch(3)
    snaps.save_dynamics(0, "pre", {"m": torch.ones(2)})
    snaps.save_dynamics(0, "post", {"m": torch.zeros(2)})
    snaps.save_dynamics(1, "pre", {"m": torch.ones(2)})  # no post: incomplete
    with pytest.raises(ValueError):
        snaps.save_dynamics(0, "mid", {})
    assert snaps.dynamics_steps() == [0]
    lazy = LazyDynamics(snaps, lambda pre, post: pre["m"] - post["m"])
    assert list(lazy) == [0] and 0 in lazy and 1 not in lazy
    torch.testing.assert_close(lazy[0], torch.ones(2))


def test_missing_parameter_is_named(tmp_path):
    snaps = TrajectorySnapshots(tmp_path / "t")
    snaps.save_parameters(0, nn.Linear(3, 2))
    snaps.save_batch(0, {})
    bigger = nn.Sequential(nn.Linear(3, 2), nn.Linear(2, 2))
    with pytest.raises(KeyError, match="0.weight"):
        snaps.load_parameters(0, bigger)


def _store(tmp_path, steps=(0, 1, 2), per_file=2):
    store = GradientStorageManager(str(tmp_path / "s"))
    for s in steps:
        for f in range(per_file):
            g = torch.Generator().manual_seed(10 * s + f)
            grad = Gradient({"a": "materialized", "b": "materialized"},
                            {"a": torch.randn(2, 3, generator=g), "b": torch.randn(2, 5, generator=g)},
                            {"a": "nn.Linear", "b": "nn.Linear"}, {"a": "batch", "b": "batch"})
            store.save_bulk([GradientRecord(s, [f"{s}-{f}-{i}" for i in range(2)], grad)])
    store.close()
    return GradientStorageManager(str(tmp_path / "s"))


@pytest.mark.parametrize("workers", [0, 2])
def test_iter_blocks_yields_each_stored_block_once(tmp_path, workers):
    store = _store(tmp_path)
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), dataloader_num_workers=workers)
    seen = []
    for step, block, hashes in iter_gradient_blocks(store, [0, 2], args, layer_name=["b"]):
        assert set(block.data) == {"b"}
        assert block.batch_size == len(hashes) == 2
        seen.extend((step, h) for h in hashes)
    assert sorted(seen) == sorted((s, f"{s}-{f}-{i}") for s in (0, 2) for f in range(2) for i in range(2))
    store.close()


def test_resolve_steps(tmp_path):
    store = _store(tmp_path)
    assert resolve_steps(store, None) == [0, 1, 2]
    assert resolve_steps(store, [2, 9, 0]) == [0, 2]
    with pytest.raises(ValueError, match="available steps"):
        resolve_steps(store, [5, 6])
    store.close()
