"""Shared machinery of the trajectory-sweeping attributors (DVEmb, AdamW-influence).

A trajectory method trains the model from checkpoint 0 (``enable_update=True``),
storing each step's per-sample gradients (or, with ``args.recompute_gradients``,
each step's parameters and batch as :class:`TrajectorySnapshots`, replayed later
by :class:`ReplayGradientSource`) plus the learning-rate schedule, then sweeps the
steps backwards propagating either the train side (a parameter-space operator) or
the test side (the query matrix).  Parity: reference
``dattri_llm/attribution/algorithm/trajectory.py:85-452``.
"""

from __future__ import annotations

import pathlib
import warnings
from collections.abc import Iterable
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.base import BaseInnerProductAttributor
from dattri_llm_b200.attribution.utils import normalize_layer_names, read_lr_schedule, write_lr_schedule
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.snapshots import TrajectorySnapshots
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.gradient.streaming import DiskGradientSource, ReplayGradientSource

TRAIN_GRADS_DIR = "train_grads"
TRAIN_SNAPSHOTS_DIR = "train_snapshots"
TEST_GRADS_DIR = "test_grads"
PROPAGATIONS = ("train", "test")


def _dense_float(block, dtype: torch.dtype = torch.float32):
    return block.map_layers(lambda _n, v, t: ops.materialize(v, t).to(dtype))


class TrajectoryAttributor(BaseInnerProductAttributor):
    """Base class of the trajectory-sweeping attributors."""

    algorithm: ClassVar[str] = "Trajectory"

    def __init__(self, args, *, task=None) -> None:
        super().__init__(args, task=task)
        self._hook_config = None

    @property
    def recompute(self) -> bool:
        """Store snapshots and recompute gradients instead of storing them."""
        return bool(getattr(self.args, "recompute_gradients", False))

    def checkpoints(self) -> list[int]:
        """Checkpoint 0 only (the trajectory is regenerated from it)."""
        n = self.num_checkpoints()
        if n > 1:
            warnings.warn(f"{self.algorithm} regenerates the trajectory from checkpoint 0; the other {n - 1} "
                          "checkpoint(s) are ignored.", stacklevel=2)
        return [0]

    def cache(self, train_dataset, test_dataset, *, cache_dir: str | None = None, hook_config=None,
              offload_interval: int = 1) -> list[tuple[str, str]]:
        """Run the trajectory into ``<cache_dir>/train_grads`` (or ``train_snapshots``) and
        ``test_grads``, with the learning-rate schedule beside the train side."""
        self.require_task("cache")
        root = pathlib.Path(cache_dir if cache_dir is not None else self.args.output_dir)
        train_dir = str(root / (TRAIN_SNAPSHOTS_DIR if self.recompute else TRAIN_GRADS_DIR))
        test_dir = str(root / TEST_GRADS_DIR)
        lrs = self.collect_trajectory(TrajectorySnapshots(train_dir) if self.recompute
                                      else GradientStorageManager(train_dir), GradientStorageManager(test_dir),
                                      train_dataset, test_dataset, hook_config=hook_config,
                                      offload_interval=offload_interval)
        write_lr_schedule(train_dir, lrs)
        return [(train_dir, test_dir)]

    def collect_trajectory(self, train_target, test_store, train_dataset, test_dataset, *, hook_config=None,
                           offload_interval: int = 1) -> dict[int, float]:
        """Train from checkpoint 0 collecting the train side, then the queries at the
        final parameters; returns ``{step: lr}``."""
        self.checkpoints()
        model = self.load_checkpoint(0)
        self._hook_config = hook_config
        snaps = train_target if isinstance(train_target, TrajectorySnapshots) else None
        streamer = self.generate_train_rep(train_dataset, enable_update=True, hook_config=hook_config, snapshots=snaps)
        for cb in self.trajectory_callbacks(model, streamer, snaps):
            streamer.hook_manager.add_callback(cb)
        on_block = self.on_trajectory_block()
        if snaps is not None:
            with streamer:
                for step, block, hashes in streamer:
                    if on_block is not None:
                        on_block(step, block, hashes)
        else:
            self.collect_gradients(streamer, train_target, offload_interval=offload_interval, on_block=on_block)
        self.collect_gradients(self.generate_test_rep(test_dataset, hook_config=hook_config), test_store,
                               offload_interval=offload_interval)
        self.finish_trajectory(train_target)
        self.require_task("collect_trajectory").invalidate_checkpoint()
        return streamer.learning_rates

    def trajectory_callbacks(self, model, streamer, snapshots) -> list:
        """Callbacks to attach to the trajectory's manager (none by default)."""
        return []

    def on_trajectory_block(self):
        """Per-block hook during the trajectory (none by default)."""
        return None

    def finish_trajectory(self, train_target) -> None:
        """Work after the trajectory (none by default)."""

    def open_train_source(self, train_source, *, steps: Iterable[int] | None = None, layer_name=None,
                          hook_config=None, verbose: bool = False):
        """A train source from a store, a snapshot directory or an existing source."""
        layer_name = normalize_layer_names(layer_name)
        if isinstance(train_source, ReplayGradientSource):
            return train_source if steps is None else train_source.for_steps(steps)
        if isinstance(train_source, TrajectorySnapshots) or TrajectorySnapshots.is_snapshot_dir(train_source):
            task = self.require_task("attribute_from_cache (replaying snapshots)")
            snaps = train_source if isinstance(train_source, TrajectorySnapshots) else TrajectorySnapshots(train_source)
            return ReplayGradientSource(task.get_model(), self.args, snaps, loss_fn=self.train_loss_fn(),
                                        config=hook_config if hook_config is not None else self._hook_config,
                                        steps=steps, layer_name=layer_name, desc=f"{self.algorithm}: replay",
                                        verbose=verbose)
        return self.load_train_rep(self.resolve_store(train_source), steps=steps, layer_name=layer_name,
                                   verbose=verbose)

    @staticmethod
    def train_dir_of(train_source) -> str:
        """Directory of a train source."""
        if isinstance(train_source, ReplayGradientSource):
            return str(train_source.snapshots.root)
        return str(train_source.file_manager.save_dir)

    @staticmethod
    def available_steps(train_source) -> list[int]:
        """Steps a train source holds."""
        if isinstance(train_source, ReplayGradientSource):
            return sorted(train_source.snapshots.steps())
        return sorted(train_source.file_manager.available_steps())

    def recorded_lr_of(self, train_source) -> dict[int, float] | None:
        """The learning-rate schedule stored beside a train source."""
        return read_lr_schedule(self.train_dir_of(train_source))

    @staticmethod
    def close_source(source) -> None:
        """Release a replay source's model state."""
        if isinstance(source, ReplayGradientSource):
            source.close()

    def source_meta(self, train_source, test_store) -> dict:
        """Provenance of the sources."""
        if isinstance(train_source, ReplayGradientSource):
            return {"train_source": "snapshots", "train_dir": self.train_dir_of(train_source),
                    "sample_id_key": {"train": None, "test": test_store.sample_id_key}}
        return {"train_source": "gradients", **self.stores_meta(train_source.file_manager, test_store)}

    @staticmethod
    def validate_propagation(propagation: str, loop_over_test: bool) -> None:
        """Check a propagation side.

        Raises:
            ValueError: for an unknown side, or ``loop_over_test`` with train-side propagation.
        """
        if propagation not in PROPAGATIONS:
            raise ValueError(f"propagation must be one of {PROPAGATIONS}, got {propagation!r}.")
        if propagation == "train" and loop_over_test:
            raise ValueError("loop_over_test applies only to propagation='test': the train-side sweep is "
                             "test-independent, so there is nothing to block over.")

    @staticmethod
    def resolve_steps(available: list[int], selected_training_steps, final_step):
        """``(propagated steps, output steps, final_step)`` (steps below *final_step*).

        Raises:
            ValueError: when no step qualifies.
        """
        if final_step is None:
            final_step = (max(available) + 1) if available else 0
        prop = [s for s in available if s < final_step]
        if not prop:
            raise ValueError(f"No training step satisfies step < final_step ({final_step}); available steps: "
                             f"{available}.")
        if selected_training_steps is None:
            out = set(prop)
        else:
            out = {int(s) for s in selected_training_steps} & set(prop)
            if not out:
                raise ValueError(f"selected_training_steps matches none of the propagated steps {prop[:10]}...")
        return prop, out, final_step

    def steps_bar(self, prop_steps: list[int], desc: str, verbose: bool) -> Iterable:
        """Steps in backward order, with a progress bar when *verbose*."""
        steps = sorted(prop_steps, reverse=True)
        if not verbose or not self.args.should_log:
            return steps
        from tqdm.auto import tqdm

        return tqdm(steps, desc=desc, unit="step", leave=False)

    def collect_test_matrix(self, test_source) -> tuple[dict[str, torch.Tensor], list[str]]:
        """``({layer: (n_test, d) fp32}, test_ids)`` of a stored test set."""
        dev = self.args.device
        ids: list[str] = []
        index: dict[str, int] = {}
        pending = []
        for _s, tg, th in test_source:
            mat = _dense_float(tg.to(dev))
            cols = []
            for h in th:
                if h not in index:
                    index[h] = len(ids)
                    ids.append(h)
                cols.append(index[h])
            pending.append((mat, cols))
        layers = list(pending[0][0].data) if pending else []
        w = {n: torch.zeros(len(ids), pending[0][0].data[n].shape[1], device=dev) for n in layers}
        for mat, cols in pending:
            idx = torch.as_tensor(cols, device=dev)
            for n in layers:
                w[n].index_copy_(0, idx, mat.data[n])
        return w, ids

    @staticmethod
    def test_column_order(test_source) -> tuple[list[str], dict[str, int]]:
        """Test identities in first-seen order, with their column index."""
        ids: list[str] = []
        index: dict[str, int] = {}
        for _s, _g, hashes in test_source:
            for h in hashes:
                if h not in index:
                    index[h] = len(ids)
                    ids.append(h)
        return ids, index
