"""Common ground of the attributors that sweep a training trajectory (DVEmb, AdamW-influence).

Such a method first RUNS the trajectory: it trains the model from checkpoint 0 with
``enable_update=True`` and keeps, for every step, either the per-sample gradients (a
gradient store) or -- with ``args.recompute_gradients`` -- the parameters and batch that
regenerate them (a :class:`TrajectorySnapshots` directory, replayed later through
:class:`ReplayGradientSource`), together with the learning rate applied at each step.  The
query gradients are taken at the final parameters.  It then SWEEPS the stored steps from
last to first, propagating either a parameter-space operator (train side) or the query
matrix (test side).

This base class provides the run, the opening of stored sources, the step selection and the
query matrix; subclasses provide the sweep.  Directory names and the learning-rate file are
the reference's (``dattri_llm/attribution/algorithm/trajectory.py``) so that caches are
interchangeable.
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
from dattri_llm_b200.gradient.streaming import DiskGradientSource, ReplayGradientSource  # noqa: F401

TRAIN_GRADS_DIR = "train_grads"
TRAIN_SNAPSHOTS_DIR = "train_snapshots"
TEST_GRADS_DIR = "test_grads"
PROPAGATIONS = ("train", "test")


def dense_block(block, dtype: torch.dtype = torch.float32):
    """*block* with every layer materialized dense in *dtype* (the sweeps' operand form)."""
    return block.map_layers(lambda _n, v, t: ops.materialize(v, t).to(dtype))


def _first_seen_columns(hash_lists: Iterable[list[str]]) -> tuple[list[str], dict[str, int]]:
    """Identities in first-seen order and their column index."""
    order: list[str] = []
    column: dict[str, int] = {}
    for hashes in hash_lists:
        for h in hashes:
            if h not in column:
                column[h] = len(order)
                order.append(h)
    return order, column


class TrajectoryAttributor(BaseInnerProductAttributor):
    """Base of the trajectory-sweeping attributors (see the module docstring)."""

    algorithm: ClassVar[str] = "Trajectory"

    def __init__(self, args, *, task=None) -> None:
        super().__init__(args, task=task)
        self.trajectory_hook_config = None  # the capture config of the last run, reused by replays

    @property
    def recompute(self) -> bool:
        """Whether runs keep snapshots (regenerating gradients on demand) instead of gradients."""
        return bool(getattr(self.args, "recompute_gradients", False))

    def checkpoints(self) -> list[int]:
        """Always ``[0]``: the trajectory starts from the first checkpoint; others are ignored."""
        extra = self.num_checkpoints() - 1
        if extra > 0:
            warnings.warn(f"{self.algorithm} runs its trajectory from checkpoint 0 and ignores the other {extra}.",
                          stacklevel=2)
        return [0]

    # ------------------------------------------------------------------ running the trajectory
    def cache(self, train_dataset, test_dataset, *, cache_dir: str | None = None, hook_config=None,
              offload_interval: int = 1) -> list[tuple[str, str]]:
        """Run the trajectory into ``<cache_dir>/train_grads`` (``train_snapshots`` when
        recomputing) and ``<cache_dir>/test_grads``; the learning rates go beside the train
        side.  Returns ``[(train_dir, test_dir)]``."""
        self.require_task("cache")
        root = pathlib.Path(self.args.output_dir if cache_dir is None else cache_dir)
        train_dir = root / (TRAIN_SNAPSHOTS_DIR if self.recompute else TRAIN_GRADS_DIR)
        test_dir = root / TEST_GRADS_DIR
        train_target = TrajectorySnapshots(train_dir) if self.recompute else GradientStorageManager(str(train_dir))
        lrs = self.collect_trajectory(train_target, GradientStorageManager(str(test_dir)), train_dataset,
                                      test_dataset, hook_config=hook_config, offload_interval=offload_interval)
        write_lr_schedule(str(train_dir), lrs)
        return [(str(train_dir), str(test_dir))]

    def collect_trajectory(self, train_target, test_store, train_dataset, test_dataset, *, hook_config=None,
                           offload_interval: int = 1) -> dict[int, float]:
        """Train from checkpoint 0 while collecting the training side into *train_target* (a
        store or a snapshot directory), then the queries at the final parameters into
        *test_store*.  Returns ``{step: learning rate}``."""
        self.checkpoints()
        model = self.load_checkpoint(0)
        self.trajectory_hook_config = hook_config
        snapshots = train_target if isinstance(train_target, TrajectorySnapshots) else None
        streamer = self.generate_train_rep(train_dataset, enable_update=True, hook_config=hook_config,
                                           snapshots=snapshots)
        for callback in self.trajectory_callbacks(model, streamer, snapshots):
            streamer.hook_manager.add_callback(callback)
        per_block = self.on_trajectory_block()
        if snapshots is None:
            self.collect_gradients(streamer, train_target, offload_interval=offload_interval, on_block=per_block)
        else:  # the streamer writes the snapshots itself; just drive it
            with streamer:
                for step, block, hashes in streamer:
                    if per_block is not None:
                        per_block(step, block, hashes)
        queries = self.generate_test_rep(test_dataset, hook_config=hook_config)
        self.collect_gradients(queries, test_store, offload_interval=offload_interval)
        self.finish_trajectory(train_target)
        # the run trained the parameters in place: checkpoint 0 must be reloaded next time
        self.require_task("collect_trajectory").invalidate_checkpoint()
        return streamer.learning_rates

    def trajectory_callbacks(self, model, streamer, snapshots) -> list:
        """Extra capture callbacks for the run (none here)."""
        return []

    def on_trajectory_block(self):
        """A ``(step, block, hashes)`` hook called on every training block of the run (none here)."""
        return None

    def finish_trajectory(self, train_target) -> None:
        """Called once the run is stored (nothing here)."""

    # ------------------------------------------------------------------ stored sources
    def open_train_source(self, train_source, *, steps: Iterable[int] | None = None, layer_name=None,
                          hook_config=None, verbose: bool = False):
        """A training source over a gradient store, a snapshot directory (replayed), or an
        existing replay source (restricted to *steps*)."""
        layers = normalize_layer_names(layer_name)
        if isinstance(train_source, ReplayGradientSource):
            return train_source.for_steps(steps) if steps is not None else train_source
        replay = isinstance(train_source, TrajectorySnapshots) or TrajectorySnapshots.is_snapshot_dir(train_source)
        if not replay:
            return self.load_train_rep(self.resolve_store(train_source), steps=steps, layer_name=layers,
                                       verbose=verbose)
        task = self.require_task("attribute_from_cache (replaying snapshots)")
        snapshots = train_source if isinstance(train_source, TrajectorySnapshots) else TrajectorySnapshots(train_source)
        config = hook_config if hook_config is not None else self.trajectory_hook_config
        return ReplayGradientSource(task.get_model(), self.args, snapshots, loss_fn=self.train_loss_fn(), config=config,
                                    steps=steps, layer_name=layers, desc=f"{self.algorithm}: replay", verbose=verbose)

    @staticmethod
    def train_dir_of(train_source) -> str:
        """The directory a training source reads."""
        if isinstance(train_source, ReplayGradientSource):
            return str(train_source.snapshots.root)
        return str(train_source.file_manager.save_dir)

    @staticmethod
    def available_steps(train_source) -> list[int]:
        """The steps a training source can provide, ascending."""
        if isinstance(train_source, ReplayGradientSource):
            return sorted(train_source.snapshots.steps())
        return sorted(train_source.file_manager.available_steps())

    def recorded_lr_of(self, train_source) -> dict[int, float] | None:
        """The learning rates recorded beside a training source, if any."""
        return read_lr_schedule(self.train_dir_of(train_source))

    @staticmethod
    def close_source(source) -> None:
        """Give back the model state a replay source borrowed (other sources need nothing)."""
        if isinstance(source, ReplayGradientSource):
            source.close()

    def source_meta(self, train_source, test_store) -> dict:
        """Where the scores' inputs came from (recorded in the score metadata)."""
        if not isinstance(train_source, ReplayGradientSource):
            return {"train_source": "gradients", **self.stores_meta(train_source.file_manager, test_store)}
        return {"train_source": "snapshots", "train_dir": self.train_dir_of(train_source),
                "sample_id_key": {"train": None, "test": test_store.sample_id_key}}

    # ------------------------------------------------------------------ sweep setup
    @staticmethod
    def validate_propagation(propagation: str, loop_over_test: bool) -> None:
        """Check the propagated side.

        Raises:
            ValueError: an unknown side, or ``loop_over_test`` with the train-side sweep (which
                does not depend on the queries, so there is nothing to split).
        """
        if propagation not in PROPAGATIONS:
            raise ValueError(f"unknown propagation {propagation!r}; choose from {PROPAGATIONS}.")
        if loop_over_test and propagation == "train":
            raise ValueError("loop_over_test splits the queries, which only the test-side sweep "
                             "(propagation='test') carries; the train-side sweep is query-independent.")

    @staticmethod
    def resolve_steps(available: list[int], selected_training_steps, final_step):
        """``(steps to sweep, steps to report, final_step)``: the sweep covers every stored
        step before *final_step* (default: after the last stored step); the report covers the
        selected ones among them (default: all).

        Raises:
            ValueError: nothing to sweep, or no selected step among the swept ones.
        """
        end = final_step if final_step is not None else (max(available) + 1 if available else 0)
        swept = [s for s in available if s < end]
        if not swept:
            raise ValueError(f"no stored step lies before final_step={end} (stored: {available}).")
        if selected_training_steps is None:
            return swept, set(swept), end
        reported = set(swept).intersection(int(s) for s in selected_training_steps)
        if not reported:
            raise ValueError(f"none of selected_training_steps is among the swept steps ({swept[:10]} ...).")
        return swept, reported, end

    def steps_bar(self, prop_steps: list[int], desc: str, verbose: bool) -> Iterable:
        """*prop_steps* from last to first (with a progress bar when *verbose* on the logging rank)."""
        backwards = sorted(prop_steps, reverse=True)
        if verbose and self.args.should_log:
            from tqdm.auto import tqdm

            return tqdm(backwards, desc=desc, unit="step", leave=False)
        return backwards

    def collect_test_matrix(self, test_source) -> tuple[dict[str, torch.Tensor], list[str]]:
        """The stored queries as dense fp32 matrices ``{layer: (n_test, d)}`` on the device,
        rows in first-seen identity order (a repeated identity keeps its last rows), with the
        identities."""
        device = self.args.device
        blocks = []
        for _step, grad, hashes in test_source:
            dense = dense_block(grad.to(device))
            blocks.append((dense, list(hashes)))
        ids, column = _first_seen_columns(h for _d, h in blocks)
        if not blocks:
            return {}, ids
        layers = list(blocks[0][0].data)
        out = {name: torch.zeros(len(ids), blocks[0][0].data[name].shape[1], device=device) for name in layers}
        for dense, hashes in blocks:
            rows = torch.tensor([column[h] for h in hashes], device=device)
            for name in layers:
                out[name].index_copy_(0, rows, dense.data[name])
        return out, ids

    @staticmethod
    def test_column_order(test_source) -> tuple[list[str], dict[str, int]]:
        """Query identities in first-seen order and their column index."""
        return _first_seen_columns(hashes for _s, _g, hashes in test_source)
