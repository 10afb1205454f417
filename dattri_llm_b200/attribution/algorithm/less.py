"""LESS: a query's gradient against each training sample's optimizer update direction.

The training side is captured optimizer-preconditioned (``HookManager(optimizer=...)``):
every sample's projected gradient goes through the Adam rule ``m_hat / (sqrt(v_hat) + eps)``
(one fused kernel per layer on sm_100).  Each training row is scaled to unit norm and then
weighted -- by the learning rate applied at its step in the trajectory form
(``enable_update=True``), or by a per-checkpoint weight in the frozen form (one optimizer
state per checkpoint).  Query rows are unit-normalised raw gradients.  The score is the
weighted cosine, summed over steps or checkpoints.  Public API and score metadata keys as
in the reference's ``dattri_llm/attribution/algorithm/less.py``.
"""

from __future__ import annotations

from collections.abc import Iterator, Mapping, Sequence
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.base import BaseInnerProductAttributor
from dattri_llm_b200.attribution.utils import read_lr_schedule, write_lr_schedule
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.streaming import GradientStreamer


def _normalised(block, target_norm: float):
    """*block* with every layer dense fp32 and each sample's whole-model row (all layers
    together) rescaled to length *target_norm*."""
    flat = {}
    for name, value in block.data.items():
        dense = value if isinstance(value, torch.Tensor) else ops.materialize(value, block.layer_types[name])
        flat[name] = dense.reshape(dense.shape[0], -1).float()
    sq = torch.stack([(x * x).sum(dim=1) for x in flat.values()]).sum(dim=0)
    scale = target_norm * sq.clamp_min(1e-16).rsqrt()
    return block.map_layers(lambda name, _v, _lt: flat[name] * scale[:, None])


class _StepWeights:
    """The weight of a training step's rows: one constant, a ``{step: weight}`` table, or
    (``None``) the learning rates the source recorded for the trajectory."""

    def __init__(self, spec: float | dict[int, float] | None) -> None:
        self.spec = spec

    def __call__(self, step: int, source) -> float:
        if self.spec is None:
            lrs = getattr(source, "learning_rates", None)
            if not lrs or step not in lrs:
                raise ValueError(f"step {step} has no recorded learning rate, which weights its rows in "
                                 "the trajectory form.")
            return float(lrs[step])
        if isinstance(self.spec, dict):
            if step not in self.spec:
                raise ValueError(f"step {step} has no weight (weighted steps: {sorted(self.spec)}).")
            return self.spec[step]
        return float(self.spec)


class _NormalisedSource:
    """Yields *source*'s blocks on *device*, normalised and weighted per step."""

    def __init__(self, source, device, weights: _StepWeights) -> None:
        self.source, self.device, self.weights = source, device, weights

    @property
    def reusable(self) -> bool:
        return bool(getattr(self.source, "reusable", False))

    def __iter__(self) -> Iterator:
        for step, block, hashes in self.source:
            yield step, _normalised(block.to(self.device), self.weights(step, self.source)), hashes


class LESSAttributor(BaseInnerProductAttributor):
    """LESS attributor.

    Args:
        args / task: as for every attributor.
        optimizers: frozen form only: one optimizer per checkpoint, holding its state there.
        checkpoint_weights: frozen form only: one weight per checkpoint (e.g. its learning rate).
    """

    algorithm: ClassVar[str] = "LESS"

    def __init__(self, args, *, task=None, optimizers: Sequence[torch.optim.Optimizer] | None = None,
                 checkpoint_weights: Sequence[float] | None = None) -> None:
        super().__init__(args, task=task)
        self.optimizers = list(optimizers or ())
        self.checkpoint_weights = [float(w) for w in checkpoint_weights or ()]
        if self.checkpoint_weights and len(self.checkpoint_weights) != len(self.optimizers):
            raise ValueError(f"{len(self.checkpoint_weights)} checkpoint weights for {len(self.optimizers)} "
                             "optimizers: give one weight per optimizer.")
        self.trajectory_form = False
        self.step_weights = _StepWeights(1.0)

    def uses_plain_inner_product(self) -> bool:
        """Normalisation and weights are applied to the rows, so the score is a plain dot."""
        return True

    def checkpoints(self) -> list[int]:
        """Checkpoint 0 in the trajectory form, else one index per optimizer.

        Raises:
            ValueError: the frozen form's optimizers do not match the task's checkpoints.
        """
        if self.trajectory_form:
            return [0]
        count = self.num_checkpoints()
        if len(self.optimizers) != count:
            raise ValueError(f"the task has {count} checkpoint(s); LESS without enable_update needs that many "
                             f"optimizers, got {len(self.optimizers)}.")
        return list(range(count))

    def generate_train_rep(self, train_dataset, *, checkpoint_step: int = 0, enable_update: bool = False,
                           hook_config=None, **_kw) -> GradientStreamer:
        """A streamer that captures preconditioned training gradients (with the trajectory's
        own optimizer, or the checkpoint's)."""
        task = self.require_task("attribute")
        optimizer = None if enable_update else self.optimizers[checkpoint_step]
        return GradientStreamer(task.model, train_dataset, self.args,
                                batch_size=self.args.per_device_train_batch_size, enable_update=enable_update,
                                loss_fn=self.train_loss_fn(), checkpoint_step=checkpoint_step, config=hook_config,
                                optimizer=optimizer, precondition=True, forward_model=task.forward_model)

    def collect_gradients(self, streamer, store, **kwargs):
        """Collect into *store*; a trajectory's learning rates are written beside it."""
        result = super().collect_gradients(streamer, store, **kwargs)
        if getattr(streamer, "enable_update", False):
            write_lr_schedule(str(store.save_dir), streamer.learning_rates)
        return result

    def cache(self, train_dataset, test_dataset, *, enable_update: bool = False, **kwargs):
        """Collect train / test stores (the trajectory form with ``enable_update``)."""
        self.trajectory_form = enable_update
        return super().cache(train_dataset, test_dataset, enable_update=enable_update, **kwargs)

    def transform_test_rep(self, test_rep):
        """Query rows at unit norm."""
        return _normalised(test_rep, 1.0)

    def score_sources(self, train_source, test_source, *, loop_over_test: bool = False, transform_test=None,
                      attribution_granularity: str = "instance"):
        """Score with the training rows normalised and weighted by their step."""
        weighted = _NormalisedSource(train_source, self.args.device, self.step_weights)
        return super().score_sources(weighted, test_source, loop_over_test=loop_over_test,
                                     transform_test=transform_test, attribution_granularity=attribution_granularity)

    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, enable_update: bool = False, gradient_cache_residency=None,
                  attribution_granularity: str = "instance"):
        """Live LESS: the trajectory form (``enable_update``) weighs steps by their learning
        rates; the frozen form uses one optimizer, and weight, per checkpoint."""
        self.trajectory_form = enable_update
        if enable_update:
            self.step_weights = _StepWeights(None)
        else:
            self.step_weights = _StepWeights(dict(enumerate(self.checkpoint_weights)) if self.checkpoint_weights
                                             else 1.0)
        return super().attribute(train_dataset, test_dataset, hook_config=hook_config, verbose=verbose,
                                 loop_over_test=loop_over_test, enable_update=enable_update,
                                 gradient_cache_residency=gradient_cache_residency,
                                 attribution_granularity=attribution_granularity)

    def attribute_from_cache(self, train_source, test_source, *, checkpoint_weight: float | None = None,
                             learning_rates: float | Mapping[int, float] | None = None, algorithm_meta=None,
                             **kwargs):
        """LESS over stored gradients.  Step weights, by precedence: *learning_rates* (one
        value or ``{step: lr}``), *checkpoint_weight*, the schedule recorded beside the train
        store, else the weights already set (1 by default)."""
        store = self.resolve_store(train_source)
        recorded_meta: dict = {}
        if learning_rates is not None:
            spec = ({int(s): float(lr) for s, lr in learning_rates.items()} if isinstance(learning_rates, Mapping)
                    else float(learning_rates))
            self.step_weights = _StepWeights(spec)
            recorded_meta["learning_rates"] = learning_rates
        elif checkpoint_weight is not None:
            self.step_weights = _StepWeights(float(checkpoint_weight))
            recorded_meta["checkpoint_weight"] = checkpoint_weight
        else:
            schedule = read_lr_schedule(str(store.save_dir))
            if schedule is not None:
                self.step_weights = _StepWeights(schedule)
            elif self.step_weights.spec is None:
                self.step_weights = _StepWeights(1.0)
        merged = {**recorded_meta, **(algorithm_meta or {})}
        return super().attribute_from_cache(store, test_source, algorithm_meta=merged, **kwargs)
