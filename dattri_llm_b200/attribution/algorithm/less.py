"""LESS: cosine between a query's gradient and a sample's Adam update direction.

Train gradients are captured optimizer-preconditioned (``HookManager(optimizer=...)``:
the per-sample Adam direction ``m_hat / (sqrt(v_hat) + eps)``, one fused kernel per
layer on sm_100), each train row is normalised to unit norm and weighted by the
step's learning rate (trajectory form, ``enable_update=True``) or by a per-
checkpoint weight (frozen form, one optimizer state per checkpoint); test rows are
unit-normalised raw gradients; scores are summed over steps / checkpoints.
Parity: reference ``dattri_llm/attribution/algorithm/less.py``.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.base import BaseInnerProductAttributor
from dattri_llm_b200.attribution.utils import read_lr_schedule, write_lr_schedule
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.streaming import GradientStreamer


def _unit_rows(block, scale: float):
    """Every layer dense fp32, each sample's full-model row scaled to norm *scale*."""
    dense = {}
    for name, v in block.data.items():
        e = v if isinstance(v, torch.Tensor) else ops.materialize(v, block.layer_types[name])
        dense[name] = e.reshape(e.shape[0], -1).float()
    norm_sq = None
    for x in dense.values():
        n = (x * x).sum(dim=1)
        norm_sq = n if norm_sq is None else norm_sq + n
    factor = scale / norm_sq.clamp_min(1e-16).sqrt()
    return block.map_layers(lambda name, _v, _lt: dense[name] * factor[:, None])


class _WeightedSource:
    """A source whose blocks are unit-normalised and weighted by their step's weight."""

    def __init__(self, source, device, weight) -> None:
        self._source, self._device, self._weight = source, device, weight

    @property
    def reusable(self) -> bool:
        return getattr(self._source, "reusable", False)

    def __iter__(self):
        for step, block, hashes in self._source:
            yield step, _unit_rows(block.to(self._device), self._weight(step)), hashes


class LESSAttributor(BaseInnerProductAttributor):
    """LESS attributor.

    Args:
        args / task: As for every attributor.
        optimizers: Frozen form: one optimizer (its state at each checkpoint) per checkpoint.
        checkpoint_weights: Frozen form: a weight per checkpoint (e.g. its learning rate).
    """

    algorithm: ClassVar[str] = "LESS"

    def __init__(self, args, *, task=None, optimizers: Sequence[torch.optim.Optimizer] | None = None,
                 checkpoint_weights: Sequence[float] | None = None) -> None:
        super().__init__(args, task=task)
        self._optimizers = list(optimizers or [])
        self._weights = [float(w) for w in checkpoint_weights or []]
        if self._weights and len(self._weights) != len(self._optimizers):
            raise ValueError(f"checkpoint_weights must match optimizers one to one, got {len(self._weights)} "
                             f"weights for {len(self._optimizers)} optimizers.")
        self._enable_update = False
        self._step_weights: float | dict[int, float] | None = 1.0

    def uses_plain_inner_product(self) -> bool:
        """After the unit-row transforms the inner product is plain."""
        return True

    def checkpoints(self) -> list[int]:
        """Trajectory form: checkpoint 0; frozen form: one per optimizer.

        Raises:
            ValueError: when the frozen form lacks one optimizer per checkpoint.
        """
        if self._enable_update:
            return [0]
        n = self.num_checkpoints()
        if len(self._optimizers) != n:
            raise ValueError(f"LESS's frozen form needs one optimizer per checkpoint: the task has {n} "
                             f"checkpoint(s) but {len(self._optimizers)} optimizers were given.")
        return list(range(n))

    def generate_train_rep(self, train_dataset, *, checkpoint_step: int = 0, enable_update: bool = False,
                           hook_config=None, **_kw) -> GradientStreamer:
        """A preconditioning streamer (the trajectory's own optimizer, or the checkpoint's)."""
        task = self.require_task("attribute")
        return GradientStreamer(task.model, train_dataset, self.args, batch_size=self.args.per_device_train_batch_size,
                                enable_update=enable_update, loss_fn=self.train_loss_fn(),
                                checkpoint_step=checkpoint_step, config=hook_config,
                                optimizer=None if enable_update else self._optimizers[checkpoint_step],
                                precondition=True, forward_model=task.forward_model)

    def collect_gradients(self, streamer, store, **kwargs):
        """Collect, and store the trajectory's learning rates beside the store."""
        out = super().collect_gradients(streamer, store, **kwargs)
        if getattr(streamer, "enable_update", False):
            write_lr_schedule(str(store.save_dir), streamer.learning_rates)
        return out

    def cache(self, train_dataset, test_dataset, *, enable_update: bool = False, **kwargs):
        """Collect stores (trajectory form with ``enable_update``)."""
        self._enable_update = enable_update
        return super().cache(train_dataset, test_dataset, enable_update=enable_update, **kwargs)

    def transform_test_rep(self, test_rep):
        """Unit-normalised query rows."""
        return _unit_rows(test_rep, 1.0)

    def score_sources(self, train_source, test_source, *, loop_over_test: bool = False, transform_test=None,
                      attribution_granularity: str = "instance"):
        """Score with train rows unit-normalised and weighted per step."""
        weights = self._step_weights

        def weight(step: int) -> float:
            if weights is None:
                lrs = getattr(train_source, "learning_rates", None)
                if lrs is None or step not in lrs:
                    raise ValueError(f"no learning rate recorded for step {step}; the per-step form weights each "
                                     "step by the applied learning rate.")
                return float(lrs[step])
            if isinstance(weights, dict):
                if step not in weights:
                    raise ValueError(f"no weight for step {step}; provided steps: {sorted(weights)}.")
                return weights[step]
            return weights

        return super().score_sources(_WeightedSource(train_source, self.args.device, weight), test_source,
                                     loop_over_test=loop_over_test, transform_test=transform_test,
                                     attribution_granularity=attribution_granularity)

    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, enable_update: bool = False, gradient_cache_residency=None,
                  attribution_granularity: str = "instance"):
        """Live LESS (trajectory form with ``enable_update``; else one optimizer per checkpoint)."""
        self._enable_update = enable_update
        self._step_weights = None if enable_update else (dict(enumerate(self._weights)) if self._weights else 1.0)
        return super().attribute(train_dataset, test_dataset, hook_config=hook_config, verbose=verbose,
                                 loop_over_test=loop_over_test, enable_update=enable_update,
                                 gradient_cache_residency=gradient_cache_residency,
                                 attribution_granularity=attribution_granularity)

    def attribute_from_cache(self, train_source, test_source, *, checkpoint_weight: float | None = None,
                             learning_rates: float | Mapping[int, float] | None = None, algorithm_meta=None,
                             **kwargs):
        """LESS over stores; step weights from *learning_rates*, *checkpoint_weight*, or the
        schedule recorded beside the train store."""
        store = self.resolve_store(train_source)
        meta: dict = {}
        if learning_rates is not None:
            self._step_weights = ({int(k): float(v) for k, v in learning_rates.items()}
                                  if isinstance(learning_rates, Mapping) else float(learning_rates))
            meta["learning_rates"] = learning_rates
        elif checkpoint_weight is not None:
            self._step_weights = float(checkpoint_weight)
            meta["checkpoint_weight"] = checkpoint_weight
        else:
            recorded = read_lr_schedule(str(store.save_dir))
            if recorded is not None:
                self._step_weights = recorded
            elif self._step_weights is None:
                self._step_weights = 1.0
        return super().attribute_from_cache(store, test_source, algorithm_meta={**meta, **(algorithm_meta or {})},
                                            **kwargs)
