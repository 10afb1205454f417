"""Attributor bases: the shared inner-product attribution workflow.

:class:`BaseInnerProductAttributor` scores ``<transform_train(g_train),
transform_test(g_test)>`` layerwise.  Subclasses override the hook surface
(``generate_*_rep`` / ``load_*_rep`` sources, ``prepare_scoring``,
``transform_*_rep``, ``inner_product``, ``checkpoints``) and inherit collection
into a store of any residency, the checkpoint ensemble, the scoring loop with
``loop_over_test``, token granularity and :class:`AttributionScore` assembly.
Parity: reference ``dattri_llm/attribution/base.py:59-1152``.

Test-side routing (:meth:`_route_test_rep`): a factorized test layer is
materialized when the flop rule prefers it against a train batch, greedily by
saving and within the device memory budget; the rest is preprocessed once.
"""

from __future__ import annotations

from dattri_llm_b200.options import AttributionGranularity  # noqa: F401  (re-exported option types)
import tempfile
import warnings
from abc import ABC, abstractmethod
from collections.abc import Callable, Iterable
from pathlib import Path
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.score import AttributionScore
from dattri_llm_b200.attribution.utils import collect_gradients, finalize_factors, normalize_layer_names, score_sources
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.gradient.streaming import DiskGradientSource, GradientStreamer
from dattri_llm_b200.task import AttributionTask, as_task
from dattri_llm_b200.utils.cache import CACHE_RESIDENCIES, CacheBudget

ATTRIBUTION_GRANULARITIES = ("instance", "token")


def _check_granularity(g: str) -> None:
    if g not in ATTRIBUTION_GRANULARITIES:
        raise ValueError(f"attribution_granularity must be one of {ATTRIBUTION_GRANULARITIES}, got {g!r}.")


class BaseAttributor(ABC):
    """Base class for all attributors."""

    algorithm: ClassVar[str] = "Base"

    @abstractmethod
    def __init__(self, args, *, task: AttributionTask | None = None, **kwargs) -> None:
        """Bind the run configuration and (for live attribution) a task."""

    @abstractmethod
    def cache(self, train_dataset, test_dataset, *, cache_dir: str | None = None, hook_config=None,
              **cache_kwargs) -> list[tuple[str, str]]:
        """Collect gradients into stores; ``[(train_dir, test_dir)]`` per checkpoint."""

    @abstractmethod
    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  **attribution_kwargs) -> AttributionScore:
        """Live attribution of *train_dataset* against *test_dataset*."""

    @abstractmethod
    def attribute_from_cache(self, train_source, test_source, *, selected_training_steps=None,
                             layer_name=None, verbose: bool = False, **attribution_kwargs) -> AttributionScore:
        """Attribution over stored gradients (no model needed)."""


class BaseInnerProductAttributor(BaseAttributor):
    """Base class for inner-product attributors (see the module docstring)."""

    algorithm: ClassVar[str] = "InnerProduct"
    #: Whether :meth:`inner_product` is the plain layerwise dot product (enables the
    #: packed one-GEMM scoring of fully dense blocks).
    plain_inner_product: ClassVar[bool] = True

    def __init__(self, args, *, task: AttributionTask | None = None) -> None:
        self.args = args
        self.task = None if task is None else as_task(task)

    # ------------------------------------------------------------ task plumbing
    def require_task(self, method: str) -> AttributionTask:
        """The task, or a clear error naming the live *method*."""
        if self.task is None:
            raise ValueError(f"{method}() (live collection) requires a ``task`` with a model; pass "
                             "pre-collected gradients to attribute_from_cache() instead.")
        return self.task

    def num_checkpoints(self) -> int:
        """Checkpoints of the task."""
        return self.require_task("attribute").num_checkpoints()

    def load_checkpoint(self, index: int):
        """Load checkpoint *index* into the task's model."""
        return self.require_task("attribute").load_checkpoint(index)

    def checkpoints(self) -> list[int]:
        """Checkpoint indices :meth:`attribute` ensembles over (all, by default)."""
        return list(range(self.num_checkpoints()))

    def train_loss_fn(self) -> Callable:
        """The task's training loss."""
        return self.require_task("attribute").loss_func

    def test_loss_fn(self) -> Callable:
        """The task's target function."""
        return self.require_task("attribute").target_func

    # ------------------------------------------------------------ sources
    def generate_train_rep(self, train_dataset, *, checkpoint_step: int = 0, enable_update: bool = False,
                           hook_config=None, snapshots=None, forward_model=None) -> GradientStreamer:
        """Live train gradients: a streamer over *train_dataset*."""
        task = self.require_task("attribute")
        return GradientStreamer(task.model, train_dataset, self.args,
                                batch_size=self.args.per_device_train_batch_size, enable_update=enable_update,
                                loss_fn=self.train_loss_fn(), checkpoint_step=checkpoint_step, config=hook_config,
                                snapshots=snapshots,
                                forward_model=task.forward_model if forward_model is None else forward_model)

    def generate_test_rep(self, test_dataset, *, checkpoint_step: int = 0, hook_config=None, hook_manager=None,
                          forward_model=None, shard: bool = True) -> GradientStreamer:
        """Live test gradients: a frozen streamer against the task's target function."""
        task = self.require_task("attribute")
        return GradientStreamer(task.model, test_dataset, self.args,
                                batch_size=self.args.per_device_eval_batch_size, enable_update=False,
                                loss_fn=self.test_loss_fn(), checkpoint_step=checkpoint_step, config=hook_config,
                                hook_manager=hook_manager,
                                forward_model=task.forward_model if forward_model is None else forward_model,
                                shard=shard)

    def load_train_rep(self, train_gradients, *, steps=None, layer_name=None, verbose: bool = False,
                       desc: str | None = None) -> DiskGradientSource:
        """Stored train gradients as a re-iterable source."""
        store = (train_gradients if isinstance(train_gradients, GradientStorageManager)
                 else GradientStorageManager(train_gradients))
        return DiskGradientSource(store, self.args, steps=steps, layer_name=normalize_layer_names(layer_name),
                                  desc=desc if desc is not None else f"{self.algorithm}: train", verbose=verbose)

    def load_test_rep(self, test_gradients, *, layer_name=None, verbose: bool = False,
                      desc: str | None = None) -> DiskGradientSource:
        """Stored test gradients as a re-iterable source."""
        store = (test_gradients if isinstance(test_gradients, GradientStorageManager)
                 else GradientStorageManager(test_gradients))
        return DiskGradientSource(store, self.args, layer_name=normalize_layer_names(layer_name),
                                  desc=desc if desc is not None else f"{self.algorithm}: test", verbose=verbose)

    # ------------------------------------------------------------ collection
    def collect_gradients(self, streamer, store, *, offload_interval: int = 1, on_block=None,
                          resume: bool = False):
        """Run *streamer* into *store* (*resume*: skip the batches already stored)."""
        return collect_gradients(streamer, store, offload_interval=offload_interval, on_block=on_block,
                                 resume=resume)

    def cache_representations(self, source, store, *, transform=None, sample_id_key=None):
        """Persist ``transform(block)`` (materialized) for every block of *source*."""
        transform = transform if transform is not None else self.transform_test_rep
        for step, block, hashes in source:
            rep = transform(block.to(self.args.device)).materialize().to("cpu")
            store.save_bulk([GradientRecord(step, list(hashes), rep, sample_id_key)])
        return store

    def cache(self, train_dataset, test_dataset, *, cache_dir: str | None = None, hook_config=None,
              enable_update: bool = False, on_train_block=None, resume: bool = False) -> list[tuple[str, str]]:
        """Collect test then train gradients per checkpoint into ``<cache_dir>/ckpt_<k>/``.

        *resume* continues an interrupted run in the same *cache_dir*: batches already
        stored are skipped (frozen probes only)."""
        if resume and enable_update:
            raise ValueError("resume=True needs a frozen probe (enable_update=False).")
        self.require_task("cache")
        cache_dir = cache_dir if cache_dir is not None else self.args.output_dir
        pairs = []
        for k in self.checkpoints():
            self.load_checkpoint(k)
            root = Path(cache_dir) / f"ckpt_{k}"
            train_dir, test_dir = str(root / "train_grads"), str(root / "test_grads")
            self.collect_gradients(self.generate_test_rep(test_dataset, checkpoint_step=k, hook_config=hook_config,
                                                          shard=False), GradientStorageManager(test_dir), resume=resume)
            self.collect_gradients(self.generate_train_rep(train_dataset, checkpoint_step=k,
                                                           enable_update=enable_update, hook_config=hook_config),
                                   GradientStorageManager(train_dir), on_block=on_train_block, resume=resume)
            pairs.append((train_dir, test_dir))
            if enable_update:
                break
        return pairs

    # ------------------------------------------------------------ scoring hooks
    def prepare_scoring(self, train_source, test_source) -> None:
        """One-time work before a scoring pass (e.g. fitting a preconditioner)."""

    def transform_train_rep(self, train_rep: Gradient) -> Gradient:
        """Per-block train transform (identity)."""
        return train_rep

    def transform_test_rep(self, test_rep: Gradient) -> Gradient:
        """Per-block test transform (identity)."""
        return test_rep

    def _route_test_rep(self, test_rep: Gradient) -> Gradient:
        b_train = self.args.per_device_train_batch_size or 1
        candidates: list[tuple[float, str]] = []
        for name, value in test_rep.data.items():
            if not isinstance(value, Factorized):
                continue
            lt = test_rep.layer_types[name]
            if not (ops.is_linear(lt) or ops.is_conv(lt) or ops.is_conv_transpose(lt)):
                candidates.append((float("inf"), name))
                continue
            b_test, s, k, d = ops.effective_dims(value, lt)
            if ops.maybe_use_materialized_gram(b_train, b_test, s, k, d):
                cost_f = b_train * b_test * s * s * (d + k)
                cost_m = (b_train + b_test) * s * d * k + b_train * b_test * d * k
                candidates.append((cost_f - cost_m, name))
        budget = CacheBudget(test_rep.device)
        held = 0
        dense = []
        for _saving, name in sorted(candidates, reverse=True):
            layer = test_rep.select_layers([name])
            growth = max(layer.materialized_nbytes - layer.nbytes, 0)
            if budget.fits(growth, held):
                dense.append(name)
                held += growth
        if dense:
            test_rep = test_rep.map_layers(lambda _n, v, t: ops.materialize(v, t), layers=dense, consume=True)
        return finalize_factors(test_rep, budget=budget, held=held)

    def inner_product(self, train_rep: Gradient, test_rep: Gradient, *, dense_cache=None) -> torch.Tensor:
        """``(B_train, B_test)`` layerwise cross-gram."""
        if not any(n in test_rep.data for n in train_rep.data):
            return torch.zeros(train_rep.batch_size, test_rep.batch_size)
        return ops.layerwise_cross_dot(train_rep, test_rep, dense_cache=dense_cache)

    def inner_product_per_token(self, train_rep: Gradient, test_rep: Gradient) -> torch.Tensor:
        """``(B_train, T_train, B_test)`` per-token decomposition of :meth:`inner_product`."""
        if not any(n in test_rep.data for n in train_rep.data):
            toks = [t for t in train_rep.token_dim.values() if t is not None]
            return torch.zeros(train_rep.batch_size, max(toks) if toks else 1, test_rep.batch_size)
        return ops.layerwise_cross_dot_per_token(train_rep, test_rep)

    def uses_plain_inner_product(self) -> bool:
        """Whether scoring is the plain layerwise dot product of untransformed train blocks
        (then fully dense pairs are scored as one packed GEMM)."""
        return (type(self).inner_product is BaseInnerProductAttributor.inner_product
                and type(self).transform_train_rep is BaseInnerProductAttributor.transform_train_rep
                and self.plain_inner_product)

    def score_sources(self, train_source, test_source, *, loop_over_test: bool = False, transform_test=None,
                      attribution_granularity: str = "instance"):
        """Run the scoring loop with this attributor's hooks."""
        self.prepare_scoring(train_source, test_source)
        transform = transform_test if transform_test is not None else self.transform_test_rep
        plain = self.uses_plain_inner_product()
        return score_sources(train_source, test_source, self.args.device, inner_product=self.inner_product,
                             transform_train=lambda b: finalize_factors(self.transform_train_rep(b)),
                             transform_test=lambda b: self._route_test_rep(transform(b)),
                             batch_size=self.args.per_device_train_batch_size or 1, loop_over_test=loop_over_test,
                             granularity=attribution_granularity,
                             inner_product_per_token=self.inner_product_per_token, packed_inner_product=plain)

    def build_score(self, scores, row_train_ids, row_steps, test_ids, *, algorithm_meta=None, layer_name=None,
                    row_token_ids=None) -> AttributionScore:
        """Assemble and save (``args.output_dir``) the :class:`AttributionScore`."""
        result = AttributionScore(scores=scores, row_train_ids=row_train_ids, row_steps=row_steps,
                                  test_ids=test_ids, algorithm_meta=dict(algorithm_meta or {}),
                                  algorithm=self.algorithm, layer_name=layer_name, row_token_ids=row_token_ids)
        result.save(self.args.output_path)
        return result

    @staticmethod
    def stores_meta(train_store, test_store) -> dict:
        """Provenance of two stores' identifier schemes."""
        return {"sample_id_key": {"train": train_store.sample_id_key, "test": test_store.sample_id_key}}

    # ------------------------------------------------------------ workflows
    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, enable_update: bool = False,
                  gradient_cache_residency: str | None = None, attribution_granularity: str = "instance",
                  **attribution_kwargs) -> AttributionScore:
        """Live attribution: per checkpoint, stream the test set (on every rank) and the
        train set (this rank's shard) through one set of hooks and score them; with
        ``gradient_cache_residency`` the gradients are collected into stores first."""
        del verbose
        self.require_task("attribute")
        _check_granularity(attribution_granularity)
        if gradient_cache_residency is not None:
            if enable_update and loop_over_test:
                raise ValueError(
                    "loop_over_test=True with enable_update=True takes the query gradient at every step's "
                    "parameters, which needs gradient_cache_residency=None: a gradient store holds the query "
                    "gradients taken once, before the trajectory.")
            if gradient_cache_residency not in CACHE_RESIDENCIES:
                raise ValueError(f"gradient_cache_residency must be one of {list(CACHE_RESIDENCIES)} or None, "
                                 f"got {gradient_cache_residency!r}.")
            return self._attribute_via_stores(train_dataset, test_dataset, residency=gradient_cache_residency,
                                              hook_config=hook_config, loop_over_test=loop_over_test,
                                              enable_update=enable_update,
                                              attribution_granularity=attribution_granularity,
                                              **attribution_kwargs)
        ckpts = self.checkpoints()
        if enable_update and len(ckpts) > 1:
            warnings.warn(f"enable_update=True regenerates the trajectory from checkpoint 0; the other "
                          f"{len(ckpts) - 1} provided checkpoint(s) are ignored.", stacklevel=2)
            ckpts = ckpts[:1]
        blocks, ids, steps, toks = [], [], [], []
        test_ids = None
        hooked: list[str] = []
        for k in ckpts:
            self.load_checkpoint(k)
            train = self.generate_train_rep(train_dataset, checkpoint_step=k, enable_update=enable_update,
                                            hook_config=hook_config)
            test = self.generate_test_rep(test_dataset, checkpoint_step=k, hook_manager=train.hook_manager,
                                          forward_model=train.forward_model, shard=False)
            hooked = list(train.hook_manager.layer_name)
            if enable_update and loop_over_test:
                if not isinstance(train, GradientStreamer):
                    raise TypeError("loop_over_test=True with enable_update=True needs generate_train_rep() to "
                                    f"return a GradientStreamer, got {type(train).__name__}.")
                train.defer_update = True
            with train, test:
                sc, rids, rsteps, tids, rtoks = self.score_sources(
                    train, test, loop_over_test=loop_over_test, attribution_granularity=attribution_granularity)
            blocks.append(sc)
            ids.extend(rids)
            steps.extend(rsteps)
            toks.extend(rtoks or [])
            test_ids = tids if test_ids is None else test_ids
        return self.build_score(
            torch.cat(blocks, dim=0) if blocks else torch.zeros(0, 0), ids, steps, test_ids or [],
            algorithm_meta={"n_checkpoints": len(ckpts), "enable_update": enable_update,
                            "query_at": (("theta_t" if loop_over_test else "theta_0") if enable_update
                                         else "checkpoint"),
                            "attribution_granularity": attribution_granularity, **attribution_kwargs},
            layer_name=hooked or None, row_token_ids=toks if attribution_granularity == "token" else None)

    def _attribute_via_stores(self, train_dataset, test_dataset, *, residency: str, hook_config,
                              loop_over_test: bool, enable_update: bool, **attribution_kwargs) -> AttributionScore:
        if residency == "disk":
            pairs = self.cache(train_dataset, test_dataset, hook_config=hook_config, enable_update=enable_update)
            results = [self.attribute_from_cache(tr, te, loop_over_test=loop_over_test, **attribution_kwargs)
                       for tr, te in pairs]
            return self._stack_scores(results, len(pairs))
        ckpts = self.checkpoints()[:1] if enable_update else self.checkpoints()
        results = []
        for k in ckpts:
            self.load_checkpoint(k)
            with (GradientStorageManager(tempfile.mkdtemp(prefix=f"{self.algorithm.lower()}_train_"),
                                         residency=residency) as train_store,
                  GradientStorageManager(tempfile.mkdtemp(prefix=f"{self.algorithm.lower()}_test_"),
                                         residency=residency) as test_store):
                self.collect_gradients(self.generate_test_rep(test_dataset, checkpoint_step=k,
                                                              hook_config=hook_config, shard=False), test_store)
                self.collect_gradients(self.generate_train_rep(train_dataset, checkpoint_step=k,
                                                               enable_update=enable_update,
                                                               hook_config=hook_config), train_store)
                results.append(self.attribute_from_cache(
                    train_store, test_store, loop_over_test=loop_over_test,
                    algorithm_meta={"gradient_cache_residency": residency}, **attribution_kwargs))
        return self._stack_scores(results, len(ckpts))

    def _stack_scores(self, results: list[AttributionScore], n_checkpoints: int) -> AttributionScore:
        if len(results) == 1:
            return results[0]
        first = results[0]
        return self.build_score(
            torch.cat([r.scores for r in results], dim=0), [i for r in results for i in r.row_train_ids],
            [s for r in results for s in r.row_steps], first.test_ids,
            algorithm_meta={**first.algorithm_meta, "n_checkpoints": n_checkpoints}, layer_name=first.layer_name,
            row_token_ids=None if first.row_token_ids is None else [t for r in results for t in r.row_token_ids])

    @staticmethod
    def resolve_store(source) -> GradientStorageManager:
        """A store from a directory, a store, or a :class:`DiskGradientSource`.

        Raises:
            TypeError: for anything else.
        """
        if isinstance(source, GradientStorageManager):
            return source
        if isinstance(source, DiskGradientSource):
            return source.file_manager
        if isinstance(source, (str, Path)):
            return GradientStorageManager(str(source))
        raise TypeError("expected a store directory, a GradientStorageManager, or a DiskGradientSource, got "
                        f"{type(source).__name__}.")

    def attribute_from_cache(self, train_source, test_source, *, selected_training_steps: Iterable[int] | None = None,
                             layer_name=None, verbose: bool = False, loop_over_test: bool = False,
                             algorithm_meta: dict | None = None, attribution_granularity: str = "instance",
                             **attribution_kwargs) -> AttributionScore:
        """Score stored train gradients against stored test gradients."""
        _check_granularity(attribution_granularity)
        train_store, test_store = self.resolve_store(train_source), self.resolve_store(test_source)
        layer_name = normalize_layer_names(layer_name)
        train = self.load_train_rep(train_store, steps=selected_training_steps, layer_name=layer_name,
                                    verbose=verbose, desc=f"{self.algorithm}: scoring")
        test = self.load_test_rep(test_store, layer_name=layer_name, verbose=verbose,
                                  desc=f"{self.algorithm}: loading test")
        scores, rids, rsteps, tids, rtoks = self.score_sources(
            train, test, loop_over_test=loop_over_test, attribution_granularity=attribution_granularity)
        return self.build_score(scores, rids, rsteps, tids,
                                algorithm_meta={"selected_training_steps": train.steps,
                                                **self.stores_meta(train_store, test_store),
                                                "attribution_granularity": attribution_granularity,
                                                **(algorithm_meta or {}), **attribution_kwargs},
                                layer_name=layer_name, row_token_ids=rtoks)
