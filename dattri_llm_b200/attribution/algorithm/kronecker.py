"""K-FAC and EK-FAC influence attributors.

Score = ``<g_train, F^-1 g_test>`` with the Fisher ``F`` approximated per layer by
a Kronecker product ``A (x) G`` of activation / output-gradient covariances
(K-FAC: ``G^-1 dW A^-1`` with damped inverses), or in the Kronecker eigenbasis
with empirically fitted eigenvalues (EK-FAC: ``U_G ((U_G^T dW U_A) / (lambda +
damping)) U_A^T``).  The test side is preconditioned once; train blocks are scored
raw.  Layers without factorized captures fall back to a dense empirical Fisher
(``non_kfac_strategy="direct"`` also covers norm layers), bounded by
``direct_fim_max_params``.  Covariances can come from a fit pass over the train
store, or from :class:`KroneckerCovarianceCallback` at capture time.  Fits are
saved to / loaded from ``<fisher_dir>/fisher_factors.pt`` (atomic rename), with
the options that define them recorded and checked.  Parity: reference
``dattri_llm/attribution/algorithm/kronecker.py:92-1601`` (workflow, options and
the fisher-file format).

B200: covariance accumulation runs as split-K tcgen05 Gram GEMMs into fp32 sums;
every layer's sums are reduced across ranks in one packed collective.
"""

from __future__ import annotations

import contextlib
import tempfile
import warnings
from abc import abstractmethod
from collections.abc import Iterable, Iterator, Mapping
from pathlib import Path
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.base import BaseInnerProductAttributor
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks import KroneckerCovarianceCallback
from dattri_llm_b200.gradient.datasets import resolve_steps
from dattri_llm_b200.gradient.gradient import Factorized
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.utils.cache import CACHE_RESIDENCIES, CacheBudget, TensorCache
from dattri_llm_b200.utils.distributed import all_reduce_sum, dist_rank


def _map_tensors(obj, fn):
    if isinstance(obj, torch.Tensor):
        return fn(obj)
    if isinstance(obj, _FactorCache):
        return obj
    if isinstance(obj, dict):
        return {k: _map_tensors(v, fn) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_map_tensors(v, fn) for v in obj)
    return obj


class _FactorCache(Mapping):
    """Per-layer factors held in a host cache of a given residency (entries the budget
    refuses stay where they are)."""

    def __init__(self, residency: str) -> None:
        self._cache = TensorCache(residency, budget=CacheBudget())
        self._kept: dict = {}
        self._order: list[str] = []

    def __setitem__(self, layer: str, factors) -> None:
        self._kept.pop(layer, None)
        if not self._cache.put(layer, _map_tensors(factors, lambda t: t.to("cpu"))):
            self._kept[layer] = factors
        if layer not in self._order:
            self._order.append(layer)

    def __getitem__(self, layer: str):
        if layer in self._kept:
            return self._kept[layer]
        if layer not in self._cache:
            raise KeyError(layer)
        return self._cache.get(layer)

    def __iter__(self) -> Iterator[str]:
        return iter(self._order)

    def __len__(self) -> int:
        return len(self._order)

    def close(self) -> None:
        self._cache.close()
        self._kept.clear()
        self._order.clear()


def _mean_eigenvalue(m: torch.Tensor) -> torch.Tensor:
    return m.diagonal(dim1=-2, dim2=-1).float().mean()


class KroneckerAttributor(BaseInnerProductAttributor):
    """Shared workflow of the K-FAC family; subclass ``fit_factors`` / ``damp`` /
    ``precondition_test_layer`` for a variant."""

    algorithm: ClassVar[str] = "Kronecker"
    _COVARIANCE_FILE: ClassVar[str] = "kronecker_covariances.pt"
    _FISHER_FILE: ClassVar[str] = "fisher_factors.pt"
    _FISHER_PROVENANCE = ("damping", "relative_damping")

    def __init__(self, args, *, task=None) -> None:
        super().__init__(args, task=task)
        self._relative_damping = False
        self._covariances_at_capture = True
        self._capture_streamer = None
        self._collected_covariances: dict[str, dict] = {}
        self._factor_cache_residency: str | None = None
        self._factor_caches: list[_FactorCache] = []
        self._damping = 1e-3
        self._non_kfac_strategy = "ignore"
        self._direct_fim_max_params = 4096
        self._raw_fit = None
        self._preconditioner = None
        self._fit_scope: dict = {"layer_name": None, "selected_training_steps": None}
        self._save_fit_to: str | None = None
        self._fisher_dir_fit = None
        self._fisher_saw_embedding: set[str] = set()
        self._skipped_materialized: set[str] = set()
        self._direct_norm_layers = False
        self._capture_covariances = None

    def uses_plain_inner_product(self) -> bool:
        """Train blocks are raw, the inner product plain (the test side is preconditioned)."""
        return True

    @abstractmethod
    def fit_factors(self, train_source, fisher_acc: ops.FisherAccumulator) -> dict:
        """Raw per-layer factors from the train source (accumulating the direct Fisher)."""

    @abstractmethod
    def damp(self, raw_factors: dict, damping: float) -> dict:
        """Damped, inverted (or rescaled) factors ready to precondition."""

    @abstractmethod
    def precondition_test_layer(self, value, layer_type: str, factors):
        """One test layer preconditioned by its factors."""

    def checkpoints(self) -> list[int]:
        """Single checkpoint (the first; others ignored with a warning)."""
        n = self.num_checkpoints()
        if n > 1:
            warnings.warn(f"{type(self).__name__} is single-checkpoint; only checkpoint 0 is used and the other "
                          f"{n - 1} provided checkpoint(s) are ignored.", stacklevel=2)
        return [0]

    # ------------------------------------------------------------ fitting
    def fit_raw(self, train_source):
        """``(raw_factors, raw_direct_fisher)`` of a re-iterable train source.

        Raises:
            ValueError: for a single-shot source, or when no layer is eligible.
        """
        if not getattr(train_source, "reusable", False):
            raise ValueError(f"{type(self).__name__} needs a re-iterable train source: the Fisher pre-pass "
                             "re-reads the train gradients before scoring. Use on-disk gradients, a frozen "
                             "GradientStreamer (enable_update=False), or attribute(gradient_cache_residency=...).")
        self._fisher_saw_embedding = set()
        self._skipped_materialized = set()
        self._direct_norm_layers = self._non_kfac_strategy == "direct"
        acc = ops.FisherAccumulator(self._direct_fim_max_params)
        raw = self.fit_factors(train_source, acc)
        if self._skipped_materialized:
            n = len(self._skipped_materialized)
            warnings.warn(
                f"{n} of the {n + len(raw)} K-FAC-eligible layers are not preconditioned by {self.algorithm}: "
                "layers stored materialized carry no (a, g) factors for Kronecker covariances; they use the "
                f"direct dense empirical Fisher bounded by direct_fim_max_params={self._direct_fim_max_params}: "
                f"{sorted(self._skipped_materialized)}. Capture them factorized, or pass capture-time "
                "covariances (KroneckerCovarianceCallback) to fit(covariances=...).", stacklevel=2)
        fisher = self._finalize_fisher(acc)
        if not raw and not fisher:
            raise ValueError("No eligible layers found in the training gradients: no K-FAC-eligible (linear/conv) "
                             "layer" + (f" and no direct-Fisher layer within direct_fim_max_params="
                                        f"{self._direct_fim_max_params}" if self._non_kfac_strategy == "direct"
                                        else " (pass non_kfac_strategy='direct' to include norm layers)") + ".")
        return raw, fisher

    def _damping_for(self, damping: float, spectrum_mean) -> float:
        return damping * float(spectrum_mean) if self._relative_damping else damping

    def damp_fit(self, raw_fit, damping: float):
        """``(damped factors, {layer: inverse direct Fisher})``."""
        raw, fisher = raw_fit
        dev = self.args.device
        factors = self._factor_map()
        for layer, r in raw.items():
            factors[layer] = self.damp({layer: _map_tensors(r, lambda t: t.to(dev))}, damping)[layer]
        fisher = _map_tensors(fisher, lambda t: t.to(dev))
        return factors, {n: ops.dense_inverse(F, self._damping_for(damping, _mean_eigenvalue(F)))
                         for n, F in fisher.items()}

    def _factor_map(self):
        if self._factor_cache_residency is None:
            return {}
        c = _FactorCache(self._factor_cache_residency)
        self._factor_caches.append(c)
        return c

    def _release_factor_caches(self, keep: tuple = ()) -> None:
        for c in [c for c in self._factor_caches if not any(c is k for k in keep)]:
            c.close()
            self._factor_caches.remove(c)

    def generate_train_rep(self, train_dataset, **kwargs):
        """The train streamer; a frozen probe also gathers capture-time covariances."""
        s = super().generate_train_rep(train_dataset, **kwargs)
        self._capture_streamer = s if self._covariances_at_capture and not kwargs.get("enable_update") else None
        return s

    def collect_gradients(self, streamer, store, **kwargs):
        """Collect; for the capture streamer also accumulate ``(A, G)`` and save them beside the store."""
        if streamer is not self._capture_streamer:
            return super().collect_gradients(streamer, store, **kwargs)
        self._capture_streamer = None
        if kwargs.get("resume") and any(step == streamer.checkpoint_step for step, _ in store.own_records()):
            # the skipped batches would be missing from covariances gathered now: the fit
            # sweeps the completed store instead (or reads the file a finished run saved)
            return super().collect_gradients(streamer, store, **kwargs)
        cb = KroneckerCovarianceCallback()
        streamer.hook_manager.add_callback(cb)
        result = super().collect_gradients(streamer, store, **kwargs)
        cb.all_reduce()
        cov = self._move_raw(cb.result(), torch.device("cpu"))
        root = Path(store.save_dir)
        self._collected_covariances[str(root.resolve())] = cov
        if store.residency == "disk" and dist_rank() in (None, 0):
            torch.save(cov, root / self._COVARIANCE_FILE)
        return result

    def cache(self, train_dataset, test_dataset, *, covariances_at_capture: bool | None = None, **kwargs):
        """Collect the stores (covariances gathered at capture by default)."""
        if covariances_at_capture is not None:
            self._covariances_at_capture = covariances_at_capture
        return super().cache(train_dataset, test_dataset, **kwargs)

    def _covariances_for(self, train_source):
        store = getattr(train_source, "file_manager", None)
        if not self._covariances_at_capture or store is None:
            return None
        if sorted(train_source.steps) != sorted(resolve_steps(store, None)):
            return None
        root = Path(store.save_dir)
        cov = self._collected_covariances.get(str(root.resolve()))
        if cov is None and (root / self._COVARIANCE_FILE).exists():
            cov = torch.load(root / self._COVARIANCE_FILE, map_location="cpu", weights_only=True)
        layers = getattr(train_source, "layer_name", None)
        if cov is not None and layers is not None:
            cov = {k: v for k, v in cov.items() if k in layers} or None
        return cov

    def prepare_scoring(self, train_source, test_source) -> None:
        """Fit (or reuse) the factors and damp them."""
        if self._preconditioner is not None:
            return
        if self._raw_fit is None:
            collected = self._covariances_for(train_source)
            if collected is not None and self._capture_covariances is None:
                self._capture_covariances = self._move_raw(collected, self.args.device)
                try:
                    self._raw_fit = self.fit_raw(train_source)
                finally:
                    self._capture_covariances = None
            else:
                self._raw_fit = self.fit_raw(train_source)
        self._preconditioner = self.damp_fit(self._raw_fit, self._damping)
        self._raw_fit = _map_tensors(self._raw_fit, lambda t: t.to("cpu"))
        if self._save_fit_to is not None:
            self.save_fisher(self._raw_fit[0], self._save_fit_to, fisher=self._raw_fit[1])
            self._fisher_dir_fit = (self._fisher_dir_key(self._save_fit_to), self._raw_fit)
            self._save_fit_to = None
        kept = () if self._fisher_dir_fit is None else (self._fisher_dir_fit[1][0],)
        self._release_factor_caches(keep=(self._raw_fit[0], self._preconditioner[0], *kept))

    def _set_options(self, damping, non_kfac_strategy, direct_fim_max_params, relative_damping,
                     factor_cache_residency, covariances_at_capture) -> None:
        if damping < 0:
            raise ValueError(f"damping must be non-negative, got {damping}.")
        if non_kfac_strategy not in ("ignore", "direct"):
            raise ValueError(f"non_kfac_strategy must be 'ignore' or 'direct', got {non_kfac_strategy!r}.")
        if direct_fim_max_params <= 0:
            raise ValueError(f"direct_fim_max_params must be positive, got {direct_fim_max_params}.")
        if factor_cache_residency is not None and factor_cache_residency not in CACHE_RESIDENCIES:
            raise ValueError(f"factor_cache_residency must be one of {list(CACHE_RESIDENCIES)} or None, got "
                             f"{factor_cache_residency!r}.")
        self._damping, self._non_kfac_strategy = damping, non_kfac_strategy
        self._direct_fim_max_params, self._relative_damping = direct_fim_max_params, relative_damping
        self._factor_cache_residency, self._covariances_at_capture = factor_cache_residency, covariances_at_capture
        self._raw_fit = self._preconditioner = None
        self._fit_scope = {"layer_name": None, "selected_training_steps": None}
        self._save_fit_to = None

    def transform_test_rep(self, test_rep):
        """Precondition every fitted test layer (layers without a fit are dropped).

        Raises:
            RuntimeError: before :meth:`prepare_scoring`.
        """
        if self._preconditioner is None:
            raise RuntimeError("prepare_scoring() must run before transform_test_rep().")
        factors, finv = self._preconditioner
        dev = test_rep.device

        def precondition(name, value, lt):
            if name in factors:
                return self.precondition_test_layer(value, lt, _map_tensors(factors[name], lambda t: t.to(dev)))
            if name in finv:
                return ops.materialize(value, lt).float() @ finv[name]
            return None

        return test_rep.map_layers(precondition)

    def kfac_layers(self, grad) -> list[str]:
        """Layers of *grad* that enter K-FAC (factorized, or with supplied covariances)."""
        supplied = self._capture_covariances or {}
        out = []
        for name, v in grad.data.items():
            if not ops.is_kfac_eligible(grad.layer_types[name]):
                continue
            if isinstance(v, Factorized) or name in supplied:
                out.append(name)
            else:
                self._skipped_materialized.add(name)
        return out

    def fisher_layers(self, grad) -> list[str]:
        """Layers preconditioned by the direct dense Fisher."""
        supplied = self._capture_covariances or {}
        out = []
        for name, v in grad.data.items():
            lt = grad.layer_types[name]
            if lt == ops.PARAM_GRAD_TYPES or (isinstance(v, torch.Tensor) and name in supplied):
                continue
            if isinstance(v, torch.Tensor) or (self._direct_norm_layers and ops.is_norm(lt)):
                out.append(name)
        return out

    def accumulate_fisher(self, fisher_acc: ops.FisherAccumulator, grad) -> None:
        """Add one block to the direct-Fisher accumulator."""
        fisher_acc.update(grad, self.fisher_layers(grad))
        if self._direct_norm_layers:
            self._fisher_saw_embedding.update(n for n, v in grad.data.items()
                                              if ops.is_embedding(grad.layer_types[n]) and isinstance(v, Factorized))

    def _finalize_fisher(self, acc: ops.FisherAccumulator) -> dict:
        if acc.skipped:
            warnings.warn("The direct dense-Fisher fallback skipped layers whose parameter count exceeds "
                          f"direct_fim_max_params={self._direct_fim_max_params}: {dict(sorted(acc.skipped.items()))}.",
                          stacklevel=2)
        if self._fisher_saw_embedding:
            warnings.warn("non_kfac_strategy='direct' does not cover embedding layers (heavily parametrised); "
                          f"leaving ignored: {sorted(self._fisher_saw_embedding)}.", stacklevel=2)
        return dict(acc.result())

    # ------------------------------------------------------------ fisher files
    def _fisher_meta(self) -> dict:
        meta = {"algorithm": self.algorithm, "non_kfac_strategy": self._non_kfac_strategy,
                "direct_fim_max_params": self._direct_fim_max_params, **self._fit_scope,
                "damping": self._damping, "relative_damping": self._relative_damping}
        if getattr(self, "mode", None) is not None:
            meta["mode"] = self.mode
        return meta

    def _set_fit_scope(self, layer_name, selected_training_steps) -> None:
        if isinstance(layer_name, str):
            layer_name = [layer_name]
        self._fit_scope = {"layer_name": None if layer_name is None else sorted(layer_name),
                           "selected_training_steps": None if selected_training_steps is None
                           else sorted(int(s) for s in selected_training_steps)}

    def _fisher_dir_key(self, fisher_dir: str) -> tuple:
        path = Path(fisher_dir) / self._FISHER_FILE
        defining = {k: v for k, v in self._fisher_meta().items() if k not in self._FISHER_PROVENANCE}
        return str(path.resolve()), path.stat().st_mtime_ns, repr(sorted(defining.items())), self._factor_cache_residency

    def _use_fisher_dir(self, fisher_dir: str | None) -> None:
        if fisher_dir is None:
            return
        if not (Path(fisher_dir) / self._FISHER_FILE).exists():
            self._save_fit_to = fisher_dir
            return
        key = self._fisher_dir_key(fisher_dir)
        if self._fisher_dir_fit is not None and self._fisher_dir_fit[0] == key:
            self._raw_fit = self._fisher_dir_fit[1]
            return
        self._raw_fit = self.load_fisher(fisher_dir)
        self._fisher_dir_fit = (key, self._raw_fit)

    @staticmethod
    def _move_raw(raw: dict, device) -> dict:
        return {k: tuple(t.to(device) for t in v) if isinstance(v, tuple) else v.to(device) for k, v in raw.items()}

    def _default_fisher_dir(self) -> str:
        return str(Path(self.args.output_dir) / f"{self.algorithm.lower()}_fisher")

    def save_fisher(self, covariances: dict, fisher_dir: str | None = None, *, fisher: dict | None = None) -> str:
        """Write ``fisher_factors.pt`` (raw factors, direct Fisher, defining options) atomically."""
        fisher_dir = fisher_dir or self._default_fisher_dir()
        path = Path(fisher_dir)
        path.mkdir(parents=True, exist_ok=True)
        cpu = torch.device("cpu")
        partial = path / f"{self._FISHER_FILE}.rank{dist_rank() or 0}.partial"
        torch.save({"meta": self._fisher_meta(), "raw_ctx": self._move_raw(dict(covariances.items()), cpu),
                    "raw_fim": self._move_raw(fisher or {}, cpu)}, partial)
        partial.replace(path / self._FISHER_FILE)
        return fisher_dir

    def load_fisher(self, fisher_dir: str):
        """Read a saved fit, checking that it was made under the requested options.

        Raises:
            ValueError: for a missing file, another algorithm, or differing options.
        """
        path = Path(fisher_dir) / self._FISHER_FILE
        if not path.exists():
            raise ValueError(f"No fitted Fisher factors at {path}; build them with "
                             f"{type(self).__name__}.fit(train_gradients_dir, {fisher_dir!r}) first.")
        blob = torch.load(path, map_location="cpu", weights_only=True)
        meta = blob["meta"]
        if meta.get("algorithm") != self.algorithm:
            raise ValueError(f"fisher_dir {fisher_dir!r} holds {meta.get('algorithm')!r} factors, but this is a "
                             f"{self.algorithm} attributor.")
        differing = {k: (meta.get(k), v) for k, v in self._fisher_meta().items()
                     if k not in self._FISHER_PROVENANCE and meta.get(k) != v}
        if differing:
            raise ValueError(f"fisher_dir {fisher_dir!r} holds a fit made under other options (recorded, "
                             f"requested): {differing}.")
        dev = self.args.device
        fim = self._move_raw(blob["raw_fim"], dev)
        if self._factor_cache_residency is None:
            return self._move_raw(blob["raw_ctx"], dev), fim
        factors = self._factor_map()
        for layer, raw in blob["raw_ctx"].items():
            factors[layer] = raw
        return factors, fim

    def fit(self, train_gradients_dir: str, fisher_dir: str | None = None, *,
            selected_training_steps: Iterable[int] | None = None, non_kfac_strategy: str = "ignore",
            direct_fim_max_params: int = 4096, layer_name=None, verbose: bool = False, covariances=None,
            factor_cache_residency: str | None = None, covariances_at_capture: bool = True) -> str:
        """Fit the factors over a train store and save them; returns the fisher directory."""
        self._set_options(self._damping, non_kfac_strategy, direct_fim_max_params, self._relative_damping,
                          factor_cache_residency, covariances_at_capture)
        self._set_fit_scope(layer_name, selected_training_steps)
        train = self.load_train_rep(train_gradients_dir, steps=selected_training_steps, layer_name=layer_name,
                                    verbose=verbose, desc=f"{self.algorithm}: fitting Fisher")
        if covariances is None:
            covariances = self._covariances_for(train)
        self._capture_covariances = None if covariances is None else self._move_raw(covariances, self.args.device)
        try:
            raw, fim = self.fit_raw(train)
        finally:
            self._capture_covariances = None
        out = self.save_fisher(raw, fisher_dir, fisher=fim)
        if isinstance(raw, _FactorCache):
            raw.close()
            self._factor_caches.remove(raw)
        return out

    # ------------------------------------------------------------ workflows
    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, gradient_cache_residency=None,
                  attribution_granularity: str = "instance", damping: float = 1e-3,
                  non_kfac_strategy: str = "ignore", direct_fim_max_params: int = 4096,
                  relative_damping: bool = False, factor_cache_residency=None, covariances_at_capture: bool = True,
                  fisher_dir: str | None = None):
        """Live K-FAC-family attribution at checkpoint 0."""
        self._set_options(damping, non_kfac_strategy, direct_fim_max_params, relative_damping,
                          factor_cache_residency, covariances_at_capture)
        if gradient_cache_residency is None:
            self._use_fisher_dir(fisher_dir)
        extra = {}
        if gradient_cache_residency is not None and loop_over_test:
            extra["preconditioned_test_cache_residency"] = gradient_cache_residency
        return super().attribute(
            train_dataset, test_dataset, hook_config=hook_config, verbose=verbose, loop_over_test=loop_over_test,
            enable_update=False, gradient_cache_residency=gradient_cache_residency,
            attribution_granularity=attribution_granularity, damping=damping, non_kfac_strategy=non_kfac_strategy,
            direct_fim_max_params=direct_fim_max_params, relative_damping=relative_damping,
            factor_cache_residency=factor_cache_residency, covariances_at_capture=covariances_at_capture,
            fisher_dir=fisher_dir, **extra)

    def attribute_from_cache(self, train_source, test_source, *, selected_training_steps=None, layer_name=None,
                             verbose: bool = False, loop_over_test: bool = False, algorithm_meta=None,
                             attribution_granularity: str = "instance", damping: float = 1e-3,
                             preconditioned_test_dir: str | None = None,
                             preconditioned_test_cache_residency: str | None = None, fisher_dir: str | None = None,
                             non_kfac_strategy: str = "ignore", direct_fim_max_params: int = 4096,
                             relative_damping: bool = False, factor_cache_residency=None,
                             covariances_at_capture: bool = True):
        """K-FAC-family attribution over stores (fit, precondition the test side, score)."""
        self._set_options(damping, non_kfac_strategy, direct_fim_max_params, relative_damping,
                          factor_cache_residency, covariances_at_capture)
        cache_pre = preconditioned_test_dir is not None or preconditioned_test_cache_residency is not None
        if cache_pre and not loop_over_test:
            raise ValueError("preconditioned_test_dir / preconditioned_test_cache_residency only apply to "
                             "loop_over_test=True (otherwise the preconditioned test set is held in memory).")
        if preconditioned_test_cache_residency is not None and preconditioned_test_cache_residency not in CACHE_RESIDENCIES:
            raise ValueError(f"preconditioned_test_cache_residency must be one of {list(CACHE_RESIDENCIES)} or None, "
                             f"got {preconditioned_test_cache_residency!r}.")
        self._set_fit_scope(layer_name, selected_training_steps)
        self._use_fisher_dir(fisher_dir)
        train_store, test_store = self.resolve_store(train_source), self.resolve_store(test_source)
        meta = {"damping": damping, "relative_damping": relative_damping,
                "factor_cache_residency": factor_cache_residency, "non_kfac_strategy": non_kfac_strategy,
                "fisher_dir": fisher_dir, **(algorithm_meta or {})}
        if not cache_pre:
            res = super().attribute_from_cache(train_store, test_store, selected_training_steps=selected_training_steps,
                                               layer_name=layer_name, verbose=verbose, loop_over_test=loop_over_test,
                                               algorithm_meta=meta, attribution_granularity=attribution_granularity)
            return self._stamp(res)
        train = self.load_train_rep(train_store, steps=selected_training_steps, layer_name=layer_name, verbose=verbose)
        test = self.load_test_rep(test_store, layer_name=layer_name, verbose=verbose)
        self.prepare_scoring(train, test)
        with contextlib.ExitStack() as stack:
            if preconditioned_test_dir is not None:
                store = GradientStorageManager(preconditioned_test_dir)
            else:
                store = stack.enter_context(GradientStorageManager(
                    tempfile.mkdtemp(prefix=f"{self.algorithm.lower()}_precond_"),
                    residency=preconditioned_test_cache_residency))
            self.cache_representations(test, store, sample_id_key=test_store.sample_id_key)
            pre = self.load_test_rep(store, desc=f"{self.algorithm}: preconditioned test")
            scores, rids, rsteps, tids, rtoks = self.score_sources(
                train, pre, loop_over_test=True, transform_test=lambda b: b,
                attribution_granularity=attribution_granularity)
        res = self.build_score(scores, rids, rsteps, tids,
                               algorithm_meta={"selected_training_steps": train.steps,
                                               **self.stores_meta(train_store, test_store),
                                               "attribution_granularity": attribution_granularity, **meta},
                               layer_name=train.layer_name, row_token_ids=rtoks)
        return self._stamp(res)

    def _stamp(self, result):
        if self._preconditioner is not None:
            result.algorithm_meta["direct_fim_layers"] = sorted(self._preconditioner[1])
        return result

    def cache_preconditioned_test(self, train_gradients_dir: str, test_gradients_dir: str,
                                  preconditioned_test_dir: str | None = None, *, damping: float = 1e-3,
                                  selected_training_steps=None, non_kfac_strategy: str = "ignore",
                                  direct_fim_max_params: int = 4096, layer_name=None, verbose: bool = False,
                                  relative_damping: bool = False, factor_cache_residency=None,
                                  covariances_at_capture: bool = True) -> str:
        """Fit on the train store and write the preconditioned test set as a store (score it
        later with ``TracInAttributor.attribute_from_cache``)."""
        preconditioned_test_dir = preconditioned_test_dir or str(
            Path(self.args.output_dir) / f"{self.algorithm.lower()}_preconditioned_test")
        self._set_options(damping, non_kfac_strategy, direct_fim_max_params, relative_damping,
                          factor_cache_residency, covariances_at_capture)
        train = self.load_train_rep(train_gradients_dir, steps=selected_training_steps, layer_name=layer_name,
                                    verbose=verbose, desc=f"{self.algorithm}: train (fitting)")
        ts = GradientStorageManager(test_gradients_dir)
        test = self.load_test_rep(ts, layer_name=layer_name, verbose=verbose, desc=f"{self.algorithm}: test (raw)")
        self.prepare_scoring(train, test)
        self.cache_representations(test, GradientStorageManager(preconditioned_test_dir), sample_id_key=ts.sample_id_key)
        return preconditioned_test_dir


class KFACAttributor(KroneckerAttributor):
    """K-FAC influence: one sweep of covariances, damped eigen-inverses."""

    algorithm: ClassVar[str] = "KFAC"

    def fit_factors(self, train_source, fisher_acc):
        """``{layer: (A, G)}`` (supplied capture-time covariances are used as is)."""
        supplied = self._capture_covariances or {}
        kron = ops.KroneckerAccumulator()
        for _s, block, _h in train_source:
            g = block.to(self.args.device)
            kron.update(g, [n for n in self.kfac_layers(g) if n not in supplied])
            self.accumulate_fisher(fisher_acc, g)
        kron.all_reduce()
        fisher_acc.all_reduce()
        factors = self._factor_map()
        for layer, cov in {**kron.result(consume=True), **supplied}.items():
            factors[layer] = cov
        return factors

    def damp(self, raw_factors, damping):
        """``(A + dI)^-1, (G + dI)^-1``."""
        return {layer: (ops.sym_inverse(A, self._damping_for(damping, _mean_eigenvalue(A))),
                        ops.sym_inverse(G, self._damping_for(damping, _mean_eigenvalue(G))))
                for layer, (A, G) in raw_factors.items()}

    def precondition_test_layer(self, value, layer_type, factors):
        """``G^-1 dW A^-1`` (factorized test layers stay factorized)."""
        a_inv, g_inv = factors
        if isinstance(value, torch.Tensor):
            return ops.kfac_precondition_materialized(value, a_inv, g_inv)
        a, g = ops.kfac_precondition(value, layer_type, a_inv, g_inv)
        return Factorized(a, g, module_kwargs=None, batch_first=True)


class EKFACAttributor(KroneckerAttributor):
    """EK-FAC influence: Kronecker eigenbases, then a second sweep fitting the eigenvalues."""

    algorithm: ClassVar[str] = "EKFAC"
    EKFAC_MODES = ("exact", "approx")

    def __init__(self, args, *, task=None, mode: str = "exact") -> None:
        if mode not in self.EKFAC_MODES:
            raise ValueError(f"mode must be one of {self.EKFAC_MODES}, got {mode!r}.")
        super().__init__(args, task=task)
        self.mode = mode

    def fit_factors(self, train_source, fisher_acc):
        """``{layer: (U_A, U_G, lambda)}`` with ``lambda = E[(U_G^T dW U_A)^2]``."""
        dev = self.args.device
        supplied = self._capture_covariances
        eig = self._factor_map()
        if supplied is None:
            kron = ops.KroneckerAccumulator()
            for _s, block, _h in train_source:
                g = block.to(dev)
                kron.update(g, self.kfac_layers(g))
                self.accumulate_fisher(fisher_acc, g)
            kron.all_reduce()
            fisher_acc.all_reduce()
            cov = kron.result(consume=True)
        else:
            cov = dict(supplied)
        for layer in list(cov):
            A, G = cov.pop(layer)
            _, u_a, _, u_g = ops.kfac_eigh(A.to(dev), G.to(dev))
            eig[layer] = (u_a, u_g)
        lam: dict[str, torch.Tensor] = {}
        counts: dict[str, int] = {}
        for _s, block, _h in (train_source if (eig or supplied) else ()):
            g = block.to(dev)
            if supplied is not None:
                missing = [n for n in self.kfac_layers(g) if n not in eig]
                if missing:
                    raise ValueError("fit(covariances=...) must cover every K-FAC-eligible layer of the store; "
                                     f"missing: {sorted(missing)}.")
                self.accumulate_fisher(fisher_acc, g)
            for layer, (u_a, u_g) in eig.items():
                if layer not in g.data:
                    continue
                lam[layer], n = ops.ekfac_lambda_accumulate(g.data[layer], g.layer_types[layer], u_a.to(dev),
                                                            u_g.to(dev), lam.get(layer))
                counts[layer] = counts.get(layer, 0) + n
        for layer in sorted(lam):
            all_reduce_sum(lam[layer])
            counts[layer] = int(all_reduce_sum(torch.tensor([counts[layer]], dtype=torch.int64)).item())
        if supplied is not None:
            fisher_acc.all_reduce()
        factors = self._factor_map()
        for layer in list(eig):
            u_a, u_g = eig[layer]
            factors[layer] = (u_a, u_g, lam.pop(layer).div_(counts[layer]))
        if isinstance(eig, _FactorCache):
            eig.close()
            self._factor_caches.remove(eig)
        return factors

    def damp(self, raw_factors, damping):
        """Eigenvalues damped by ``damping`` (relative: times their mean)."""
        return {layer: (u_a, u_g, lam + self._damping_for(damping, lam.mean()))
                for layer, (u_a, u_g, lam) in raw_factors.items()}

    def precondition_test_layer(self, value, layer_type, factors):
        """``U_G ((U_G^T dW U_A) / lambda) U_A^T`` (dense)."""
        u_a, u_g, lam = factors
        return ops.ekfac_precondition(ops.ekfac_materialize(value, layer_type, u_a, u_g), u_a, u_g, lam, layer_type)
