"""K-FAC and EK-FAC influence attributors.

Score = ``<g_train, F^-1 g_test>`` with the Fisher ``F`` of every linear layer taken as a
Kronecker product ``A (x) G`` of its input-activation and output-gradient covariances:

* K-FAC preconditions a query layer as ``G^-1 dW A^-1`` with damped inverses;
* EK-FAC works in the eigenbases ``U_A``, ``U_G`` of the two factors and replaces the
  Kronecker eigenvalues by ones fitted on the data, ``lambda = E[(U_G^T dW U_A)^2]``:
  ``U_G ((U_G^T dW U_A) / (lambda + damping)) U_A^T``.

Only the queries are preconditioned; training rows are scored raw with a plain dot.
Layers without Kronecker factors (stored materialized, or norm layers under
``non_kfac_strategy="direct"``) use a dense empirical Fisher, bounded by
``direct_fim_max_params``.  ``A`` and ``G`` come either from the capture itself (a
:class:`KroneckerCovarianceCallback` riding on the training stream, the default) or from a
fit pass over the stored training gradients.  A fit can be saved to and reused from
``<fisher_dir>/fisher_factors.pt``; the options that define it are stored with it and
checked on load.

Reference behaviour: ``dattri_llm/attribution/algorithm/kronecker.py`` (workflow, options,
the fisher-file keys ``meta`` / ``raw_ctx`` / ``raw_fim``).

On the B200 the covariances are split-K tcgen05 Gram GEMMs accumulated in fp32, and every
layer's sums cross ranks in one packed all-reduce.
"""

from __future__ import annotations

import contextlib
import dataclasses
import tempfile
import warnings
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

FISHER_FILE = "fisher_factors.pt"
COVARIANCE_FILE = "kronecker_covariances.pt"
_STRATEGIES = ("ignore", "direct")


def _on(value, device):
    """*value* (a tensor, or a tuple of tensors) on *device*."""
    if isinstance(value, tuple):
        return tuple(t.to(device) for t in value)
    return value.to(device)


def _all_on(table: Mapping, device) -> dict:
    return {k: _on(v, device) for k, v in table.items()}


def _trace_mean(m: torch.Tensor) -> torch.Tensor:
    """The mean eigenvalue of a square matrix (its trace over its order)."""
    return m.diagonal(dim1=-2, dim2=-1).float().mean()


@dataclasses.dataclass(frozen=True)
class KroneckerOptions:
    """The options that shape a K-FAC-family fit and its damping."""

    damping: float = 1e-3
    non_kfac_strategy: str = "ignore"
    direct_fim_max_params: int = 4096
    relative_damping: bool = False
    factor_cache_residency: str | None = None
    covariances_at_capture: bool = True

    def __post_init__(self) -> None:
        if self.damping < 0:
            raise ValueError(f"damping cannot be negative (got {self.damping}).")
        if self.non_kfac_strategy not in _STRATEGIES:
            raise ValueError(f"non_kfac_strategy is one of {_STRATEGIES}, got {self.non_kfac_strategy!r}.")
        if self.direct_fim_max_params <= 0:
            raise ValueError(f"direct_fim_max_params must be at least 1 (got {self.direct_fim_max_params}).")
        if self.factor_cache_residency not in (None, *CACHE_RESIDENCIES):
            raise ValueError(f"factor_cache_residency is None or one of {list(CACHE_RESIDENCIES)}, got "
                             f"{self.factor_cache_residency!r}.")

    def damping_of(self, spectrum_mean) -> float:
        """The damping added to a spectrum: absolute, or relative to its mean eigenvalue."""
        return self.damping * float(spectrum_mean) if self.relative_damping else self.damping


class _FactorTable(Mapping):
    """``{layer: factors}`` held in a host cache of some residency; an entry the cache's
    budget refuses is kept as given."""

    def __init__(self, residency: str) -> None:
        self._cache = TensorCache(residency, budget=CacheBudget())
        self._refused: dict = {}
        self._layers: list[str] = []

    def __setitem__(self, layer: str, factors) -> None:
        self._refused.pop(layer, None)
        if not self._cache.put(layer, _on(factors, "cpu")):
            self._refused[layer] = factors
        if layer not in self._layers:
            self._layers.append(layer)

    def __getitem__(self, layer: str):
        if layer in self._refused:
            return self._refused[layer]
        if layer not in self._cache:
            raise KeyError(layer)
        return self._cache.get(layer)

    def __iter__(self) -> Iterator[str]:
        return iter(self._layers)

    def __len__(self) -> int:
        return len(self._layers)

    def close(self) -> None:
        self._cache.close()
        self._refused.clear()
        self._layers.clear()


class _Tables:
    """The factor tables an attributor has opened, to close those no fit refers to any more."""

    def __init__(self) -> None:
        self.open: list[_FactorTable] = []

    def new(self, residency: str | None):
        if residency is None:
            return {}
        table = _FactorTable(residency)
        self.open.append(table)
        return table

    def drop(self, table) -> None:
        if isinstance(table, _FactorTable):
            table.close()
            self.open = [t for t in self.open if t is not table]

    def retain(self, *keep) -> None:
        for table in [t for t in self.open if not any(t is k for k in keep)]:
            self.drop(table)


class _LayerRouting:
    """Per fit: which layers of a block enter the Kronecker fit and which the dense direct
    Fisher, with what was left out along the way (reported as warnings at the end)."""

    def __init__(self, supplied: Mapping | None, strategy: str, max_params: int) -> None:
        self.supplied = supplied or {}
        self.direct_norms = strategy == "direct"
        self.max_params = max_params
        self.materialized_eligible: set[str] = set()  # K-FAC-eligible, but stored without (a, g)
        self.embeddings: set[str] = set()             # factorized embeddings the direct Fisher skips

    def kronecker(self, block) -> list[str]:
        chosen = []
        for name, value in block.data.items():
            if not ops.is_kfac_eligible(block.layer_types[name]):
                continue
            if isinstance(value, Factorized) or name in self.supplied:
                chosen.append(name)
            else:
                self.materialized_eligible.add(name)
        return chosen

    def direct(self, block) -> list[str]:
        chosen = []
        for name, value in block.data.items():
            kind = block.layer_types[name]
            if kind == ops.PARAM_GRAD_TYPES:
                continue
            dense = isinstance(value, torch.Tensor)
            if dense and name in self.supplied:
                continue  # its Kronecker factors were supplied
            if dense or (self.direct_norms and ops.is_norm(kind)):
                chosen.append(name)
        return chosen

    def add_direct(self, acc: ops.FisherAccumulator, block) -> None:
        acc.update(block, self.direct(block))
        if self.direct_norms:
            self.embeddings.update(n for n, v in block.data.items()
                                   if ops.is_embedding(block.layer_types[n]) and isinstance(v, Factorized))

    def report(self, acc: ops.FisherAccumulator, algorithm: str, n_kronecker: int) -> None:
        if self.materialized_eligible:
            names = sorted(self.materialized_eligible)
            warnings.warn(
                f"{algorithm}: {len(names)} of {len(names) + n_kronecker} linear layers were stored materialized, "
                f"without the (activation, output-gradient) pair a Kronecker factor is built from; they fall back "
                f"to the dense direct Fisher (at most {self.max_params} parameters per layer): {names}. Capture "
                "them factorized, or give fit() capture-time covariances.", stacklevel=3)
        if acc.skipped:
            warnings.warn(f"{algorithm}: layers above direct_fim_max_params={self.max_params} get no direct "
                          f"Fisher: {dict(sorted(acc.skipped.items()))}.", stacklevel=3)
        if self.embeddings:
            warnings.warn(f"{algorithm}: the direct Fisher does not cover embedding layers; left unpreconditioned: "
                          f"{sorted(self.embeddings)}.", stacklevel=3)


class _CaptureCovariances:
    """Kronecker covariances gathered while a training store was being written, kept per
    store (and saved beside a disk store)."""

    def __init__(self) -> None:
        self.by_store: dict[str, dict] = {}
        self.pending = None  # the streamer whose collection should gather them

    @staticmethod
    def _key(root) -> str:
        return str(Path(root).resolve())

    def gather(self, collect, streamer, store, kwargs):
        """Run ``collect(streamer, store, **kwargs)`` with a covariance callback attached."""
        callback = KroneckerCovarianceCallback()
        streamer.hook_manager.add_callback(callback)
        result = collect(streamer, store, **kwargs)
        callback.all_reduce()
        sums = _all_on(callback.result(), torch.device("cpu"))
        self.by_store[self._key(store.save_dir)] = sums
        if store.residency == "disk" and dist_rank() in (None, 0):
            torch.save(sums, Path(store.save_dir) / COVARIANCE_FILE)
        return result

    def lookup(self, source) -> dict | None:
        """The covariances of *source*'s store when they cover the whole source."""
        store = getattr(source, "file_manager", None)
        if store is None or sorted(source.steps) != sorted(resolve_steps(store, None)):
            return None
        root = Path(store.save_dir)
        sums = self.by_store.get(self._key(root))
        if sums is None and (root / COVARIANCE_FILE).exists():
            sums = torch.load(root / COVARIANCE_FILE, map_location="cpu", weights_only=True)
        layers = getattr(source, "layer_name", None)
        if sums is not None and layers is not None:
            sums = {k: v for k, v in sums.items() if k in layers} or None
        return sums


class KroneckerAttributor(BaseInnerProductAttributor):
    """The K-FAC family's workflow.  A variant provides three steps: ``sweep_factors``
    (per-layer factors from the training gradients), ``damped`` (factors ready to
    precondition) and ``precondition_layer`` (one query layer)."""

    algorithm: ClassVar[str] = "Kronecker"
    _UNCHECKED = ("damping", "relative_damping")  # recorded with a fit, free to differ on reuse

    def __init__(self, args, *, task=None) -> None:
        super().__init__(args, task=task)
        self.options = KroneckerOptions()
        self._scope: dict = {"layer_name": None, "selected_training_steps": None}
        self._tables = _Tables()
        self._captured = _CaptureCovariances()
        self._raw: tuple | None = None       # (factors, direct Fisher) before damping
        self._ready: tuple | None = None     # (damped factors, inverse direct Fisher) on the device
        self._supplied: dict | None = None   # covariances to use instead of sweeping A, G
        self._routing: _LayerRouting | None = None
        self._save_to: str | None = None     # fisher_dir to write the next fit into
        self._memo: tuple | None = None      # (fisher-file key, raw fit) of the last fisher_dir read or written

    def uses_plain_inner_product(self) -> bool:
        """Queries are preconditioned, training rows raw: the score is a plain dot."""
        return True

    def sweep_factors(self, train_source, fisher_acc: ops.FisherAccumulator) -> Mapping:
        """Per-layer raw factors from the training source (adding its blocks to the direct Fisher)."""
        raise NotImplementedError

    def damped(self, raw_factors: Mapping) -> dict:
        """Damped (inverted or rescaled) factors."""
        raise NotImplementedError

    def precondition_layer(self, value, layer_type: str, factors):
        """One query layer preconditioned by its factors."""
        raise NotImplementedError

    def checkpoints(self) -> list[int]:
        """``[0]``: the Fisher is taken at one checkpoint; others are ignored."""
        extra = self.num_checkpoints() - 1
        if extra > 0:
            warnings.warn(f"{self.algorithm} uses checkpoint 0 only; the other {extra} checkpoint(s) are ignored.",
                          stacklevel=2)
        return [0]

    # ------------------------------------------------------------ configuration
    def _configure(self, **options) -> None:
        self.options = KroneckerOptions(**options)
        self._raw = self._ready = None
        self._scope = {"layer_name": None, "selected_training_steps": None}
        self._save_to = None

    def _set_scope(self, layer_name, steps) -> None:
        layers = [layer_name] if isinstance(layer_name, str) else layer_name
        self._scope = {"layer_name": None if layers is None else sorted(layers),
                       "selected_training_steps": None if steps is None else sorted(int(s) for s in steps)}

    # ------------------------------------------------------------ fitting
    def fit_raw(self, train_source) -> tuple:
        """``(raw factors, raw direct Fisher)`` of a re-iterable training source.

        Raises:
            ValueError: a single-pass source, or nothing to fit.
        """
        if not getattr(train_source, "reusable", False):
            raise ValueError(f"{self.algorithm} reads the training gradients twice (fit, then score): give it a "
                             "store, a frozen GradientStreamer (enable_update=False), or "
                             "attribute(gradient_cache_residency=...).")
        opts = self.options
        self._routing = _LayerRouting(self._supplied, opts.non_kfac_strategy, opts.direct_fim_max_params)
        acc = ops.FisherAccumulator(opts.direct_fim_max_params)
        factors = self.sweep_factors(train_source, acc)
        self._routing.report(acc, self.algorithm, len(factors))
        direct = dict(acc.result())
        if not factors and not direct:
            hint = ("; non_kfac_strategy='direct' would add norm layers" if opts.non_kfac_strategy == "ignore"
                    else f" and no layer within direct_fim_max_params={opts.direct_fim_max_params}")
            raise ValueError(f"{self.algorithm}: the training gradients hold no linear layer to fit{hint}.")
        return factors, direct

    def _prepare(self, raw: tuple) -> tuple:
        """Damp a raw fit onto the device: ``(damped factors, {layer: inverse direct Fisher})``."""
        factors, direct = raw
        dev = self.args.device
        damped = self._tables.new(self.options.factor_cache_residency)
        for layer in factors:
            damped[layer] = self.damped({layer: _on(factors[layer], dev)})[layer]
        inverses = {}
        for layer, fisher in _all_on(direct, dev).items():
            inverses[layer] = ops.dense_inverse(fisher, self.options.damping_of(_trace_mean(fisher)))
        return damped, inverses

    def prepare_scoring(self, train_source, test_source) -> None:
        """Fit (unless a fit is at hand) and damp the preconditioner."""
        if self._ready is not None:
            return
        if self._raw is None:
            captured = self._captured.lookup(train_source) if self.options.covariances_at_capture else None
            if captured is not None and self._supplied is None:
                self._supplied = _all_on(captured, self.args.device)
                try:
                    self._raw = self.fit_raw(train_source)
                finally:
                    self._supplied = None
            else:
                self._raw = self.fit_raw(train_source)
        self._ready = self._prepare(self._raw)
        factors, direct = self._raw
        self._raw = (factors, _all_on(direct, "cpu")) if isinstance(factors, _FactorTable) else (
            _all_on(factors, "cpu"), _all_on(direct, "cpu"))
        if self._save_to is not None:
            self.save_fisher(self._raw[0], self._save_to, fisher=self._raw[1])
            self._memo = (self._file_key(self._save_to), self._raw)
            self._save_to = None
        memo_factors = () if self._memo is None else (self._memo[1][0],)
        self._tables.retain(self._raw[0], self._ready[0], *memo_factors)

    def transform_test_rep(self, test_rep):
        """Every query layer with a fit, preconditioned (layers without one are dropped).

        Raises:
            RuntimeError: before :meth:`prepare_scoring`.
        """
        if self._ready is None:
            raise RuntimeError(f"{self.algorithm}: prepare_scoring() runs before queries can be preconditioned.")
        factors, inverses = self._ready
        dev = test_rep.device

        def precondition(name, value, kind):
            if name in factors:
                return self.precondition_layer(value, kind, _on(factors[name], dev))
            if name in inverses:
                return ops.materialize(value, kind).float() @ inverses[name]
            return None

        return test_rep.map_layers(precondition)

    # ------------------------------------------------------------ capture-time covariances
    def generate_train_rep(self, train_dataset, **kwargs):
        """The training streamer; a frozen probe's collection also gathers its covariances."""
        streamer = super().generate_train_rep(train_dataset, **kwargs)
        wanted = self.options.covariances_at_capture and not kwargs.get("enable_update")
        self._captured.pending = streamer if wanted else None
        return streamer

    def collect_gradients(self, streamer, store, **kwargs):
        """Collect into *store*; the pending training streamer also gathers ``(A, G)``."""
        base = super().collect_gradients
        if streamer is not self._captured.pending:
            return base(streamer, store, **kwargs)
        self._captured.pending = None
        if kwargs.get("resume") and any(step == streamer.checkpoint_step for step, _ in store.own_records()):
            # a resumed collection would miss the skipped batches: the fit sweeps the store instead
            return base(streamer, store, **kwargs)
        return self._captured.gather(base, streamer, store, kwargs)

    def cache(self, train_dataset, test_dataset, *, covariances_at_capture: bool | None = None, **kwargs):
        """Collect the training and query stores (covariances gathered during capture unless
        *covariances_at_capture* is false)."""
        if covariances_at_capture is not None:
            self.options = dataclasses.replace(self.options, covariances_at_capture=covariances_at_capture)
        return super().cache(train_dataset, test_dataset, **kwargs)

    # ------------------------------------------------------------ fisher files
    def _file_meta(self) -> dict:
        opts = self.options
        meta = {"algorithm": self.algorithm, "non_kfac_strategy": opts.non_kfac_strategy,
                "direct_fim_max_params": opts.direct_fim_max_params, **self._scope,
                "damping": opts.damping, "relative_damping": opts.relative_damping}
        mode = getattr(self, "mode", None)
        if mode is not None:
            meta["mode"] = mode
        return meta

    def _file_key(self, fisher_dir: str) -> tuple:
        path = Path(fisher_dir) / FISHER_FILE
        checked = sorted((k, v) for k, v in self._file_meta().items() if k not in self._UNCHECKED)
        return str(path.resolve()), path.stat().st_mtime_ns, repr(checked), self.options.factor_cache_residency

    def _from_fisher_dir(self, fisher_dir: str | None) -> None:
        """Reuse the fit in *fisher_dir*, or arrange for the next fit to be written there."""
        if fisher_dir is None:
            return
        if not (Path(fisher_dir) / FISHER_FILE).exists():
            self._save_to = fisher_dir
            return
        key = self._file_key(fisher_dir)
        if self._memo is None or self._memo[0] != key:
            self._memo = (key, self.load_fisher(fisher_dir))
        self._raw = self._memo[1]

    def _default_fisher_dir(self) -> str:
        return str(Path(self.args.output_dir) / f"{self.algorithm.lower()}_fisher")

    def save_fisher(self, covariances: Mapping, fisher_dir: str | None = None, *, fisher: dict | None = None) -> str:
        """Write ``fisher_factors.pt`` -- raw factors, raw direct Fisher and the options that
        define them -- by an atomic rename.  Returns the directory."""
        fisher_dir = fisher_dir or self._default_fisher_dir()
        root = Path(fisher_dir)
        root.mkdir(parents=True, exist_ok=True)
        blob = {"meta": self._file_meta(), "raw_ctx": _all_on(covariances, "cpu"),
                "raw_fim": _all_on(fisher or {}, "cpu")}
        staging = root / f"{FISHER_FILE}.rank{dist_rank() or 0}.partial"
        torch.save(blob, staging)
        staging.replace(root / FISHER_FILE)
        return fisher_dir

    def load_fisher(self, fisher_dir: str) -> tuple:
        """A saved fit, after checking it was made by this algorithm under the same options.

        Raises:
            ValueError: no fit there, another algorithm's, or other options.
        """
        path = Path(fisher_dir) / FISHER_FILE
        if not path.exists():
            raise ValueError(f"{path} does not exist: build it first with {type(self).__name__}.fit("
                             f"train_gradients_dir, {fisher_dir!r}).")
        blob = torch.load(path, map_location="cpu", weights_only=True)
        saved = blob["meta"]
        if saved.get("algorithm") != self.algorithm:
            raise ValueError(f"{path} is a {saved.get('algorithm')!r} fit, not {self.algorithm}.")
        clash = {k: (saved.get(k), v) for k, v in self._file_meta().items()
                 if k not in self._UNCHECKED and saved.get(k) != v}
        if clash:
            raise ValueError(f"{path} was fitted under other options ((saved, requested) per option): {clash}.")
        dev = self.args.device
        direct = _all_on(blob["raw_fim"], dev)
        if self.options.factor_cache_residency is None:
            return _all_on(blob["raw_ctx"], dev), direct
        table = self._tables.new(self.options.factor_cache_residency)
        for layer, value in blob["raw_ctx"].items():
            table[layer] = value
        return table, direct

    def fit(self, train_gradients_dir: str, fisher_dir: str | None = None, *,
            selected_training_steps: Iterable[int] | None = None, non_kfac_strategy: str = "ignore",
            direct_fim_max_params: int = 4096, layer_name=None, verbose: bool = False, covariances=None,
            factor_cache_residency: str | None = None, covariances_at_capture: bool = True) -> str:
        """Fit over a training store and save the fit; returns the fisher directory."""
        self._configure(damping=self.options.damping, non_kfac_strategy=non_kfac_strategy,
                        direct_fim_max_params=direct_fim_max_params, relative_damping=self.options.relative_damping,
                        factor_cache_residency=factor_cache_residency, covariances_at_capture=covariances_at_capture)
        self._set_scope(layer_name, selected_training_steps)
        train = self.load_train_rep(train_gradients_dir, steps=selected_training_steps, layer_name=layer_name,
                                    verbose=verbose, desc=f"{self.algorithm}: fitting")
        if covariances is None and covariances_at_capture:
            covariances = self._captured.lookup(train)
        self._supplied = None if covariances is None else _all_on(covariances, self.args.device)
        try:
            factors, direct = self.fit_raw(train)
        finally:
            self._supplied = None
        out = self.save_fisher(factors, fisher_dir, fisher=direct)
        self._tables.drop(factors)
        return out

    # ------------------------------------------------------------ workflows
    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, gradient_cache_residency=None,
                  attribution_granularity: str = "instance", damping: float = 1e-3,
                  non_kfac_strategy: str = "ignore", direct_fim_max_params: int = 4096,
                  relative_damping: bool = False, factor_cache_residency=None, covariances_at_capture: bool = True,
                  fisher_dir: str | None = None):
        """Live attribution at checkpoint 0 (a frozen probe: the Fisher needs fixed parameters)."""
        options = {"damping": damping, "non_kfac_strategy": non_kfac_strategy,
                   "direct_fim_max_params": direct_fim_max_params, "relative_damping": relative_damping,
                   "factor_cache_residency": factor_cache_residency, "covariances_at_capture": covariances_at_capture}
        self._configure(**options)
        if gradient_cache_residency is None:
            self._from_fisher_dir(fisher_dir)
        forwarded = dict(options, fisher_dir=fisher_dir)
        if gradient_cache_residency is not None and loop_over_test:
            forwarded["preconditioned_test_cache_residency"] = gradient_cache_residency
        return super().attribute(train_dataset, test_dataset, hook_config=hook_config, verbose=verbose,
                                 loop_over_test=loop_over_test, enable_update=False,
                                 gradient_cache_residency=gradient_cache_residency,
                                 attribution_granularity=attribution_granularity, **forwarded)

    def attribute_from_cache(self, train_source, test_source, *, selected_training_steps=None, layer_name=None,
                             verbose: bool = False, loop_over_test: bool = False, algorithm_meta=None,
                             attribution_granularity: str = "instance", damping: float = 1e-3,
                             preconditioned_test_dir: str | None = None,
                             preconditioned_test_cache_residency: str | None = None, fisher_dir: str | None = None,
                             non_kfac_strategy: str = "ignore", direct_fim_max_params: int = 4096,
                             relative_damping: bool = False, factor_cache_residency=None,
                             covariances_at_capture: bool = True):
        """Attribution over stores: fit (or reuse a fit), precondition the queries, score.
        With ``loop_over_test`` the preconditioned queries can go through a store of their
        own (*preconditioned_test_dir*, or a temporary one of the given residency)."""
        self._configure(damping=damping, non_kfac_strategy=non_kfac_strategy,
                        direct_fim_max_params=direct_fim_max_params, relative_damping=relative_damping,
                        factor_cache_residency=factor_cache_residency, covariances_at_capture=covariances_at_capture)
        staged = preconditioned_test_dir is not None or preconditioned_test_cache_residency is not None
        if staged and not loop_over_test:
            raise ValueError("a preconditioned query store (preconditioned_test_dir / "
                             "preconditioned_test_cache_residency) is used with loop_over_test=True only; without "
                             "it the preconditioned queries stay in memory.")
        if preconditioned_test_cache_residency not in (None, *CACHE_RESIDENCIES):
            raise ValueError(f"preconditioned_test_cache_residency is None or one of {list(CACHE_RESIDENCIES)}, "
                             f"got {preconditioned_test_cache_residency!r}.")
        self._set_scope(layer_name, selected_training_steps)
        self._from_fisher_dir(fisher_dir)
        train_store, test_store = self.resolve_store(train_source), self.resolve_store(test_source)
        meta = {"damping": damping, "relative_damping": relative_damping,
                "factor_cache_residency": factor_cache_residency, "non_kfac_strategy": non_kfac_strategy,
                "fisher_dir": fisher_dir, **(algorithm_meta or {})}
        if not staged:
            result = super().attribute_from_cache(
                train_store, test_store, selected_training_steps=selected_training_steps, layer_name=layer_name,
                verbose=verbose, loop_over_test=loop_over_test, algorithm_meta=meta,
                attribution_granularity=attribution_granularity)
            return self._with_direct_layers(result)
        train = self.load_train_rep(train_store, steps=selected_training_steps, layer_name=layer_name, verbose=verbose)
        test = self.load_test_rep(test_store, layer_name=layer_name, verbose=verbose)
        self.prepare_scoring(train, test)
        with contextlib.ExitStack() as scope:
            if preconditioned_test_dir is not None:
                staging = GradientStorageManager(preconditioned_test_dir)
            else:
                staging = scope.enter_context(GradientStorageManager(
                    tempfile.mkdtemp(prefix=f"{self.algorithm.lower()}_precond_"),
                    residency=preconditioned_test_cache_residency))
            self.cache_representations(test, staging, sample_id_key=test_store.sample_id_key)
            queries = self.load_test_rep(staging, desc=f"{self.algorithm}: preconditioned queries")
            scores, rids, rsteps, tids, rtoks = self.score_sources(
                train, queries, loop_over_test=True, transform_test=lambda block: block,
                attribution_granularity=attribution_granularity)
        result = self.build_score(scores, rids, rsteps, tids,
                                  algorithm_meta={"selected_training_steps": train.steps,
                                                  **self.stores_meta(train_store, test_store),
                                                  "attribution_granularity": attribution_granularity, **meta},
                                  layer_name=train.layer_name, row_token_ids=rtoks)
        return self._with_direct_layers(result)

    def _with_direct_layers(self, result):
        if self._ready is not None:
            result.algorithm_meta["direct_fim_layers"] = sorted(self._ready[1])
        return result

    def cache_preconditioned_test(self, train_gradients_dir: str, test_gradients_dir: str,
                                  preconditioned_test_dir: str | None = None, *, damping: float = 1e-3,
                                  selected_training_steps=None, non_kfac_strategy: str = "ignore",
                                  direct_fim_max_params: int = 4096, layer_name=None, verbose: bool = False,
                                  relative_damping: bool = False, factor_cache_residency=None,
                                  covariances_at_capture: bool = True) -> str:
        """Fit on the training store and write the preconditioned queries as a store of their
        own (scored later by ``TracInAttributor.attribute_from_cache``).  Returns its directory."""
        out_dir = preconditioned_test_dir or str(Path(self.args.output_dir)
                                                 / f"{self.algorithm.lower()}_preconditioned_test")
        self._configure(damping=damping, non_kfac_strategy=non_kfac_strategy,
                        direct_fim_max_params=direct_fim_max_params, relative_damping=relative_damping,
                        factor_cache_residency=factor_cache_residency, covariances_at_capture=covariances_at_capture)
        train = self.load_train_rep(train_gradients_dir, steps=selected_training_steps, layer_name=layer_name,
                                    verbose=verbose, desc=f"{self.algorithm}: fitting")
        queries_store = GradientStorageManager(test_gradients_dir)
        queries = self.load_test_rep(queries_store, layer_name=layer_name, verbose=verbose,
                                     desc=f"{self.algorithm}: raw queries")
        self.prepare_scoring(train, queries)
        self.cache_representations(queries, GradientStorageManager(out_dir),
                                   sample_id_key=queries_store.sample_id_key)
        return out_dir

    # ------------------------------------------------------------ shared sweep
    def _sweep_covariances(self, train_source, fisher_acc, skip: Mapping = ()) -> dict:
        """One pass: ``{layer: (A, G)}`` over the Kronecker layers not in *skip*, and the
        direct Fisher, both summed over ranks."""
        kron = ops.KroneckerAccumulator()
        for _step, block, _ids in train_source:
            block = block.to(self.args.device)
            kron.update(block, [n for n in self._routing.kronecker(block) if n not in skip])
            self._routing.add_direct(fisher_acc, block)
        kron.all_reduce()
        fisher_acc.all_reduce()
        return kron.result(consume=True)


class KFACAttributor(KroneckerAttributor):
    """K-FAC influence: one covariance pass, damped inverses of both factors."""

    algorithm: ClassVar[str] = "KFAC"

    def sweep_factors(self, train_source, fisher_acc):
        """``{layer: (A, G)}``; supplied capture-time covariances are taken as they are."""
        supplied = self._supplied or {}
        covariances = self._sweep_covariances(train_source, fisher_acc, skip=supplied)
        table = self._tables.new(self.options.factor_cache_residency)
        for layer, pair in {**covariances, **supplied}.items():
            table[layer] = pair
        return table

    def damped(self, raw_factors):
        """``((A + d_A I)^-1, (G + d_G I)^-1)`` per layer."""
        out = {}
        for layer, (a_cov, g_cov) in raw_factors.items():
            out[layer] = (ops.sym_inverse(a_cov, self.options.damping_of(_trace_mean(a_cov))),
                          ops.sym_inverse(g_cov, self.options.damping_of(_trace_mean(g_cov))))
        return out

    def precondition_layer(self, value, layer_type, factors):
        """``G^-1 dW A^-1``; a factorized query stays factorized."""
        a_inv, g_inv = factors
        if isinstance(value, torch.Tensor):
            return ops.kfac_precondition_materialized(value, a_inv, g_inv)
        a, g = ops.kfac_precondition(value, layer_type, a_inv, g_inv)
        return Factorized(a, g, module_kwargs=None, batch_first=True)


class EKFACAttributor(KroneckerAttributor):
    """EK-FAC influence: the Kronecker eigenbases, then a second pass fitting the
    eigenvalues in them."""

    algorithm: ClassVar[str] = "EKFAC"
    EKFAC_MODES = ("exact", "approx")

    def __init__(self, args, *, task=None, mode: str = "exact") -> None:
        if mode not in self.EKFAC_MODES:
            raise ValueError(f"mode is one of {self.EKFAC_MODES}, got {mode!r}.")
        super().__init__(args, task=task)
        self.mode = mode

    def _eigenbases(self, covariances: dict) -> Mapping:
        """``{layer: (U_A, U_G)}``.  Factors of one size are eigendecomposed together, one
        batched call per size and memory budget (capture-time projections make every factor
        k x k: two calls instead of two per layer, each of which waits for the device)."""
        dev = self.args.device
        bases = self._tables.new(self.options.factor_cache_residency)
        layers = list(covariances)
        by_size: dict[int, list[tuple[str, int, torch.Tensor]]] = {}
        for layer in layers:
            for side, cov in enumerate(covariances.pop(layer)):
                by_size.setdefault(int(cov.shape[-1]), []).append((layer, side, cov))
        vectors: dict[tuple[str, int], torch.Tensor] = {}
        budget = 1 << 30  # bytes of fp32 factors per batched call
        for n, items in by_size.items():
            per_call = max(1, budget // (4 * n * n))
            for i in range(0, len(items), per_call):
                chunk = items[i:i + per_call]
                stacked = torch.stack([cov.to(dev).float() for _, _, cov in chunk])
                _, u = torch.linalg.eigh(stacked)
                for (layer, side, _), u_i in zip(chunk, u.unbind(0), strict=True):
                    vectors[(layer, side)] = u_i
        for layer in layers:
            bases[layer] = (vectors[(layer, 0)], vectors[(layer, 1)])
        return bases

    def sweep_factors(self, train_source, fisher_acc):
        """``{layer: (U_A, U_G, lambda)}`` with ``lambda = E[(U_G^T dW U_A)^2]`` over samples."""
        dev = self.args.device
        supplied = self._supplied
        covariances = dict(supplied) if supplied is not None else self._sweep_covariances(train_source, fisher_acc)
        bases = self._eigenbases(covariances)
        sums: dict[str, torch.Tensor] = {}
        counts: dict[str, int] = {}
        if bases or supplied is not None:
            for _step, block, _ids in train_source:
                block = block.to(dev)
                if supplied is not None:
                    # the covariance pass was skipped: this pass also checks coverage and feeds the direct Fisher
                    uncovered = [n for n in self._routing.kronecker(block) if n not in bases]
                    if uncovered:
                        raise ValueError("capture-time covariances given to fit() must cover every linear layer "
                                         f"of the store; missing: {sorted(uncovered)}.")
                    self._routing.add_direct(fisher_acc, block)
                for layer in bases:
                    if layer not in block.data:
                        continue
                    u_a, u_g = bases[layer]
                    sums[layer], n = ops.ekfac_lambda_accumulate(block.data[layer], block.layer_types[layer],
                                                                 u_a.to(dev), u_g.to(dev), sums.get(layer))
                    counts[layer] = counts.get(layer, 0) + n
        for layer in sorted(sums):
            all_reduce_sum(sums[layer])
            counts[layer] = int(all_reduce_sum(torch.tensor([counts[layer]], dtype=torch.int64)).item())
        if supplied is not None:
            fisher_acc.all_reduce()
        table = self._tables.new(self.options.factor_cache_residency)
        for layer in list(bases):
            u_a, u_g = bases[layer]
            table[layer] = (u_a, u_g, sums.pop(layer).div_(counts[layer]))
        self._tables.drop(bases)
        return table

    def damped(self, raw_factors):
        """The fitted eigenvalues plus the damping (relative: times their mean)."""
        return {layer: (u_a, u_g, lam + self.options.damping_of(lam.mean()))
                for layer, (u_a, u_g, lam) in raw_factors.items()}

    def precondition_layer(self, value, layer_type, factors):
        """``U_G ((U_G^T dW U_A) / lambda) U_A^T``, dense."""
        u_a, u_g, lam = factors
        rotated = ops.ekfac_materialize(value, layer_type, u_a, u_g)
        return ops.ekfac_precondition(rotated, u_a, u_g, lam, layer_type)
