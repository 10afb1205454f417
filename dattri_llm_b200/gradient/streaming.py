"""Gradient sources: stored (:class:`DiskGradientSource`), live (:class:`GradientStreamer`)
and replayed from trajectory snapshots (:class:`ReplayGradientSource`).

Every source yields ``(step, Gradient, hashes)`` blocks -- the one contract the attributors
consume.  Public names and constructor keywords are the reference's
(``dattri_llm/gradient/streaming.py``).

:class:`GradientStreamer` runs a training-step loop under a :class:`HookManager`: a loader
(``DistributedSampler`` under distributed execution), the model on this device or wrapped
for DDP / FSDP (a frozen probe under ``fsdp=full_shard`` on sm_100 GPUs shards its linears
in place instead, with the weight all-gather inside their GEMMs), and per batch one
``loss_fn(model, batch)`` + backward.  Two modes:

* frozen probe (``enable_update=False``): gradients at fixed parameters; whatever the pass
  changed (parameter ``.grad``, train/eval modes, RNG states) is put back afterwards, so a
  probe can share a model with a training loop;
* trajectory (``enable_update=True``): optimizer / scheduler steps per accumulation window,
  gradient clipping, one step label per batch, learning rates recorded per step,
  optionally the parameters and batches saved for replay.

Data path on the B200: host batches are pinned and moved with ``non_blocking=True``; their
content hashes are computed on a side thread from the host copy while the GPU runs the
step, and handed to the manager once the first step shows they equal the hash of what the
model was fed.
"""

from __future__ import annotations

import contextlib
import functools
import logging
import warnings
from collections.abc import Callable, Iterable, Iterator
from concurrent.futures import Future, ThreadPoolExecutor
from contextlib import AbstractContextManager
from typing import Protocol, runtime_checkable

import torch
from torch import nn
from torch.utils.data import DataLoader, Dataset, DistributedSampler

from dattri_llm_b200.gradient.callbacks import CaptureCallback
from dattri_llm_b200.gradient.datasets import iter_gradient_blocks, resolve_steps
from dattri_llm_b200.gradient.gradient import Gradient
from dattri_llm_b200.gradient.hooks import REGISTER_ALL, HookManager, HookManagerConfig
from dattri_llm_b200.gradient.snapshots import TrajectorySnapshots
from dattri_llm_b200.utils.hashing import hash_batch
from dattri_llm_b200.utils.tracing import trace_range

logger = logging.getLogger(__name__)
StreamBatch = tuple[int, Gradient, list[str]]
LossFn = Callable[[nn.Module, object], torch.Tensor]


@runtime_checkable
class GradientSource(Protocol):
    """Iterable of ``(step, Gradient, hashes)``; ``reusable`` sources can be iterated again."""

    def __iter__(self) -> Iterator[StreamBatch]: ...

    def __len__(self) -> int: ...

    @property
    def reusable(self) -> bool: ...


def _layer_list(layer_name: str | list[str] | None) -> list[str] | None:
    if layer_name is None:
        return None
    return [layer_name] if isinstance(layer_name, str) else list(layer_name)


def _record_hashes(record) -> list[str]:
    return list(record.input_hash) if isinstance(record.input_hash, list) else [record.input_hash]


class DiskGradientSource(GradientSource):
    """A re-iterable source over a :class:`GradientStorageManager` (any residency), optionally
    restricted to some steps and layers."""

    def __init__(self, file_manager, args, *, steps: Iterable[int] | None = None,
                 layer_name: str | list[str] | None = None, desc: str | None = None,
                 verbose: bool = False) -> None:
        self.file_manager = file_manager
        self.args = args
        self._layers = _layer_list(layer_name)
        self._steps = resolve_steps(file_manager, steps)
        self._desc, self._verbose = desc, verbose

    @property
    def reusable(self) -> bool:
        """Always true: the store can be read again."""
        return True

    @property
    def steps(self) -> list[int]:
        """The steps this source yields."""
        return list(self._steps)

    @property
    def layer_name(self) -> list[str] | None:
        """The layer filter (``None``: every layer)."""
        return None if self._layers is None else list(self._layers)

    def __len__(self) -> int:
        return sum(len(records) for _step, records in self.file_manager.iter_steps(self._steps))

    def __iter__(self) -> Iterator[StreamBatch]:
        return iter_gradient_blocks(self.file_manager, self._steps, self.args, layer_name=self._layers,
                                    desc=self._desc, verbose=self._verbose)

    def for_steps(self, steps: Iterable[int]) -> DiskGradientSource:
        """The same store restricted to *steps*."""
        return DiskGradientSource(self.file_manager, self.args, steps=steps, layer_name=self._layers,
                                  desc=self._desc, verbose=False)


class _MergedBlocks:
    """Dense blocks being concatenated along the sample axis.  A sample-indexed layer that
    some blocks lack (a routed expert that none of their tokens reached) gets zero rows for
    them: its gradient for those samples is zero."""

    def __init__(self) -> None:
        self.parts: dict[str, list[torch.Tensor]] = {}
        self.kinds: dict[str, tuple] = {}  # layer -> (representation, layer type, indexing)
        self.ids: list[str] = []
        self.steps: list[int] = []

    def fits(self, block) -> bool:
        """Whether *block* can join: every layer only one side has is sample-indexed."""
        for name in set(block.data) ^ set(self.parts):
            indexing = block.indexing[name] if name in block.data else self.kinds[name][2]
            if indexing != "batch":
                return False
        return True

    def add(self, step: int, block, hashes) -> None:
        before, n = len(self.ids), block.batch_size
        for name, t in block.data.items():
            if name not in self.parts:
                self.parts[name] = [t.new_zeros((before, *t.shape[1:]))] if before else []
                self.kinds[name] = (block.representation[name], block.layer_types[name], block.indexing[name])
            self.parts[name].append(t)
        for name, ts in self.parts.items():
            if name not in block.data:
                ts.append(ts[-1].new_zeros((n, *ts[-1].shape[1:])))
        self.ids.extend(hashes)
        self.steps.extend([step] * n)

    def take(self):
        data = {n: ts[0] if len(ts) == 1 else torch.cat(ts) for n, ts in self.parts.items()}
        rep = {n: k[0] for n, k in self.kinds.items()}
        types = {n: k[1] for n, k in self.kinds.items()}
        idx = {n: k[2] for n, k in self.kinds.items()}
        merged = (self.steps, Gradient(rep, data, types, idx, validate_on_init=False), self.ids)
        self.__init__()
        return merged


def rebatch_blocks(source: Iterable[StreamBatch], batch_size: int):
    """Merge consecutive all-dense blocks until each holds at least *batch_size* samples
    (a block with factorized layers is passed through on its own, after flushing what is
    pending).  Yields ``(step of every row, block, hashes)``."""
    if batch_size < 1:
        raise ValueError(f"batch_size must be at least 1, got {batch_size}.")
    pending = _MergedBlocks()
    for step, block, hashes in source:
        if not all(isinstance(v, torch.Tensor) for v in block.data.values()):
            if pending.ids:
                yield pending.take()
            yield [step] * block.batch_size, block, list(hashes)
            continue
        if not pending.fits(block):
            yield pending.take()
        pending.add(step, block, hashes)
        if len(pending.ids) >= batch_size:
            yield pending.take()
    if pending.ids:
        yield pending.take()


def _auto_wrap_policy(model: nn.Module, fsdp_config: dict) -> Callable | None:
    """FSDP's auto-wrap policy from the Hugging Face-style ``fsdp_config`` keys
    (``transformer_layer_cls_to_wrap`` or ``min_num_params``), removing them from the dict."""
    if "auto_wrap_policy" in fsdp_config:
        return None
    by_class = fsdp_config.pop("transformer_layer_cls_to_wrap", None)
    by_size = fsdp_config.pop("min_num_params", None)
    if by_class is not None and by_size is not None:
        raise ValueError("fsdp_config takes transformer_layer_cls_to_wrap or min_num_params, not both.")
    if by_size is not None:
        from torch.distributed.fsdp.wrap import size_based_auto_wrap_policy

        return functools.partial(size_based_auto_wrap_policy, min_num_params=int(by_size))
    if by_class is None:
        return None
    from torch.distributed.fsdp.wrap import transformer_auto_wrap_policy

    names = {by_class} if isinstance(by_class, str) else set(by_class)
    found = {type(m) for m in model.modules() if type(m).__name__ in names}
    absent = names - {cls.__name__ for cls in found}
    if absent:
        raise ValueError(f"transformer_layer_cls_to_wrap: the model has no module of class {sorted(absent)}.")
    return functools.partial(transformer_auto_wrap_policy, transformer_layer_cls=found)


def _default_loss_fn(model: nn.Module, batch: object) -> torch.Tensor:
    if not isinstance(batch, dict):
        raise TypeError(f"without a loss_fn the streamer calls model(**batch).loss, which needs a dict batch, "
                        f"got {type(batch).__name__}.")
    loss = getattr(model(**batch), "loss", None)
    if loss is None:
        raise ValueError("model(**batch) returned no loss (labels missing?); give the streamer a loss_fn.")
    return loss


class _ProbeGuard:
    """Everything a frozen-probe pass must leave as it found it: parameter gradients,
    train/eval modes of every module, and the RNG states."""

    def __init__(self, model: nn.Module, forward_model: nn.Module) -> None:
        self.grads = [(p, None if p.grad is None else p.grad.detach().clone()) for p in model.parameters()]
        self.holds_grads = any(g is not None for _p, g in self.grads)
        self.modes = [(m, m.training) for m in forward_model.modules()]
        self.cpu_rng = torch.get_rng_state()
        cuda_live = torch.cuda.is_available() and torch.cuda.is_initialized()
        self.cuda_rng = torch.cuda.get_rng_state_all() if cuda_live else None

    def restore(self) -> None:
        errors = []
        with torch.no_grad():
            for p, saved in self.grads:
                try:
                    same = (saved is not None and p.grad is not None and p.grad.shape == saved.shape
                            and p.grad.dtype == saved.dtype)
                    if same:
                        p.grad.copy_(saved)
                    else:
                        p.grad = saved
                except RuntimeError as err:
                    errors.append(err)
        for m, training in self.modes:
            m.training = training
        torch.set_rng_state(self.cpu_rng)
        if self.cuda_rng is not None:
            torch.cuda.set_rng_state_all(self.cuda_rng)
        if errors:
            raise RuntimeError(f"the probe pass could not hand {len(errors)} parameter gradient(s) back to the "
                               f"model it shares: {errors[0]}") from errors[0]


def autocast_for(args) -> AbstractContextManager:
    """The autocast context *args* asks for (bf16 / fp16), else a null context."""
    dtype = torch.bfloat16 if args.bf16 else torch.float16 if args.fp16 else None
    if dtype is None:
        return contextlib.nullcontext()
    on_gpu = torch.cuda.is_available() and not args.use_cpu
    return torch.autocast(device_type="cuda" if on_gpu else "cpu", dtype=dtype)


def move_batch(batch: object, device: torch.device | str, non_blocking: bool = False) -> object:
    """*batch* (dict, sequence or tensor) with its tensors moved to *device*."""
    def move(v):
        return v.to(device, non_blocking=non_blocking) if isinstance(v, torch.Tensor) else v

    if isinstance(batch, dict):
        return {k: move(v) for k, v in batch.items()}
    if isinstance(batch, (list, tuple)):
        return type(batch)(move(v) for v in batch)
    return move(batch)


def _device_to_host(host: object, device_copy: object) -> dict[int, torch.Tensor]:
    """``{id(device tensor): its host tensor}`` over a host batch and its moved copy."""
    if isinstance(host, dict) and isinstance(device_copy, dict):
        pairs = [(host[k], device_copy[k]) for k in host if k in device_copy]
    elif isinstance(host, (list, tuple)) and isinstance(device_copy, (list, tuple)):
        pairs = list(zip(host, device_copy))
    else:
        pairs = [(host, device_copy)]
    return {id(d): h for h, d in pairs if isinstance(h, torch.Tensor) and isinstance(d, torch.Tensor)}


def _hashable_fields(batch: object) -> dict | None:
    """The tensor fields of a host batch that the manager would hash (dict batches only)."""
    if isinstance(batch, dict):
        return {k: v for k, v in batch.items() if isinstance(v, torch.Tensor)}
    return None


def _fused_fsdp_ready(device: torch.device) -> bool:
    """Peer-memory kernels can run: NCCL group of two or more ranks on sm_100 GPUs."""
    if device.type != "cuda" or torch.cuda.get_device_capability(device)[0] != 10:
        return False
    from dattri_llm_b200 import ops
    from dattri_llm_b200.parallel import symm

    return ops.available() and symm.available(device)


class _ResumeSkip:
    """Batches to skip at the start of the next pass (resuming a collection), each checked
    against the stored record's identities when those are given."""

    def __init__(self, count: int = 0, expected: list[list[str]] | None = None) -> None:
        self.left, self.expected = count, expected
        self.mismatch: int | None = None  # first skipped batch whose content hash differed

    def check(self, index: int, host_batch, id_key) -> None:
        if self.expected is None or index >= len(self.expected) or self.mismatch is not None:
            return
        if id_key is not None and isinstance(host_batch, dict) and id_key in host_batch:
            raw = host_batch[id_key]
            got = [str(v) for v in (raw.tolist() if isinstance(raw, torch.Tensor) else list(raw))]
            if got != self.expected[index]:
                raise RuntimeError(f"Cannot resume: the {id_key!r} values of batch {index} are not the stored "
                                   "record's -- the loader's order changed since the collection began.")
            return
        fields = _hashable_fields(host_batch)
        if fields and hash_batch(fields) != self.expected[index]:
            self.mismatch = index  # reported once hashes of host batches are known to be trustworthy


class GradientStreamer(GradientSource):
    """Yields per-step ``(step, Gradient, hashes)`` from a live forward+backward loop.

    Args:
        model: The model (unwrapped; hooks are registered on it).
        dataset: Batches go straight to ``loss_fn(model, batch)``.
        args: :class:`AttributionArguments`.
        batch_size: Per-process batch size.
        enable_update: Train while streaming (a trajectory) instead of a frozen probe.
        loss_fn: ``(model, batch) -> loss`` (default ``model(**batch).loss``).
        optimizer / scheduler: For ``enable_update`` (built from *args* when omitted).
        config: Capture configuration (default: every capable layer).
        collate_fn: Loader collate function.
        checkpoint_step: Step label of a frozen probe's blocks.
        hook_manager: Share another streamer's manager (one set of hooks).  A manager the
            streamer did not build is not switched to collecting by it: the caller holds
            ``hook_manager.collect()`` open around the loop.
        precondition: Capture optimizer-preconditioned gradients (LESS).
        snapshots: Record the trajectory's parameters and batches here.
        forward_model: The DDP/FSDP wrapper to run on (default: wrap per *args*).
        shard: Split the dataset across ranks (else every rank streams all of it).
        defer_update: Apply the optimizer step lazily at the next ``next()``.
    """

    def __init__(self, model: nn.Module, dataset: Dataset, args, *, batch_size: int,
                 enable_update: bool = False, loss_fn: LossFn | None = None, optimizer=None, scheduler=None,
                 config: HookManagerConfig | None = None, collate_fn: Callable | None = None,
                 checkpoint_step: int = 0, hook_manager: HookManager | None = None, precondition: bool = False,
                 snapshots: TrajectorySnapshots | str | None = None, forward_model: nn.Module | None = None,
                 shard: bool = True, defer_update: bool = False) -> None:
        if snapshots is not None:
            snapshots = snapshots if isinstance(snapshots, TrajectorySnapshots) else TrajectorySnapshots(snapshots)
            if not enable_update:
                raise ValueError("snapshots= records a training trajectory: it needs enable_update=True.")
            if args.fsdp:
                raise NotImplementedError("snapshots= cannot record FSDP-sharded parameters; record under DDP or "
                                          "on one device.")
        if precondition and not enable_update and optimizer is None:
            raise ValueError("precondition=True reads optimizer state: give optimizer= (a probe at a checkpoint's "
                             "optimizer) or use enable_update=True.")
        if args.deepspeed:
            raise NotImplementedError("DeepSpeed is not supported by the streamer; run on one device, DDP or FSDP.")
        self._model, self._dataset, self._args = model, dataset, args
        self._batch_size, self._shard = batch_size, shard
        self.enable_update, self.defer_update = enable_update, defer_update
        self._snapshots = snapshots
        self._loss_fn = loss_fn if loss_fn is not None else _default_loss_fn
        self._optimizer, self._scheduler = optimizer, scheduler
        self._collate_fn = collate_fn
        self._checkpoint_step = checkpoint_step
        self._precondition = precondition
        self._manager_is_mine = hook_manager is None
        self._manager, self._capture = self._attach_manager(hook_manager, config)
        if args.gradient_checkpointing and hasattr(model, "gradient_checkpointing_enable"):
            model.gradient_checkpointing_enable(gradient_checkpointing_kwargs=args.gradient_checkpointing_kwargs)
        self._scaler = torch.amp.GradScaler("cuda", enabled=bool(args.fp16 and enable_update and not args.use_cpu))
        model = model.to(args.device)
        if forward_model is not None:
            self._fwd = forward_model
        elif hook_manager is not None and args.world_size > 1:
            raise ValueError("sharing another streamer's hook_manager across ranks needs its forward_model= too "
                             "(pass other.forward_model).")
        else:
            self._fwd = self._wrap_model(model, args, frozen=not enable_update)
        self._loader = self._build_loader()
        self._window = max(1, int(args.gradient_accumulation_steps))
        if enable_update and self._optimizer is None:
            self._optimizer, self._scheduler = self._create_optimizer_and_scheduler()
        self._active = False            # inside the with-block
        self._batches: Iterator | None = None
        self._index = 0                 # batch index within the pass
        self._in_window = 0             # batches accumulated in the current update window
        self._window_first = 0          # first batch of the current window (snapshot references)
        self._update_owed = False       # a deferred optimizer step is due
        self._passes = 0
        self._lrs: dict[int, float] = {}
        self._trainable = True
        self._guard: _ProbeGuard | None = None
        self._collect_cm = None
        self._hash_pool: ThreadPoolExecutor | None = None
        self.host_hash_trusted: bool | None = None  # host-batch hash == hash of the model's inputs
        self._skip_next = _ResumeSkip()
        self._skip = _ResumeSkip()

    def _attach_manager(self, shared: HookManager | None, config) -> tuple[HookManager, CaptureCallback]:
        if shared is None:
            capture = CaptureCallback()
            cfg = config if config is not None else HookManagerConfig(linear_io=REGISTER_ALL)
            manager = HookManager(self._model, config=cfg, callbacks=[capture],
                                  optimizer=(lambda: self.optimizer) if self._precondition else None)
            return manager, capture
        if self._precondition and not shared.supports_preconditioning:
            raise ValueError("precondition=True needs a hook_manager built with an optimizer; the shared one has none.")
        capture = next((cb for cb in shared.callbacks if isinstance(cb, CaptureCallback)), None)
        if capture is None:
            raise ValueError("a shared hook_manager must carry a CaptureCallback -- pass another "
                             "GradientStreamer's .hook_manager.")
        return shared, capture

    # ------------------------------------------------------------------ public state
    @property
    def args(self):
        """The run configuration."""
        return self._args

    @property
    def model(self) -> nn.Module:
        """The unwrapped model."""
        return self._model

    @property
    def forward_model(self) -> nn.Module:
        """The model the forward runs on (the wrapper, if any)."""
        return self._fwd

    @property
    def hook_manager(self) -> HookManager:
        """The capture manager."""
        return self._manager

    @property
    def checkpoint_step(self) -> int:
        """The step label a frozen probe puts on its blocks."""
        return self._checkpoint_step

    @property
    def reusable(self) -> bool:
        """A frozen probe can be streamed again; a trajectory only once."""
        return not self.enable_update

    @property
    def optimizer(self) -> torch.optim.Optimizer:
        """The optimizer.

        Raises:
            RuntimeError: a frozen probe built without one.
        """
        if self._optimizer is None:
            raise RuntimeError("this frozen probe was built without an optimizer.")
        return self._optimizer

    @property
    def learning_rates(self) -> dict[int, float]:
        """``{step: learning rate}`` of the trajectory so far."""
        return dict(self._lrs)

    def __len__(self) -> int:
        return len(self._loader)

    def skip_batches(self, n: int, expected_hashes: list[list[str]] | None = None) -> None:
        """Skip the first *n* batches of the next pass: resuming a collection whose first
        *n* batches are already stored.  The skipped batches are read from the loader (so
        the order stays the same) but not run.  With *expected_hashes* (the stored records'
        hashes, one list per batch) each skipped batch is checked against its record, and
        a batch that differs raises once the first computed step shows that the host
        batch's hash is the model inputs' hash.

        Raises:
            ValueError: on a trajectory stream (``enable_update=True``), whose later steps
                depend on the skipped updates.
        """
        if n < 0:
            raise ValueError(f"cannot skip a negative number of batches ({n}).")
        if n and self.enable_update:
            raise ValueError("only a frozen probe can resume by skipping batches: a trajectory's later steps "
                             "depend on the updates of the skipped ones.")
        self._skip_next = _ResumeSkip(int(n), expected_hashes)

    # ------------------------------------------------------------------ with-block
    def __enter__(self) -> GradientStreamer:
        if self._active:
            raise RuntimeError("this GradientStreamer is already open; leave its with-block first.")
        self._active = True
        _seed_everything(self._args.seed, self._args.full_determinism)
        if self._manager_is_mine:
            self._collect_cm = self._manager.collect()
            self._collect_cm.__enter__()
        self._hash_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="bw-hash")
        return self

    def __exit__(self, *exc) -> bool:
        try:
            passed = exc
            try:
                owed, self._update_owed = self._update_owed, False
                if owed and exc[0] is None:
                    self._optimizer_step()
            except BaseException as err:
                passed = (type(err), err, err.__traceback__)
                raise
            finally:
                if self._collect_cm is not None:
                    cm, self._collect_cm = self._collect_cm, None
                    cm.__exit__(*passed)
        finally:
            try:
                self._close()
            except Exception as err:
                if exc[0] is None:
                    raise
                warnings.warn(f"while handling {exc[0].__name__}: {err}", RuntimeWarning, stacklevel=2)
            finally:
                self._active = False
        return False

    def _close(self) -> None:
        try:
            if self._manager_is_mine:
                self._manager.remove()
            if self._hash_pool is not None:
                self._hash_pool.shutdown(wait=True)
                self._hash_pool = None
        finally:
            self._restore_probe()

    def _restore_probe(self) -> None:
        guard, self._guard = self._guard, None
        if guard is not None:
            guard.restore()

    # ------------------------------------------------------------------ iteration
    def __iter__(self) -> Iterator[StreamBatch]:
        if not self._active:
            raise RuntimeError("open the streamer first: ``with streamer: for step, grad, ids in streamer: ...``.")
        if self._passes and not self.reusable:
            raise RuntimeError("a trajectory (enable_update=True) streams once; this one has been consumed.")
        self._update_owed = False
        self._skip, self._skip_next = self._skip_next, _ResumeSkip()
        if not self.enable_update:
            self._restore_probe()
            self._guard = _ProbeGuard(self._model, self._fwd)
        self._fwd.train(self.enable_update)
        # A frozen probe (no parameter requires grad) needs no per-step zero_grad walks.
        self._trainable = any(p.requires_grad for p in self._fwd.parameters())
        self._batches = iter(self._loader)
        self._index = self._in_window = 0
        self._lrs = {}
        self._manager.reset_steps()
        self._passes += 1
        return self

    def _next_host_batch(self):
        try:
            host = next(self._batches)
            while self._skip.left > 0:
                self._skip.check(self._index, host, self._manager.sample_id_key)
                self._index += 1
                self._skip.left -= 1
                host = next(self._batches)
        except StopIteration:
            self._restore_probe()
            raise
        return host

    def _hash_on_side(self, host) -> Future | None:
        if self.host_hash_trusted is False or self._hash_pool is None:
            return None
        if self._manager.sample_id_key is not None or self._manager.sample_hash_fields is not None:
            return None
        fields = _hashable_fields(host)
        return self._hash_pool.submit(hash_batch, fields) if fields else None

    def _record_snapshot(self, batch) -> None:
        if self._snapshots is None:
            return
        if self._in_window == 0:
            self._window_first = self._index
            self._snapshots.save_parameters(self._index, self._model)
        else:
            self._snapshots.save_parameters(self._index, self._model, same_as=self._window_first)
        self._snapshots.save_batch(self._index, batch)

    def __next__(self) -> StreamBatch:
        if self._batches is None:
            raise RuntimeError("start a pass with iter(streamer) before calling next().")
        if self._update_owed:
            self._update_owed = False
            self._optimizer_step()
        host = self._next_host_batch()
        pending_hash = self._hash_on_side(host)
        batch = move_batch(host, self._args.device, non_blocking=True)
        self._record_snapshot(batch)
        manager = self._manager
        manager.reset_steps(self._index)
        if manager.supports_preconditioning:
            manager.precondition = self._precondition
        host_ids = None
        if pending_hash is not None:
            try:
                host_ids = pending_hash.result()
            except ValueError:
                host_ids = None
            manager.set_sample_ids(host_ids if self.host_hash_trusted else None)
        # a field moved from this host batch is hashed from its host copy (no device read-back)
        manager.set_host_inputs(_device_to_host(host, batch))
        with trace_range(f"dattri.stream.batch[{self._index}]"):
            self._forward_backward(batch)
        if self.enable_update:
            self._after_trajectory_step()
        record = self._capture.record
        if record is None:
            raise RuntimeError("the step produced no capture: loss_fn must run the streamer's model on the batch, "
                               "the backward must reach the hooked layers, and the manager must be collecting.")
        if record.step != self._index:
            raise RuntimeError(f"the capture recorded step {record.step} for batch {self._index}: every streamed "
                               "batch must produce exactly one capture step.")
        hashes = _record_hashes(record)
        if self.host_hash_trusted is None and host_ids is not None:
            self.host_hash_trusted = list(host_ids) == hashes
        if self._skip.mismatch is not None and self.host_hash_trusted:
            raise RuntimeError(f"Cannot resume: skipped batch {self._skip.mismatch} is not its stored record -- "
                               "the loader's order changed since the collection began.")
        if self._guard is not None and not self._guard.holds_grads and self._trainable:
            self._fwd.zero_grad(set_to_none=True)
        step = self._index if self.enable_update else self._checkpoint_step
        self._index += 1
        return step, record.gradient, hashes

    def _after_trajectory_step(self) -> None:
        self._lrs[self._index] = float(self._optimizer.param_groups[0]["lr"])
        self._in_window += 1
        if self._in_window >= self._window or self._index + 1 >= len(self._loader):
            if self.defer_update:
                self._update_owed = True
            else:
                self._optimizer_step()
            self._in_window = 0

    def _forward_backward(self, batch: object) -> torch.Tensor:
        if self.enable_update:
            self._fwd.train()
        if self._in_window == 0 and self._trainable:
            keep = self._guard is not None and self._guard.holds_grads
            self._fwd.zero_grad(set_to_none=not keep)
        self._capture.record = None
        with autocast_for(self._args):
            loss = self._loss_fn(self._fwd, batch)
        if self.enable_update and self._window > 1:
            loss = loss / self._window
        (self._scaler.scale(loss) if self._scaler.is_enabled() else loss).backward()
        return loss

    # ------------------------------------------------------------------ updates
    def _optimizer_step(self) -> None:
        scaled = self._scaler.is_enabled()
        if scaled:
            self._scaler.unscale_(self._optimizer)
        norm = self._args.max_grad_norm
        if norm is not None and norm > 0:
            self._clip_gradients(norm)
        if scaled:
            self._scaler.step(self._optimizer)
            self._scaler.update()
        else:
            self._optimizer.step()
        if self._scheduler is not None:
            self._scheduler.step()

    def _clip_gradients(self, max_norm: float) -> None:
        if torch.distributed.is_available():
            from torch.distributed.fsdp import FullyShardedDataParallel

            if isinstance(self._fwd, FullyShardedDataParallel):
                self._fwd.clip_grad_norm_(max_norm)  # norms across the shards
                return
        nn.utils.clip_grad_norm_(self._model.parameters(), max_norm)

    def _create_optimizer_and_scheduler(self):
        a = self._args
        decayed, plain = [], []
        for name, p in self._model.named_parameters():
            if p.requires_grad:
                (plain if p.ndim < 2 or name.endswith(".bias") else decayed).append(p)
        groups = [{"params": decayed, "weight_decay": a.weight_decay}, {"params": plain, "weight_decay": 0.0}]
        if a.optim == "sgd":
            opt = torch.optim.SGD(groups, lr=a.learning_rate)
        elif a.optim in ("adamw_torch", "adamw"):
            # GPU parameters take torch's fused AdamW (one update kernel per dtype and device
            # instead of a dozen multi-tensor passes): the same update rule
            params = decayed + plain
            fused = bool(params) and all(p.is_cuda and p.is_floating_point() for p in params)
            opt = torch.optim.AdamW(groups, lr=a.learning_rate, betas=(a.adam_beta1, a.adam_beta2),
                                    eps=a.adam_epsilon, fused=True if fused else None)
        else:
            raise ValueError(f"optimizer {a.optim!r} is not supported by the streamer: use 'adamw_torch' or 'sgd'.")
        updates = -(-len(self._loader) // self._window)
        return opt, _make_scheduler(a.lr_scheduler_type, opt, a.warmup_steps, updates)

    # ------------------------------------------------------------------ data and wrapping
    def _build_loader(self) -> DataLoader:
        a = self._args
        shuffle = self.enable_update
        seed = a.seed if a.data_seed is None else a.data_seed
        kw: dict = {"dataset": self._dataset, "batch_size": self._batch_size, "num_workers": a.dataloader_num_workers,
                    "pin_memory": a.dataloader_pin_memory}
        if a.world_size > 1 and self._shard:
            kw["sampler"] = DistributedSampler(self._dataset, num_replicas=a.world_size, rank=a.process_index,
                                               shuffle=shuffle, seed=seed)
        else:
            kw["shuffle"] = shuffle
            if shuffle:
                kw["generator"] = torch.Generator().manual_seed(seed)
        if self._collate_fn is not None:
            kw["collate_fn"] = self._collate_fn
        if a.dataloader_num_workers > 0:
            kw["persistent_workers"] = a.dataloader_persistent_workers
            if a.dataloader_prefetch_factor is not None:
                kw["prefetch_factor"] = a.dataloader_prefetch_factor
        return DataLoader(**kw)

    @staticmethod
    def _wrap_model(model: nn.Module, args, frozen: bool = False) -> nn.Module:
        """The module forwards run through under *args*' parallelism (the model itself on
        one process)."""
        if args.world_size <= 1:
            return model
        fsdp = args.fsdp
        tokens = set(fsdp.split() if isinstance(fsdp, str) else (fsdp or []))
        if args.device.type == "cuda":
            torch.cuda.set_device(args.local_process_index)
        fused_ok = (frozen and "full_shard" in tokens and "offload" not in tokens
                    and (args.fsdp_config or {}).get("fused", True) and _fused_fsdp_ready(args.device))
        if fused_ok:
            # An attribution probe (no update) on NCCL + sm_100: the linears are sharded in
            # place and all-gather their weights inside their own GEMMs; nothing to wrap.
            from dattri_llm_b200.parallel.fsdp import shard_frozen_linears

            shard_frozen_linears(model)
            return model
        if tokens:
            from torch.distributed.fsdp import CPUOffload, ShardingStrategy
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

            kw = dict(args.fsdp_config or {})
            kw.pop("fused", None)
            policy = _auto_wrap_policy(model, kw)
            if policy is not None:
                kw["auto_wrap_policy"] = policy
            kw.setdefault("use_orig_params", True)
            strategy = ShardingStrategy.SHARD_GRAD_OP if "shard_grad_op" in tokens else ShardingStrategy.FULL_SHARD
            kw.setdefault("sharding_strategy", strategy)
            kw.setdefault("device_id", args.device)
            if "offload" in tokens:
                kw.setdefault("cpu_offload", CPUOffload(offload_params=True))
            return FSDP(model, **kw)
        from dattri_llm_b200.parallel.moe import expert_parallel_buffers

        # Expert-parallel layers hold a different expert shard on every rank: DDP must not
        # broadcast rank 0's over them.
        shards = expert_parallel_buffers(model)
        if shards:
            nn.parallel.DistributedDataParallel._set_params_and_buffers_to_ignore_for_model(model, shards)
        return nn.parallel.DistributedDataParallel(
            model, device_ids=[args.local_process_index] if args.device.type == "cuda" else None,
            find_unused_parameters=bool(args.ddp_find_unused_parameters))


def _seed_everything(seed: int, full_determinism: bool = False) -> None:
    import random

    import numpy as np

    random.seed(seed)
    np.random.seed(seed % (2**32))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if full_determinism:
        torch.use_deterministic_algorithms(True)


def _make_scheduler(kind: str, optimizer, warmup: int, total: int):
    """An LR schedule by transformers' name (``linear``, ``constant``, ``cosine``,
    ``constant_with_warmup``); transformers' own when importable."""
    try:
        from transformers import get_scheduler

        return get_scheduler(kind, optimizer, num_warmup_steps=warmup, num_training_steps=total)
    except ImportError:  # pragma: no cover - transformers is installed in the image
        import math

        def factor(step):
            if warmup and step < warmup:
                return step / max(1, warmup)
            if kind.startswith("constant"):
                return 1.0
            done = (step - warmup) / max(1, total - warmup)
            return 0.5 * (1 + math.cos(math.pi * min(1.0, done))) if kind == "cosine" else max(0.0, 1.0 - done)

        return torch.optim.lr_scheduler.LambdaLR(optimizer, factor)


class _ReplayModel:
    """The model a replay borrows: hooks installed, the original trainable parameters kept
    on the host to be put back by :meth:`close`."""

    def __init__(self, model: nn.Module, config, device) -> None:
        self.model = model.to(device)
        self.capture = CaptureCallback()
        cfg = config if config is not None else HookManagerConfig(linear_io=REGISTER_ALL)
        self.manager = HookManager(model, config=cfg, callbacks=[self.capture])
        self.saved = {n: p.detach().to("cpu", copy=True) for n, p in model.named_parameters() if p.requires_grad}
        self.closed = False

    def close(self) -> None:
        if self.closed:
            return
        self.manager.remove()
        with torch.no_grad():
            for name, p in self.model.named_parameters():
                if name in self.saved:
                    p.copy_(self.saved[name].to(p.device, p.dtype))
        self.model.zero_grad(set_to_none=True)
        self.closed = True


class ReplayGradientSource(GradientSource):
    """Per-step blocks recomputed from a trajectory's snapshots: each step's parameters are
    loaded into *model* and its batch is run forward and backward under fresh hooks."""

    def __init__(self, model: nn.Module, args, snapshots, *, loss_fn: LossFn | None = None,
                 config: HookManagerConfig | None = None, steps: Iterable[int] | None = None,
                 layer_name: str | list[str] | None = None, train_mode: bool = True, desc: str | None = None,
                 verbose: bool = False, _state: _ReplayModel | None = None) -> None:
        if args.world_size > 1:
            raise NotImplementedError("replays run in one process: the replayed steps are not split over ranks.")
        snapshots = snapshots if isinstance(snapshots, TrajectorySnapshots) else TrajectorySnapshots(snapshots)
        self._model, self.args, self.snapshots = model, args, snapshots
        self._loss_fn = loss_fn if loss_fn is not None else _default_loss_fn
        self._config = config
        recorded = snapshots.steps()
        if steps is None:
            self._steps = list(recorded)
        else:
            have = set(recorded)
            self._steps = [int(t) for t in steps if int(t) in have]
            if not self._steps:
                raise ValueError(f"no snapshot for any of the steps {sorted(set(steps))[:10]}; recorded steps: "
                                 f"{recorded[:10]}...")
        self._layers = _layer_list(layer_name)
        self._train_mode, self._desc, self._verbose = train_mode, desc, verbose
        self._state = _state

    @property
    def reusable(self) -> bool:
        """Always true: snapshots can be replayed again."""
        return True

    @property
    def steps(self) -> list[int]:
        """The replayed steps."""
        return list(self._steps)

    @property
    def layer_name(self) -> list[str] | None:
        """The layer filter (``None``: every layer)."""
        return None if self._layers is None else list(self._layers)

    def __len__(self) -> int:
        return len(self._steps)

    def for_steps(self, steps: Iterable[int]) -> ReplayGradientSource:
        """The same trajectory restricted to *steps* (sharing the borrowed model)."""
        return ReplayGradientSource(self._model, self.args, self.snapshots, loss_fn=self._loss_fn,
                                    config=self._config, steps=steps, layer_name=self._layers,
                                    train_mode=self._train_mode, desc=self._desc, verbose=self._verbose,
                                    _state=self._borrow())

    def _borrow(self) -> _ReplayModel:
        if self._state is None or self._state.closed:
            self._state = _ReplayModel(self._model, self._config, self.args.device)
        return self._state

    def _replay(self, state: _ReplayModel, step: int):
        self.snapshots.load_parameters(step, state.model)
        batch = move_batch(self.snapshots.load_batch(step), self.args.device)
        state.model.train(self._train_mode)
        state.model.zero_grad(set_to_none=True)
        state.capture.record = None
        with autocast_for(self.args):
            loss = self._loss_fn(state.model, batch)
        loss.backward()
        record = state.capture.record
        if record is None:
            raise RuntimeError(f"replaying step {step} produced no capture: loss_fn must run the model on the "
                               "batch, and the backward must reach the hooked layers.")
        grad = record.gradient if self._layers is None else record.gradient.select_layers(self._layers)
        return grad, _record_hashes(record)

    def __iter__(self) -> Iterator[StreamBatch]:
        state = self._borrow()
        steps: Iterable[int] = self._steps
        if self._verbose and self.args.should_log:
            from tqdm.auto import tqdm

            steps = tqdm(self._steps, desc=self._desc or "replay", unit="step", leave=False)
        with state.manager.collect():
            state.manager.reset_steps()
            for step in steps:
                grad, hashes = self._replay(state, step)
                yield step, grad, hashes

    def close(self) -> None:
        """Put the model's parameters back and remove the replay's hooks."""
        if self._state is not None:
            self._state.close()

    def __enter__(self) -> ReplayGradientSource:
        return self

    def __exit__(self, *exc) -> bool:
        self.close()
        return False
