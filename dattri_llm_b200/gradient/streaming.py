"""Gradient sources: stored (:class:`DiskGradientSource`), live
(:class:`GradientStreamer`) and replayed (:class:`ReplayGradientSource`).

Every source yields ``(step, Gradient, hashes)`` blocks -- the one contract all
attributors consume (parity: reference ``dattri_llm/gradient/streaming.py``).

:class:`GradientStreamer` mirrors an HF Trainer step: it builds the loader
(``DistributedSampler`` under distributed execution), wraps the model in DDP or
FSDP, runs ``loss_fn(model, batch)`` + backward under a :class:`HookManager`, and
either trains (``enable_update``: optimizer/scheduler per accumulation window,
gradient clipping, one step label per batch) or acts as a frozen probe at a
checkpoint (gradients and RNG state handed back untouched after the pass).

B200 data path: batches are pinned on the host and copied with
``non_blocking=True``; their sample identities are hashed on the host from that
same host batch while the GPU runs the step (handed to the manager with
:meth:`HookManager.set_sample_ids`), so no device tensor is read back for hashing.
"""

from __future__ import annotations

import contextlib
import functools
import logging
import warnings
from collections.abc import Callable, Iterable, Iterator
from concurrent.futures import ThreadPoolExecutor
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


class DiskGradientSource(GradientSource):
    """A re-iterable source over a :class:`GradientStorageManager` (any residency)."""

    def __init__(self, file_manager, args, *, steps: Iterable[int] | None = None,
                 layer_name: str | list[str] | None = None, desc: str | None = None,
                 verbose: bool = False) -> None:
        self._fm = file_manager
        self._args = args
        self._layer_name = [layer_name] if isinstance(layer_name, str) else (
            None if layer_name is None else list(layer_name))
        self._steps = resolve_steps(file_manager, steps)
        self._desc, self._verbose = desc, verbose

    reusable = property(lambda self: True, doc="Always re-iterable.")
    args = property(lambda self: self._args, doc="The run configuration.")
    file_manager = property(lambda self: self._fm, doc="The store.")

    @property
    def steps(self) -> list[int]:
        """The steps this source yields."""
        return list(self._steps)

    @property
    def layer_name(self) -> list[str] | None:
        """The layer filter."""
        return None if self._layer_name is None else list(self._layer_name)

    def __len__(self) -> int:
        return sum(len(b) for _, b in self._fm.iter_steps(self._steps))

    def __iter__(self) -> Iterator[StreamBatch]:
        return iter_gradient_blocks(self._fm, self._steps, self._args, layer_name=self._layer_name,
                                    desc=self._desc, verbose=self._verbose)

    def for_steps(self, steps: Iterable[int]) -> DiskGradientSource:
        """The same store restricted to *steps*."""
        return DiskGradientSource(self._fm, self._args, steps=steps, layer_name=self._layer_name,
                                  desc=self._desc, verbose=False)


def rebatch_blocks(source: Iterable[StreamBatch], batch_size: int):
    """Concatenate consecutive all-dense blocks into blocks of at least *batch_size*
    samples (factorized blocks pass through); yields ``(steps per row, block, hashes)``."""
    if batch_size < 1:
        raise ValueError(f"batch_size must be >= 1, got {batch_size}.")
    pending: dict[str, list[torch.Tensor]] = {}
    ids: list[str] = []
    steps: list[int] = []
    n = 0
    meta = None

    def build():
        nonlocal pending, ids, steps, n
        data = {k: v[0] if len(v) == 1 else torch.cat(v, dim=0) for k, v in pending.items()}
        rep, types, idx = meta
        out = (steps, Gradient(rep, data, types, idx, validate_on_init=False), ids)
        pending, ids, steps, n = {}, [], [], 0
        return out

    for step, block, hashes in source:
        if not all(isinstance(v, torch.Tensor) for v in block.data.values()):
            if n:
                yield build()
            yield [step] * block.batch_size, block, list(hashes)
            continue
        meta = (block.representation, block.layer_types, block.indexing)
        for name, t in block.data.items():
            pending.setdefault(name, []).append(t)
        ids.extend(hashes)
        steps.extend([step] * block.batch_size)
        n += block.batch_size
        if n >= batch_size:
            yield build()
    if n:
        yield build()


def _auto_wrap_policy(model: nn.Module, fsdp_config: dict) -> Callable | None:
    if "auto_wrap_policy" in fsdp_config:
        return None
    cls_names = fsdp_config.pop("transformer_layer_cls_to_wrap", None)
    min_params = fsdp_config.pop("min_num_params", None)
    if cls_names is None and min_params is None:
        return None
    if cls_names is not None and min_params is not None:
        raise ValueError("fsdp_config: pass either transformer_layer_cls_to_wrap or min_num_params, not both.")
    if cls_names is not None:
        from torch.distributed.fsdp.wrap import transformer_auto_wrap_policy

        wanted = {cls_names} if isinstance(cls_names, str) else set(cls_names)
        classes = {type(m) for m in model.modules() if type(m).__name__ in wanted}
        missing = wanted - {c.__name__ for c in classes}
        if missing:
            raise ValueError(f"transformer_layer_cls_to_wrap: no module of class {sorted(missing)} found in the model.")
        return functools.partial(transformer_auto_wrap_policy, transformer_layer_cls=classes)
    from torch.distributed.fsdp.wrap import size_based_auto_wrap_policy

    return functools.partial(size_based_auto_wrap_policy, min_num_params=int(min_params))


def _default_loss_fn(model: nn.Module, batch: object) -> torch.Tensor:
    if not isinstance(batch, dict):
        raise TypeError("The default loss_fn expects a dict batch (model(**batch).loss). Pass a custom "
                        "loss_fn for other batch formats.")
    loss = getattr(model(**batch), "loss", None)
    if loss is None:
        raise ValueError("Default loss_fn expected the model output to carry a ``.loss``; none found. "
                         "Pass an explicit loss_fn.")
    return loss


class _ProbePassState:
    """What a frozen probe must hand back: gradients, train/eval modes, RNG states."""

    def __init__(self, model: nn.Module, forward_model: nn.Module) -> None:
        self._grads = [(p, None if p.grad is None else p.grad.detach().clone()) for p in model.parameters()]
        self.holds_grads = any(g is not None for _, g in self._grads)
        self._modes = [(m, m.training) for m in forward_model.modules()]
        self._cpu_rng = torch.get_rng_state()
        self._cuda_rng = (torch.cuda.get_rng_state_all()
                          if torch.cuda.is_available() and torch.cuda.is_initialized() else None)

    def restore(self) -> None:
        failed = []
        with torch.no_grad():
            for p, g in self._grads:
                try:
                    if g is not None and p.grad is not None and p.grad.shape == g.shape and p.grad.dtype == g.dtype:
                        p.grad.copy_(g)
                    else:
                        p.grad = g
                except RuntimeError as err:
                    failed.append(err)
        for m, training in self._modes:
            m.training = training
        torch.set_rng_state(self._cpu_rng)
        if self._cuda_rng is not None:
            torch.cuda.set_rng_state_all(self._cuda_rng)
        if failed:
            raise RuntimeError(f"A frozen probe could not copy {len(failed)} saved gradient(s) back into "
                               f"the model it shares: {failed[0]}") from failed[0]


def autocast_for(args) -> AbstractContextManager:
    """The autocast context of *args* (bf16/fp16), or a null context."""
    dtype = torch.bfloat16 if args.bf16 else torch.float16 if args.fp16 else None
    if dtype is None:
        return contextlib.nullcontext()
    dev = "cuda" if (torch.cuda.is_available() and not args.use_cpu) else "cpu"
    return torch.autocast(device_type=dev, dtype=dtype)


def move_batch(batch: object, device: torch.device | str, non_blocking: bool = False) -> object:
    """*batch* (dict / sequence / tensor) with its tensors on *device*."""
    def mv(v):
        return v.to(device, non_blocking=non_blocking) if isinstance(v, torch.Tensor) else v
    if isinstance(batch, dict):
        return {k: mv(v) for k, v in batch.items()}
    if isinstance(batch, (list, tuple)):
        return type(batch)(mv(v) for v in batch)
    return mv(batch)


def _host_mirror(host: object, dev: object) -> dict[int, torch.Tensor]:
    """``{id(device tensor): host tensor}`` over a batch and its moved copy."""
    if isinstance(host, dict) and isinstance(dev, dict):
        pairs = [(host[k], dev[k]) for k in host if k in dev]
    elif isinstance(host, (list, tuple)) and isinstance(dev, (list, tuple)):
        pairs = list(zip(host, dev))
    else:
        pairs = [(host, dev)]
    return {id(d): h for h, d in pairs if isinstance(h, torch.Tensor) and isinstance(d, torch.Tensor)}


def _host_hashable(batch: object) -> dict | None:
    """The tensor fields of a host batch the manager would hash, or ``None``."""
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


class GradientStreamer(GradientSource):
    """Yields per-step ``(step, Gradient, hashes)`` from a live forward+backward pass.

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
        hook_manager: Share another streamer's manager (one set of hooks).
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
        self._model = model
        self._dataset = dataset
        self._args = args
        self._batch_size = batch_size
        self._shard = shard
        self.enable_update = enable_update
        self.defer_update = defer_update
        self._update_pending = False
        if snapshots is not None and not isinstance(snapshots, TrajectorySnapshots):
            snapshots = TrajectorySnapshots(snapshots)
        if snapshots is not None and not enable_update:
            raise ValueError("snapshots= records a trajectory; needs enable_update=True.")
        if snapshots is not None and args.fsdp:
            raise NotImplementedError("parameter snapshots are not supported under FSDP (the parameters are "
                                      "sharded); use DDP or a single device.")
        self._snapshots = snapshots
        self._window_start = 0
        self._loss_fn = loss_fn if loss_fn is not None else _default_loss_fn
        self._optimizer, self._scheduler = optimizer, scheduler
        self._collate_fn = collate_fn
        self._checkpoint_step = checkpoint_step
        self._precondition = precondition
        if precondition and not enable_update and optimizer is None:
            raise ValueError("precondition=True needs an optimizer to read the state from: pass optimizer= "
                             "(a frozen probe at a checkpoint's optimizer) or enable_update=True.")
        if hook_manager is not None:
            if precondition and not hook_manager.supports_preconditioning:
                raise ValueError("precondition=True on a shared hook_manager that was built without an optimizer.")
            self._hm = hook_manager
            self._owns_hm = False
            shared = next((cb for cb in hook_manager.callbacks if isinstance(cb, CaptureCallback)), None)
            if shared is None:
                raise ValueError("A shared hook_manager must carry a CaptureCallback; pass the "
                                 "``.hook_manager`` of another GradientStreamer.")
            self._capture = shared
        else:
            self._capture = CaptureCallback()
            self._hm = HookManager(model, config=config if config is not None else HookManagerConfig(
                linear_io=REGISTER_ALL), callbacks=[self._capture],
                optimizer=(lambda: self.optimizer) if precondition else None)
            self._owns_hm = True
        if args.deepspeed:
            raise NotImplementedError("GradientStreamer does not support DeepSpeed. Run single-process, DDP, "
                                      "or FSDP instead.")
        if args.gradient_checkpointing and hasattr(model, "gradient_checkpointing_enable"):
            model.gradient_checkpointing_enable(gradient_checkpointing_kwargs=args.gradient_checkpointing_kwargs)
        self._scaler = torch.amp.GradScaler("cuda", enabled=bool(args.fp16 and enable_update and not args.use_cpu))
        self._max_grad_norm = args.max_grad_norm
        model = model.to(args.device)
        if forward_model is not None:
            self._fwd = forward_model
        elif hook_manager is not None and args.world_size > 1:
            raise ValueError("A shared hook_manager under distributed execution needs the sharing streamer's "
                             "forward_model= as well (pass ``other.forward_model``).")
        else:
            self._fwd = self._wrap_model(model, args, frozen=not enable_update)
        self._loader = self._build_loader()
        self._accum_steps = max(1, int(args.gradient_accumulation_steps))
        self._accum = 0
        if enable_update and self._optimizer is None:
            self._optimizer, self._scheduler = self._create_optimizer_and_scheduler()
        self._it: Iterator | None = None
        self._index = 0
        self._consumed = False
        self._any_trainable = True
        self._lrs: dict[int, float] = {}
        self._entered = False
        self._collect_ctx = None
        self._pass_state: _ProbePassState | None = None
        self._hasher: ThreadPoolExecutor | None = None
        self._host_ids_ok: bool | None = None  # host batch hash == manager's model-input hash
        self._skip_pending: tuple[int, list[list[str]] | None] = (0, None)
        self._skip_left = 0
        self._skip_expected: list[list[str]] | None = None
        self._skip_mismatch: int | None = None

    args = property(lambda self: self._args, doc="The run configuration.")
    model = property(lambda self: self._model, doc="The unwrapped model.")
    forward_model = property(lambda self: self._fwd, doc="The model the forward runs on (wrapper if any).")
    hook_manager = property(lambda self: self._hm, doc="The capture manager.")
    checkpoint_step = property(lambda self: self._checkpoint_step,
                               doc="The step a frozen probe stamps on its records.")

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
            raise ValueError(f"n must be >= 0, got {n}.")
        if n and self.enable_update:
            raise ValueError("Only a frozen probe can resume: a trajectory's later steps depend on the "
                             "updates of the skipped ones.")
        self._skip_pending = (int(n), expected_hashes)

    def _skip_one(self, host_batch) -> None:
        i = self._index
        expected = self._skip_expected
        if expected is not None and i < len(expected) and self._skip_mismatch is None:
            key = self._hm.sample_id_key
            if key is not None and isinstance(host_batch, dict) and key in host_batch:
                ids = host_batch[key]
                got = [str(v) for v in (ids.tolist() if isinstance(ids, torch.Tensor) else list(ids))]
                if got != expected[i]:
                    raise RuntimeError(f"Cannot resume: batch {i}'s {key!r} values differ from the stored "
                                       "record; the loader's order changed since the collection began.")
            else:
                hashable = _host_hashable(host_batch)
                if hashable and hash_batch(hashable) != expected[i]:
                    self._skip_mismatch = i
        self._index += 1
        self._skip_left -= 1

    @property
    def reusable(self) -> bool:
        """A frozen probe can be streamed again; a trajectory cannot."""
        return not self.enable_update

    @property
    def optimizer(self) -> torch.optim.Optimizer:
        """The optimizer.

        Raises:
            RuntimeError: for a frozen probe built without one.
        """
        if self._optimizer is None:
            raise RuntimeError("No optimizer: this streamer is a frozen probe built without one.")
        return self._optimizer

    @property
    def learning_rates(self) -> dict[int, float]:
        """``{step: lr}`` of the trajectory so far."""
        return dict(self._lrs)

    def __len__(self) -> int:
        return len(self._loader)

    def __enter__(self) -> GradientStreamer:
        if self._entered:
            raise RuntimeError("GradientStreamer is already active.")
        self._entered = True
        _seed_everything(self._args.seed, self._args.full_determinism)
        if self._owns_hm:
            self._collect_ctx = self._hm.collect()
            self._collect_ctx.__enter__()
        self._hasher = ThreadPoolExecutor(max_workers=1, thread_name_prefix="bw-hash")
        return self

    def __exit__(self, *exc) -> bool:
        try:
            ctx_exc = exc
            try:
                pending, self._update_pending = self._update_pending, False
                if pending and exc[0] is None:
                    self._optimizer_step()
            except BaseException as err:
                ctx_exc = (type(err), err, err.__traceback__)
                raise
            finally:
                if self._owns_hm and self._collect_ctx is not None:
                    self._collect_ctx.__exit__(*ctx_exc)
        finally:
            try:
                self._release()
            except Exception as err:
                if exc[0] is None:
                    raise
                warnings.warn(f"While handling {exc[0].__name__}: {err}", RuntimeWarning, stacklevel=2)
            finally:
                self._entered = False
        return False

    def _release(self) -> None:
        try:
            if self._owns_hm:
                self._hm.remove()
            if self._hasher is not None:
                self._hasher.shutdown(wait=True)
                self._hasher = None
        finally:
            self._end_probe_pass()

    def __iter__(self) -> Iterator[StreamBatch]:
        if not self._entered:
            raise RuntimeError("Use the streamer as a context manager before iterating: "
                               "``with streamer as s: for ... in s: ...``.")
        if self._consumed and not self.reusable:
            raise RuntimeError("This streamer is single-shot (enable_update=True) and was already consumed; "
                               "the training trajectory cannot be replayed.")
        self._update_pending = False
        self._skip_left, self._skip_expected = self._skip_pending
        self._skip_pending = (0, None)
        self._skip_mismatch = None
        if not self.enable_update:
            self._end_probe_pass()
            self._pass_state = _ProbePassState(self._model, self._fwd)
        self._fwd.train(self.enable_update)
        # Nothing can hold a parameter gradient when every parameter is frozen (the frozen
        # probe): then the per-step zero_grad walks of the module tree are skipped.
        self._any_trainable = any(p.requires_grad for p in self._fwd.parameters())
        self._it = iter(self._loader)
        self._index = 0
        self._accum = 0
        self._lrs = {}
        self._hm.reset_steps()
        self._consumed = True
        return self

    def __next__(self) -> StreamBatch:
        if self._it is None:
            raise RuntimeError("Call iter(streamer) before next(streamer).")
        if self._update_pending:
            self._update_pending = False
            self._optimizer_step()
        try:
            host_batch = next(self._it)
            while self._skip_left > 0:
                self._skip_one(host_batch)
                host_batch = next(self._it)
        except StopIteration:
            self._end_probe_pass()
            raise
        ids = None
        hashable = _host_hashable(host_batch) if self._host_ids_ok is not False else None
        if (hashable and self._hm.sample_id_key is None and self._hm.sample_hash_fields is None
                and self._hasher is not None):
            ids = self._hasher.submit(hash_batch, hashable)
        batch = move_batch(host_batch, self._args.device, non_blocking=True)
        if self._snapshots is not None:
            if self._accum == 0:
                self._window_start = self._index
                self._snapshots.save_parameters(self._index, self._model)
            else:
                self._snapshots.save_parameters(self._index, self._model, same_as=self._window_start)
            self._snapshots.save_batch(self._index, batch)
        self._hm.reset_steps(self._index)
        if self._hm.supports_preconditioning:
            self._hm.precondition = self._precondition
        host_ids = None
        if ids is not None:
            try:
                host_ids = ids.result()
            except ValueError:
                host_ids = None
            # The host hash stands in for the manager's hash of the model's inputs only once
            # the first step has shown the two agree (the loss_fn may feed the model a subset
            # of the batch's fields); until then the manager hashes.
            self._hm.set_sample_ids(host_ids if self._host_ids_ok else None)
        # Whatever the model is fed, a field moved from this host batch is hashed from its
        # host copy (no device read-back at step end).
        self._hm.set_host_inputs(_host_mirror(host_batch, batch))
        with trace_range(f"dattri.stream.batch[{self._index}]"):
            self._forward_backward(batch)
        if self.enable_update:
            self._lrs[self._index] = float(self._optimizer.param_groups[0]["lr"])
            self._accum += 1
            if self._accum >= self._accum_steps or self._index + 1 >= len(self._loader):
                if self.defer_update:
                    self._update_pending = True
                else:
                    self._optimizer_step()
                self._accum = 0
        record = self._capture.record
        if record is None:
            raise RuntimeError("loss_fn produced no capture step: it must run the streamer's model on the "
                               "batch and its backward must reach the hooked layers.")
        if record.step != self._index:
            raise RuntimeError(f"Step desync: HookManager captured step {record.step} but the streamer is on "
                               f"batch {self._index}. Exactly one capture step is expected per streamed batch.")
        hashes = list(record.input_hash) if isinstance(record.input_hash, list) else [record.input_hash]
        if self._host_ids_ok is None and host_ids is not None:
            self._host_ids_ok = list(host_ids) == hashes
        if self._skip_mismatch is not None and self._host_ids_ok:
            raise RuntimeError(f"Cannot resume: skipped batch {self._skip_mismatch} differs from its stored "
                               "record; the loader's order changed since the collection began.")
        if self._pass_state is not None and not self._pass_state.holds_grads and self._any_trainable:
            self._fwd.zero_grad(set_to_none=True)
        step = self._index if self.enable_update else self._checkpoint_step
        self._index += 1
        return step, record.gradient, hashes

    def _forward_backward(self, batch: object) -> torch.Tensor:
        if self.enable_update:
            self._fwd.train()
        if self._accum == 0 and self._any_trainable:
            hands_back = self._pass_state is not None and self._pass_state.holds_grads
            self._fwd.zero_grad(set_to_none=not hands_back)
        self._capture.record = None
        with autocast_for(self._args):
            loss = self._loss_fn(self._fwd, batch)
        if self.enable_update and self._accum_steps > 1:
            loss = loss / self._accum_steps
        if self._scaler.is_enabled():
            self._scaler.scale(loss).backward()
        else:
            loss.backward()
        return loss

    def _optimizer_step(self) -> None:
        if self._scaler.is_enabled():
            self._scaler.unscale_(self._optimizer)
        if self._max_grad_norm is not None and self._max_grad_norm > 0:
            self._clip_gradients()
        if self._scaler.is_enabled():
            self._scaler.step(self._optimizer)
            self._scaler.update()
        else:
            self._optimizer.step()
        if self._scheduler is not None:
            self._scheduler.step()

    def _end_probe_pass(self) -> None:
        state, self._pass_state = self._pass_state, None
        if state is not None:
            state.restore()

    def _clip_gradients(self) -> None:
        fsdp_cls = None
        if torch.distributed.is_available():
            from torch.distributed.fsdp import FullyShardedDataParallel

            fsdp_cls = FullyShardedDataParallel
        if fsdp_cls is not None and isinstance(self._fwd, fsdp_cls):
            self._fwd.clip_grad_norm_(self._max_grad_norm)
        else:
            nn.utils.clip_grad_norm_(self._model.parameters(), self._max_grad_norm)

    def _create_optimizer_and_scheduler(self):
        a = self._args
        decay, no_decay = [], []
        for name, p in self._model.named_parameters():
            if p.requires_grad:
                (no_decay if (p.ndim < 2 or name.endswith(".bias")) else decay).append(p)
        groups = [{"params": decay, "weight_decay": a.weight_decay}, {"params": no_decay, "weight_decay": 0.0}]
        if a.optim == "sgd":
            opt = torch.optim.SGD(groups, lr=a.learning_rate)
        elif a.optim in ("adamw_torch", "adamw"):
            opt = torch.optim.AdamW(groups, lr=a.learning_rate, betas=(a.adam_beta1, a.adam_beta2), eps=a.adam_epsilon)
        else:
            raise ValueError(f"Unsupported args.optim={a.optim!r}; use 'adamw_torch' or 'sgd'.")
        updates = -(-len(self._loader) // self._accum_steps)
        return opt, _make_scheduler(a.lr_scheduler_type, opt, a.warmup_steps, updates)

    def _build_loader(self) -> DataLoader:
        a = self._args
        kw: dict = {"dataset": self._dataset, "batch_size": self._batch_size,
                    "num_workers": a.dataloader_num_workers, "pin_memory": a.dataloader_pin_memory}
        shuffle = self.enable_update
        seed = a.data_seed if a.data_seed is not None else a.seed
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
        fsdp = args.fsdp
        tokens = set(fsdp.split() if isinstance(fsdp, str) else (fsdp or []))
        if args.world_size <= 1:
            return model
        if args.device.type == "cuda":
            torch.cuda.set_device(args.local_process_index)
        if tokens and frozen and "full_shard" in tokens and "offload" not in tokens and \
                (args.fsdp_config or {}).get("fused", True) and _fused_fsdp_ready(args.device):
            # An attribution probe (no update) on NCCL + sm_100: the linears are sharded in
            # place and all-gather their weights inside their own GEMMs; nothing to wrap.
            from dattri_llm_b200.parallel.fsdp import shard_frozen_linears

            shard_frozen_linears(model)
            return model
        if tokens:
            from torch.distributed.fsdp import CPUOffload, ShardingStrategy
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

            kw = dict(args.fsdp_config or {})
            policy = _auto_wrap_policy(model, kw)
            if policy is not None:
                kw["auto_wrap_policy"] = policy
            kw.setdefault("use_orig_params", True)
            kw.setdefault("sharding_strategy", ShardingStrategy.SHARD_GRAD_OP if "shard_grad_op" in tokens
                          else ShardingStrategy.FULL_SHARD)
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

        def lam(step):
            if warmup and step < warmup:
                return step / max(1, warmup)
            if kind.startswith("constant"):
                return 1.0
            progress = (step - warmup) / max(1, total - warmup)
            if kind == "cosine":
                return 0.5 * (1 + math.cos(math.pi * min(1.0, progress)))
            return max(0.0, 1.0 - progress)
        return torch.optim.lr_scheduler.LambdaLR(optimizer, lam)


class _ReplayState:
    def __init__(self, model: nn.Module, config, device) -> None:
        self.model = model.to(device)
        self.capture = CaptureCallback()
        self.hm = HookManager(model, config=config if config is not None else HookManagerConfig(
            linear_io=REGISTER_ALL), callbacks=[self.capture])
        self.original = {n: p.detach().to("cpu", copy=True) for n, p in model.named_parameters() if p.requires_grad}
        self.closed = False

    def close(self) -> None:
        if self.closed:
            return
        self.hm.remove()
        with torch.no_grad():
            for n, p in self.model.named_parameters():
                if n in self.original:
                    p.copy_(self.original[n].to(p.device, p.dtype))
        self.model.zero_grad(set_to_none=True)
        self.closed = True


class ReplayGradientSource(GradientSource):
    """Per-step blocks recomputed from a trajectory's snapshots (parameters + batch)."""

    def __init__(self, model: nn.Module, args, snapshots, *, loss_fn: LossFn | None = None,
                 config: HookManagerConfig | None = None, steps: Iterable[int] | None = None,
                 layer_name: str | list[str] | None = None, train_mode: bool = True, desc: str | None = None,
                 verbose: bool = False, _state: _ReplayState | None = None) -> None:
        if args.world_size > 1:
            raise NotImplementedError("ReplayGradientSource runs single-process; the replayed steps are not "
                                      "sharded across ranks.")
        if not isinstance(snapshots, TrajectorySnapshots):
            snapshots = TrajectorySnapshots(snapshots)
        self._model, self._args, self._snapshots = model, args, snapshots
        self._loss_fn = loss_fn if loss_fn is not None else _default_loss_fn
        self._config = config
        available = snapshots.steps()
        if steps is None:
            self._steps = list(available)
        else:
            have = set(available)
            self._steps = [int(t) for t in steps if int(t) in have]
            if not self._steps:
                raise ValueError(f"none of the requested steps {sorted(set(steps))[:10]} has a snapshot; "
                                 f"available: {available[:10]}...")
        self._layer_name = [layer_name] if isinstance(layer_name, str) else (
            None if layer_name is None else list(layer_name))
        self._train_mode, self._desc, self._verbose = train_mode, desc, verbose
        self._state = _state

    reusable = property(lambda self: True, doc="Always re-iterable.")
    args = property(lambda self: self._args, doc="The run configuration.")
    snapshots = property(lambda self: self._snapshots, doc="The snapshot directory.")

    @property
    def steps(self) -> list[int]:
        """The replayed steps."""
        return list(self._steps)

    @property
    def layer_name(self) -> list[str] | None:
        """The layer filter."""
        return None if self._layer_name is None else list(self._layer_name)

    def __len__(self) -> int:
        return len(self._steps)

    def for_steps(self, steps: Iterable[int]) -> ReplayGradientSource:
        """The same trajectory restricted to *steps* (sharing the model state)."""
        return ReplayGradientSource(self._model, self._args, self._snapshots, loss_fn=self._loss_fn,
                                    config=self._config, steps=steps, layer_name=self._layer_name,
                                    train_mode=self._train_mode, desc=self._desc, verbose=self._verbose,
                                    _state=self._ensure_state())

    def _ensure_state(self) -> _ReplayState:
        if self._state is None or self._state.closed:
            self._state = _ReplayState(self._model, self._config, self._args.device)
        return self._state

    def __iter__(self) -> Iterator[StreamBatch]:
        state = self._ensure_state()
        model = state.model
        steps: Iterable[int] = self._steps
        if self._verbose and self._args.should_log:
            from tqdm.auto import tqdm

            steps = tqdm(self._steps, desc=self._desc or "replay", unit="step", leave=False)
        with state.hm.collect():
            state.hm.reset_steps()
            for step in steps:
                self._snapshots.load_parameters(step, model)
                batch = move_batch(self._snapshots.load_batch(step), self._args.device)
                model.train(self._train_mode)
                model.zero_grad(set_to_none=True)
                state.capture.record = None
                with autocast_for(self._args):
                    loss = self._loss_fn(model, batch)
                loss.backward()
                record = state.capture.record
                if record is None:
                    raise RuntimeError(f"loss_fn produced no capture step replaying step {step}: it must run "
                                       "the model on the batch and its backward must reach the hooked layers.")
                grad = record.gradient
                if self._layer_name is not None:
                    grad = grad.select_layers(self._layer_name)
                hashes = list(record.input_hash) if isinstance(record.input_hash, list) else [record.input_hash]
                yield step, grad, hashes

    def close(self) -> None:
        """Restore the model's parameters and remove the hooks."""
        if self._state is not None:
            self._state.close()

    def __enter__(self) -> ReplayGradientSource:
        return self

    def __exit__(self, *exc) -> bool:
        self.close()
        return False
