"""``HookManager``: per-layer hook fires in, one ``GradientRecord`` per backward out.

The manager owns the capture of a model: it installs the per-layer hooks (and any forward
overrides), and decides when a training step's backward is complete so that its gradient
can be assembled and handed to the callbacks.  A step is complete when

* every hooked layer that ran a forward in the step got as many backward fires as it had
  forwards (a forward that never gets one -- activation checkpointing's first pass -- is
  dropped once the backward ends), and
* the gradients of linear-IO layers' own trainable parameters are final: every
  post-accumulate hook fired, or, under FSDP (which writes gradients after those hooks),
  the engine's end-of-backward callback ran; and
* every ``param_grad`` hook fired.

:class:`_StepBarrier` holds this bookkeeping for the step in flight.  When it closes, each
layer's buffer is turned into entries (a layer called k times yields virtual layers
``name``, ``name@2`` ... ``name@k``; parts from several devices are concatenated), the
samples are identified (ids handed in with :meth:`HookManager.set_sample_ids`, a
``sample_id_key`` field, or content hashes -- computed from host copies of the inputs when
the data pipeline provides them), and the callbacks run outside the lock, so a callback may
itself run a forward/backward through the same hooks (the data-selection validation pass
does, between :meth:`save_state` and :meth:`load_state`).  A backward that reaches no hooked
layer at all raises.  Public API as in the reference's ``dattri_llm/gradient/hooks/manager.py``.

B200 specifics: the step's deferred per-sample outer products run as one grouped tcgen05
launch when the step closes, and the per-step activation-projection share (q/k/v and
gate/up read one projection) is cleared with the buffers.
"""

from __future__ import annotations

import sys

import threading
import warnings
from collections.abc import Callable, Generator, Iterable
from contextlib import contextmanager
from dataclasses import dataclass, field, replace

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
from dattri_llm_b200.gradient.hooks.config import (
    INVASIVE_LINEAR_IO,
    LINEAR_IO,
    PARAM_GRAD,
    HookManagerConfig,
    resolve_hook_assignments,
)
from dattri_llm_b200.gradient.hooks.hooks import (
    LayerBuffer,
    _projection_matrix,
    _StepShare,
    has_trainable_params,
    register_linear_io_hooks,
    register_linear_param_hooks,
    register_param_grad_hooks,
    remove_hooks,
)
from dattri_llm_b200.gradient.hooks.override_layers import (
    find_fused_experts,
    find_sequence_mixers,
    install_fused_experts,
    install_invasive_forward,
    install_sequence_mixer_forward,
)
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.hooks.override_layers.fused_experts import PROXY_EXPERTS
from dattri_llm_b200.gradient.hooks.override_layers.grouped_experts import GroupedExpertCapture
from dattri_llm_b200.gradient.hooks.routing import RoutedTokenTracker
from dattri_llm_b200.gradient.ops import PARAM_GRAD_TYPES, is_embedding
from dattri_llm_b200.utils.autograd import queue_backward_end_callback
from dattri_llm_b200.utils.hashing import hash_batch
from dattri_llm_b200.utils.tracing import trace_range

_task_id_fn = getattr(torch._C, "_current_graph_task_id", None)


def _backward_task() -> int:
    """Id of the autograd graph task running on this thread (-1 outside any backward)."""
    return -1 if _task_id_fn is None else _task_id_fn()


def _grad_leaf_of(output: object) -> torch.Tensor | None:
    """The first tensor requiring grad inside a (nested) model output."""
    if isinstance(output, torch.Tensor):
        return output if output.requires_grad else None
    items = output.values() if isinstance(output, dict) else output
    if not isinstance(items, Iterable) or isinstance(items, (str, bytes)):
        return None
    for item in items:
        found = _grad_leaf_of(item)
        if found is not None:
            return found
    return None


@dataclass
class _StepBarrier:
    """Completion bookkeeping of the step in flight.

    ``ran``: layers with a forward this step; ``finished``: those whose backward fires
    caught up with their forwards; ``fires``: backward fires per layer; ``unreached``:
    layers whose forwards all went unmatched.  ``layers_closed`` / ``params_closed`` are
    the two halves of the barrier (linear-IO side incl. its parameters' gradients, and the
    ``param_grad`` side); ``weight_fires`` / ``param_fires`` count the parameter hooks;
    ``weights_final`` is set by the end-of-backward callback; ``end_queued`` says that
    callback is queued for this step, ``end_task`` which backward it belongs to (nested
    recomputation backwards end first), and ``recomputed`` that a forward ran inside a
    backward."""

    ran: set = field(default_factory=set)
    finished: set = field(default_factory=set)
    fires: dict = field(default_factory=dict)
    unreached: set = field(default_factory=set)
    layers_closed: bool = True
    params_closed: bool = True
    weight_fires: int = 0
    param_fires: int = 0
    weights_final: bool = False
    end_queued: bool = False
    end_task: int = -1
    recomputed: bool = False

    def fresh(self, has_linear_io: bool, has_param_grad: bool) -> _StepBarrier:
        return _StepBarrier(layers_closed=not has_linear_io, params_closed=not has_param_grad)

    def copy(self) -> _StepBarrier:
        return replace(self, ran=set(self.ran), finished=set(self.finished), fires=dict(self.fires),
                       unreached=set(self.unreached))


class HookManager:
    """Collect per-sample (``linear_io``) or per-batch (``param_grad``) gradients via hooks.

    Args:
        model: The model (or its DDP/FSDP/DataParallel wrapper; hooks go on ``.module``).
        config: :class:`HookManagerConfig` (default: every capable layer).
        callbacks: :class:`HookManagerCallback` instances.
        sample_id_key: Identify samples by this input field's values instead of hashing.
        sample_hash_fields: Hash only these input fields.
        non_batch_first_layers: Layers whose inputs are sequence-first ``(T, B, ...)``.
        moe_routed_layers: MoE blocks whose router / expert rows are regrouped per sample.
        offload_to_cpu: Move every capture to host memory as it arrives.
        optimizer: Precondition captures with this optimizer's state (LESS-style);
            a callable is resolved lazily.
    """

    def __init__(self, model: nn.Module, config: HookManagerConfig | None = None,
                 callbacks: list | None = None, sample_id_key: str | int | None = None,
                 sample_hash_fields: Iterable[str | int] | None = None,
                 non_batch_first_layers: Iterable[str] | None = None,
                 moe_routed_layers: Iterable[str] | None = None, offload_to_cpu: bool = False,
                 optimizer: torch.optim.Optimizer | Callable[[], torch.optim.Optimizer] | None = None) -> None:
        if isinstance(sample_hash_fields, (str, int)):
            sample_hash_fields = [sample_hash_fields]
        hash_fields = None if sample_hash_fields is None else tuple(sample_hash_fields)
        if hash_fields is not None and sample_id_key is not None:
            raise ValueError("give either sample_id_key (identify samples by a field) or sample_hash_fields "
                             "(hash only some fields), not both.")
        if hash_fields == ():
            raise ValueError("sample_hash_fields is empty: name at least one input field to hash.")
        self._model = model
        self._config = config if config is not None else HookManagerConfig()
        self._callbacks: list = list(callbacks or [])
        self._sample_id_key = sample_id_key
        self._sample_hash_fields = hash_fields
        self._offload = offload_to_cpu
        self._non_batch_first = set(non_batch_first_layers or ())
        self._moe_blocks = set(moe_routed_layers or ())
        self._preconditioner = None
        if optimizer is not None:
            from dattri_llm_b200.gradient.optimizer_state import GradientPreconditioner, OptimizerSnapshot

            inner = getattr(model, "module", model)
            self._preconditioner = GradientPreconditioner(
                lambda: OptimizerSnapshot(inner, optimizer() if callable(optimizer) else optimizer))
        # installation state
        self._installed = False
        self._reverts: list[Callable[[], None]] = []
        self._model_hooks: list = []
        self._layer_hooks: list = []
        self._weight_hooks: list = []
        self._param_hooks: list = []
        self._layers: dict[str, LayerBuffer] = {}
        self._params: dict[str, dict] = {}
        self._n_weights = 0          # trainable parameters of linear-IO layers (post-accumulate hooks)
        self._n_param_hooks = 0      # param_grad hooks
        self._has_linear_io = False
        self._has_param_grad = False
        self._routed: RoutedTokenTracker | None = None
        self._projector: ops.DattriProjector | None = None
        self._share = _StepShare()
        self._group_forwards: dict[str, int] = {}  # grouped expert blocks: forwards of this step
        # step state
        self._lock = threading.Lock()
        self._barrier = _StepBarrier()
        self._collecting = False
        self._steps = 0
        self._inputs: dict = {}
        self._pending_ids: list[str] | None = None
        self._host_inputs: dict[int, torch.Tensor] | None = None
        self._last_gradient: Gradient | None = None
        self._warned: set = set()
        self.register()
        for cb in self._callbacks:
            if hasattr(cb, "on_register"):
                cb.on_register(self)

    # ------------------------------------------------------------------ model inputs
    def _on_model_inputs(self, _module, args: tuple, kwargs: dict) -> None:
        """Keep the forward's inputs: they identify the step's samples."""
        if not self._collecting:
            return
        if torch.is_grad_enabled():
            self._last_gradient = None

        def field_of(f):
            return f"_arg{f}" if isinstance(f, int) else f

        if self._sample_hash_fields is not None:
            picked = {}
            for f in self._sample_hash_fields:
                if isinstance(f, int) and f < len(args):
                    picked[field_of(f)] = args[f]
                elif not isinstance(f, int) and f in kwargs:
                    picked[f] = kwargs[f]
            self._inputs = picked
            return
        found = {k: v for k, v in kwargs.items() if isinstance(v, torch.Tensor)}
        if not found:
            found = {field_of(i): a for i, a in enumerate(args) if isinstance(a, torch.Tensor)}
        key = self._sample_id_key
        if isinstance(key, int) and key < len(args):
            found[field_of(key)] = args[key]
        elif isinstance(key, str) and key in kwargs:
            found[key] = kwargs[key]
        self._inputs = found

    def set_host_inputs(self, mirror: dict[int, torch.Tensor] | None) -> None:
        """Host copies of the next step's device inputs, keyed by ``id()`` of the device
        tensor (consumed by that step).  When every model input of the step is one of them,
        its content hash is computed from the host copies: the same hash, without reading
        device tensors back (which would wait for the GPU at every step)."""
        self._host_inputs = mirror

    def set_sample_ids(self, ids: list[str] | None) -> None:
        """Identities of the samples of the next completed step (consumed by that step).

        Lets a data pipeline hash the batch on the host (from the pinned copy it sends
        to the GPU) instead of the manager reading device tensors back at step end.
        """
        self._pending_ids = None if ids is None else [str(i) for i in ids]

    # ------------------------------------------------------------------ the barrier
    def _queue_end_callback(self) -> None:
        """Queue the end-of-backward callback once per step (caller holds the lock)."""
        b = self._barrier
        if not b.end_queued and queue_backward_end_callback(self._on_backward_finished):
            b.end_queued = True
            if b.end_task == -1:
                b.end_task = _backward_task()

    def _on_layer_forward(self, name, activation, layer_type, module_kwargs) -> None:
        with self._lock:
            self._barrier.ran.add(name)
            if self._collecting and _backward_task() != -1:  # a forward inside a backward: recomputation
                b = self._barrier
                b.recomputed = True
                if b.end_task == -1:
                    b.end_task = _backward_task()
                if self._n_weights:
                    self._queue_end_callback()
        for cb in self._callbacks:
            cb.on_layer_forward(name, activation, layer_type, module_kwargs)

    def _on_layer_backward(self, name, grad_output, layer_type, module_kwargs) -> None:
        for cb in self._callbacks:
            cb.on_layer_backward(name, grad_output, layer_type, module_kwargs)
        if not self._collecting:
            return
        with self._lock:
            b = self._barrier
            if self._n_weights:
                self._queue_end_callback()
            b.fires[name] = b.fires.get(name, 0) + 1
            if b.fires[name] >= self._layers[name].forwards:
                b.finished.add(name)
            record = self._close_linear_side()
        if record is not None:
            self._emit(record)

    def _on_weight_grad_final(self, _layer, _param, _grad) -> None:
        """Post-accumulate hook of a linear-IO layer's own trainable parameter."""
        if not self._collecting:
            return
        with self._lock:
            self._barrier.weight_fires += 1
            record = self._close_linear_side()
        if record is not None:
            self._emit(record)

    def _on_param_grad(self, _layer, _param, _grad) -> None:
        """A ``param_grad`` hook fired."""
        if not self._collecting:
            return
        record = None
        with self._lock:
            b = self._barrier
            b.param_fires += 1
            if b.param_fires >= self._n_param_hooks:
                b.param_fires = 0
                b.params_closed = True
                record = self._close_if_ready()
        if record is not None:
            self._emit(record)

    def _on_model_output(self, _module, _args, output) -> None:
        if self._collecting and self._layers and torch.is_grad_enabled():
            leaf = _grad_leaf_of(output)
            if leaf is not None:
                leaf.register_hook(self._on_backward_started)

    def _on_backward_started(self, _grad) -> None:
        if self._collecting:
            with self._lock:
                self._queue_end_callback()

    def _on_backward_finished(self) -> None:
        """Engine callback at the end of the step's backward."""
        if not self._collecting:
            return
        with self._lock:
            b = self._barrier
            if not b.end_queued or (b.end_task != -1 and _backward_task() != b.end_task):
                return  # not queued for us, or the end of a nested recomputation backward
            b.weights_final = True
            self._settle_unmatched()
            unreached = sorted(b.unreached)
            stalled = self._has_linear_io and bool(unreached) and not b.ran and not b.layers_closed
            record = None if stalled else self._close_linear_side()
        if stalled:
            shown = unreached[:8] + (["..."] if len(unreached) > 8 else [])
            raise RuntimeError(
                f"the backward reached none of the hooked layers that ran forward ({shown}), so the step "
                "cannot be completed. A layer gets a gradient only if the loss depends on its output through "
                "something that requires grad -- with frozen layers (include_frozen=True), a parameter or an "
                "input upstream of them must require grad.")
        if unreached and record is not None and frozenset(unreached) not in self._warned:
            self._warned.add(frozenset(unreached))
            shown = unreached[:8] + (["..."] if len(unreached) > 8 else [])
            warnings.warn(f"hooked layers {shown} ran forward but got no gradient in this step (a detached "
                          "branch, or frozen layers with nothing trainable upstream); they are left out of the "
                          "step's record. Reported once per set of layers.", stacklevel=2)
        if record is not None:
            self._emit(record)

    def _settle_unmatched(self) -> None:
        """At the end of a backward: forget forwards that met no backward (caller holds the lock)."""
        b = self._barrier
        for name, buf in self._layers.items():
            with buf.lock:
                dropped = buf.keep_matched()
                matched = buf.forwards
            if matched == 0:
                b.ran.discard(name)
                if dropped:
                    b.unreached.add(name)
            elif b.fires.get(name, 0) >= matched:
                b.finished.add(name)
        for key, forwards in self._group_forwards.items():
            fired = b.fires.get(key, 0)
            if key in b.ran and fired < forwards:
                if fired:
                    b.finished.add(key)
                else:  # its forward's graph was never backpropagated (recomputation's first pass)
                    b.ran.discard(key)

    def _layers_finished(self) -> bool:
        b = self._barrier
        return not self._layers or (bool(b.ran) and len(b.finished) == len(b.ran))

    def _close_linear_side(self) -> GradientRecord | None:
        """Barrier (a) + (b); on success try the whole step (caller holds the lock)."""
        b = self._barrier
        weights_ready = self._n_weights == 0 or b.weights_final or b.weight_fires >= self._n_weights
        if self._layers_finished() and weights_ready:
            b.layers_closed = True
            return self._close_if_ready()
        return None

    def _close_if_ready(self) -> GradientRecord | None:
        b = self._barrier
        return self._close_step() if b.layers_closed and b.params_closed else None

    # ------------------------------------------------------------------ sample identity
    def _id_field(self) -> str | None:
        key = self._sample_id_key
        return None if key is None else (f"_arg{key}" if isinstance(key, int) else key)

    def _ids_from_key(self, expected: int) -> list[str]:
        fld = self._id_field()
        if fld not in self._inputs:
            raise KeyError(f"the model inputs of this step ({sorted(self._inputs)}) lack the sample_id_key field "
                           f"{self._sample_id_key!r}; samples cannot be identified.")
        value = self._inputs[fld]
        ids = value.reshape(-1).tolist() if isinstance(value, torch.Tensor) else list(value)
        if len(ids) != expected:
            raise ValueError(f"the sample_id_key field {self._sample_id_key!r} holds {len(ids)} ids for a step of "
                             f"{expected} samples.")
        return [str(i) for i in ids]

    def _sized_inputs(self) -> list:
        """Inputs that tell the batch size (the id field itself excluded: its length is checked)."""
        skip = self._id_field()
        return [v for k, v in self._inputs.items() if k != skip]

    def _batch_size(self, gradient: Gradient) -> int:
        def leading(default):
            return next((v.shape[0] for v in self._sized_inputs() if isinstance(v, torch.Tensor) and v.ndim > 0),
                        default)

        try:
            b = gradient.batch_size
        except ValueError:
            return leading(1)
        sized = self._sized_inputs()
        if not sized:
            return b
        agrees = any((isinstance(v, torch.Tensor) and v.ndim > 0 and v.shape[0] == b)
                     or (isinstance(v, (list, tuple)) and len(v) == b) for v in sized)
        return b if agrees else leading(b)

    def _sample_identities(self, batch: int) -> list[str]:
        ids, self._pending_ids = self._pending_ids, None
        mirror, self._host_inputs = self._host_inputs, None
        if ids is not None:
            if len(ids) != batch:
                raise ValueError(f"set_sample_ids gave {len(ids)} identities for a step of {batch} samples.")
            return ids
        if self._sample_id_key is not None:
            return self._ids_from_key(batch)
        if self._sample_hash_fields is not None:
            absent = [f for f in self._sample_hash_fields
                      if (f"_arg{f}" if isinstance(f, int) else f) not in self._inputs]
            if absent:
                raise KeyError(f"sample_hash_fields {absent!r} are not among this step's model inputs; samples "
                               "cannot be identified.")
        inputs = self._inputs
        if mirror:
            on_host = {k: mirror.get(id(v)) if isinstance(v, torch.Tensor) else v for k, v in inputs.items()}
            if all(v is not None for v in on_host.values()):
                inputs = on_host
        return hash_batch(inputs, batch)

    # ------------------------------------------------------------------ closing a step
    def _close_step(self) -> GradientRecord:
        with trace_range(f"dattri.capture.step[{self._steps}]"):
            self._last_gradient = None
            gradient = self._build_gradient()
            step = self._steps
            self._steps += 1
            self._barrier = self._barrier.fresh(self._has_linear_io, self._has_param_grad)
            self._clear_captures()
            self._last_gradient = gradient
            ids = self._sample_identities(self._batch_size(gradient))
            return GradientRecord(step=step, input_hash=ids, gradient=gradient, sample_id_key=self._sample_id_key)

    def _emit(self, record: GradientRecord) -> None:
        for cb in self._callbacks:
            cb.on_step_end(record)

    @staticmethod
    def _merge_parts(parts: list) -> torch.Tensor:
        """Device parts ``[(device index, tensor)]`` in device order, on the first device."""
        tensors = [t for _dev, t in sorted(parts, key=lambda item: item[0])]
        if len(tensors) == 1:
            return tensors[0]
        home = tensors[0].device
        return torch.cat([t.to(home) for t in tensors], dim=0)

    def _flush_deferred(self) -> None:
        """Run the step's deferred per-sample outer products (one grouped launch per shape)."""
        self._share.flush_outer()
        for buf in self._layers.values():
            with buf.lock:
                _StepShare.resolve(buf.dense)

    def _entry(self, name: str, buf: LayerBuffer, acts, grads, dense):
        """``(data, representation, layer type, indexing)`` of one invocation of a layer."""
        batch_first = name not in self._non_batch_first
        style = (buf.proj_kw or {}).get("style", "logra") if buf.proj_kw else None
        if dense or style in ("dense", "mask") or self._config.capture_style == "materialized":
            if not dense:
                raise RuntimeError(f"nothing was captured for layer {name!r}: run backward() inside collect().")
            return self._merge_parts(dense), "materialized", buf.layer_type, "batch"
        if not acts or not grads:
            raise RuntimeError(f"nothing was captured for layer {name!r}: run backward() inside collect().")
        a, g = self._merge_parts(acts), self._merge_parts(grads)
        if buf.proj_kw is not None:
            tokens = a.shape[1 if batch_first else 0] > 1
            return (Factorized(a, g, module_kwargs=None, batch_first=batch_first), "factorized", "nn.Linear",
                    "batch_token" if tokens else "batch")
        if a.ndim == 1 and is_embedding(buf.layer_type):
            a, g = a.unsqueeze(0), g.unsqueeze(0)
        per_token = a.ndim >= 3 or not a.is_floating_point()
        return (Factorized(a, g, module_kwargs=buf.module_kwargs, batch_first=batch_first), "factorized",
                buf.layer_type, "batch_token" if per_token else "batch")

    def _build_gradient(self) -> Gradient:
        self._flush_deferred()
        data, rep, types, idx = {}, {}, {}, {}
        for name, buf in self._layers.items():
            if buf.forwards == 0:
                self._warn_absent(name)
                continue
            for k, (acts, grads, dense) in enumerate(buf.invocations()):
                out = name if k == 0 else f"{name}@{k + 1}"
                data[out], rep[out], types[out], idx[out] = self._entry(name, buf, acts, grads, dense)
        for layer, grads in self._params.items():
            for pname, grad in grads.items():
                if grad is not None:
                    key = f"{layer}.{pname}"
                    data[key], rep[key], types[key], idx[key] = grad, "materialized", PARAM_GRAD_TYPES, "batch"
        if not data:
            raise RuntimeError("the step assembled no gradient: run backward() inside collect().")
        self._warn_shared_rows(data, types)
        return Gradient(rep, data, types, idx)

    def _warn_absent(self, name: str) -> None:
        if ("absent", name) in self._warned:
            return
        self._warned.add(("absent", name))
        if ".dattri_experts." in name or ".dattri_router" in name:
            warnings.warn(f"the fused-MoE stand-in {name} did not run in this step; its parameters are not in the "
                          "record.", stacklevel=2)
            return
        warnings.warn(f"hooked layer {name} ran no forward in this step and is not in its record. A model that "
                      "uses the weight without calling the module (a functional call or a fused kernel) is never "
                      "captured there -- see gradient.hooks.override_layers. Reported once per layer.", stacklevel=2)

    def _warn_shared_rows(self, data: dict, types: dict) -> None:
        def rows(v):
            return v.activation.shape[0 if v.batch_first else 1] if isinstance(v, Factorized) else v.shape[0]

        batch = max((rows(v) for n, v in data.items() if types.get(n) != PARAM_GRAD_TYPES), default=0)
        if batch <= 1:
            return
        for name, v in data.items():
            if isinstance(v, Factorized) and rows(v) == 1 and ("shared", name) not in self._warned:
                self._warned.add(("shared", name))
                warnings.warn(f"layer {name!r} captured one row for a step of {batch} samples (an input shared by "
                              "the whole batch, e.g. a positional embedding): its gradient is summed over the batch "
                              "and is treated as one shared row, not per-sample.", stacklevel=3)

    def _clear_captures(self) -> None:
        self._share.clear()
        self._group_forwards.clear()
        if self._routed is not None:
            self._routed.reset()
        for buf in self._layers.values():
            buf.clear()
        for grads in self._params.values():
            for pname in grads:
                grads[pname] = None

    # ------------------------------------------------------------------ grouped expert blocks
    def routed_shape(self, x: torch.Tensor) -> tuple[int, int] | None:
        """``(batch, tokens)`` of a declared MoE block whose flattened input is *x*."""
        return None if self._routed is None else self._routed.identity_shape(x)

    def _watched_per_layer(self) -> bool:
        """Whether a callback looks at individual layers' activations or gradients."""
        base = (HookManagerCallback.on_layer_forward, HookManagerCallback.on_layer_backward)
        return any(getattr(type(cb), hook.__name__, hook) is not hook for cb in self._callbacks for hook in base)

    def grouped_matrices(self, block: GroupedExpertCapture, x: torch.Tensor, tokens: int) -> dict | None:
        """The projections of a grouped expert block (``up_a``, ``up_g``, ``down_a``,
        ``down_g``) when its captures allow the grouped path, else ``None``: every expert
        projection hooked with one LoGra projection and materialized at *tokens* tokens, no
        preconditioning or offload, no per-layer callback, not inside a backward."""
        if not self._collecting or self._offload or _backward_task() != -1 or self._watched_per_layer():
            return None
        if self._preconditioner is not None and self._preconditioner.enabled:
            return None
        sides = []
        for names in (block.up_names, block.down_names):
            bufs = [self._layers.get(n) for n in names]
            first = bufs[0]
            if first is None or first.proj_kw is None or first.proj_kw.get("style", "logra") != "logra":
                return None
            if any(b is None or b.proj_kw != first.proj_kw or b.capture_style != first.capture_style
                   or b.forwards or b.acts or b.waiting for b in bufs):
                return None
            sides.append(first)
        up, down = sides
        experts = block.experts
        widths = {"up_a": (up, "a", x.shape[1]), "up_g": (up, "g", experts.gate_up_proj.shape[1]),
                  "down_a": (down, "a", experts.down_proj.shape[2]), "down_g": (down, "g", x.shape[1])}
        out = {}
        for key, (buf, side, width) in widths.items():
            pm = _projection_matrix(buf, side, x.new_empty(1, width), self._projector)
            if pm.bias_row is not None or (x.is_cuda and pm.matrix_t is None):
                return None
            out[key] = pm
        for a_key, g_key, buf in (("up_a", "up_g", up), ("down_a", "down_g", down)):
            if not ops.should_materialize(buf.capture_style, tokens, out[a_key].proj_dim, out[g_key].proj_dim):
                return None
        return out

    def grouped_forward(self, block: GroupedExpertCapture) -> None:
        """A grouped block ran forward: the step waits for its backward."""
        key = f"{block.name}#grouped"
        with self._lock:
            self._barrier.ran.add(key)
            self._group_forwards[key] = self._group_forwards.get(key, 0) + 1

    def grouped_backward(self, block: GroupedExpertCapture, parts: dict, device: torch.device) -> None:
        """A grouped block's backward delivered ``{expert projection name: (B, k_g * k_a)}``."""
        dev = device.index if device.type == "cuda" else 0
        key = f"{block.name}#grouped"
        with self._lock:
            b = self._barrier
            invocation = b.fires.get(key, 0)
            forwards = self._group_forwards.get(key, 0)
            position = max(forwards - 1 - invocation, 0)  # backwards run in reverse forward order
            for name, mat in parts.items():
                buf = self._layers[name]
                with buf.lock:
                    buf.dense.append((dev, mat))
                    buf.pairs.append((dev, position))
                    buf.forwards += 1
            b.fires[key] = invocation + 1
            if b.fires[key] >= forwards:
                b.finished.add(key)
            record = self._close_linear_side()
        if record is not None:
            self._emit(record)

    # ------------------------------------------------------------------ secondary passes
    def save_state(self) -> dict:
        """Snapshot of the step in flight, for a secondary forward/backward through the same
        hooks (restore it with :meth:`load_state`): ``{"layers", "params", "inputs", "step",
        "last_gradient", "barrier", "pending_ids", "groups"}``."""
        self._flush_deferred()
        with self._lock:
            barrier = self._barrier.copy()
        return {"layers": {n: b.snapshot() for n, b in self._layers.items()},
                "params": {n: dict(g) for n, g in self._params.items()}, "inputs": dict(self._inputs),
                "step": self._steps, "last_gradient": self._last_gradient, "barrier": barrier,
                "pending_ids": self._pending_ids, "groups": dict(self._group_forwards)}

    def clear_state(self) -> None:
        """Empty the layer and parameter buffers (the step counter is kept)."""
        with self._lock:
            self._barrier.ran.clear()
        self._clear_captures()

    def load_state(self, state: dict) -> None:
        """Return to a :meth:`save_state` snapshot."""
        for name, buf in self._layers.items():
            buf.restore(state["layers"].get(name))
        for name, grads in self._params.items():
            grads.clear()
            grads.update(state["params"].get(name, {}))
        self._inputs = state["inputs"]
        self._last_gradient = state["last_gradient"]
        self._pending_ids = state["pending_ids"]
        self._group_forwards = dict(state.get("groups", {}))
        with self._lock:
            self._steps = state["step"]
            self._barrier = state["barrier"].copy()

    # ------------------------------------------------------------------ lifecycle
    @contextmanager
    def collect(self, deregister_on_exit: bool = False) -> Generator[HookManager, None, None]:
        """Capture every backward inside the block; callbacks' ``on_context_end`` runs at exit."""
        self.register()
        self._clear_captures()
        with self._lock:
            self._barrier = self._barrier.fresh(self._has_linear_io, self._has_param_grad)
        self._last_gradient = None
        self._inputs = {}
        self._collecting = True
        try:
            yield self
        finally:
            self._collecting = False
            for cb in self._callbacks:
                cb.on_context_end()
            if deregister_on_exit:
                kept = self._last_gradient
                self.remove()
                self._last_gradient = kept

    def _install_overrides(self, root: nn.Module, assignment: dict, layer_types: dict) -> None:
        """Forward overrides: fused-expert stand-ins for declared MoE blocks (their proxies
        replace the blocks in the assignment) and module-by-module sequence mixers."""
        if self._moe_blocks:
            self._routed = RoutedTokenTracker(root, self._moe_blocks)
            fused = [n for n in find_fused_experts(root) if self._routed.covers(n)]
            if fused:
                tracker = self._routed
                proxies, reverts = install_fused_experts(
                    root, fused, lambda: self._collecting,
                    grouped=lambda name, experts: GroupedExpertCapture(self, name, experts, PROXY_EXPERTS),
                    place=lambda x: tracker.place if tracker.identity_shape(x) is not None else None)
                self._reverts.extend(reverts)
                layer_types.update(proxies)
                for proxy in proxies:
                    owner = proxy.rsplit(".", 3 if ".dattri_experts." in proxy else 1)[0]
                    assignment.pop(owner, None)
                    assignment[proxy] = LINEAR_IO
        mixers = find_sequence_mixers(root)
        if mixers:
            self._reverts.extend(install_sequence_mixer_forward(root, list(mixers), lambda: self._collecting))
        self._bind_expert_parallel(root)

    def _bind_expert_parallel(self, root: nn.Module) -> None:
        """Let every fused expert-parallel block take its expert taps' captures itself (the
        grouped capture inside the peer-memory kernels) when the captures allow it."""
        if "dattri_llm_b200.parallel.moe" not in sys.modules:
            return  # no expert-parallel block can exist
        from dattri_llm_b200.parallel.moe import EPGroupedCapture, ExpertParallelMoE

        for name, mod in root.named_modules():
            if isinstance(mod, ExpertParallelMoE) and mod.fused:
                mod.grouped_capture = EPGroupedCapture(self, name, mod)
                self._reverts.append(lambda m=mod: setattr(m, "grouped_capture", None))

    def register(self) -> None:
        """Install every hook and override (idempotent)."""
        if self._installed:
            return
        model = self._model
        root = getattr(model, "module", model)
        self._model_hooks = [root.register_forward_pre_hook(self._on_model_inputs, with_kwargs=True),
                             root.register_forward_hook(self._on_model_output)]
        assignment = resolve_hook_assignments(root, self._config)
        layer_types = dict(self._config.layer_types or {})
        self._install_overrides(root, assignment, layer_types)
        plain = {n for n, kind in assignment.items() if kind == LINEAR_IO}
        invasive = {n for n, kind in assignment.items() if kind == INVASIVE_LINEAR_IO}
        per_batch = {n for n, kind in assignment.items() if kind == PARAM_GRAD}
        captured = plain | invasive
        self._has_linear_io, self._has_param_grad = bool(captured), bool(per_batch)
        if self._preconditioner is not None:
            self._check_preconditionable(per_batch)
        self._n_weights = 0
        if captured:
            if self._config.projection_kwargs is not None and self._projector is None:
                self._projector = ops.DattriProjector(self._config.projector)
            if self._preconditioner is not None:
                self._preconditioner.projector = self._projector
            self._layers, self._layer_hooks = register_linear_io_hooks(
                model, layer_names=captured, on_layer_forward=self._on_layer_forward,
                on_layer_backward=self._on_layer_backward, type_overrides=layer_types,
                kwargs_overrides=self._config.module_kwargs, projection_kwargs=self._config.projection_kwargs,
                capture_style=self._config.capture_style, projector=self._projector, offload_to_cpu=self._offload,
                preconditioner=self._preconditioner, include_frozen=self._config.include_frozen,
                routed=self._routed, step_share=self._share)
            self._warn_frozen(root, captured)
            self._n_weights, self._weight_hooks = register_linear_param_hooks(
                model, layer_names=plain, on_linear_param_grad=self._on_weight_grad_final)
            if invasive:
                self._reverts.extend(install_invasive_forward(model, invasive, lambda: self._collecting))
        self._n_param_hooks = 0
        if per_batch:
            self._params, self._param_hooks = register_param_grad_hooks(
                model, layer_names=per_batch, on_param_grad=self._on_param_grad, offload_to_cpu=self._offload)
            self._n_param_hooks = len(self._param_hooks)
        self._barrier = self._barrier.fresh(self._has_linear_io, self._has_param_grad)
        self._warn_unused_options(layer_types)
        self._installed = True

    def _warn_unused_options(self, layer_types: dict) -> None:
        hooked = set(self._layers) | set(self._params)
        unused = sorted(set(self._config.layer_types or {}) - hooked)
        if unused:
            warnings.warn(f"HookManagerConfig.layer_types names layers that are not hooked ({unused}); those type "
                          "overrides do nothing.", stacklevel=3)
        unused = sorted(self._non_batch_first - set(self._layers))
        if unused:
            warnings.warn(f"non_batch_first_layers names layers without factorized (linear_io) capture ({unused}); "
                          "the flag does nothing for them.", stacklevel=3)
        if self._routed is not None:
            self._routed.bind(self._layers)
            unused = sorted(blk for blk in self._moe_blocks
                            if not any(n == blk or n.startswith(blk + ".") for n in self._routed.layers))
            if unused:
                warnings.warn(f"moe_routed_layers names modules with no factorized (linear_io) capture inside "
                              f"({unused}); the flag does nothing for them.", stacklevel=3)

    def remove(self) -> None:
        """Remove every hook and override (idempotent)."""
        if not self._installed:
            return
        remove_hooks(self._model_hooks)
        remove_hooks(self._layer_hooks)
        remove_hooks(self._weight_hooks)
        remove_hooks(self._param_hooks)
        for revert in self._reverts:
            revert()
        self._reverts = []
        if self._routed is not None:
            self._routed.remove()
            self._routed = None
        self._layers.clear()
        self._params.clear()
        self._last_gradient = None
        self._share.clear()
        if self._projector is not None:
            self._projector.close()
            self._projector = None
        self._installed = False

    def _warn_frozen(self, root: nn.Module, candidates: set[str]) -> None:
        modules = dict(root.named_modules())

        def frozen(name):
            m = modules.get(name)
            return m is not None and not has_trainable_params(m)

        if self._config.include_frozen:
            names = sorted(n for n in self._layers if frozen(n))
            if names:
                warnings.warn(
                    f"{len(names)} hooked layer(s) have no trainable parameter (include_frozen=True), e.g. "
                    f"{names[:3]}. Such a layer gets a gradient only through something upstream that requires "
                    "grad (typically the input embedding); a step in which no hooked layer gets one cannot be "
                    "completed and raises at the end of its backward -- under DDP/FSDP the other ranks may then "
                    "wait in their collectives.", stacklevel=3)
        elif not self._layers:
            skipped = sorted(n for n in candidates if frozen(n))
            if skipped:
                warnings.warn(f"no layer is hooked: the {len(skipped)} linear-IO candidate(s) (e.g. {skipped[:3]}) "
                              "have no trainable parameter and include_frozen is False; pass "
                              "HookManagerConfig(include_frozen=True) to capture frozen layers.", stacklevel=3)

    def _check_preconditionable(self, per_batch_layers: set[str]) -> None:
        if per_batch_layers:
            raise ValueError("HookManager(optimizer=...) preconditions per-sample (linear_io) captures, but these "
                             f"layers are assigned param_grad: {sorted(per_batch_layers)[:5]}.")
        for name, kw in (self._config.projection_kwargs or {}).items():
            if kw.get("style", "logra") == "logra":
                raise ValueError(f"projection_kwargs[{name!r}] uses the 'logra' style, whose factors cannot go "
                                 "through the optimizer's per-coordinate map; use no projection, 'mask' or 'dense'.")

    # ------------------------------------------------------------------ properties
    @property
    def supports_preconditioning(self) -> bool:
        """Whether the manager was given an optimizer."""
        return self._preconditioner is not None

    @property
    def precondition(self) -> bool:
        """Whether captures are currently preconditioned."""
        return self._preconditioner is not None and self._preconditioner.enabled

    @precondition.setter
    def precondition(self, enabled: bool) -> None:
        if self._preconditioner is None:
            if enabled:
                raise ValueError("this HookManager was built without an optimizer; pass optimizer= at "
                                 "construction to precondition captures.")
            return
        self._preconditioner.enabled = bool(enabled)

    def add_callback(self, callback) -> None:
        """Append a callback (``on_register`` runs at once)."""
        self._callbacks.append(callback)
        if hasattr(callback, "on_register"):
            callback.on_register(self)

    @property
    def callbacks(self) -> list:
        """The registered callbacks."""
        return self._callbacks

    @property
    def model(self) -> nn.Module:
        """The model the manager was built on."""
        return self._model

    @property
    def config(self) -> HookManagerConfig:
        """The capture configuration."""
        return self._config

    @property
    def projector(self) -> ops.DattriProjector | None:
        """The shared projector (``None`` without projection)."""
        return self._projector

    @property
    def sample_id_key(self):
        """The identifier field, or ``None`` for content hashing."""
        return self._sample_id_key

    @property
    def sample_hash_fields(self):
        """The hashed input fields, or ``None`` for every field."""
        return self._sample_hash_fields

    @property
    def layer_names(self) -> list[str]:
        """Layers hooked with linear-IO capture."""
        return list(self._layers)

    @property
    def layer_name(self) -> list[str]:
        """Alias of :attr:`layer_names`."""
        return list(self._layers)

    @property
    def param_layer_names(self) -> list[str]:
        """Layers hooked with param_grad capture."""
        return list(self._params)

    @property
    def steps_collected(self) -> int:
        """Completed steps so far."""
        return self._steps

    def reset_steps(self, to: int = 0) -> None:
        """Restart the step counter at *to*."""
        with self._lock:
            self._steps = to

    def get_gradient(self) -> Gradient:
        """The last completed step's gradient.

        Raises:
            RuntimeError: before any step completed.
        """
        if self._last_gradient is None:
            raise RuntimeError("no step has completed yet: call get_gradient() after a backward() run inside "
                               "collect().")
        return self._last_gradient
