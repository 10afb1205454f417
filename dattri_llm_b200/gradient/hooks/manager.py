"""``HookManager``: turns per-layer hook fires into one ``GradientRecord`` per backward.

Step-completion barrier (parity: reference ``dattri_llm/gradient/hooks/manager.py``):

(a) every hooked layer that ran forward this step has received as many backward
    fires as it had forwards, and
(b) when linear-IO layers own trainable parameters, their gradients are final --
    every post-accumulate-grad hook fired, or (under FSDP, whose reduce-scatter
    writes gradients after the hooks) the end-of-backward engine callback ran;
(c) every ``param_grad`` hook fired.

When all hold, the step is assembled (invocations split into ``name@k`` virtual
layers, parts from several devices concatenated), identified (content hashes,
``sample_id_key`` values, or ids handed in with :meth:`HookManager.set_sample_ids`)
and dispatched to the callbacks outside the lock, so a callback may run a
secondary forward/backward through the same hooks.  Forwards left unmatched at
the end of the backward (activation checkpointing's first pass) are reconciled
away; a step in which no hooked layer received a gradient raises.

B200-specific: the manager clears the per-step activation-projection share of
the hooks (q/k/v, gate/up read one projection), and sample identities can be
supplied by the data pipeline (hashed on the host from the pinned batch while
the GPU runs) instead of being computed from device tensors at step end.
"""

from __future__ import annotations

import operator
import threading
import warnings
from collections.abc import Callable, Generator, Iterable
from contextlib import contextmanager

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
from dattri_llm_b200.gradient.hooks.routing import RoutedTokenTracker
from dattri_llm_b200.gradient.ops import PARAM_GRAD_TYPES, is_embedding
from dattri_llm_b200.utils.autograd import queue_backward_end_callback
from dattri_llm_b200.utils.hashing import hash_batch
from dattri_llm_b200.utils.tracing import trace_range

_TASK_ID = getattr(torch._C, "_current_graph_task_id", None)


def _graph_task_id() -> int:
    """Id of the running backward graph task (-1 outside a backward)."""
    return _TASK_ID() if _TASK_ID is not None else -1


def _first_grad_tensor(output: object) -> torch.Tensor | None:
    if isinstance(output, torch.Tensor):
        return output if output.requires_grad else None
    try:
        values = output.values() if isinstance(output, dict) else output
        for v in values:
            found = _first_grad_tensor(v)
            if found is not None:
                return found
    except TypeError:
        return None
    return None


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
        self._model = model
        self._callbacks: list = list(callbacks or [])
        self._preconditioner = None
        if optimizer is not None:
            from dattri_llm_b200.gradient.optimizer_state import GradientPreconditioner, OptimizerSnapshot

            root = getattr(model, "module", model)
            self._preconditioner = GradientPreconditioner(
                lambda: OptimizerSnapshot(root, optimizer() if callable(optimizer) else optimizer))
        if isinstance(sample_hash_fields, (str, int)):
            sample_hash_fields = [sample_hash_fields]
        self._sample_hash_fields = None if sample_hash_fields is None else tuple(sample_hash_fields)
        if self._sample_hash_fields is not None:
            if sample_id_key is not None:
                raise ValueError("sample_id_key and sample_hash_fields are alternative identifier "
                                 "schemes; pass one of them.")
            if not self._sample_hash_fields:
                raise ValueError("sample_hash_fields must name at least one field.")
        self._sample_id_key = sample_id_key
        self._offload = offload_to_cpu
        self._non_batch_first = set(non_batch_first_layers or ())
        self._moe_declared = set(moe_routed_layers or ())
        self._routed: RoutedTokenTracker | None = None
        self._override_reverts: list = []
        self._invasive_reverts: list = []
        self._warned_silent: set[str] = set()
        self._warned_broadcast: set[str] = set()
        self._warned_orphans: set[frozenset] = set()
        self._config = config if config is not None else HookManagerConfig()
        self._projector: ops.DattriProjector | None = None
        self._share = _StepShare()
        self._next_ids: list[str] | None = None
        self._host_mirror: dict[int, torch.Tensor] | None = None

        self._step_count = 0
        self._collecting = False
        self._last_gradient: Gradient | None = None
        self._step_lock = threading.Lock()
        self._seen_bwd: set[str] = set()
        self._bwd_counts: dict[str, int] = {}
        self._active: set[str] = set()
        self._orphaned: set[str] = set()
        self._bwd_done = True
        self._grad_done = True
        self._mlp_hook_count = 0
        self._n_mlp_params = 0
        self._mlp_ready = False
        self._end_scheduled = False
        self._saw_recompute = False
        self._outer_task = -1
        self._last_inputs: dict = {}
        self._registered = False
        self._fwd_handle = None
        self._out_handle = None
        self._has_linear_io = False
        self._has_param_grad = False
        self._buffers: dict = {}
        self._handles: list = []
        self._mlp_handles: list = []
        self._n_layers = 0
        self._param_buffers: dict = {}
        self._param_handles: list = []
        self._n_params_hooked = 0
        self._param_hook_count = 0
        self.register()
        for cb in self._callbacks:
            if hasattr(cb, "on_register"):
                cb.on_register(self)

    # ------------------------------------------------------------------ inputs
    def _capture_model_input(self, _module, args: tuple, kwargs: dict) -> None:
        if not self._collecting:
            return
        if torch.is_grad_enabled():
            self._last_gradient = None
        if self._sample_hash_fields is not None:
            self._last_inputs = {
                (f"_arg{f}" if isinstance(f, int) else f): (args[f] if isinstance(f, int) else kwargs[f])
                for f in self._sample_hash_fields
                if (f < len(args) if isinstance(f, int) else f in kwargs)
            }
            return
        captured = {k: v for k, v in kwargs.items() if isinstance(v, torch.Tensor)}
        if not captured:
            captured = {f"_arg{i}": a for i, a in enumerate(args) if isinstance(a, torch.Tensor)}
        key = self._sample_id_key
        if key is not None:
            if isinstance(key, int):
                if key < len(args):
                    captured[f"_arg{key}"] = args[key]
            elif key in kwargs:
                captured[key] = kwargs[key]
        self._last_inputs = captured

    def set_host_inputs(self, mirror: dict[int, torch.Tensor] | None) -> None:
        """Host copies of the next step's device inputs, keyed by ``id()`` of the device
        tensor (consumed by that step).  When every model input of the step is one of them,
        its content hash is computed from the host copies: the same hash, without reading
        device tensors back (which would wait for the GPU at every step)."""
        self._host_mirror = mirror

    def set_sample_ids(self, ids: list[str] | None) -> None:
        """Identities of the samples of the next completed step (consumed by that step).

        Lets a data pipeline hash the batch on the host (from the pinned copy it sends
        to the GPU) instead of the manager reading device tensors back at step end.
        """
        self._next_ids = None if ids is None else [str(i) for i in ids]

    # ------------------------------------------------------------------ barrier
    def _dispatch_layer_forward(self, name, activation, layer_type, module_kwargs) -> None:
        if name not in self._active:
            with self._step_lock:
                self._active.add(name)
        if self._collecting:
            task = _graph_task_id()
            if task != -1:  # a forward inside a backward: checkpoint recomputation
                with self._step_lock:
                    self._saw_recompute = True
                    if self._outer_task == -1:
                        self._outer_task = task
                    if (self._n_mlp_params > 0 and not self._end_scheduled
                            and queue_backward_end_callback(self._on_backward_end)):
                        self._end_scheduled = True
        for cb in self._callbacks:
            cb.on_layer_forward(name, activation, layer_type, module_kwargs)

    def _check_step_bwd_complete(self, name, grad_output, layer_type, module_kwargs) -> None:
        for cb in self._callbacks:
            cb.on_layer_backward(name, grad_output, layer_type, module_kwargs)
        if not self._collecting:
            return
        record = None
        with self._step_lock:
            if (self._n_mlp_params > 0 and not self._end_scheduled
                    and queue_backward_end_callback(self._on_backward_end)):
                self._end_scheduled = True
                if self._outer_task == -1:
                    self._outer_task = _graph_task_id()
            self._bwd_counts[name] = self._bwd_counts.get(name, 0) + 1
            if self._bwd_counts[name] >= self._buffers[name]["_fwd_fires"]:
                self._seen_bwd.add(name)
            if self._bwd_hooks_done():
                record = self._check_mlp_done()
        if record is not None:
            self._dispatch_step_end(record)

    def _on_backward_end(self) -> None:
        if not self._collecting:
            return
        record = None
        with self._step_lock:
            if not self._end_scheduled:
                return
            if self._outer_task != -1 and _graph_task_id() != self._outer_task:
                return  # end of a nested (recomputation) backward, not ours
            self._mlp_ready = True
            self._reconcile_unmatched_forwards()
            orphaned = sorted(self._orphaned)
            stalled = self._has_linear_io and bool(orphaned) and not self._active and not self._bwd_done
            record = None if stalled else self._check_mlp_done()
        if stalled:
            raise RuntimeError(
                f"No hooked layer received a gradient this step: {orphaned[:8]}"
                f"{'...' if len(orphaned) > 8 else ''} ran forward but the backward pass did not "
                "reach them, so the step cannot complete. A layer receives a gradient only when the "
                "loss depends on its output through something that requires grad; with frozen layers "
                "(include_frozen=True) a parameter or input upstream of them must require grad.",
            )
        if orphaned and record is not None:
            key = frozenset(orphaned)
            if key not in self._warned_orphans:
                self._warned_orphans.add(key)
                warnings.warn(
                    f"Hooked layers {orphaned[:8]}{'...' if len(orphaned) > 8 else ''} ran forward "
                    "but received no gradient this step and are left out of its record (a detached "
                    "branch, or a frozen layer with nothing trainable upstream). Reported once per "
                    "layer set.",
                    stacklevel=2,
                )
        if record is not None:
            self._dispatch_step_end(record)

    def _capture_model_output(self, _module, _args, output) -> None:
        if not self._collecting or self._n_layers == 0 or not torch.is_grad_enabled():
            return
        t = _first_grad_tensor(output)
        if t is not None:
            t.register_hook(self._on_backward_begin)

    def _on_backward_begin(self, _grad) -> None:
        if not self._collecting:
            return
        with self._step_lock:
            if not self._end_scheduled and queue_backward_end_callback(self._on_backward_end):
                self._end_scheduled = True
                if self._outer_task == -1:
                    self._outer_task = _graph_task_id()

    def _reconcile_unmatched_forwards(self) -> None:
        for name, buf in self._buffers.items():
            with buf["_lock"]:
                had_orphans = any(buf["_pending"].values())
                if had_orphans:
                    self._drop_orphan_forwards(buf)
                buf["_pending"] = {}
                matched = len(buf["_pair_pos"])
                buf["_fwd_fires"] = matched
            if matched == 0 and had_orphans:
                self._active.discard(name)
                self._orphaned.add(name)
            elif matched == 0:
                self._active.discard(name)
            elif self._bwd_counts.get(name, 0) >= matched:
                self._seen_bwd.add(name)

    @staticmethod
    def _drop_orphan_forwards(buf: dict) -> None:
        """Keep only matched forwards and renumber invocation positions densely."""
        matched: dict[int, list[int]] = {}
        for dev, pos in buf["_pair_pos"]:
            matched.setdefault(dev, []).append(pos)
        remap = {dev: {p: r for r, p in enumerate(sorted(ps))} for dev, ps in matched.items()}
        if buf["_proj_kw"] is None:
            seen: dict[int, int] = {}
            kept = []
            for dev, part in buf["_act_parts"]:
                pos = seen.get(dev, 0)
                seen[dev] = pos + 1
                if pos in remap.get(dev, {}):
                    kept.append((dev, part))
            buf["_act_parts"] = kept
        buf["_pair_pos"] = [(dev, remap[dev][pos]) for dev, pos in buf["_pair_pos"]]

    def _check_step_mlp_param_complete(self, _l, _p, _g) -> None:
        if not self._collecting:
            return
        record = None
        with self._step_lock:
            self._mlp_hook_count += 1
            if self._mlp_hook_count >= self._n_mlp_params:
                record = self._check_mlp_done()
        if record is not None:
            self._dispatch_step_end(record)

    def _bwd_hooks_done(self) -> bool:
        if self._n_layers == 0:
            return True
        return len(self._active) > 0 and len(self._seen_bwd) == len(self._active)

    def _check_mlp_done(self) -> GradientRecord | None:
        params_done = (self._n_mlp_params == 0 or self._mlp_ready
                       or self._mlp_hook_count >= self._n_mlp_params)
        if self._bwd_hooks_done() and params_done:
            self._bwd_done = True
            return self._check_step_complete()
        return None

    def _check_step_grad_complete(self, _l, _p, _g) -> None:
        if not self._collecting:
            return
        record = None
        with self._step_lock:
            self._param_hook_count += 1
            if self._param_hook_count >= self._n_params_hooked:
                self._param_hook_count = 0
                self._grad_done = True
                record = self._check_step_complete()
        if record is not None:
            self._dispatch_step_end(record)

    def _check_step_complete(self) -> GradientRecord | None:
        return self._finalize_step() if self._bwd_done and self._grad_done else None

    # ------------------------------------------------------------------ assembly
    def _extract_sample_ids(self, expected: int) -> list[str]:
        key = self._sample_id_key
        fld = f"_arg{key}" if isinstance(key, int) else key
        if fld not in self._last_inputs:
            raise KeyError(
                f"sample_id_key={key!r} was not found among the captured model inputs "
                f"{sorted(self._last_inputs)}; cannot assign sample identities.",
            )
        v = self._last_inputs[fld]
        ids = v.reshape(-1).tolist() if isinstance(v, torch.Tensor) else list(v)
        if len(ids) != expected:
            raise ValueError(f"sample_id_key={key!r} yielded {len(ids)} identifiers but the step's "
                             f"batch size is {expected}.")
        return [str(i) for i in ids]

    def _shape_inputs(self) -> list:
        """The captured model inputs that can tell the batch size: every one but the
        sample-identifier field (its length is what gets checked against the batch)."""
        key = self._sample_id_key
        skip = None if key is None else (f"_arg{key}" if isinstance(key, int) else key)
        return [v for k, v in self._last_inputs.items() if k != skip]

    def _input_batch_size(self, default: int = 1) -> int:
        for v in self._shape_inputs():
            if isinstance(v, torch.Tensor) and v.ndim > 0:
                return v.shape[0]
        return default

    def _step_batch_size(self, gradient: Gradient) -> int:
        try:
            b = gradient.batch_size
        except ValueError:
            return self._input_batch_size()
        inputs = self._shape_inputs()
        for v in inputs:
            if (isinstance(v, torch.Tensor) and v.ndim > 0 and v.shape[0] == b) or (
                    isinstance(v, (list, tuple)) and len(v) == b):
                return b
        return self._input_batch_size(default=b) if inputs else b

    def _finalize_step(self) -> GradientRecord:
        with trace_range(f"dattri.capture.step[{self._step_count}]"):
            return self._finalize_step_inner()

    def _finalize_step_inner(self) -> GradientRecord:
        self._last_gradient = None
        gradient = self._assemble_gradient()
        step = self._step_count
        self._step_count += 1
        self._seen_bwd.clear()
        self._bwd_counts.clear()
        self._orphaned.clear()
        self._mlp_hook_count = 0
        self._param_hook_count = 0
        self._mlp_ready = False
        self._end_scheduled = False
        self._saw_recompute = False
        self._outer_task = -1
        self._bwd_done = not self._has_linear_io
        self._grad_done = not self._has_param_grad
        self._reset_layer_buffers()
        self._reset_param_buffers()
        self._last_gradient = gradient
        batch = self._step_batch_size(gradient)
        ids, self._next_ids = self._next_ids, None
        mirror, self._host_mirror = self._host_mirror, None
        if ids is not None:
            if len(ids) != batch:
                raise ValueError(f"set_sample_ids supplied {len(ids)} identities for a step of {batch} samples.")
            input_hash = ids
        elif self._sample_id_key is not None:
            input_hash = self._extract_sample_ids(batch)
        else:
            if self._sample_hash_fields is not None:
                missing = [f for f in self._sample_hash_fields
                           if (f"_arg{f}" if isinstance(f, int) else f) not in self._last_inputs]
                if missing:
                    raise KeyError(f"sample_hash_fields {missing!r} were not found among the model "
                                   "inputs of this step; cannot assign sample identities.")
            inputs = self._last_inputs
            if mirror:
                hosted = {k: mirror.get(id(v)) if isinstance(v, torch.Tensor) else v for k, v in inputs.items()}
                if all(h is not None for h in hosted.values()):
                    inputs = hosted
            input_hash = hash_batch(inputs, batch)
        return GradientRecord(step=step, input_hash=input_hash, gradient=gradient,
                              sample_id_key=self._sample_id_key)

    def _dispatch_step_end(self, record: GradientRecord) -> None:
        for cb in self._callbacks:
            cb.on_step_end(record)

    @staticmethod
    def _concat_parts(parts: list) -> torch.Tensor:
        ordered = [t for _, t in sorted(parts, key=operator.itemgetter(0))]
        if len(ordered) == 1:
            return ordered[0]
        dev = ordered[0].device
        return torch.cat([t if t.device == dev else t.to(dev) for t in ordered], dim=0)

    @staticmethod
    def _split_invocations(buf: dict) -> list[tuple[list, list, list]]:
        pair_pos = buf["_pair_pos"]
        n_inv = max((p for _, p in pair_pos), default=0) + 1
        if n_inv <= 1:
            return [(buf["_act_parts"], buf["_grad_parts"], buf["_proj_parts"])]
        acts = [[] for _ in range(n_inv)]
        grads = [[] for _ in range(n_inv)]
        projs = [[] for _ in range(n_inv)]
        if buf["_proj_parts"]:
            for (dev, part), (_, pos) in zip(buf["_proj_parts"], pair_pos, strict=True):
                projs[pos].append((dev, part))
        elif buf["_proj_kw"] is None:
            seen: dict[int, int] = {}
            for dev, part in buf["_act_parts"]:
                pos = seen.get(dev, 0)
                seen[dev] = pos + 1
                acts[pos].append((dev, part))
            for (dev, part), (_, pos) in zip(buf["_grad_parts"], pair_pos, strict=True):
                grads[pos].append((dev, part))
        else:
            for (dev, part), (_, pos) in zip(buf["_act_parts"], pair_pos, strict=True):
                acts[pos].append((dev, part))
            for (dev, part), (_, pos) in zip(buf["_grad_parts"], pair_pos, strict=True):
                grads[pos].append((dev, part))
        return list(zip(acts, grads, projs, strict=True))

    def _flush_deferred(self) -> None:
        """Run the step's deferred per-sample outer products and put their results in place."""
        self._share.flush_outer()
        for buf in self._buffers.values():
            with buf["_lock"]:
                _StepShare.resolve(buf["_proj_parts"])

    def _assemble_gradient(self) -> Gradient:
        self._flush_deferred()
        data, rep, types, idx = {}, {}, {}, {}
        for lname, buf in self._buffers.items():
            if buf["_fwd_fires"] == 0:
                self._warn_silent(lname)
                continue
            batch_first = lname not in self._non_batch_first
            proj_kw = buf["_proj_kw"]
            style = proj_kw.get("style", "logra") if proj_kw else None
            for k, (acts, grads, projs) in enumerate(self._split_invocations(buf)):
                out = lname if k == 0 else f"{lname}@{k + 1}"
                if projs or style in ("dense", "mask") or self._config.capture_style == "materialized":
                    if not projs:
                        raise RuntimeError(f"Layer '{lname}' has no buffered data. Ensure backward() "
                                           "was called inside the collect() context.")
                    data[out], rep[out], types[out], idx[out] = (
                        self._concat_parts(projs), "materialized", buf["_class_name"], "batch")
                    continue
                if not acts or not grads:
                    raise RuntimeError(f"Layer '{lname}' has no buffered data. Ensure backward() was "
                                       "called inside the collect() context.")
                a, g = self._concat_parts(acts), self._concat_parts(grads)
                if proj_kw is not None:
                    data[out] = Factorized(a, g, module_kwargs=None, batch_first=batch_first)
                    rep[out], types[out] = "factorized", "nn.Linear"
                    idx[out] = "batch_token" if a.shape[1 if batch_first else 0] > 1 else "batch"
                    continue
                if a.ndim == 1 and is_embedding(buf["_class_name"]):
                    a, g = a.unsqueeze(0), g.unsqueeze(0)
                data[out] = Factorized(a, g, module_kwargs=buf["_module_kwargs"], batch_first=batch_first)
                rep[out], types[out] = "factorized", buf["_class_name"]
                idx[out] = "batch_token" if a.ndim >= 3 or not a.is_floating_point() else "batch"
        for lname, pbuf in self._param_buffers.items():
            for pname, grad in pbuf.items():
                if grad is None:
                    continue
                key = f"{lname}.{pname}"
                data[key], rep[key], types[key], idx[key] = grad, "materialized", PARAM_GRAD_TYPES, "batch"
        if not data:
            raise RuntimeError("No gradient data assembled. Ensure backward() was called inside the "
                               "collect() context.")
        self._warn_broadcast(data, types)
        return Gradient(rep, data, types, idx)

    def _warn_silent(self, lname: str) -> None:
        if lname in self._warned_silent:
            return
        self._warned_silent.add(lname)
        if ".dattri_experts." in lname or ".dattri_router" in lname:
            warnings.warn(f"Fused MoE proxy {lname} did not run in this step, so its parameters are "
                          "absent from the record.", stacklevel=2)
            return
        warnings.warn(
            f"Hooked layer {lname} ran no forward in this step and is absent from its record. If the "
            "model uses the layer's weight without calling the module (a functional call or a fused "
            "kernel), it is never captured; see gradient.hooks.override_layers. Reported once per layer.",
            stacklevel=2,
        )

    def _warn_broadcast(self, data: dict, types: dict) -> None:
        batch = max((v.activation.shape[0 if v.batch_first else 1] if isinstance(v, Factorized) else v.shape[0]
                     for n, v in data.items() if types.get(n) != PARAM_GRAD_TYPES), default=0)
        if batch <= 1:
            return
        for name, v in data.items():
            if not isinstance(v, Factorized) or name in self._warned_broadcast:
                continue
            if v.activation.shape[0 if v.batch_first else 1] == 1:
                self._warned_broadcast.add(name)
                warnings.warn(
                    f"Layer '{name}' produced a broadcast (batch-collapsed) gradient: batch size 1 while "
                    f"the step batch is {batch} (e.g. a positional embedding added to every sample). Its "
                    "gradient is summed over the batch and is NOT per-sample; per-sample attribution "
                    "treats it as a single shared row.",
                    stacklevel=3,
                )

    def _reset_layer_buffers(self) -> None:
        self._active.clear()
        self._share.clear()
        if self._routed is not None:
            self._routed.reset()
        for buf in self._buffers.values():
            buf["activation"] = None
            buf["grad_output"] = None
            buf["_act_parts"] = []
            buf["_grad_parts"] = []
            buf["_proj_parts"] = []
            buf["_pending"] = {}
            buf["_fwd_fires"] = 0
            buf["_pair_pos"] = []

    def _reset_param_buffers(self) -> None:
        for buf in self._param_buffers.values():
            for p in buf:
                buf[p] = None

    # ------------------------------------------------------------------ state
    def save_state(self) -> dict:
        """Snapshot of the in-flight step (for a secondary pass through the same hooks)."""
        self._flush_deferred()
        return {
            "layer_buffers": {n: {
                "_act_parts": list(b["_act_parts"]), "_grad_parts": list(b["_grad_parts"]),
                "_proj_parts": list(b["_proj_parts"]),
                "_pending": {k: list(v) for k, v in b["_pending"].items()},
                "_fwd_fires": b["_fwd_fires"], "_pair_pos": list(b["_pair_pos"]),
                "activation": b["activation"], "grad_output": b["grad_output"],
            } for n, b in self._buffers.items()},
            "param_buffers": {n: dict(b) for n, b in self._param_buffers.items()},
            "last_inputs": dict(self._last_inputs), "step_count": self._step_count,
            "last_gradient": self._last_gradient, "seen_bwd": set(self._seen_bwd),
            "active_layers": set(self._active), "bwd_replica_counts": dict(self._bwd_counts),
            "mlp_param_hook_count": self._mlp_hook_count, "param_hook_count": self._param_hook_count,
            "bwd_done": self._bwd_done, "grad_done": self._grad_done, "mlp_params_ready": self._mlp_ready,
            "backward_end_scheduled": self._end_scheduled, "saw_recompute": self._saw_recompute,
            "outer_task_id": self._outer_task, "next_ids": self._next_ids,
        }

    def clear_state(self) -> None:
        """Empty the layer and parameter buffers (the step counter is kept)."""
        self._reset_layer_buffers()
        self._reset_param_buffers()

    def load_state(self, state: dict) -> None:
        """Restore a :meth:`save_state` snapshot."""
        for name, buf in self._buffers.items():
            s = state["layer_buffers"].get(name, {})
            buf["_act_parts"] = s.get("_act_parts", [])
            buf["_grad_parts"] = s.get("_grad_parts", [])
            buf["_proj_parts"] = s.get("_proj_parts", [])
            buf["_pending"] = s.get("_pending", {})
            buf["_fwd_fires"] = s.get("_fwd_fires", 0)
            buf["_pair_pos"] = s.get("_pair_pos", [])
            buf["activation"] = s.get("activation")
            buf["grad_output"] = s.get("grad_output")
        for name, buf in self._param_buffers.items():
            buf.clear()
            buf.update(state["param_buffers"].get(name, {}))
        self._last_inputs = state["last_inputs"]
        self._last_gradient = state["last_gradient"]
        self._next_ids = state.get("next_ids")
        with self._step_lock:
            self._step_count = state["step_count"]
            self._seen_bwd = state["seen_bwd"]
            self._active = state.get("active_layers", set())
            self._bwd_counts = state["bwd_replica_counts"]
            self._mlp_hook_count = state["mlp_param_hook_count"]
            self._param_hook_count = state["param_hook_count"]
            self._bwd_done = state["bwd_done"]
            self._grad_done = state["grad_done"]
            self._mlp_ready = state["mlp_params_ready"]
            self._end_scheduled = state["backward_end_scheduled"]
            self._saw_recompute = state.get("saw_recompute", False)
            self._outer_task = state.get("outer_task_id", -1)

    # ------------------------------------------------------------------ lifecycle
    @contextmanager
    def collect(self, deregister_on_exit: bool = False) -> Generator[HookManager, None, None]:
        """Capture every backward inside the block; callbacks' ``on_context_end`` runs at exit."""
        self.register()
        self._reset_layer_buffers()
        self._reset_param_buffers()
        self._last_gradient = None
        self._param_hook_count = 0
        self._mlp_ready = False
        self._end_scheduled = False
        self._seen_bwd.clear()
        self._bwd_counts.clear()
        self._orphaned.clear()
        self._last_inputs = {}
        self._collecting = True
        try:
            yield self
        finally:
            self._collecting = False
            for cb in self._callbacks:
                cb.on_context_end()
            if deregister_on_exit:
                last = self._last_gradient
                self.remove()
                self._last_gradient = last

    def register(self) -> None:
        """Install every hook and override (idempotent)."""
        if self._registered:
            return
        model = self._model
        root = getattr(model, "module", model)
        self._fwd_handle = root.register_forward_pre_hook(self._capture_model_input, with_kwargs=True)
        self._out_handle = root.register_forward_hook(self._capture_model_output)
        assignment = resolve_hook_assignments(root, self._config)
        type_overrides = dict(self._config.layer_types or {})
        if self._moe_declared:
            self._routed = RoutedTokenTracker(root, self._moe_declared)
            fused = [n for n in find_fused_experts(root) if self._routed.covers(n)]
            if fused:
                proxy_types, reverts = install_fused_experts(root, fused, lambda: self._collecting)
                self._override_reverts.extend(reverts)
                type_overrides.update(proxy_types)
                for proxy in proxy_types:
                    depth = 3 if ".dattri_experts." in proxy else 1
                    assignment.pop(proxy.rsplit(".", depth)[0], None)
                    assignment[proxy] = LINEAR_IO
        mixers = find_sequence_mixers(root)
        if mixers:
            self._override_reverts.extend(
                install_sequence_mixer_forward(root, list(mixers), lambda: self._collecting))
        lin = {n for n, t in assignment.items() if t == LINEAR_IO}
        pgrad = {n for n, t in assignment.items() if t == PARAM_GRAD}
        inv = {n for n, t in assignment.items() if t == INVASIVE_LINEAR_IO}
        capture = lin | inv
        self._has_linear_io = bool(capture)
        self._has_param_grad = bool(pgrad)
        self._bwd_done = True
        self._n_mlp_params = 0
        self._n_layers = 0
        if self._preconditioner is not None:
            self._validate_preconditioning(pgrad)
        if self._has_linear_io:
            self._bwd_done = False
            if self._config.projection_kwargs is not None and self._projector is None:
                self._projector = ops.DattriProjector(self._config.projector)
            if self._preconditioner is not None:
                self._preconditioner.projector = self._projector
            self._buffers, self._handles = register_linear_io_hooks(
                model, layer_names=capture, on_layer_forward=self._dispatch_layer_forward,
                on_layer_backward=self._check_step_bwd_complete, type_overrides=type_overrides,
                kwargs_overrides=self._config.module_kwargs,
                projection_kwargs=self._config.projection_kwargs,
                capture_style=self._config.capture_style, projector=self._projector,
                offload_to_cpu=self._offload, preconditioner=self._preconditioner,
                include_frozen=self._config.include_frozen, routed=self._routed,
                step_share=self._share)
            self._n_layers = len(self._buffers)
            self._warn_frozen(root, capture)
            self._n_mlp_params, self._mlp_handles = register_linear_param_hooks(
                model, layer_names=lin, on_linear_param_grad=self._check_step_mlp_param_complete)
            if inv:
                self._invasive_reverts = install_invasive_forward(model, inv, lambda: self._collecting)
        self._grad_done = True
        self._n_params_hooked = 0
        if self._has_param_grad:
            self._grad_done = False
            self._param_buffers, self._param_handles = register_param_grad_hooks(
                model, layer_names=pgrad, on_param_grad=self._check_step_grad_complete,
                offload_to_cpu=self._offload)
            self._n_params_hooked = len(self._param_handles)
        if self._config.layer_types:
            unused = sorted(set(self._config.layer_types) - set(self._buffers) - set(self._param_buffers))
            if unused:
                warnings.warn(f"HookManagerConfig.layer_types designated a type for layers that were "
                              f"not hooked: {unused}. These overrides had no effect.", stacklevel=2)
        if self._non_batch_first:
            unused = sorted(self._non_batch_first - set(self._buffers))
            if unused:
                warnings.warn("non_batch_first_layers names layers not hooked with factorized "
                              f"(linear_io) capture; the flag had no effect: {unused}.", stacklevel=2)
        if self._routed is not None:
            self._routed.bind(self._buffers)
            unused = sorted(d for d in self._moe_declared
                            if not any(n == d or n.startswith(d + ".") for n in self._routed.layers))
            if unused:
                warnings.warn("moe_routed_layers names modules with no layer hooked with factorized "
                              f"(linear_io) capture; the flag had no effect: {unused}.", stacklevel=2)
        self._registered = True

    def remove(self) -> None:
        """Remove every hook and override (idempotent)."""
        if not self._registered:
            return
        self._fwd_handle.remove()
        self._fwd_handle = None
        if self._out_handle is not None:
            self._out_handle.remove()
            self._out_handle = None
        remove_hooks(self._handles)
        for revert in self._override_reverts:
            revert()
        self._override_reverts = []
        if self._routed is not None:
            self._routed.remove()
            self._routed = None
        for revert in self._invasive_reverts:
            revert()
        self._invasive_reverts = []
        self._buffers.clear()
        remove_hooks(self._mlp_handles)
        remove_hooks(self._param_handles)
        self._param_buffers.clear()
        self._last_gradient = None
        self._share.clear()
        if self._projector is not None:
            self._projector.close()
            self._projector = None
        self._registered = False

    def _warn_frozen(self, root: nn.Module, candidates: set[str]) -> None:
        modules = dict(root.named_modules())

        def frozen(n):
            m = modules.get(n)
            return m is not None and not has_trainable_params(m)

        if self._config.include_frozen:
            names = sorted(n for n in self._buffers if frozen(n))
            if names:
                warnings.warn(
                    f"{len(names)} hooked layer(s) have no trainable parameter (include_frozen=True), "
                    f"e.g. {names[:3]}. They receive a gradient only through something upstream that "
                    "requires grad (typically the input embedding); a step in which no hooked layer "
                    "receives one cannot complete and raises at the end of that backward -- under "
                    "DDP/FSDP the other ranks may then wait in their collectives.",
                    stacklevel=3,
                )
        elif not self._buffers:
            skipped = sorted(n for n in candidates if frozen(n))
            if skipped:
                warnings.warn(
                    f"No layer hooked: the {len(skipped)} linear-IO candidate(s) (e.g. {skipped[:3]}) "
                    "have no trainable parameter and include_frozen is False. Pass "
                    "HookManagerConfig(include_frozen=True) to capture frozen layers.",
                    stacklevel=3,
                )

    def _validate_preconditioning(self, param_grad_layers: set[str]) -> None:
        if param_grad_layers:
            raise ValueError("HookManager(optimizer=...) preconditions per-sample (linear_io) captures; "
                             f"these layers are assigned param_grad: {sorted(param_grad_layers)[:5]}.")
        for name, kw in (self._config.projection_kwargs or {}).items():
            if kw.get("style", "logra") == "logra":
                raise ValueError(
                    f"projection_kwargs[{name!r}] uses style 'logra', which cannot be preconditioned: "
                    "the optimizer map needs exact gradient entries. Use no projection, 'mask', or 'dense'.",
                )

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
                raise ValueError("This HookManager has no optimizer; pass optimizer= at construction "
                                 "to precondition captures.")
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
        return list(self._buffers)

    @property
    def layer_name(self) -> list[str]:
        """Alias of :attr:`layer_names`."""
        return list(self._buffers)

    @property
    def param_layer_names(self) -> list[str]:
        """Layers hooked with param_grad capture."""
        return list(self._param_buffers)

    @property
    def steps_collected(self) -> int:
        """Completed steps so far."""
        return self._step_count

    def reset_steps(self, to: int = 0) -> None:
        """Restart the step counter at *to*."""
        with self._step_lock:
            self._step_count = to

    def get_gradient(self) -> Gradient:
        """The last completed step's gradient.

        Raises:
            RuntimeError: before any step completed.
        """
        if self._last_gradient is None:
            raise RuntimeError("No gradient available: no step has completed yet. Ensure backward() "
                               "was called inside the collect() context before calling get_gradient().")
        return self._last_gradient
