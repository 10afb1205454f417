"""Forward/backward capture hooks on individual layers.

``register_linear_io_hooks`` puts a forward hook (input activation) and a full
backward hook (output gradient) on each selected layer and buffers what they
see per device.  Forwards are matched to backwards LIFO per device (autograd
runs a device's graph in reverse creation order), which keeps repeated
invocations (weight tying, unrolled loops) and DataParallel replica threads
apart; a forward left unmatched at the end of the backward (activation
checkpointing's first pass) is discarded by the manager.  Parity: reference
``dattri_llm/gradient/hooks/hooks.py:81-866``.

Projected capture (``projection_kwargs``): for a linear layer under the
``logra`` style the activation is projected in the forward hook, so only
``a P_a`` is held until the backward.  On an sm_100 device with bf16 factors:

* the projection is a tcgen05 GEMM against the cached ``P^T``;
* layers reading the *same* input tensor with the same matrix (q/k/v, gate/up)
  share one activation projection per step;
* when the layer will be materialized (``capture_style`` ``"materialized"`` or
  ``"auto"`` with ``T >= k_a k_g / (k_a + k_g)``) the projected factors are
  written token-major ``(B, k, T)`` straight from the GEMM epilogue, so the
  per-sample ``g_p^T a_p`` is a second tcgen05 GEMM with no transpose copy;
* a layer whose class declares ``__bw_fused_capture__`` (the library's models use
  :class:`dattri_llm_b200.models.layers.TcLinear`) computes both projections inside its own
  GEMMs: a :class:`_FusedCaptureLink` hands its forward ``P_a^T`` to append as a narrow
  last column tile (``x P_a`` token-major from the same read of ``x``) and its backward
  ``P_g^T`` plus a sink that receives ``dy P_g`` from the input-gradient GEMM -- no
  separate projection launches and no second read of ``x`` or ``dy``.
"""

from __future__ import annotations

import threading
import warnings
import weakref
from collections.abc import Callable

import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.ops import (
    canonical_class_name,
    dtypes,
    extract_module_kwargs,
    is_embedding,
    is_linear,
    to_3d,
)

try:
    from transformers.pytorch_utils import Conv1D as HF_Conv1D
except ImportError:  # pragma: no cover - transformers is optional
    HF_Conv1D = None

_LINEAR_IO_TYPES: tuple[type, ...] = (
    nn.Embedding, nn.EmbeddingBag, nn.LayerNorm, nn.GroupNorm, nn.InstanceNorm1d,
    nn.InstanceNorm2d, nn.InstanceNorm3d, nn.Linear, nn.Bilinear, nn.Conv1d, nn.Conv2d,
    nn.Conv3d, nn.ConvTranspose1d, nn.ConvTranspose2d, nn.ConvTranspose3d,
) + ((HF_Conv1D,) if HF_Conv1D is not None else ()) + ((nn.RMSNorm,) if hasattr(nn, "RMSNorm") else ())

def is_linear_io_capable(module: nn.Module) -> bool:
    """Whether *module*'s per-sample gradient factorizes as an outer product (by type).

    A capture tap (a class with ``__bw_capture_tap__``, e.g. an expert-parallel expert's
    stand-in) counts as the layer type its ``__bw_layer_type__`` names.
    """
    return isinstance(module, _LINEAR_IO_TYPES) or getattr(type(module), "__bw_capture_tap__", False)


def has_trainable_params(module: nn.Module) -> bool:
    """Whether *module* owns (or proxies) a parameter that requires grad.

    A capture tap that stands for a weight held elsewhere (``__bw_capture_frozen__``) is
    always captured.
    """
    if getattr(type(module), "__bw_capture_frozen__", False):
        return True
    proxied = getattr(module, "proxied_parameters", None)
    if proxied is not None:
        return any(p.requires_grad for p in proxied())
    return any(p.requires_grad for _, p in module.named_parameters(recurse=False))


def _flatten_tokens(t: torch.Tensor, layer_type: str) -> torch.Tensor:
    if t.ndim > 3 and is_linear(layer_type):
        return t.reshape(t.shape[0], -1, t.shape[-1])
    return t


class LayerBuffer:
    """What one hooked layer captures in the current step.

    ``acts`` / ``grads`` hold ``(device, tensor)`` parts of the kept factors (raw, or
    projected); ``dense`` holds materialized per-sample blocks (or :class:`_DeferredOuter`
    stand-ins until the step's grouped launch); ``waiting[device]`` is the LIFO of forward
    entries that still wait for their backward (autograd runs a device's graph in reverse
    creation order); ``pairs`` records, per matched forward/backward, the device and the
    invocation position (``k`` of the virtual ``name@k`` layers); ``forwards`` counts the
    grad-enabled forwards of the step.  ``lock`` guards the lists against DataParallel
    replica threads.
    """

    __slots__ = ("layer_type", "module_kwargs", "proj_kw", "capture_style", "matrices", "lock", "acts", "grads",
                 "dense", "waiting", "forwards", "pairs", "last_activation", "last_grad")

    def __init__(self, layer_type: str, module_kwargs: dict | None, proj_kw: dict | None,
                 capture_style: str) -> None:
        self.layer_type, self.module_kwargs = layer_type, module_kwargs
        self.proj_kw, self.capture_style = proj_kw, capture_style
        self.matrices: dict = {}  # {"a" / "g": ProjectionMatrix}, resolved on first use
        self.lock = threading.Lock()
        self.clear()

    def clear(self) -> None:
        """Forget the step's captures (configuration and matrices stay)."""
        self.acts: list = []
        self.grads: list = []
        self.dense: list = []
        self.waiting: dict = {}
        self.forwards = 0
        self.pairs: list = []
        self.last_activation = None
        self.last_grad = None

    def snapshot(self) -> dict:
        """Copies of the step's lists and counters (for a secondary pass)."""
        return {"acts": list(self.acts), "grads": list(self.grads), "dense": list(self.dense),
                "waiting": {dev: list(stack) for dev, stack in self.waiting.items()}, "forwards": self.forwards,
                "pairs": list(self.pairs), "last_activation": self.last_activation, "last_grad": self.last_grad}

    def restore(self, snap: dict | None) -> None:
        """Undo to a :meth:`snapshot` (``None``: an empty step)."""
        self.clear()
        for field, value in (snap or {}).items():
            setattr(self, field, value)

    def keep_matched(self) -> bool:
        """Drop forwards that never met a backward (activation checkpointing's first pass)
        and renumber the matched invocations densely per device.  Returns whether any was
        dropped."""
        dropped = any(self.waiting.values())
        if dropped:
            positions: dict[int, list[int]] = {}
            for dev, pos in self.pairs:
                positions.setdefault(dev, []).append(pos)
            dense_pos = {dev: {p: i for i, p in enumerate(sorted(ps))} for dev, ps in positions.items()}
            if self.proj_kw is None:  # raw activations are appended at the forward, in call order
                count: dict[int, int] = {}
                kept = []
                for dev, part in self.acts:
                    pos = count.get(dev, 0)
                    count[dev] = pos + 1
                    if pos in dense_pos.get(dev, {}):
                        kept.append((dev, part))
                self.acts = kept
            self.pairs = [(dev, dense_pos[dev][pos]) for dev, pos in self.pairs]
        self.waiting = {}
        self.forwards = len(self.pairs)
        return dropped

    def invocations(self) -> list[tuple[list, list, list]]:
        """``[(acts, grads, dense)]`` per invocation position (one entry when the layer ran once)."""
        n = 1 + max((pos for _dev, pos in self.pairs), default=0)
        if n == 1:
            return [(self.acts, self.grads, self.dense)]
        by_pos: list[tuple[list, list, list]] = [([], [], []) for _ in range(n)]
        if self.dense:
            for part, (_dev, pos) in zip(self.dense, self.pairs, strict=True):
                by_pos[pos][2].append(part)
            return by_pos
        if self.proj_kw is None:  # activations in forward order, per device
            count: dict[int, int] = {}
            for dev, part in self.acts:
                pos = count.get(dev, 0)
                count[dev] = pos + 1
                by_pos[pos][0].append((dev, part))
        else:  # projected activations are kept at the matched backward, like the gradients
            for part, (_dev, pos) in zip(self.acts, self.pairs, strict=True):
                by_pos[pos][0].append(part)
        for part, (_dev, pos) in zip(self.grads, self.pairs, strict=True):
            by_pos[pos][1].append(part)
        return by_pos


#: One layer's ``param_grad`` buffer: ``{param_name: tensor | None}``.
ParamGradBuffer = dict


class _Projected:
    """A projected activation waiting for its backward; ``token_major`` marks the
    ``(B, k, T)`` layout written for the fused materialize path."""

    __slots__ = ("a", "token_major")

    def __init__(self, a: torch.Tensor, token_major: bool) -> None:
        self.a, self.token_major = a, token_major


class _DeferredOuter:
    """A layer's per-sample ``g_p^T a_p`` awaiting the step's grouped launch; stands in
    the layer's buffer until :meth:`_StepShare.flush_outer` replaces it with the result."""

    __slots__ = ("a", "g", "result")

    def __init__(self, g: torch.Tensor, a: torch.Tensor) -> None:
        self.g, self.a, self.result = g, a, None


class _TokenMajorGrad:
    """A layer's output gradient delivered already projected, token-major ``(B, k, T)``
    (from the input-gradient GEMM of a fused-capture layer)."""

    __slots__ = ("g_pt",)

    def __init__(self, g_pt: torch.Tensor) -> None:
        self.g_pt = g_pt


class _FusedCaptureLink:
    """What a fused-capture layer's forward and backward need from its capture.

    :meth:`before_forward` returns ``(P_a^T or None, slot or None)``: the slot when this
    call's capture can take the fused route (LoGra, token-major materialize, native bf16,
    nothing routed or offloaded), and ``P_a^T`` only when no sibling layer reading the same
    input has projected it already this step.  The layer stores what it computed with
    :meth:`after_forward`; the forward hook consumes it (:meth:`take`)."""

    def __init__(self, name: str, buffers: dict, projector, offload: bool, routed, share) -> None:
        self.name, self.buffers, self.projector = name, buffers, projector
        self.offload, self.routed, self.share = offload, routed, share

    def _eligible(self, x: torch.Tensor) -> bool:
        buf = self.buffers[self.name]
        return (torch.is_grad_enabled() and self.share is not None and not self.offload
                and (self.routed is None or self.name not in self.routed.layers)
                and _style(buf) == "logra" and _preprojects_activation(buf.layer_type, "logra")
                and buf.capture_style != "factorized" and x.ndim == 3 and x.is_cuda)

    def before_forward(self, module, x: torch.Tensor):
        from dattri_llm_b200.ops.linear import CaptureSlot

        if not self._eligible(x):
            return None, None
        buf = self.buffers[self.name]
        (xa,) = dtypes.align(x)
        pm = _projection_matrix(buf, "a", xa, self.projector)
        k = pm.proj_dim
        if not (ops.should_materialize(buf.capture_style, x.shape[1], k, k) and _token_major_ok(pm, xa)):
            return None, None
        key, root = _share_key(x, pm, True)
        hit = self.share.get(key)
        shared = hit is not None and hit[0]() is root
        return (None if shared else pm.matrix_t), CaptureSlot(x.shape[1])

    @staticmethod
    def after_forward(module, a_pt: torch.Tensor | None, slot) -> None:
        module.__dict__["_bw_fused_out"] = (a_pt, slot)

    @staticmethod
    def take(module):
        return module.__dict__.pop("_bw_fused_out", None)


class _AttrHandle:
    """Hook-handle stand-in that deletes a module attribute on ``remove()``."""

    def __init__(self, module: nn.Module, attr: str) -> None:
        self.module, self.attr = weakref.ref(module), attr

    def remove(self) -> None:
        m = self.module()
        if m is not None:
            m.__dict__.pop(self.attr, None)


class _StepShare:
    """Per-step state shared by a manager's hooks: the activation projections shared by
    layers that read the same input tensor (q/k/v, gate/up), and the deferred per-sample
    outer products that one grouped tcgen05 launch computes at step end.  Cleared by the
    manager at every step end."""

    def __init__(self) -> None:
        self._store: dict = {}
        self._outer: list[_DeferredOuter] = []
        self._lock = threading.Lock()

    def get(self, key):
        with self._lock:
            return self._store.get(key)

    def put(self, key, value) -> None:
        with self._lock:
            self._store[key] = value

    def defer_outer(self, g_pt: torch.Tensor, a_pt: torch.Tensor) -> _DeferredOuter:
        """Queue ``(B, k_g, k_a) = g_pt a_pt^T`` (token-major ``(B, k, T)`` operands)."""
        job = _DeferredOuter(g_pt, a_pt)
        with self._lock:
            self._outer.append(job)
        return job

    def flush_outer(self) -> None:
        """Run every queued outer product, one grouped launch per operand shape."""
        from dattri_llm_b200 import ops as native_ops

        with self._lock:
            jobs, self._outer = self._outer, []
        groups: dict = {}
        for j in jobs:
            key = (tuple(j.g.shape), tuple(j.a.shape), j.g.device, j.g.dtype)
            groups.setdefault(key, []).append(j)
        for (gs, as_, dev, dt), grp in groups.items():
            out = torch.empty(len(grp), gs[0], gs[1], as_[1], dtype=dt, device=dev)
            native_ops.gemm_grouped([j.g for j in grp], [j.a for j in grp], list(out.unbind(0)),
                                    mode=native_ops.STORE_BF16)
            flat = out.reshape(len(grp), gs[0], -1)
            for i, j in enumerate(grp):
                j.result = flat[i]

    @staticmethod
    def resolve(parts: list) -> None:
        """Replace finished :class:`_DeferredOuter` stand-ins in a buffer's part list."""
        for i, (dev, part) in enumerate(parts):
            if isinstance(part, _DeferredOuter):
                if part.result is None:
                    raise RuntimeError("a deferred outer product was never flushed")
                parts[i] = (dev, part.result)

    def clear(self) -> None:
        with self._lock:
            self._store.clear()
            self._outer.clear()


def register_linear_io_hooks(
    model: nn.Module,
    layer_names: set[str] | None = None,
    on_layer_forward: Callable | None = None,
    on_layer_backward: Callable | None = None,
    type_overrides: dict[str, str] | None = None,
    kwargs_overrides: dict[str, dict] | None = None,
    projection_kwargs: dict[str, dict] | None = None,
    capture_style: str = "factorized",
    projector: ops.DattriProjector | None = None,
    offload_to_cpu: bool = False,
    preconditioner=None,
    include_frozen: bool = False,
    routed=None,
    step_share: _StepShare | None = None,
) -> tuple[dict[str, LayerBuffer], list]:
    """Register forward and backward hooks on linear-family layers.

    Returns ``(buffers, handles)``: ``{layer_name: LayerBuffer}`` and the hook handles.
    Callbacks receive ``(layer_name, tensor, layer_type, module_kwargs)``; for a
    pre-projected layer the tensor is the projected factor and the type ``"nn.Linear"``.
    """
    root = getattr(model, "module", model)
    buffers: dict[str, LayerBuffer] = {}
    handles: list = []
    share = step_share
    for name, module in root.named_modules():
        if (type_overrides is None or name not in type_overrides) and not is_linear_io_capable(module):
            continue
        if layer_names is not None and name not in layer_names:
            continue
        if not include_frozen and not has_trainable_params(module):
            continue
        layer_type = (type_overrides or {}).get(name) or canonical_class_name(module)
        if kwargs_overrides is not None and name in kwargs_overrides:
            module_kwargs = dict(kwargs_overrides[name])
        else:
            module_kwargs = extract_module_kwargs(module, layer_type)
        proj_kw = None
        if projection_kwargs is not None:
            proj_kw = projection_kwargs.get(name, projection_kwargs.get("__default__"))
        buffers[name] = LayerBuffer(layer_type, module_kwargs, proj_kw, capture_style)
        bwd = _backward_hook(name, buffers, projector, preconditioner, offload_to_cpu, routed, share,
                             on_layer_backward)
        if getattr(type(module), "__bw_fused_capture__", False) and not _preconditioning(preconditioner):
            module.__dict__["_bw_capture_link"] = _FusedCaptureLink(name, buffers, projector, offload_to_cpu,
                                                                    routed, share)
            handles.append(_AttrHandle(module, "_bw_capture_link"))
        # The output gradient is taken by a hook on the autograd node that produced the
        # layer's output, registered in the forward hook: a full module backward hook would
        # wrap every call's inputs and outputs in an extra autograd function (host time per
        # layer and step) and forbids in-place ops on the layer's output.
        handles.append(module.register_forward_hook(
            _forward_hook(name, buffers, projector, preconditioner, offload_to_cpu, routed, share,
                          on_layer_forward, bwd)))
    return buffers, handles


def _device_index(t: torch.Tensor) -> int:
    return t.device.index if t.is_cuda else 0


def _on_output_grad(out: torch.Tensor, fire) -> None:
    """Call ``fire(dL/d out)`` during the backward.

    The hook sits on the autograd node that produced *out* (for a reshaped view such as
    ``F.linear``'s 3-D output, on the node of its base), as a pre-hook: the node still runs
    with the gradient w.r.t. the value the layer returned even when that value is modified
    in place afterwards (an inplace activation), which a hook on the tensor would miss.
    """
    base = out._base
    if base is not None:
        if (base.grad_fn is not None and base.numel() == out.numel() and out.is_contiguous()
                and base.is_contiguous()):
            node, idx, shape = base.grad_fn, base.output_nr, out.shape
        else:  # a general view: a plain tensor hook
            out.register_hook(lambda g: fire(g) and None)
            return
    else:
        node, idx, shape = out.grad_fn, out.output_nr, None

    def pre(grads):
        g = grads[idx]
        if g is not None:
            fire(g if shape is None else g.reshape(shape))

    node.register_prehook(pre)


def _forward_hook(name, buffers, projector, preconditioner, offload, routed, share, callback, on_grad):
    def hook(module, inp, out):
        fused = _FusedCaptureLink.take(module)
        if not torch.is_grad_enabled():
            return  # no backward will follow (eval / log-prob pass)
        entry = record_forward(module, inp, fused[0] if fused is not None else None)
        if not (isinstance(out, torch.Tensor) and out.requires_grad and out.grad_fn is not None):
            return
        slot = fused[1] if fused is not None else None
        if slot is not None and isinstance(entry, _Projected) and entry.token_major:
            buf = buffers[name]
            (oa,) = dtypes.align(out)
            pm_g = _projection_matrix(buf, "g", oa, projector)
            if _token_major_ok(pm_g, oa):
                # the layer's input-gradient GEMM projects dy itself and delivers it here
                slot.grad_tail_t = pm_g.matrix_t
                slot.sink = lambda g_pt, _m=module: on_grad(_m, None, (_TokenMajorGrad(g_pt),))
                return
        _on_output_grad(out, lambda g, _m=module: on_grad(_m, None, (g,)))

    def record_forward(_module, inp, given_a_pt=None):
        x = inp[0]
        a = x.detach()
        dev = _device_index(x)
        buf = buffers[name]
        if routed is not None and name in routed.layers:
            layout = routed.push(name, a, dev)
            if layout is not None:
                a = layout.regroup(a)
        a = _flatten_tokens(a, buf.layer_type)
        emit, emit_type, emit_kw = a, buf.layer_type, buf.module_kwargs
        if _raw_capture(buf, preconditioner):
            if offload:
                a = a.cpu()
            with buf.lock:
                buf.waiting.setdefault(dev, []).append(len(buf.acts))
                buf.acts.append((dev, a))
                buf.forwards += 1
            buf.last_activation = a
            emit = a
        else:
            entry = a
            if _preprojects_activation(buf.layer_type, _style(buf)):
                entry = _project_activation(buf, a, projector, share, x, given_a_pt)
                emit = entry.a.transpose(1, 2) if entry.token_major else entry.a
                emit_type, emit_kw = "nn.Linear", None
            with buf.lock:
                buf.waiting.setdefault(dev, []).append(entry)
                buf.forwards += 1
        if callback is not None:
            callback(name, emit, emit_type, emit_kw)
        return entry if not _raw_capture(buf, preconditioner) else None

    return hook


def _backward_hook(name, buffers, projector, preconditioner, offload, routed, share, callback):
    def hook(_module, _grad_input, grad_output):
        buf = buffers[name]
        if isinstance(grad_output[0], _TokenMajorGrad):  # projected inside the layer's own GEMM
            g_pt = grad_output[0].g_pt
            matched, g_p = _capture_projected(buf, None, _device_index(g_pt), projector, offload, preconditioner,
                                              name, share, g_pt=g_pt)
            if not matched:
                _warn_orphan_backward(name)
                return
            if callback is not None:
                callback(name, g_p, "nn.Linear", None)
            return
        g = grad_output[0].detach()
        dev = _device_index(grad_output[0])
        if routed is not None and name in routed.layers:
            layout = routed.pop(name, dev)
            if layout is not None:
                g = layout.regroup(g)
        g = _flatten_tokens(g, buf.layer_type)
        emit, emit_type, emit_kw = g, buf.layer_type, buf.module_kwargs
        if _raw_capture(buf, preconditioner):
            if offload:
                g = g.cpu()
            with buf.lock:
                stack = buf.waiting.get(dev)
                if not stack:
                    _warn_orphan_backward(name)
                    return
                stack.pop()
                buf.pairs.append((dev, len(stack)))
                buf.grads.append((dev, g))
            buf.last_grad = g
            emit = g
        else:
            matched, g_p = _capture_projected(buf, g, dev, projector, offload, preconditioner, name, share)
            if not matched:
                _warn_orphan_backward(name)
                return
            if g_p is not None:
                emit, emit_type, emit_kw = g_p, "nn.Linear", None
        if callback is not None:
            callback(name, emit, emit_type, emit_kw)

    return hook


def _warn_orphan_backward(layer_name: str) -> None:
    warnings.warn(
        f"Discarding a backward fire on layer '{layer_name}' with no matching forward capture "
        "(e.g. a repeated backward over a retained graph); this is not a normal forward+backward step.",
        stacklevel=3,
    )


def _projection_matrix(buf: LayerBuffer, side: str, x: torch.Tensor, projector) -> ops.ProjectionMatrix:
    """The layer's projection for *side* ``"a"`` / ``"g"``, resolved once per dtype/device."""
    (x,) = dtypes.align(x)
    pm = buf.matrices.get(side)
    if pm is not None and pm.matches(x):
        return pm
    kw = {k: v for k, v in buf.proj_kw.items() if k != "style"}
    seed = kw.pop("proj_seed", 0)
    mk = buf.module_kwargs
    with_bias = side == "a" and mk is not None and mk.get("has_bias", False)
    pm = ops.DattriProjector.coerce(projector).resolve(
        x.shape[-1], proj_seed=seed + 1 if side == "a" else seed, include_bias=with_bias,
        device=x.device, dtype=x.dtype, **kw)
    buf.matrices[side] = pm
    return pm


def _token_major_ok(pm: ops.ProjectionMatrix, x: torch.Tensor) -> bool:
    """The fused token-major path: native bf16 on sm_100, bias-free, 8-aligned widths."""
    from dattri_llm_b200 import ops as native_ops

    return (pm.matrix_t is not None and pm.bias_row is None and x.dtype == torch.bfloat16
            and x.ndim == 3 and x.shape[1] % 8 == 0 and x.shape[-1] % 8 == 0
            and pm.proj_dim % 8 == 0 and native_ops.use_native(x))


def project_token_major(pm: ops.ProjectionMatrix, x: torch.Tensor) -> torch.Tensor:
    """``(x P)`` of ``x (B, T, d)`` written token-major: a ``(B, k, T)`` view whose rows
    are contiguous over tokens (the tcgen05 epilogue stores the transpose directly)."""
    from dattri_llm_b200 import ops as native_ops

    b, t, _ = x.shape
    flat = x.reshape(b * t, x.shape[-1])
    return native_ops.gemm_tn_seg(flat, pm.matrix_t, t)


def _share_key(source: torch.Tensor, pm: ops.ProjectionMatrix, token_major: bool):
    """``(key, root)`` under which layers reading the same input tensor with the same matrix
    (q/k/v, gate/up) share one activation projection per step.  A module with full backward
    hooks sees its input through a per-module view (same storage, same version counter), so
    siblings are matched through the view's base.  id() alone could be recycled once the
    input is freed (frozen layers do not save it for backward); the weak reference to the
    base proves it is the same tensor."""
    root = source._base if source._base is not None else source
    key = (id(root), source._version, source.data_ptr(), tuple(source.shape), tuple(source.stride()),
           id(pm.matrix), token_major)
    return key, root


def _project_activation(buf, a, projector, share, source, given_a_pt=None) -> _Projected:
    """The layer's projected activation: *given_a_pt* (token-major, computed by a fused
    layer's own GEMM), a sibling's shared projection, or a fresh projection GEMM."""
    a3 = to_3d(dtypes.align(a)[0])
    pm = _projection_matrix(buf, "a", a3, projector)
    seq_len = a3.shape[1]
    k = pm.proj_dim
    token_major = given_a_pt is not None or (ops.should_materialize(buf.capture_style, seq_len, k, k)
                                             and _token_major_ok(pm, a3))
    key = None
    if share is not None and a3.is_cuda:
        key, root = _share_key(source, pm, token_major)
        hit = share.get(key)
        if hit is not None and hit[0]() is root:
            return hit[1]
    if given_a_pt is not None:
        entry = _Projected(given_a_pt, True)
    else:
        entry = _Projected(project_token_major(pm, a3) if token_major else pm(a3), token_major)
    if key is not None:
        share.put(key, (weakref.ref(root), entry))
    return entry


def _preprojects_activation(layer_type: str, style: str | None) -> bool:
    return ops.is_linear(layer_type) and style == "logra"


def _preconditioning(preconditioner) -> bool:
    return preconditioner is not None and preconditioner.enabled


def _style(buf: LayerBuffer) -> str | None:
    return None if buf.proj_kw is None else buf.proj_kw.get("style", "logra")


def _raw_capture(buf: LayerBuffer, preconditioner) -> bool:
    return (buf.proj_kw is None and buf.capture_style == "factorized"
            and not _preconditioning(preconditioner))


def _keep_factors(buf: LayerBuffer, seq_len: int, k_a: int, k_g: int) -> bool:
    if buf.acts:
        return True
    if buf.dense:
        return False
    return not ops.should_materialize(buf.capture_style, seq_len, k_a, k_g)


def _capture_projected(buf, g, dev, projector, offload, preconditioner, layer_name, share=None, g_pt=None):
    """Pair *g* with its forward and store the projected / materialized / preconditioned
    capture.  Returns ``(matched, projected g to hand the callbacks or None)``.  *g_pt*: the
    output gradient already projected token-major ``(B, k, T)`` (then *g* is ``None``)."""
    with buf.lock:
        stack = buf.waiting.get(dev)
        entry = stack.pop() if stack else None
        pos = (dev, len(stack)) if entry is not None else None
    if entry is None:
        return False, None
    proj_kw = buf.proj_kw
    kw = dict(proj_kw or {})
    style = kw.pop("style", "logra") if proj_kw is not None else None
    pre = preconditioner if _preconditioning(preconditioner) else None
    layer_type, mk = buf.layer_type, buf.module_kwargs

    def keep_factors(a_f, g_f):
        if offload:
            a_f, g_f = a_f.cpu(), g_f.cpu()
        with buf.lock:
            buf.acts.append((dev, a_f))
            buf.grads.append((dev, g_f))
            buf.pairs.append(pos)

    def keep_dense(mat):
        if offload:
            mat = mat.cpu()
        with buf.lock:
            buf.dense.append((dev, mat))
            buf.pairs.append(pos)

    if style == "logra":
        if isinstance(entry, _Projected):
            g_p = None
            if g_pt is None:
                g3 = to_3d(dtypes.align(g)[0])
                pm_g = _projection_matrix(buf, "g", g3, projector)
                if entry.token_major and _token_major_ok(pm_g, g3) and not buf.acts:
                    g_pt = project_token_major(pm_g, g3)
                else:
                    g_p = pm_g(g3)
            if g_pt is not None and entry.token_major and not buf.acts:
                from dattri_llm_b200 import ops as native_ops

                b = g_pt.shape[0]
                if share is not None and not offload:
                    # The per-sample outer product g_p^T a_p of every layer of the step runs
                    # in one grouped launch at step end (StepShare.flush_outer).
                    keep_dense(share.defer_outer(g_pt, entry.a))
                    return True, g_pt.transpose(1, 2)
                dense = torch.empty(b, g_pt.shape[1], entry.a.shape[1], dtype=g_pt.dtype, device=g_pt.device)
                native_ops.gemm_tn(g_pt, entry.a, dense, mode=native_ops.STORE_BF16)
                keep_dense(dense.reshape(b, -1))
                return True, g_pt.transpose(1, 2)
            if g_p is None:
                g_p = g_pt.transpose(1, 2)
            a_p = entry.a.transpose(1, 2) if entry.token_major else entry.a
            emit = g_p
        else:
            a = entry
            if a.ndim == 1 and is_embedding(layer_type):
                a, g = a.unsqueeze(0), g.unsqueeze(0)
            a_p, g_p = ops.project_factors(a, g, layer_type, projector, mk, **kw)
            emit = None
        seq_len = a_p.shape[1] if a_p.ndim >= 3 else 1
        if _keep_factors(buf, seq_len, a_p.shape[-1], g_p.shape[-1]):
            keep_factors(a_p, g_p)
        else:
            keep_dense(ops.materialize_factors(a_p, g_p, "nn.Linear"))
        return True, emit
    a = entry
    if a.ndim == 1 and is_embedding(layer_type):
        a, g = a.unsqueeze(0), g.unsqueeze(0)
    if style == "mask":
        mat = ops.mask_factors(a, g, layer_type, projector, mk, **kw)
        keep_dense(pre(layer_name, mat, proj_kw) if pre is not None else mat)
        return True, None
    if style == "dense":
        if pre is not None:
            include_bias = bool(kw.pop("include_bias", True))
            mat = ops.materialize_factors(a, g, layer_type, mk, include_bias)
            mat = ops.apply_projection(projector, pre(layer_name, mat, proj_kw), **kw)
        else:
            mat = ops.project_materialized_factors(a, g, layer_type, projector, mk, **kw)
        keep_dense(mat)
        return True, None
    if pre is not None:
        keep_dense(pre(layer_name, ops.materialize_factors(a, g, layer_type, mk), None))
        return True, None
    seq_len = a.shape[1] if a.ndim >= 3 else 1
    if _keep_factors(buf, seq_len, a.shape[-1] + 1, g.shape[-1]):
        keep_factors(a, g)
    else:
        keep_dense(ops.materialize_factors(a, g, layer_type, mk))
    return True, None


def remove_hooks(handles: list) -> None:
    """Remove every handle and clear the list."""
    for h in handles:
        h.remove()
    handles.clear()


def register_param_grad_hooks(model: nn.Module, layer_names: set[str] | None = None,
                              on_param_grad: Callable | None = None, offload_to_cpu: bool = False):
    """Tensor hooks on every trainable parameter of the selected modules: the batch-level
    gradient lands in ``buffers[layer][param]``.  Returns ``(buffers, handles)``."""
    root = getattr(model, "module", model)
    buffers: dict[str, ParamGradBuffer] = {}
    handles: list = []
    for lname, module in root.named_modules():
        if layer_names is not None and lname not in layer_names:
            continue
        trainable = [(pn, p) for pn, p in module.named_parameters(recurse=False) if p.requires_grad]
        if not trainable:
            continue
        buffers[lname] = {pn: None for pn, _ in trainable}
        for pn, p in trainable:
            def hook(grad, ln=lname, pn=pn):
                g = grad.detach()
                if offload_to_cpu:
                    g = g.cpu()
                buffers[ln][pn] = g
                if on_param_grad is not None:
                    on_param_grad(ln, pn, g)
            handles.append(p.register_hook(hook))
    return buffers, handles


def register_linear_param_hooks(model: nn.Module, layer_names: set[str] | None = None,
                                on_linear_param_grad: Callable | None = None):
    """Post-accumulate-grad hooks on the trainable parameters of linear-IO layers (the
    per-step barrier that weight gradients have been written).  Returns ``(count, handles)``."""
    root = getattr(model, "module", model)
    count, handles = 0, []
    for name, module in root.named_modules():
        if not is_linear_io_capable(module) or (layer_names is not None and name not in layer_names):
            continue
        for pn, p in module.named_parameters(recurse=False):
            if not p.requires_grad:
                continue
            count += 1

            def hook(param, ln=name, pn=pn):
                if on_linear_param_grad is not None:
                    on_linear_param_grad(ln, pn, param.grad.detach() if param.grad is not None else None)
            handles.append(p.register_post_accumulate_grad_hook(hook))
    return count, handles
