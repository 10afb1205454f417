"""Gradient data model: ``Factorized`` factor pairs and multi-layer ``Gradient`` blocks.

Parity: reference ``dattri_llm/gradient/gradient.py:20-1238``.  A ``Gradient`` is
one step's per-sample gradients over several layers; each layer is either
*factorized* (activation, output-gradient) -- ``"batch_token"`` indexed when it
keeps a token axis -- or *materialized* ``(B, d)``.  A layer invoked ``k`` times in
a step is recorded as virtual layers ``name``, ``name@2``, ...  A layer whose batch
axis is 1 while the step batch is larger is a *broadcast* gradient (e.g. a
positional embedding shared by every sample) and is expanded, sliced and
averaged as one shared row.  These semantics are part of the stored format.
"""

from __future__ import annotations

from dattri_llm_b200.options import CaptureStyle  # noqa: F401  (re-exported option types)
from collections.abc import Callable, Iterable, Sequence
from dataclasses import InitVar, dataclass, field
from typing import Literal

import torch

from dattri_llm_b200.gradient import ops

GradientRepresentation = Literal["materialized", "factorized"]
Indexing = Literal["batch", "batch_token"]



def _dense_to_gpu_together(data: dict, device) -> dict[str, torch.Tensor]:
    """``{name: tensor on device}`` for the host-resident dense tensors of *data* when *device*
    is a GPU and there are several: per dtype, one pinned staging buffer, one copy, and views
    of the device buffer (the layers' own storages are not shared with the host)."""
    if device is None or torch.device(device).type != "cuda":
        return {}
    names = [n for n, v in data.items() if isinstance(v, torch.Tensor) and v.device.type == "cpu"]
    if len(names) < 8:
        return {}
    target = torch.device(device)
    out: dict[str, torch.Tensor] = {}
    by_dtype: dict[torch.dtype, list[str]] = {}
    for n in names:
        by_dtype.setdefault(data[n].dtype, []).append(n)
    for dt, group in by_dtype.items():
        sizes = [data[n].numel() for n in group]
        staging = torch.empty(sum(sizes), dtype=dt, pin_memory=True)
        torch.cat([data[n].reshape(-1) for n in group], out=staging)
        flat = staging.to(target, non_blocking=True)
        for n, piece in zip(group, flat.split(sizes), strict=True):
            out[n] = piece.view(data[n].shape)
    return out

@dataclass(frozen=True, eq=False)
class Factorized:
    """A per-layer factorized ("ghost") gradient: an (activation, output-gradient) pair.

    ``module_kwargs`` are the layer hyperparameters preprocessing needs (``None`` for
    final factors such as projected ones); ``batch_first=False`` marks a
    sequence-first ``(T, B, ...)`` capture.
    """

    activation: torch.Tensor
    pre_activation_grad: torch.Tensor
    module_kwargs: dict | None = field(default=None, compare=False, repr=False, hash=False)
    batch_first: bool = field(default=True, compare=False)

    def _rebuild(self, a, g, batch_first=None) -> Factorized:
        return Factorized(a, g, module_kwargs=self.module_kwargs,
                          batch_first=self.batch_first if batch_first is None else batch_first)

    def to(self, device=None, dtype=None, non_blocking: bool = False) -> Factorized:
        """Both factors moved to *device* / cast to *dtype* (floating factors only for dtype)."""
        def mv(t):
            dt = dtype if (dtype is not None and t.is_floating_point()) else None
            return t.to(device=device, dtype=dt, non_blocking=non_blocking)
        return self._rebuild(mv(self.activation), mv(self.pre_activation_grad))

    def pin_memory(self) -> Factorized:
        """Both factors in pinned host memory (idempotent)."""
        def pin(t):
            return t if t.device.type != "cpu" or t.is_pinned() else t.pin_memory()
        return self._rebuild(pin(self.activation), pin(self.pre_activation_grad))

    @property
    def nbytes(self) -> int:
        """Bytes held by the two factors."""
        return sum(t.numel() * t.element_size() for t in (self.activation, self.pre_activation_grad))

    def as_batch_first(self) -> Factorized:
        """A ``(B, T, ...)`` view (swaps the leading axes of a sequence-first capture)."""
        if self.batch_first:
            return self
        return self._rebuild(self.activation.transpose(0, 1), self.pre_activation_grad.transpose(0, 1),
                             batch_first=True)


GradientData = torch.Tensor | Factorized


def base_layer_name(name: str) -> str:
    """Strip the ``@k`` invocation suffix of a virtual layer name."""
    return name.split("@", 1)[0]


def _grow_tokens(t: torch.Tensor, length: int, axis: int, fill: float = 0) -> torch.Tensor:
    """*t* right-padded with *fill* along *axis* to *length* positions."""
    short = length - t.shape[axis]
    if short <= 0:
        return t
    pad_shape = list(t.shape)
    pad_shape[axis] = short
    return torch.cat([t, t.new_full(pad_shape, fill)], dim=axis)


def _same_token_length(x: Factorized, y: Factorized) -> tuple[Factorized, Factorized]:
    """Both factor pairs right-padded to the longer token axis.  A padded position carries
    a zero output gradient, so it contributes nothing anywhere; integer activations (token
    ids) are padded with the layer's ``padding_idx`` (or 0)."""
    axis = 1 if x.batch_first else 0
    length = max(x.activation.shape[axis], y.activation.shape[axis])

    def grown(f: Factorized) -> Factorized:
        if f.activation.shape[axis] == length:
            return f
        pad_id = (f.module_kwargs or {}).get("padding_idx")
        fill = 0 if f.activation.is_floating_point() or pad_id is None else pad_id
        return f._rebuild(_grow_tokens(f.activation, length, axis, fill),
                          _grow_tokens(f.pre_activation_grad, length, axis))

    return grown(x), grown(y)


def _layer_batch(value: GradientData) -> int:
    """Samples held by one layer's payload."""
    if isinstance(value, Factorized):
        return value.activation.shape[0 if value.batch_first else 1]
    return value.shape[0]


def _factorized_rows(name: str, kind: str, value) -> tuple[int, tuple]:
    """Check one factorized payload; returns ``(samples, activation shape)``."""
    if not isinstance(value, Factorized):
        raise TypeError(f"layer {name!r} is declared factorized but holds a {type(value).__name__}.")
    bf = value.as_batch_first()
    a, g = bf.activation, bf.pre_activation_grad
    if kind == "nn.EmbeddingBag":
        ok = a.ndim == 2 and g.ndim == 2 and a.shape[0] == g.shape[0]
        want = "2-D bags and 2-D gradients with one row per bag"
    elif ops.is_embedding(kind):
        ok = a.ndim == 2 and g.ndim == 3 and a.shape == g.shape[:2]
        want = "(B, T) ids and (B, T, E) gradients"
    elif ops.is_conv(kind) or ops.is_conv_transpose(kind):
        ok = a.shape[0] == g.shape[0]
        want = "factors with the same leading sample axis"
    else:
        ok = a.shape[:-1] == g.shape[:-1]
        want = "factors that agree on every axis but the feature axis"
    if not ok:
        raise ValueError(f"layer {name!r} ({kind}): expected {want}, got activation {tuple(a.shape)} and gradient "
                         f"{tuple(g.shape)}.")
    return a.shape[0], tuple(value.activation.shape)


def _dense_rows(name: str, kind: str, value, indexing: str) -> tuple[int, tuple]:
    """Check one materialized payload; returns ``(samples, shape)``."""
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"layer {name!r} is declared materialized but holds a {type(value).__name__}.")
    if value.ndim == 0:
        raise ValueError(f"layer {name!r} holds a scalar; a per-sample payload needs a leading sample axis.")
    if kind != ops.PARAM_GRAD_TYPES and indexing == "batch_token" and value.ndim != 3:
        raise ValueError(f"layer {name!r} is batch_token indexed, which needs a (B, T, d) tensor, not "
                         f"{value.ndim}-D.")
    return value.shape[0], tuple(value.shape)


def _mix_shared_rows(name: str, kind: str, x, y, wx: float, wy: float):
    """The shared (broadcast) row of two blocks merged as their sample-weighted mean."""
    total = wx + wy
    if isinstance(x, torch.Tensor) and isinstance(y, torch.Tensor):
        return (wx * x + wy * y) / total, None
    if not (isinstance(x, Factorized) and isinstance(y, Factorized)):
        raise TypeError(f"layer {name!r} is factorized in one block and materialized in the other.")
    xb, yb = x.as_batch_first(), y.as_batch_first()
    if xb.activation.shape == yb.activation.shape and torch.equal(xb.activation, yb.activation):
        grad = (wx * xb.pre_activation_grad + wy * yb.pre_activation_grad) / total
        return Factorized(xb.activation, grad, module_kwargs=xb.module_kwargs), None
    dense = (wx * ops.materialize(x, kind) + wy * ops.materialize(y, kind)) / total
    return dense, "materialized"


@dataclass(frozen=True, eq=False)
class Gradient:
    """A per-step, multi-layer container of per-sample gradients with metadata."""

    representation: dict[str, GradientRepresentation]
    data: dict[str, GradientData]
    layer_types: dict[str, str]
    indexing: dict[str, Indexing] = field(default_factory=dict)
    validate_on_init: InitVar[bool] = True

    def __post_init__(self, validate_on_init: bool) -> None:
        object.__setattr__(self, "indexing", {n: self.indexing.get(n, "batch") for n in self.data})
        if validate_on_init:
            self.validate()

    def _layer_indexing(self, name: str) -> Indexing:
        return self.indexing[name]

    @property
    def layer_names(self) -> set[str]:
        """Names of the layers this block covers."""
        return set(self.data)

    @property
    def batch_size(self) -> int:
        """The step batch: the largest per-layer sample count (``param_grad`` excluded).

        Raises:
            ValueError: when only batch-level ``param_grad`` layers are present.
        """
        best = 0
        for name, x in self.data.items():
            if self.layer_types.get(name) == ops.PARAM_GRAD_TYPES:
                continue
            best = max(best, _layer_batch(x))
        if best:
            return best
        raise ValueError(
            "batch_size is undefined for a gradient holding only batch-level param_grad layers "
            "(their tensors have no per-sample axis).",
        )

    @property
    def token_dim(self) -> dict[str, int | None]:
        """Per-layer token count (``None`` for ``"batch"`` layers)."""
        out: dict[str, int | None] = {}
        for name, v in self.data.items():
            if self._layer_indexing(name) != "batch_token":
                out[name] = None
            elif isinstance(v, Factorized):
                out[name] = v.activation.shape[1 if v.batch_first else 0]
            else:
                out[name] = v.shape[1]
        return out

    @property
    def device(self) -> torch.device:
        """Device of the payloads."""
        x = next(iter(self.data.values()))
        return x.activation.device if isinstance(x, Factorized) else x.device

    @property
    def dtype(self) -> torch.dtype:
        """Dtype of the payloads (the activation's for factorized layers)."""
        x = next(iter(self.data.values()))
        return x.activation.dtype if isinstance(x, Factorized) else x.dtype

    @property
    def nbytes(self) -> int:
        """Bytes as stored."""
        return sum(v.nbytes if isinstance(v, Factorized) else v.numel() * v.element_size()
                   for v in self.data.values())

    @property
    def materialized_nbytes(self) -> int:
        """Bytes :meth:`materialize` would produce, from the shapes alone."""
        total = 0
        for name, v in self.data.items():
            if not isinstance(v, Factorized):
                total += v.numel() * v.element_size()
                continue
            bf = v.as_batch_first()
            a, g = bf.activation, bf.pre_activation_grad
            lt = self.layer_types.get(name, "nn.Linear")
            size = g.element_size()
            if ops.is_norm(lt):
                total += a.shape[0] * a.shape[-1] * size
            elif ops.is_embedding(lt):
                vocab = (bf.module_kwargs or {}).get("num_embeddings") or int(a.max().item()) + 1
                total += a.shape[0] * vocab * g.shape[-1] * size
            else:
                total += a.shape[0] * a.shape[-1] * g.shape[-1] * size
        return total

    def map_layers(self, fn: Callable[[str, GradientData, str], GradientData | None], *,
                   layers: Iterable[str] | None = None, consume: bool = False) -> Gradient:
        """Rebuild the block from ``fn(name, value, layer_type)`` on the selected layers
        (``None`` drops the layer; a tensor result is materialized ``"batch"``).
        ``consume=True`` releases each old payload as its replacement is built."""
        selected = set(self.data) if layers is None else set(layers)
        data, rep, idx = {}, {}, {}
        for name in list(self.data):
            release = consume and name in selected
            old = self.data.pop(name) if release else self.data[name]
            value = fn(name, old, self.layer_types[name]) if name in selected else old
            del old
            if value is None:
                continue
            data[name] = value
            if isinstance(value, Factorized):
                rep[name], idx[name] = "factorized", self.indexing[name]
            else:
                rep[name] = "materialized"
                idx[name] = "batch" if name in selected else self.indexing[name]
        return Gradient(rep, data, {k: v for k, v in self.layer_types.items() if k in data}, idx,
                        validate_on_init=False)

    def validate(self) -> None:
        """Check internal consistency.

        Raises:
            ValueError / TypeError: on an empty block, a missing representation, a
                payload of the wrong kind, inconsistent factor shapes, or layers that
                disagree on the batch size.
        """
        if not self.data:
            raise ValueError("a Gradient block needs at least one layer.")
        unlisted = sorted(set(self.data) - set(self.representation))
        if unlisted:
            raise ValueError(f"layers without a representation entry: {unlisted}.")
        reference_rows = None  # (samples, layer, shape) of the first per-sample layer
        for name, value in self.data.items():
            kind = self.layer_types[name]
            if self.representation[name] == "factorized":
                rows, shape = _factorized_rows(name, kind, value)
            else:
                rows, shape = _dense_rows(name, kind, value, self._layer_indexing(name))
            if kind == ops.PARAM_GRAD_TYPES or rows == 1:
                continue  # batch-level or broadcast: no per-sample axis to agree on
            if reference_rows is None:
                reference_rows = (rows, name, shape)
            elif rows != reference_rows[0]:
                raise ValueError(
                    f"layers disagree on the batch size: {reference_rows[1]!r} has {reference_rows[0]} samples "
                    f"(shape {reference_rows[2]}), {name!r} has {rows} (shape {shape}). Every per-sample layer "
                    "carries its samples on axis 0: declare sequence-first (T, B, ...) inputs in "
                    "HookManager(non_batch_first_layers=...) and routed token rows (MoE routers / experts) in "
                    "HookManager(moe_routed_layers=...).")

    def clone(self) -> Gradient:
        """Deep copy with every tensor cloned."""
        data = {n: (v._rebuild(v.activation.clone(), v.pre_activation_grad.clone())
                    if isinstance(v, Factorized) else v.clone()) for n, v in self.data.items()}
        return Gradient(dict(self.representation), data, dict(self.layer_types), dict(self.indexing))

    def to(self, device=None, dtype=None, non_blocking: bool = False) -> Gradient:
        """Every payload moved to *device* / cast to *dtype*.  Host-resident dense layers bound
        for a GPU travel together, one copy per dtype (a record carries one tensor per
        captured layer, and one blocking copy each would stall the host hundreds of times)."""
        moved = _dense_to_gpu_together(self.data, device) if dtype is None else {}
        data = {n: moved[n] if n in moved
                else v.to(device=device, dtype=dtype, non_blocking=non_blocking) if isinstance(v, Factorized)
                else v.to(device=device, dtype=dtype if (dtype is not None and v.is_floating_point()) else None,
                          non_blocking=non_blocking)
                for n, v in self.data.items()}
        return Gradient(dict(self.representation), data, self.layer_types, dict(self.indexing))

    def pin_memory(self) -> Gradient:
        """Every CPU payload in pinned memory (idempotent)."""
        data = {n: v.pin_memory() if isinstance(v, Factorized) or (v.device.type == "cpu" and not v.is_pinned())
                else v for n, v in self.data.items()}
        return Gradient(dict(self.representation), data, self.layer_types, dict(self.indexing))

    def materialize(self) -> Gradient:
        """Every factorized layer turned into its dense ``(B, d)`` gradient."""
        if all(r == "materialized" for r in self.representation.values()):
            return self
        data, rep, idx = {}, {}, dict(self.indexing)
        for name, v in self.data.items():
            if self.representation[name] == "factorized" and isinstance(v, Factorized):
                data[name] = ops.materialize(v, self.layer_types[name])
                rep[name], idx[name] = "materialized", "batch"
            else:
                data[name], rep[name] = v, self.representation[name]
        return Gradient(rep, data, self.layer_types, idx)

    def project(self, projector, proj_kwargs: dict[str, dict], *, capture_style: str = "factorized") -> Gradient:
        """Each layer reduced per ``proj_kwargs[name]`` (or ``"__default__"``) in the
        ``logra`` / ``dense`` / ``mask`` style; layers without a config pass through."""
        data, rep, types, idx = {}, {}, {}, {}
        projector = ops.DattriProjector.coerce(projector)
        for name, v in self.data.items():
            kw = proj_kwargs.get(name, proj_kwargs.get("__default__"))
            if kw is None:
                data[name], rep[name] = v, self.representation[name]
                types[name], idx[name] = self.layer_types[name], self.indexing[name]
                continue
            kw = dict(kw)
            style = kw.pop("style", "logra")
            payload, is_fact = ops.project_layer(v, self.layer_types[name], projector, style=style,
                                                 capture_style=capture_style, **kw)
            if is_fact:
                data[name], rep[name] = Factorized(*payload), "factorized"
                types[name], idx[name] = "nn.Linear", self.indexing[name]
            else:
                data[name], rep[name] = payload, "materialized"
                types[name], idx[name] = self.layer_types[name], "batch"
        return Gradient(rep, data, types, idx)

    def select_layers(self, layer_names: Iterable[str], include_derived: bool = False) -> Gradient:
        """A copy restricted to *layer_names* (with ``include_derived``: plus their ``@k``
        invocation layers).

        Raises:
            KeyError: for unknown names.
        """
        wanted = set(layer_names)
        if include_derived:
            wanted.update(n for n in self.data if base_layer_name(n) in wanted)
        unknown = sorted(wanted - set(self.data))
        if unknown:
            raise KeyError(f"the block has no layers {unknown}.")
        keep = [n for n in self.data if n in wanted]
        return Gradient({n: self.representation[n] for n in keep}, {n: self.data[n] for n in keep},
                        {n: self.layer_types[n] for n in keep}, {n: self.indexing[n] for n in keep})

    def _require_token_axis(self, what: str) -> None:
        flat = sorted(n for n in self.data if self._layer_indexing(n) != "batch_token")
        if flat:
            raise ValueError(f"{what} along tokens needs every layer batch_token indexed; {flat} are not.")

    def concatenate(self, other: Gradient, dim: Literal["batch", "token"] = "batch") -> Gradient:
        """Concatenate along the batch (unequal token lengths zero-padded; broadcast layers
        averaged by batch size) or the token axis."""
        self._check_compatible(other, require_same_batch=False)
        rows_self, rows_other = self.batch_size, other.batch_size
        if dim == "token":
            self._require_token_axis("concatenation")
            if rows_self != rows_other:
                raise ValueError(f"concatenating along tokens needs equal batch sizes, got {rows_self} and "
                                 f"{rows_other}.")
        data, rep, idx = {}, dict(self.representation), dict(self.indexing)
        for name in self.data:
            x, y = self.data[name], other.data[name]
            shared_x, shared_y = _layer_batch(x) == 1 < rows_self, _layer_batch(y) == 1 < rows_other
            if dim == "batch" and (shared_x or shared_y):
                if shared_x != shared_y:
                    raise ValueError(f"layer {name!r} holds one shared row in one block and per-sample rows in "
                                     "the other; they cannot be stacked along the batch.")
                data[name], new_rep = _mix_shared_rows(name, self.layer_types[name], x, y, float(rows_self),
                                                       float(rows_other))
                if new_rep is not None:
                    rep[name], idx[name] = new_rep, "batch"
                continue
            data[name] = self._joined(name, x, y, dim)
        joined = Gradient(rep, data, self.layer_types, idx)
        joined.validate()
        return joined

    def _joined(self, name: str, x, y, dim: str):
        """One layer's payloads of two blocks joined along *dim*."""
        tokens_indexed = self._layer_indexing(name) == "batch_token"
        if isinstance(x, Factorized) and isinstance(y, Factorized):
            if x.batch_first != y.batch_first:
                raise ValueError(f"layer {name!r} is batch-first in one block and sequence-first in the other.")
            if dim == "batch" and tokens_indexed:
                x, y = _same_token_length(x, y)
            sample_axis = 0 if x.batch_first else 1
            axis = sample_axis if dim == "batch" else 1 - sample_axis
            return x._rebuild(torch.cat([x.activation, y.activation], dim=axis),
                              torch.cat([x.pre_activation_grad, y.pre_activation_grad], dim=axis))
        if isinstance(x, torch.Tensor) and isinstance(y, torch.Tensor):
            if dim == "batch" and tokens_indexed:
                length = max(x.shape[1], y.shape[1])
                x, y = _grow_tokens(x, length, 1), _grow_tokens(y, length, 1)
            return torch.cat([x, y], dim=0 if dim == "batch" else 1)
        raise TypeError(f"layer {name!r} is factorized in one block and materialized in the other.")

    def aggregate(self, dim: Literal["token"] = "token") -> Gradient:
        """Sum out the token axis of ``"batch_token"`` layers (the chain rule:
        ``dL/dW = sum_t g_t a_t^T``); every layer ends ``"batch"`` indexed."""
        if dim != "token":
            raise NotImplementedError(f"aggregate() sums out the token axis; dim={dim!r} is not one.")
        data, rep = {}, {}
        for name, value in self.data.items():
            data[name], rep[name] = value, self.representation[name]
            if self._layer_indexing(name) != "batch_token":
                continue
            if isinstance(value, Factorized):
                data[name], rep[name] = ops.materialize(value, self.layer_types[name]), "materialized"
            else:
                data[name] = value.sum(dim=1)
        return Gradient(rep, data, self.layer_types, {})

    def slice(self, dim: Literal["batch", "token"], index: int | Sequence[int] | torch.Tensor) -> Gradient:
        """Slice every layer along the batch or token axis (a broadcast layer's shared row
        is copied to every requested sample)."""
        if dim == "token":
            self._require_token_axis("slicing")
        scalar = isinstance(index, int)
        count = 1 if scalar else (index.numel() if torch.is_tensor(index) else len(index))

        def take(t: torch.Tensor, axis: int) -> torch.Tensor:
            picks = index
            if dim == "batch" and t.shape[axis] == 1:  # a shared row serves every sample
                picks = 0 if scalar else torch.zeros(count, dtype=torch.long, device=t.device)
            if scalar:
                return t.narrow(axis, picks, 1)
            return t.index_select(axis, torch.as_tensor(picks, device=t.device).reshape(-1))

        def axis_of(batch_first: bool) -> int:
            sample = 0 if batch_first else 1
            return sample if dim == "batch" else 1 - sample

        data = {}
        for name, value in self.data.items():
            if self.layer_types[name] == ops.PARAM_GRAD_TYPES:
                data[name] = value
            elif isinstance(value, Factorized):
                ax = axis_of(value.batch_first)
                data[name] = value._rebuild(take(value.activation, ax), take(value.pre_activation_grad, ax))
            else:
                data[name] = take(value, axis_of(True))
        return Gradient(dict(self.representation), data, self.layer_types, dict(self.indexing))

    def similarity(self, other: Gradient, metric: Literal["dot", "cosine"] = "dot",
                   reduce: Literal["none", "all"] = "none",
                   mode: Literal["factorized", "materialized", "auto"] = "auto", eps: float = 1e-8):
        """Per-layer ``{layer: (B_self, B_other)}`` cross-grams (``reduce="none"``) or their
        sum over layers (``"all"``), as dot products or cosines."""
        if metric not in {"dot", "cosine"}:
            raise ValueError("metric must be 'dot' or 'cosine'")
        if reduce not in {"none", "all"}:
            raise ValueError("reduce must be 'none' or 'all'")
        if mode not in {"factorized", "materialized", "auto"}:
            raise ValueError("mode must be 'factorized', 'materialized', or 'auto'")
        per_layer = ops.layerwise_cross_dot(self, other, mode=mode, reduce="none")
        if reduce == "none":
            if metric == "cosine":
                for name in per_layer:
                    ns = self._layer_norm_sq(name, mode).clamp_min(0).sqrt()
                    no = other._layer_norm_sq(name, mode).clamp_min(0).sqrt()
                    per_layer[name] /= ns[:, None] * no[None, :] + eps
            return per_layer
        if not per_layer:
            raise ValueError("No shared layers to compute an overall similarity")
        total = ops.layerwise_cross_dot(self, other, layers=list(per_layer), mode=mode, reduce="sum")
        if metric == "cosine":
            b_s, b_o = self.batch_size, other.batch_size

            def vec(v, b):
                return v.expand(b) if v.shape[0] == 1 else v

            ns = torch.stack([vec(self._layer_norm_sq(n, mode), b_s) for n in per_layer]).sum(0).clamp_min(0)
            no = torch.stack([vec(other._layer_norm_sq(n, mode), b_o) for n in per_layer]).sum(0).clamp_min(0)
            total /= ns.sqrt()[:, None] * no.sqrt()[None, :] + eps
        return total

    def similarity_per_token(self, other: Gradient, reduce: Literal["none", "all"] = "all"):
        """``(B_self, T_self, B_other)``: each of this block's token positions' share of
        :meth:`similarity` (factorized ``batch_token`` layers only; sums back over ``T``)."""
        if reduce not in {"none", "all"}:
            raise ValueError("reduce must be 'none' or 'all'")
        per_layer = {}
        for name in self.layer_names:
            if name not in other.data:
                continue
            sv = self.data[name]
            if not (isinstance(sv, Factorized) and self._layer_indexing(name) == "batch_token"):
                continue
            per_layer[name] = ops.cross_dot_per_token(sv, other.data[name], self.layer_types[name])
        if reduce == "none":
            return per_layer
        if not per_layer:
            raise ValueError("No shared factorized batch_token layers for per-token similarity")
        return torch.stack(list(per_layer.values())).sum(0)

    def _layer_norm_sq(self, name: str, mode: str) -> torch.Tensor:
        return ops.grad_norm_sq(self.data[name], self.layer_types[name], mode=mode)

    def _check_compatible(self, other: Gradient, require_same_batch: bool) -> None:
        if set(self.data) != set(other.data):
            raise ValueError(f"the blocks hold different layers: {sorted(set(self.data) ^ set(other.data))}.")
        for what, mine, theirs in (("representation", self.representation, other.representation),
                                   ("indexing", {n: self._layer_indexing(n) for n in self.data},
                                    {n: other._layer_indexing(n) for n in other.data}),
                                   ("layer type", self.layer_types, other.layer_types)):
            odd = sorted(n for n in self.data if mine.get(n) != theirs.get(n))
            if odd:
                raise ValueError(f"the blocks disagree on the {what} of layers {odd}.")
        if require_same_batch:
            if self.batch_size != other.batch_size:
                raise ValueError(f"the blocks have different batch sizes ({self.batch_size} and "
                                 f"{other.batch_size}).")
            mine_t, theirs_t = self.token_dim, other.token_dim
            odd = sorted(n for n in self.data if mine_t[n] != theirs_t[n])
            if odd:
                raise ValueError(f"the blocks have different token lengths in layers {odd}.")


@dataclass
class GradientRecord:
    """A gradient block with its identity: ``step`` (global backward counter),
    ``input_hash`` (one id per sample -- content hashes, or ``sample_id_key`` values),
    the :class:`Gradient`, and which ``sample_id_key`` produced the ids (``None`` for
    content hashing)."""

    step: int
    input_hash: str | list[str]
    gradient: Gradient
    sample_id_key: str | int | None = None

    def __repr__(self) -> str:
        if isinstance(self.input_hash, list):
            h = f"[{self.input_hash[0][:16]}...+{len(self.input_hash) - 1}]" if self.input_hash else "[]"
        else:
            h = f"{self.input_hash[:16]}..."
        return f"GradientRecord(step={self.step}, input_hash={h})"
