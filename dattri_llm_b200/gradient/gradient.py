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


def _pad_tokens(t: torch.Tensor, target: int, axis: int, value: float = 0) -> torch.Tensor:
    if t.shape[axis] == target:
        return t
    shape = list(t.shape)
    shape[axis] = target - shape[axis]
    return torch.cat([t, t.new_full(shape, value)], dim=axis)


def _pad_to_common_tokens(a: Factorized, b: Factorized) -> tuple[Factorized, Factorized]:
    """Right-pad the shorter token axis; padded positions get an exactly-zero gradient
    (integer ids get the layer's ``padding_idx`` or 0), which every consumer treats as inert."""
    axis = 1 if a.batch_first else 0
    target = max(a.activation.shape[axis], b.activation.shape[axis])

    def pad(f: Factorized) -> Factorized:
        if f.activation.shape[axis] == target:
            return f
        fill = 0
        if not f.activation.is_floating_point():
            p = (f.module_kwargs or {}).get("padding_idx")
            fill = p if p is not None else 0
        return f._rebuild(_pad_tokens(f.activation, target, axis, fill),
                          _pad_tokens(f.pre_activation_grad, target, axis))

    return pad(a), pad(b)


def _layer_batch(value: GradientData) -> int:
    if isinstance(value, Factorized):
        return value.activation.shape[0 if value.batch_first else 1]
    return value.shape[0]


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
            raise ValueError("data cannot be empty")
        missing = set(self.data) - set(self.representation)
        if missing:
            raise ValueError(f"Missing representation for layers: {sorted(missing)}")
        batch = first = None
        for name, value in self.data.items():
            lt = self.layer_types[name]
            if self.representation[name] == "factorized":
                if not isinstance(value, Factorized):
                    raise TypeError(f"{name} must be Factorized")
                shape = tuple(value.activation.shape)
                bf = value.as_batch_first()
                a, g = bf.activation, bf.pre_activation_grad
                if lt == "nn.EmbeddingBag":
                    if a.ndim != 2 or g.ndim != 2:
                        raise ValueError(f"{name} has invalid embedding-bag factor dimensions")
                    if a.shape[0] != g.shape[0]:
                        raise ValueError(f"{name} embedding-bag batch dimension mismatch")
                elif ops.is_embedding(lt):
                    if a.ndim != 2 or g.ndim != 3:
                        raise ValueError(f"{name} has invalid embedding factor dimensions")
                    if a.shape != g.shape[:2]:
                        raise ValueError(f"{name} embedding batch/token dimensions mismatch")
                elif ops.is_conv(lt) or ops.is_conv_transpose(lt):
                    if a.shape[0] != g.shape[0]:
                        raise ValueError(f"{name} conv factor batch size mismatch: {a.shape[0]} != {g.shape[0]}")
                elif a.shape[:-1] != g.shape[:-1]:
                    raise ValueError(f"{name} factor batch/token dimensions mismatch")
                cur = a.shape[0]
            else:
                if not isinstance(value, torch.Tensor):
                    raise TypeError(f"{name} must be Tensor")
                if value.ndim < 1:
                    raise ValueError(f"{name} must be at least 1D")
                if lt != ops.PARAM_GRAD_TYPES and self._layer_indexing(name) == "batch_token" and value.ndim != 3:
                    raise ValueError(f"{name} declared as batch_token but tensor is {value.ndim}D, expected 3D")
                cur, shape = value.shape[0], tuple(value.shape)
            if lt == ops.PARAM_GRAD_TYPES or cur == 1:
                continue
            if batch is None:
                batch, first = cur, (name, shape)
            elif batch != cur:
                raise ValueError(
                    f"All layers must have the same batch size: {first[0]} has {batch} samples "
                    f"(captured shape {first[1]}) but {name} has {cur} (captured shape {shape}). "
                    "The sample axis is read from dim 0 of every per-sample layer; a layer whose "
                    "input is sequence-first (T, B, ...) must be declared in "
                    "HookManager(non_batch_first_layers=...), and a layer fed flattened or routed "
                    "token rows (an MoE router or expert) in HookManager(moe_routed_layers=...).",
                )

    def clone(self) -> Gradient:
        """Deep copy with every tensor cloned."""
        data = {n: (v._rebuild(v.activation.clone(), v.pre_activation_grad.clone())
                    if isinstance(v, Factorized) else v.clone()) for n, v in self.data.items()}
        return Gradient(dict(self.representation), data, dict(self.layer_types), dict(self.indexing))

    def to(self, device=None, dtype=None, non_blocking: bool = False) -> Gradient:
        """Every payload moved to *device* / cast to *dtype*."""
        data = {n: v.to(device=device, dtype=dtype, non_blocking=non_blocking) if isinstance(v, Factorized)
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
        names = set(layer_names)
        if include_derived:
            names |= {n for n in self.layer_names if base_layer_name(n) in names}
        missing = names - self.layer_names
        if missing:
            raise KeyError(f"Unknown layers: {sorted(missing)}")
        return Gradient({n: self.representation[n] for n in names}, {n: self.data[n] for n in names},
                        {k: v for k, v in self.layer_types.items() if k in names},
                        {n: i for n, i in self.indexing.items() if n in names})

    def concatenate(self, other: Gradient, dim: Literal["batch", "token"] = "batch") -> Gradient:
        """Concatenate along the batch (unequal token lengths zero-padded; broadcast layers
        averaged by batch size) or the token axis."""
        self._check_compatible(other, require_same_batch=False)
        if dim == "token":
            bad = [n for n in self.layer_names if self._layer_indexing(n) != "batch_token"]
            if bad:
                raise ValueError(
                    f"Token concatenation requires all layers to have indexing='batch_token'. "
                    f"Non-conforming: {sorted(bad)}",
                )
            if self.batch_size != other.batch_size:
                raise ValueError("Token concatenation requires the same batch size")
        data, rep, idx = {}, dict(self.representation), dict(self.indexing)
        b_self, b_other = self.batch_size, other.batch_size

        def axis(batch_first: bool) -> int:
            return (0 if batch_first else 1) if dim == "batch" else (1 if batch_first else 0)

        for name in self.layer_names:
            a, b = self.data[name], other.data[name]
            bc_a = _layer_batch(a) == 1 and b_self > 1
            bc_b = _layer_batch(b) == 1 and b_other > 1
            if dim == "batch" and (bc_a or bc_b):
                if bc_a != bc_b:
                    raise ValueError(
                        f"{name} is a broadcast (batch-collapsed) gradient on one side but "
                        "per-sample on the other; the two cannot be concatenated along the batch axis.",
                    )
                wa, wb = float(b_self), float(b_other)
                if isinstance(a, Factorized) and isinstance(b, Factorized):
                    abf, bbf = a.as_batch_first(), b.as_batch_first()
                    if abf.activation.shape == bbf.activation.shape and torch.equal(abf.activation, bbf.activation):
                        g = (wa * abf.pre_activation_grad + wb * bbf.pre_activation_grad) / (wa + wb)
                        data[name] = Factorized(abf.activation, g, module_kwargs=abf.module_kwargs)
                    else:
                        lt = self.layer_types[name]
                        data[name] = (wa * ops.materialize(a, lt) + wb * ops.materialize(b, lt)) / (wa + wb)
                        rep[name], idx[name] = "materialized", "batch"
                elif isinstance(a, torch.Tensor) and isinstance(b, torch.Tensor):
                    data[name] = (wa * a + wb * b) / (wa + wb)
                else:
                    raise TypeError(f"{name} has mismatched data types")
                continue
            if isinstance(a, Factorized) and isinstance(b, Factorized):
                if a.batch_first != b.batch_first:
                    raise ValueError(f"{name} has mismatched batch_first layout between gradients")
                if dim == "batch" and self._layer_indexing(name) == "batch_token":
                    a, b = _pad_to_common_tokens(a, b)
                ax = axis(a.batch_first)
                data[name] = a._rebuild(torch.cat([a.activation, b.activation], dim=ax),
                                        torch.cat([a.pre_activation_grad, b.pre_activation_grad], dim=ax))
            elif isinstance(a, torch.Tensor) and isinstance(b, torch.Tensor):
                if dim == "batch" and self._layer_indexing(name) == "batch_token":
                    t = max(a.shape[1], b.shape[1])
                    a, b = _pad_tokens(a, t, 1), _pad_tokens(b, t, 1)
                data[name] = torch.cat([a, b], dim=axis(True))
            else:
                raise TypeError(f"{name} has mismatched data types")
        out = Gradient(rep, data, self.layer_types, idx)
        out.validate()
        return out

    def aggregate(self, dim: Literal["token"] = "token") -> Gradient:
        """Sum out the token axis of ``"batch_token"`` layers (the chain rule:
        ``dL/dW = sum_t g_t a_t^T``); every layer ends ``"batch"`` indexed."""
        if dim != "token":
            raise NotImplementedError("Only token aggregation is supported")
        data, rep = {}, {}
        for name, v in self.data.items():
            if self._layer_indexing(name) == "batch_token":
                if isinstance(v, Factorized):
                    data[name], rep[name] = ops.materialize(v, self.layer_types[name]), "materialized"
                else:
                    data[name], rep[name] = v.sum(dim=1), self.representation[name]
            else:
                data[name], rep[name] = v, self.representation[name]
        return Gradient(rep, data, self.layer_types, {})

    def slice(self, dim: Literal["batch", "token"], index: int | Sequence[int] | torch.Tensor) -> Gradient:
        """Slice every layer along the batch or token axis (a broadcast layer's shared row
        is copied to every requested sample)."""
        if dim == "token":
            bad = [n for n in self.layer_names if self._layer_indexing(n) != "batch_token"]
            if bad:
                raise ValueError(
                    f"Token slicing requires all layers to have indexing='batch_token'. "
                    f"Non-conforming: {sorted(bad)}",
                )

        def cut(x: torch.Tensor, ax: int) -> torch.Tensor:
            li = index
            if dim == "batch" and x.shape[ax] == 1:
                if isinstance(index, int):
                    li = 0
                else:
                    n = index.numel() if torch.is_tensor(index) else len(index)
                    li = torch.zeros(n, dtype=torch.long, device=x.device)
            sl = [slice(None)] * x.ndim
            sl[ax] = li
            y = x[tuple(sl)]
            return y.unsqueeze(ax) if isinstance(li, int) else y

        def axis(bf: bool) -> int:
            return (0 if bf else 1) if dim == "batch" else (1 if bf else 0)

        data = {}
        for name, v in self.data.items():
            if self.layer_types[name] == ops.PARAM_GRAD_TYPES:
                data[name] = v
            elif isinstance(v, Factorized):
                ax = axis(v.batch_first)
                data[name] = v._rebuild(cut(v.activation, ax), cut(v.pre_activation_grad, ax))
            else:
                data[name] = cut(v, axis(True))
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
        if self.layer_names != other.layer_names:
            raise ValueError("Layer sets differ")
        bad = {n for n in self.layer_names if self.representation.get(n) != other.representation.get(n)}
        if bad:
            raise ValueError(f"Layers have differing representations: {sorted(bad)}")
        bad = {n for n in self.layer_names if self._layer_indexing(n) != other._layer_indexing(n)}
        if bad:
            raise ValueError(f"Layers have differing indexing: {sorted(bad)}")
        if self.layer_types != other.layer_types:
            raise ValueError(f"Layer types differ: {self.layer_types} vs {other.layer_types}")
        if require_same_batch:
            if self.batch_size != other.batch_size:
                raise ValueError("Batch sizes differ")
            st, ot = self.token_dim, other.token_dim
            bad = {n for n in self.layer_names if st[n] != ot[n]}
            if bad:
                raise ValueError(f"Token dimensions differ for layers: {sorted(bad)}")


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
