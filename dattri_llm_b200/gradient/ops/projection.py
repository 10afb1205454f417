"""Random projection of per-sample gradients: ``logra``, ``dense`` and ``mask`` styles.

* ``logra`` projects the two factors, ``a_p = a P_a``, ``g_p = g P_g`` (seeds
  ``proj_seed + 1`` and ``proj_seed``), keeping the Kronecker structure at width
  ``proj_dim``; a linear layer's bias column is folded in as the matrix's last row.
* ``dense`` materializes the per-sample gradient and projects it (TRAK style).
* ``mask`` keeps ``proj_dim`` fixed random coordinates of the per-sample gradient,
  gathered from the factors without materializing it.

A projector is a factory following dattri's ``random_project`` protocol,
``factory(feature, batch_size, proj_dim=, proj_seed=, device=, **kw)`` returning
``x -> x P``.  :class:`DattriProjector` turns a factory into explicit ``(d_in, k)``
matrices and caches them (parity: reference
``dattri_llm/gradient/ops/projection.py:50-944``).

B200 design: with no factory the projector is the library's counter-based
generator (:func:`counter_projector`), whose matrices are produced directly on the
GPU by a kernel (no identity pushed through a factory) and kept in the
tensor-core layout ``P^T`` (K-major bf16), so every projection is one tcgen05 GEMM.
Any protocol factory still works: its matrix is built once and cached.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from dattri_llm_b200.gradient.ops import dtypes
from dattri_llm_b200.gradient.ops.materialize import materialize_factors
from dattri_llm_b200.gradient.ops.preprocess import preprocess_factors, to_3d
from dattri_llm_b200.gradient.ops.types import is_conv_transpose, is_embedding, is_linear, is_norm
from dattri_llm_b200.utils.cache import TensorCache
from dattri_llm_b200.utils.rng import counter_projection_matrix

PROJECTION_STYLES = ("logra", "dense", "mask")
CAPTURE_STYLES = ("factorized", "materialized", "auto")
MASK_KEYS = frozenset({"style", "proj_dim", "proj_seed", "include_bias", "device"})
_MASK_CHUNK_ELEMS = 1 << 24
_IDENTITY_CHUNK_ROWS = 8192


def counter_projector(feature: torch.Tensor, batch_size: int, proj_dim: int, proj_seed: int = 0,
                      device: torch.device | str | None = None, proj_type: str = "rademacher",
                      **_ignored) -> Callable[[torch.Tensor], torch.Tensor]:
    """Protocol-compatible factory of the library's counter-based projections.

    Returns ``x -> x @ P`` with ``P`` the ``(d, proj_dim)`` counter-based matrix of
    ``(proj_seed, d, proj_dim)`` (``d = feature.shape[-1]``); entries
    ``+-1/sqrt(proj_dim)`` (``proj_type="rademacher"``) or scaled normals.
    """
    d = feature.shape[-1]
    dev = torch.device(device) if device is not None else feature.device
    kind = "normal" if proj_type in ("normal", "gaussian") else "rademacher"
    matrix = _counter_matrix(d, proj_dim, proj_seed, kind, torch.float32, dev)

    def project(x: torch.Tensor) -> torch.Tensor:
        return x.to(matrix.dtype) @ matrix

    return project


counter_projector.__bw_counter__ = True  # marks the generator the GPU kernel reproduces


def _counter_matrix(d, k, seed, kind, dtype, device):
    from dattri_llm_b200 import ops as native_ops

    if device.type == "cuda" and native_ops.use_native(torch.empty(0, device=device)):
        return native_ops.projection_matrix_t(d, k, seed, kind=kind, dtype=torch.float32,
                                              device=device).t().to(dtype)
    return counter_projection_matrix(d, k, seed, kind=kind, dtype=dtype, device=device)


def _projector_key(projector: Callable) -> str:
    return f"{getattr(projector, '__module__', '')}.{getattr(projector, '__qualname__', repr(projector))}"


def _mask_seed(proj_seed: int, d: int, proj_dim: int) -> int:
    """Seed of a mask's coordinate draw (a function of seed, width and size only)."""
    return ((proj_seed * 1_000_003 + d) * 1_000_003 + proj_dim) & ((1 << 63) - 1)


def _check_mask_kwargs(kw: dict) -> None:
    extra = set(kw) - MASK_KEYS
    if extra:
        raise ValueError(
            f"style 'mask' keeps coordinates rather than projecting, so it takes only "
            f"{sorted(MASK_KEYS - {'style'})}; got unexpected {sorted(extra)}.",
        )


class DattriProjector:
    """A projection factory plus the cache of the matrices it builds."""

    def __init__(self, projector: Callable | None = None, *, cache: TensorCache | None = None) -> None:
        self._factory = projector
        self._cache = cache if cache is not None else TensorCache("memory")

    @classmethod
    def coerce(cls, projector: Callable | DattriProjector | None) -> DattriProjector:
        """A :class:`DattriProjector` for a factory, a projector, or ``None`` (default)."""
        return projector if isinstance(projector, DattriProjector) else cls(projector)

    @property
    def factory(self) -> Callable:
        """The factory (the library's counter-based projector when none was given)."""
        return self._factory if self._factory is not None else counter_projector

    @property
    def cache(self) -> TensorCache:
        """The matrix cache."""
        return self._cache

    def _is_counter(self) -> bool:
        return getattr(self.factory, "__bw_counter__", False)

    def matrix(self, d_in: int, *, proj_dim: int, proj_seed: int, device: torch.device,
               dtype: torch.dtype, **proj_kwargs) -> torch.Tensor:
        """The ``(d_in, proj_dim)`` matrix of this factory (cached)."""
        device = torch.device(device)
        key = (_projector_key(self.factory), d_in, proj_dim, proj_seed, str(device), dtype,
               tuple(sorted((k, repr(v)) for k, v in proj_kwargs.items())))
        cached = self._cache.get(key)
        if cached is not None:
            return cached
        if self._is_counter():
            kind = proj_kwargs.get("proj_type", "rademacher")
            kind = "normal" if kind in ("normal", "gaussian") else "rademacher"
            matrix = _counter_matrix(d_in, proj_dim, proj_seed, kind, dtype, device)
        else:
            rows = []
            for start in range(0, d_in, _IDENTITY_CHUNK_ROWS):
                stop = min(start + _IDENTITY_CHUNK_ROWS, d_in)
                block = torch.zeros(stop - start, d_in, device=device, dtype=torch.float32)
                idx = torch.arange(stop - start, device=device)
                block[idx, idx + start] = 1.0
                rows.append(self.factory(block, block.shape[0], proj_dim=proj_dim,
                                         proj_seed=proj_seed, device=device, **proj_kwargs)(block))
            matrix = torch.cat(rows, dim=0).to(dtype)
        self._cache.put(key, matrix)
        return matrix

    def matrix_t(self, d_in: int, **kw) -> torch.Tensor:
        """``matrix(d_in, ...)^T`` contiguous, ``(proj_dim, d_in)``: the tensor-core
        B-operand layout (cached)."""
        key = ("T", d_in, tuple(sorted((k, repr(v)) for k, v in kw.items())))
        cached = self._cache.get(key)
        if cached is None:
            cached = self.matrix(d_in, **kw).t().contiguous()
            self._cache.put(key, cached)
        return cached

    def mask_indices(self, d: int, *, proj_dim: int, proj_seed: int, device) -> torch.Tensor:
        """Sorted ``proj_dim`` coordinates out of ``d`` (CPU-seeded, device-independent)."""
        if not 0 < proj_dim <= d:
            raise ValueError(f"a mask needs 0 < proj_dim <= d, got proj_dim={proj_dim} for a width-{d} layer.")
        key = ("subset", d, proj_dim, proj_seed, str(device))
        cached = self._cache.get(key)
        if cached is not None:
            return cached
        gen = torch.Generator(device="cpu").manual_seed(_mask_seed(proj_seed, d, proj_dim))
        idx = torch.randperm(d, generator=gen)[:proj_dim].sort().values.to(device)
        self._cache.put(key, idx)
        return idx

    def apply(self, x: torch.Tensor, *, proj_dim: int, proj_seed: int = 0, include_bias: bool = False,
              **proj_kwargs) -> torch.Tensor:
        """``x @ P`` over the last axis (``include_bias``: ``P``'s last row is added)."""
        lead = x.shape[:-1]
        (x,) = dtypes.as_float(x)
        flat = x.reshape(-1, x.shape[-1])
        device = torch.device(proj_kwargs.pop("device", flat.device))
        flat = flat.to(device)
        pm = self.resolve(flat.shape[-1], proj_dim=proj_dim, proj_seed=proj_seed,
                          include_bias=include_bias, device=device, dtype=flat.dtype, **proj_kwargs)
        return pm(flat).reshape(*lead, proj_dim)

    def resolve(self, d_in: int, *, proj_dim: int, proj_seed: int = 0, include_bias: bool = False,
                device, dtype: torch.dtype, **proj_kwargs) -> ProjectionMatrix:
        """One layer-side's :class:`ProjectionMatrix` (matrix, bias row, tensor-core layout)."""
        device = torch.device(proj_kwargs.pop("device", device))
        kw = dict(proj_dim=proj_dim, proj_seed=proj_seed, device=device, dtype=dtype, **proj_kwargs)
        n = d_in + (1 if include_bias else 0)
        matrix = self.matrix(n, **kw)
        matrix_t = None
        if device.type == "cuda" and dtype == torch.bfloat16:
            matrix_t = self.matrix_t(n, **kw)
        return ProjectionMatrix(matrix, include_bias, d_in, dtype, device, matrix_t=matrix_t)

    def clear(self) -> None:
        """Drop every cached matrix."""
        self._cache.clear()

    def close(self) -> None:
        """Release the cache."""
        self._cache.clear()

    def __enter__(self) -> DattriProjector:
        return self

    def __exit__(self, *_exc: object) -> bool:
        self.close()
        return False


class ProjectionMatrix:
    """One layer-side's projection with everything but the GEMM resolved."""

    __slots__ = ("bias_row", "d_in", "device", "dtype", "matrix", "matrix_t", "proj_dim")

    def __init__(self, matrix: torch.Tensor, include_bias: bool, d_in: int, dtype: torch.dtype,
                 device: torch.device, *, matrix_t: torch.Tensor | None = None) -> None:
        self.matrix = matrix[:-1] if include_bias else matrix
        self.bias_row = matrix[-1] if include_bias else None
        self.matrix_t = None
        if matrix_t is not None:
            self.matrix_t = matrix_t[:, :-1].contiguous() if include_bias else matrix_t
        self.d_in, self.dtype, self.device = d_in, dtype, device
        self.proj_dim = matrix.shape[1]

    def matches(self, x: torch.Tensor) -> bool:
        """Whether *x* is the width, dtype and device this matrix was resolved for."""
        return x.shape[-1] == self.d_in and x.dtype == self.dtype and x.device == self.device

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """``x P (+ bias row)`` over the last axis (tcgen05 GEMM for bf16 on sm_100)."""
        flat = x.reshape(-1, self.d_in)
        if self.matrix_t is not None and self.d_in % 8 == 0:
            from dattri_llm_b200 import ops as native_ops

            if native_ops.use_native(flat):
                out = torch.empty(flat.shape[0], self.proj_dim, dtype=self.dtype, device=flat.device)
                if self.bias_row is not None:
                    f32 = torch.empty(flat.shape[0], self.proj_dim, device=flat.device)
                    native_ops.gemm_tn(flat, self.matrix_t, f32, mode=native_ops.STORE_F32)
                    out.copy_(f32 + self.bias_row.float())
                else:
                    native_ops.gemm_tn(flat, self.matrix_t, out, mode=native_ops.STORE_BF16)
                return out.reshape(*x.shape[:-1], self.proj_dim)
        out = flat @ self.matrix if self.bias_row is None else torch.addmm(self.bias_row, flat, self.matrix)
        return out.reshape(*x.shape[:-1], self.proj_dim)


def apply_projection(projector, x: torch.Tensor, *, proj_dim: int, proj_seed: int = 0,
                     include_bias: bool = False, **proj_kwargs) -> torch.Tensor:
    """:meth:`DattriProjector.apply` for a factory **or** a projector."""
    return DattriProjector.coerce(projector).apply(x, proj_dim=proj_dim, proj_seed=proj_seed,
                                                   include_bias=include_bias, **proj_kwargs)


def project_materialized_factors(a, g, layer_type, projector, module_kwargs=None,
                                 include_bias: bool = True, *, proj_dim: int, proj_seed: int = 0,
                                 **proj_kwargs) -> torch.Tensor:
    """TRAK style: materialize the per-sample gradient, then project it ``(B, proj_dim)``."""
    mat = materialize_factors(a, g, layer_type, module_kwargs, include_bias)
    return apply_projection(projector, mat, proj_dim=proj_dim, proj_seed=proj_seed, **proj_kwargs)


def project_factors(a, g, layer_type, projector, module_kwargs=None, include_bias: bool = True,
                    *, proj_dim: int, proj_seed: int = 0, **proj_kwargs):
    """LoGra style: ``(a_p, g_p)`` -- each factor projected, the structure kept."""
    if is_norm(layer_type):
        raise ValueError(
            f"factorized projection is undefined for {layer_type!r}: its gradient is not an "
            "outer product of the factors -- use materialized projection",
        )
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    if is_embedding(layer_type):
        if module_kwargs is None:
            raise ValueError("Factorized projection of an embedding requires module_kwargs with 'num_embeddings'.")
        a = torch.nn.functional.one_hot(a.long(), num_classes=module_kwargs["num_embeddings"])
    a, g = dtypes.align(a, g)
    a_f, g_f = to_3d(a), to_3d(g)
    g_p = apply_projection(projector, g_f, proj_dim=proj_dim, proj_seed=proj_seed, **proj_kwargs)
    a_p = apply_projection(projector, a_f, proj_dim=proj_dim, proj_seed=proj_seed + 1, **proj_kwargs)
    return a_p, g_p


def project_activation(a, layer_type, projector, module_kwargs, include_bias: bool = True, *,
                       proj_dim: int, proj_seed: int = 0, **proj_kwargs) -> torch.Tensor:
    """The a-side of :func:`project_factors` for a linear layer (bias folded as a row)."""
    if not is_linear(layer_type):
        raise ValueError(f"project_activation is for linear layers only, got {layer_type!r}.")
    with_bias = module_kwargs is not None and module_kwargs["has_bias"] and include_bias
    a_f = to_3d(dtypes.align(a)[0])
    return apply_projection(projector, a_f, proj_dim=proj_dim, proj_seed=proj_seed + 1,
                            include_bias=with_bias, **proj_kwargs)


def project_gradient(g, layer_type, projector, module_kwargs, *, proj_dim: int, proj_seed: int = 0,
                     **proj_kwargs) -> torch.Tensor:
    """The g-side of :func:`project_factors` for a linear layer."""
    del module_kwargs
    if not is_linear(layer_type):
        raise ValueError(f"project_gradient is for linear layers only, got {layer_type!r}.")
    return apply_projection(projector, to_3d(dtypes.align(g)[0]), proj_dim=proj_dim,
                            proj_seed=proj_seed, **proj_kwargs)


def project_materialized(f, layer_type, projector, *, proj_dim: int, include_bias: bool = True,
                         proj_seed: int = 0, **proj_kwargs) -> torch.Tensor:
    """:func:`project_materialized_factors` on a :class:`Factorized` (or a dense block)."""
    if isinstance(f, torch.Tensor):
        return apply_projection(projector, f, proj_dim=proj_dim, proj_seed=proj_seed, **proj_kwargs)
    bf = f.as_batch_first()
    return project_materialized_factors(bf.activation, bf.pre_activation_grad, layer_type, projector,
                                        bf.module_kwargs, include_bias, proj_dim=proj_dim,
                                        proj_seed=proj_seed, **proj_kwargs)


def project_factorized(f, layer_type, projector, *, proj_dim: int, include_bias: bool = True,
                       proj_seed: int = 0, **proj_kwargs):
    """:func:`project_factors` on a :class:`Factorized` (batch-first-safe)."""
    bf = f.as_batch_first()
    return project_factors(bf.activation, bf.pre_activation_grad, layer_type, projector,
                           bf.module_kwargs, include_bias, proj_dim=proj_dim, proj_seed=proj_seed,
                           **proj_kwargs)


def mask_coordinates(projection: dict | None, layer_name: str, width: int, projector,
                     device="cpu") -> torch.Tensor | None:
    """The coordinates a ``"mask"`` capture keeps for a layer (``None`` without a config).

    Raises:
        ValueError: when the layer is configured with another style.
    """
    if projection is None:
        return None
    kw = projection.get(layer_name, projection.get("__default__"))
    if kw is None:
        return None
    if kw.get("style", "logra") != "mask":
        raise ValueError(
            f"layer {layer_name!r} is captured with style {kw.get('style')!r}; coordinate-wise "
            "maps need exact gradient entries, i.e. no projection or style 'mask'.",
        )
    return DattriProjector.coerce(projector).mask_indices(
        width, proj_dim=kw["proj_dim"], proj_seed=kw.get("proj_seed", 0), device=torch.device(device))


def mask_materialized(x: torch.Tensor, projector, *, proj_dim: int, proj_seed: int = 0,
                      **proj_kwargs) -> torch.Tensor:
    """Keep ``proj_dim`` fixed random coordinates of a dense ``(..., D)`` tensor."""
    _check_mask_kwargs(proj_kwargs)
    device = torch.device(proj_kwargs.get("device", x.device))
    x = x.to(device)
    idx = DattriProjector.coerce(projector).mask_indices(x.shape[-1], proj_dim=proj_dim,
                                                         proj_seed=proj_seed, device=device)
    return x.index_select(-1, idx)


def _gather_pairs(rows_src, cols_src, rows, cols, *, one_hot: bool = False) -> torch.Tensor:
    """``out[:, m] = sum_t rows_src[:, t, rows[m]] * cols_src[:, t, cols[m]]`` chunked over m.

    On sm_100 with bf16 factors this is one gather-contract kernel (``csrc/mask_gather.cu``)
    that stages token tiles of both factors in shared memory."""
    from dattri_llm_b200 import ops as native_ops

    if (not one_hot and rows_src.ndim == 3 and native_ops.use_native(rows_src, cols_src)
            and rows_src.dtype == torch.bfloat16 and cols_src.dtype == torch.bfloat16
            and (rows_src.shape[-1] + cols_src.shape[-1]) * 2 <= 192 * 1024):
        return native_ops.mask_gather(rows_src, cols_src, rows, cols).to(rows_src.dtype)
    b, t = cols_src.shape[:2]
    chunk = max(1, _MASK_CHUNK_ELEMS // max(1, b * t))
    out = []
    for start in range(0, rows.numel(), chunk):
        r, c = rows[start : start + chunk], cols[start : start + chunk]
        left = rows_src[..., start : start + chunk] if one_hot else rows_src.index_select(-1, r)
        out.append((left * cols_src.index_select(-1, c)).sum(1))
    return torch.cat(out, dim=-1)


def mask_factors(a, g, layer_type, projector, module_kwargs=None, include_bias: bool = True, *,
                 proj_dim: int, proj_seed: int = 0, **proj_kwargs) -> torch.Tensor:
    """``materialize_factors(...)[:, mask]`` computed without materializing."""
    _check_mask_kwargs(proj_kwargs)
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    projector = DattriProjector.coerce(projector)
    device = torch.device(proj_kwargs.get("device", g.device))
    if is_embedding(layer_type):
        if module_kwargs is None:
            raise ValueError("Subsetting an embedding gradient requires module_kwargs with 'num_embeddings'.")
        ids = a.to(device)
        (grad,) = dtypes.align(g)
        grad = grad.to(device)
        vocab, embed = module_kwargs["num_embeddings"], grad.shape[-1]
        idx = projector.mask_indices(vocab * embed, proj_dim=proj_dim, proj_seed=proj_seed, device=device)
        rows, cols = idx // embed, idx % embed
        return _gather_pairs((ids.unsqueeze(-1) == rows).to(grad.dtype), grad, rows, cols, one_hot=True)
    a, g = dtypes.align(a, g)
    a_f, g_f = to_3d(a).to(device), to_3d(g).to(device)
    if a_f.ndim == 4:
        groups, k_g = a_f.shape[2], a_f.shape[-1]
        d_g = g_f.shape[-1]
        a_flat = a_f.reshape(*a_f.shape[:2], groups * k_g)
        g_flat = g_f.reshape(*g_f.shape[:2], groups * d_g)
        idx = projector.mask_indices(groups * d_g * k_g, proj_dim=proj_dim, proj_seed=proj_seed, device=device)
        grp, rem = idx // (d_g * k_g), idx % (d_g * k_g)
        if is_conv_transpose(layer_type):
            return _gather_pairs(a_flat, g_flat, grp * k_g + rem // d_g, grp * d_g + rem % d_g)
        return _gather_pairs(g_flat, a_flat, grp * d_g + rem // k_g, grp * k_g + rem % k_g)
    if is_norm(layer_type):
        dense = (a_f * g_f).sum(1)
        idx = projector.mask_indices(dense.shape[-1], proj_dim=proj_dim, proj_seed=proj_seed, device=device)
        return dense.index_select(-1, idx)
    if is_conv_transpose(layer_type):
        n_cols = g_f.shape[-1]
        idx = projector.mask_indices(a_f.shape[-1] * n_cols, proj_dim=proj_dim, proj_seed=proj_seed, device=device)
        return _gather_pairs(a_f, g_f, idx // n_cols, idx % n_cols)
    n_cols = a_f.shape[-1]
    idx = projector.mask_indices(g_f.shape[-1] * n_cols, proj_dim=proj_dim, proj_seed=proj_seed, device=device)
    return _gather_pairs(g_f, a_f, idx // n_cols, idx % n_cols)


def mask_factorized(f, layer_type, projector, *, proj_dim: int, include_bias: bool = True,
                    proj_seed: int = 0, **proj_kwargs) -> torch.Tensor:
    """:func:`mask_factors` on a :class:`Factorized` (or a dense block)."""
    if isinstance(f, torch.Tensor):
        return mask_materialized(f, projector, proj_dim=proj_dim, proj_seed=proj_seed, **proj_kwargs)
    bf = f.as_batch_first()
    return mask_factors(bf.activation, bf.pre_activation_grad, layer_type, projector, bf.module_kwargs,
                        include_bias, proj_dim=proj_dim, proj_seed=proj_seed, **proj_kwargs)


def maybe_materialize_projected(seq_len: int, k_a: int, k_g: int, kappa: float = 1.0) -> bool:
    """``True`` when the projected factors are larger than their outer product:
    ``seq_len >= kappa * k_a k_g / (k_a + k_g)``."""
    denom = k_a + k_g
    return denom > 0 and seq_len >= kappa * (k_a * k_g) / denom


def should_materialize(capture_style: str, seq_len: int, k_a: int, k_g: int) -> bool:
    """Whether a layer's factors are materialized at capture under *capture_style*."""
    if capture_style == "factorized":
        return False
    if capture_style == "materialized":
        return True
    if capture_style != "auto":
        raise ValueError(f"capture_style must be one of {CAPTURE_STYLES}, got {capture_style!r}.")
    return maybe_materialize_projected(seq_len, k_a, k_g)


def project_layer(f, layer_type, projector, *, style: str = "logra", capture_style: str = "factorized",
                  **proj_kwargs) -> tuple[object, bool]:
    """Route one layer through a projection style: ``(payload, is_factorized)``."""
    if style not in PROJECTION_STYLES:
        raise ValueError(f"style must be one of {PROJECTION_STYLES}, got {style!r}.")
    if style == "mask":
        return mask_factorized(f, layer_type, projector, **proj_kwargs), False
    if style == "logra" and not isinstance(f, torch.Tensor):
        a_p, g_p = project_factorized(f, layer_type, projector, **proj_kwargs)
        seq_len = a_p.shape[1] if a_p.ndim >= 3 else 1
        if should_materialize(capture_style, seq_len, a_p.shape[-1], g_p.shape[-1]):
            return materialize_factors(a_p, g_p, "nn.Linear"), False
        return (a_p, g_p), True
    return project_materialized(f, layer_type, projector, **proj_kwargs), False
