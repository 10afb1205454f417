"""Inner products of per-sample gradients and the factorized-vs-materialized cost rule.

For one layer with factors ``a_i (S, K)`` and ``g_i (S, D)`` the per-sample
gradient is ``dW_i = g_i^T a_i``.  Two exact ways to form the cross-gram
``K[i, j] = <dW1_i, dW2_j>``:

* factorized ("ghost"):  ``sum_{s,t} (a1_i a2_j^T) * (g1_i g2_j^T)`` -- cost
  ``B1 B2 S^2 (D + K)``;
* materialized: ``vec(dW1) . vec(dW2)`` -- cost ``(B1 + B2) S D K + B1 B2 D K``.

:func:`maybe_use_materialized_gram` picks the cheaper one (parity: reference
``dattri_llm/gradient/ops/dot.py:728-753``; the rule and every layout are the
reference's).  On an sm_100 device both routes run on native kernels: the
ghost route is one fused tcgen05 kernel that keeps both Gram tiles in TMEM and
reduces their Hadamard product per sample pair in the epilogue, so the
``(B1 S) x (B2 S2)`` intermediates never reach HBM.
"""

from __future__ import annotations

import math
from collections.abc import Iterable

import torch

from dattri_llm_b200.gradient.ops import dtypes
from dattri_llm_b200.gradient.ops.materialize import materialize
from dattri_llm_b200.gradient.ops.preprocess import preprocess_factors, to_3d
from dattri_llm_b200.gradient.ops.types import (
    PARAM_GRAD_TYPES,
    is_conv,
    is_conv_transpose,
    is_embedding,
    is_norm,
)

# Bound on the (B1*T1) x (B2*T2) token-match temporaries of the embedding gram.
_EMB_CHUNK_ELEMS = 1 << 26


def _native(*ts):
    from dattri_llm_b200 import ops as native_ops

    return native_ops.use_native(*ts) and all(t.dtype == torch.bfloat16 for t in ts)


def _embedding_gram(tok1, g1, tok2, g2, per_token: bool = False) -> torch.Tensor:
    """``K[i, j] = sum_{t, s} [tok1_it == tok2_js] <g1_it, g2_js>`` without a vocab-sized
    buffer (chunked over side 2); ``per_token`` keeps side 1's ``t`` axis."""
    g1, g2 = dtypes.align(g1, g2)
    b1, t1 = tok1.shape
    b2, t2 = tok2.shape
    e = g1.shape[-1]
    if _native(g1, g2) and tok1.is_cuda and tok2.is_cuda:
        from dattri_llm_b200 import ops as native_ops

        if per_token:  # every side-1 token is its own "sample"
            k = native_ops.ghost_gram_tokens(tok1.reshape(-1, 1), g1.reshape(b1 * t1, 1, e), tok2, g2)
            return k.view(b1, t1, b2).to(g1.dtype)
        return native_ops.ghost_gram_tokens(tok1, g1, tok2, g2).to(g1.dtype)
    out = torch.zeros((b1, t1, b2) if per_token else (b1, b2), dtype=g1.dtype, device=g1.device)
    flat1, gf1 = tok1.reshape(-1), g1.reshape(-1, e)
    step = max(1, _EMB_CHUNK_ELEMS // max(1, b1 * t1 * t2))
    for j0 in range(0, b2, step):
        j1 = min(b2, j0 + step)
        flat2 = tok2[j0:j1].reshape(-1)
        gf2 = g2[j0:j1].reshape(-1, e)
        match = (flat1[:, None] == flat2[None, :]).to(gf1.dtype)
        prod = (gf1 @ gf2.T) * match
        prod = prod.view(b1, t1, j1 - j0, t2).sum(3)
        if per_token:
            out[:, :, j0:j1] = prod
        else:
            out[:, j0:j1] = prod.sum(1)
    return out


def cross_gram(a1, g1, a2, g2, layer_type: str, mode: str = "auto") -> torch.Tensor:
    """Cross-gram ``K[i, j] = <dW1_i, dW2_j>`` on already-preprocessed factors."""
    if is_embedding(layer_type):
        return _embedding_gram(a1, g1, a2, g2)
    a1, g1, a2, g2 = dtypes.align(a1, g1, a2, g2)
    a1, g1, a2, g2 = to_3d(a1), to_3d(g1), to_3d(a2), to_3d(g2)
    if is_norm(layer_type):
        return (a1 * g1).sum(1) @ (a2 * g2).sum(1).T
    b1, s, k = a1.shape[0], a1.shape[1], a1.shape[-1]
    b2, d = a2.shape[0], g1.shape[-1]
    if mode == "auto":
        mode = "materialized" if maybe_use_materialized_gram(b1, b2, s, k, d) else "factorized"
    if a1.ndim == 4:
        if mode == "materialized":
            m1 = torch.einsum("bsgk,bsgd->bgkd", a1, g1).reshape(b1, -1)
            m2 = torch.einsum("bsgk,bsgd->bgkd", a2, g2).reshape(b2, -1)
            return m1 @ m2.T
        ka = torch.einsum("bsgk,ctgk->bcgst", a1, a2)
        kg = torch.einsum("bsgd,ctgd->bcgst", g1, g2)
        return (ka * kg).sum((2, 3, 4))
    if mode == "materialized":
        if _native(a1, g1, a2, g2):
            from dattri_llm_b200 import ops as native_ops

            m1 = native_ops.per_sample_outer(a1, g1, out_dtype=torch.bfloat16).reshape(b1, -1)
            m2 = native_ops.per_sample_outer(a2, g2, out_dtype=torch.bfloat16).reshape(b2, -1)
            return native_ops.matmul_tn(m1, m2).to(a1.dtype)
        m1 = torch.bmm(a1.transpose(1, 2), g1).reshape(b1, -1)
        m2 = torch.bmm(a2.transpose(1, 2), g2).reshape(b2, -1)
        return m1 @ m2.T
    if _native(a1, g1, a2, g2):
        from dattri_llm_b200 import ops as native_ops

        return native_ops.ghost_gram(a1, g1, a2, g2).to(a1.dtype)
    s2 = a2.shape[1]
    ka = a1.reshape(b1 * s, k) @ a2.reshape(b2 * s2, k).T
    kg = g1.reshape(b1 * s, d) @ g2.reshape(b2 * s2, d).T
    return (ka * kg).view(b1, s, b2, s2).sum((1, 3))


def cross_dot_factors(a1, g1, a2, g2, layer_type, module_kwargs1=None, module_kwargs2=None,
                      include_bias: bool = True, mode: str = "auto") -> torch.Tensor:
    """``(B1, B2)`` cross-gram of two raw factor pairs."""
    a1, g1 = preprocess_factors(a1, g1, layer_type, module_kwargs1, include_bias)
    a2, g2 = preprocess_factors(a2, g2, layer_type, module_kwargs2, include_bias)
    return cross_gram(a1, g1, a2, g2, layer_type, mode)


def pairwise_dot_factors(a, g, layer_type, module_kwargs=None, include_bias: bool = True,
                         mode: str = "auto") -> torch.Tensor:
    """``(B, B)`` Gram matrix of one batch's per-sample gradients."""
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    return cross_gram(a, g, a, g, layer_type, mode)


# Bound on the (B1*T1, D*K) per-token outer products of the native per-token gram.
_TOKEN_OUTER_ELEMS = 1 << 27


def _per_token_gram_native(a1: torch.Tensor, g1: torch.Tensor, m2: torch.Tensor) -> torch.Tensor:
    """``K[i, t, j] = <g1_it a1_it^T, M2_j> = g1_it . (M2_j a1_it)`` for bf16 ``a1 (B, T, K)``,
    ``g1 (B, T, D)`` and side 2 dense ``m2 (C, D*K)`` in the materialized ``(out, in)``
    layout.  One tcgen05 GEMM maps every token's activation through every ``M2_j`` at once,
    ``Y = a1 [M2_1; ...; M2_C]^T`` (fp32), and the dot with ``g1`` reduces ``Y`` over ``D``:
    the ``(D, K)`` outer product of a token is never formed (``T C D`` intermediate values per
    sample instead of ``T D K``: fewer whenever side 2 has fewer samples than the layer has
    inputs).  Chunked over side 2 to bound ``Y``."""
    from dattri_llm_b200 import ops as native_ops

    b, t, k = a1.shape
    d = g1.shape[-1]
    n = b * t
    rows_a, rows_g = a1.reshape(n, k), g1.reshape(n, d).float()
    m2 = m2.reshape(m2.shape[0], d, k).to(torch.bfloat16).contiguous()
    out = torch.empty(n, m2.shape[0], dtype=torch.float32, device=a1.device)
    step = max(1, _TOKEN_OUTER_ELEMS // (n * d))
    for c0 in range(0, m2.shape[0], step):
        block = m2[c0:c0 + step]
        mapped = native_ops.matmul_tn(rows_a, block.reshape(-1, k), out_dtype=torch.float32)
        out[:, c0:c0 + block.shape[0]] = torch.einsum("ncd,nd->nc", mapped.view(n, block.shape[0], d), rows_g)
    return out.view(b, t, -1)


def cross_gram_per_token(a1, g1, a2, g2, layer_type: str) -> torch.Tensor:
    """``K[i, t, j]``: side-1 token ``t``'s share of ``<dW1_i, dW2_j>`` (sums to the gram).

    On sm_100 with bf16 factors the linear-family contraction runs on the tensor cores
    (:func:`_per_token_gram_native`), side 2 summed over its tokens by the per-sample
    outer-product GEMM first."""
    if is_embedding(layer_type):
        return _embedding_gram(a1, g1, a2, g2, per_token=True)
    a1, g1, a2, g2 = dtypes.align(a1, g1, a2, g2)
    a1, g1, a2, g2 = to_3d(a1), to_3d(g1), to_3d(a2), to_3d(g2)
    if is_norm(layer_type):
        return torch.einsum("btd,cd->btc", a1 * g1, (a2 * g2).sum(1))
    if a1.ndim == 3 and _native(a1, g1, a2, g2):
        from dattri_llm_b200 import ops as native_ops

        m2 = native_ops.per_sample_outer(g2, a2, out_dtype=torch.bfloat16)  # (C, D, K) = g2^T a2
        return _per_token_gram_native(a1, g1, m2).to(g1.dtype)
    if a1.ndim == 4:
        m2 = torch.einsum("csgk,csgd->cgkd", a2, g2)
        return torch.einsum("btgk,btgd,cgkd->btc", a1, g1, m2)
    m2 = torch.einsum("csk,csd->ckd", a2, g2)
    return torch.einsum("btk,btd,ckd->btc", a1, g1, m2)


def cross_gram_per_token_dense(a1, g1, m2, layer_type: str) -> torch.Tensor:
    """:func:`cross_gram_per_token` with side 2 already dense ``(B2, d)`` in
    :func:`materialize`'s layout (e.g. a preconditioned test block)."""
    b2 = m2.shape[0]
    if is_embedding(layer_type):
        g1f, m2 = dtypes.align(to_3d(g1), m2)
        e = g1f.shape[-1]
        rows = m2.reshape(b2, -1, e)[:, a1.reshape(-1)].reshape(b2, *a1.shape, e)
        return torch.einsum("bte,cbte->btc", g1f, rows)
    a1f, g1f, m2 = dtypes.align(to_3d(a1), to_3d(g1), m2)
    if is_norm(layer_type):
        return torch.einsum("btd,cd->btc", a1f * g1f, m2)
    if a1f.ndim == 4:
        groups = a1f.shape[2]
        if is_conv_transpose(layer_type):
            m2 = m2.reshape(b2, groups, a1f.shape[-1], g1f.shape[-1])
            return torch.einsum("blgc,blgp,ngcp->bln", a1f, g1f, m2)
        m2 = m2.reshape(b2, groups, g1f.shape[-1], a1f.shape[-1])
        return torch.einsum("btgk,btgd,cgdk->btc", a1f, g1f, m2)
    if is_conv_transpose(layer_type):
        m2 = m2.reshape(b2, a1f.shape[-1], g1f.shape[-1])
        return torch.einsum("blc,blp,ncp->bln", a1f, g1f, m2)
    if _native(a1f, g1f) and m2.is_cuda:
        return _per_token_gram_native(a1f, g1f, m2).to(g1f.dtype)
    m2 = m2.reshape(b2, g1f.shape[-1], a1f.shape[-1])
    return torch.einsum("btk,btd,cdk->btc", a1f, g1f, m2)


def cross_dot_per_token(f1, f2, layer_type: str, include_bias: bool = True) -> torch.Tensor:
    """Per-token-position cross-gram of a :class:`Factorized` side 1 against side 2 in
    either form (batch-first-safe)."""
    b1 = f1.as_batch_first()
    a1, g1 = preprocess_factors(b1.activation, b1.pre_activation_grad, layer_type,
                                b1.module_kwargs, include_bias)
    if isinstance(f2, torch.Tensor):
        return cross_gram_per_token_dense(a1, g1, f2.reshape(f2.shape[0], -1), layer_type)
    b2 = f2.as_batch_first()
    a2, g2 = preprocess_factors(b2.activation, b2.pre_activation_grad, layer_type,
                                b2.module_kwargs, include_bias)
    return cross_gram_per_token(a1, g1, a2, g2, layer_type)


def dot_factors(a1, g1, a2, g2, layer_type, module_kwargs1=None, module_kwargs2=None,
                include_bias: bool = True) -> torch.Tensor:
    """``(B,)`` aligned per-sample dot products ``<dW1_i, dW2_i>``."""
    a1, g1 = preprocess_factors(a1, g1, layer_type, module_kwargs1, include_bias)
    a2, g2 = preprocess_factors(a2, g2, layer_type, module_kwargs2, include_bias)
    if is_embedding(layer_type):
        if _native(g1, g2) and a1.is_cuda and a2.is_cuda:
            from dattri_llm_b200 import ops as native_ops

            return native_ops.ghost_gram_tokens(a1, g1, a2, g2, diag_only=True).diagonal().to(g1.dtype)
        return torch.stack([
            _embedding_gram(a1[i : i + 1], g1[i : i + 1], a2[i : i + 1], g2[i : i + 1])[0, 0]
            for i in range(a1.shape[0])
        ])
    a1, g1, a2, g2 = dtypes.align(a1, g1, a2, g2)
    a1, g1, a2, g2 = to_3d(a1), to_3d(g1), to_3d(a2), to_3d(g2)
    if is_norm(layer_type):
        return ((a1 * g1).sum(1) * (a2 * g2).sum(1)).sum(-1)
    if a1.ndim == 4:
        ka = torch.einsum("btgd,bsgd->bgts", a1, a2)
        kg = torch.einsum("btge,bsge->bgts", g1, g2)
        return (ka * kg).sum((1, 2, 3))
    if _native(a1, g1, a2, g2):
        from dattri_llm_b200 import ops as native_ops

        return native_ops.ghost_dot(a1, g1, a2, g2).to(a1.dtype)
    ka = torch.einsum("btd,bsd->bts", a1, a2)
    kg = torch.einsum("bte,bse->bts", g1, g2)
    return (ka * kg).sum((1, 2))


def grad_norm_sq_factors(a, g, layer_type, module_kwargs=None, include_bias: bool = True,
                         mode: str = "auto") -> torch.Tensor:
    """``(B,)`` per-sample squared Frobenius norms of the weight gradients."""
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    if is_embedding(layer_type):
        if _native(g) and a.is_cuda:
            from dattri_llm_b200 import ops as native_ops

            return native_ops.ghost_gram_tokens(a, g, a, g, diag_only=True).diagonal().to(g.dtype)
        return torch.stack([
            _embedding_gram(a[i : i + 1], g[i : i + 1], a[i : i + 1], g[i : i + 1])[0, 0]
            for i in range(a.shape[0])
        ])
    a, g = dtypes.align(a, g)
    a, g = to_3d(a), to_3d(g)
    if is_norm(layer_type):
        return (a * g).sum(1).square().sum(-1)
    s, k, d = a.shape[1], a.shape[-1], g.shape[-1]
    if mode == "auto":
        mode = "materialized" if maybe_use_materialized_norm(s, k, d) else "factorized"
    if a.ndim == 4:
        if mode == "materialized":
            m = torch.einsum("btgk,btgd->bgkd", a, g).flatten(1)
            return (m * m).sum(-1)
        ka = torch.einsum("btgk,bsgk->bgts", a, a)
        kg = torch.einsum("btgd,bsgd->bgts", g, g)
        return (ka * kg).sum((1, 2, 3))
    if mode == "materialized":
        if _native(a, g):
            from dattri_llm_b200 import ops as native_ops

            m = native_ops.per_sample_outer(a, g, out_dtype=torch.float32).flatten(1)
            return (m * m).sum(-1).to(a.dtype)
        m = torch.einsum("btk,btd->bkd", a, g).flatten(1)
        return (m * m).sum(-1)
    if _native(a, g):
        from dattri_llm_b200 import ops as native_ops

        return native_ops.ghost_dot(a, g, a, g).to(a.dtype)
    ka = torch.einsum("btk,bsk->bts", a, a)
    kg = torch.einsum("btd,bsd->bts", g, g)
    return (ka * kg).sum((1, 2))


def grad_norm_sq(f, layer_type: str, include_bias: bool = True, mode: str = "auto") -> torch.Tensor:
    """Per-sample squared gradient norms ``(B,)`` of one layer, whatever its form."""
    if isinstance(f, torch.Tensor):
        (flat,) = dtypes.align(f.reshape(f.shape[0], -1))
        return (flat * flat).sum(-1)
    bf = f.as_batch_first()
    return grad_norm_sq_factors(bf.activation, bf.pre_activation_grad, layer_type,
                                bf.module_kwargs, include_bias, mode)


def pairwise_dot(f, layer_type: str, include_bias: bool = True, mode: str = "auto") -> torch.Tensor:
    """:func:`pairwise_dot_factors` on a :class:`Factorized` (batch-first-safe)."""
    bf = f.as_batch_first()
    return pairwise_dot_factors(bf.activation, bf.pre_activation_grad, layer_type,
                                bf.module_kwargs, include_bias, mode)


def dot(f1, f2, layer_type: str, include_bias: bool = True) -> torch.Tensor:
    """:func:`dot_factors` on two :class:`Factorized` (batch-first-safe)."""
    b1, b2 = f1.as_batch_first(), f2.as_batch_first()
    return dot_factors(b1.activation, b1.pre_activation_grad, b2.activation,
                       b2.pre_activation_grad, layer_type, b1.module_kwargs, b2.module_kwargs,
                       include_bias)


def cross_dot(f1, f2, layer_type: str, include_bias: bool = True, mode: str = "auto") -> torch.Tensor:
    """``(B1, B2)`` cross-gram of one layer in whatever form each side holds; a dense
    side materializes the other."""
    if isinstance(f1, torch.Tensor) or isinstance(f2, torch.Tensor):
        m1 = materialize(f1, layer_type, include_bias)
        m2 = materialize(f2, layer_type, include_bias)
        m1, m2 = dtypes.align(m1, m2)
        if _native(m1, m2):
            from dattri_llm_b200 import ops as native_ops

            return native_ops.matmul_tn(m1, m2).to(m1.dtype)
        return m1 @ m2.T
    b1, b2 = f1.as_batch_first(), f2.as_batch_first()
    return cross_dot_factors(b1.activation, b1.pre_activation_grad, b2.activation,
                             b2.pre_activation_grad, layer_type, b1.module_kwargs,
                             b2.module_kwargs, include_bias, mode)


def _expand_broadcast(m: torch.Tensor, b1: int, b2: int) -> torch.Tensor:
    return m.expand(b1 if m.shape[0] == 1 else m.shape[0], b2 if m.shape[1] == 1 else m.shape[1])


def layerwise_cross_dot(train, test, *, layers: Iterable[str] | None = None, mode: str = "auto",
                        dense_cache=None, reduce: str = "sum"):
    """Layer-by-layer cross-gram of two gradient blocks, summed over layers (or per layer
    with ``reduce="none"``).  A broadcast layer (batch 1) is expanded to every sample.
    With a dense test side, the train side is materialized once per layer (reused
    through *dense_cache*)."""
    if reduce not in {"sum", "none"}:
        raise ValueError("reduce must be 'sum' or 'none'")
    names = list(train.data) if layers is None else list(layers)
    per_layer: dict[str, torch.Tensor] = {}
    for name in names:
        if name not in train.data or name not in test.data:
            continue
        lt = train.layer_types[name]
        if lt == PARAM_GRAD_TYPES:
            continue
        tr, te = train.data[name], test.data[name]
        if isinstance(te, torch.Tensor) and not isinstance(tr, torch.Tensor):
            tr = (dense_cache.get_or_compute(name, lambda tr=tr, lt=lt: materialize(tr, lt))
                  if dense_cache is not None else materialize(tr, lt))
        per_layer[name] = cross_dot(tr, te, lt, mode=mode)
    if reduce == "none":
        return per_layer
    if not per_layer:
        raise ValueError("No shared layers between the two gradient blocks.")
    b_tr, b_te = train.batch_size, test.batch_size
    total = None
    for m in per_layer.values():
        e = _expand_broadcast(m, b_tr, b_te)
        total = e.clone() if total is None else total + e
    return total


def layerwise_cross_dot_per_token(train, test, *, layers: Iterable[str] | None = None,
                                  reduce: str = "sum"):
    """``(B_train, T_train, B_test)`` contribution of every train token position to
    :func:`layerwise_cross_dot` (sums back to it over ``T``)."""
    if reduce not in {"sum", "none"}:
        raise ValueError("reduce must be 'sum' or 'none'")
    names = list(train.data) if layers is None else list(layers)
    per_layer: dict[str, torch.Tensor] = {}
    for name in names:
        if name not in train.data or name not in test.data:
            continue
        if train.layer_types[name] == PARAM_GRAD_TYPES:
            continue
        tr = train.data[name]
        if isinstance(tr, torch.Tensor) or train.indexing[name] != "batch_token":
            raise ValueError(
                f"layer {name!r} has no token axis on the train side (stored "
                f"{train.representation[name]}, indexing {train.indexing[name]!r}); token-level "
                "attribution needs the train gradients captured factorized.",
            )
        per_layer[name] = cross_dot_per_token(tr, test.data[name], train.layer_types[name])
    if reduce == "none":
        return per_layer
    if not per_layer:
        raise ValueError("No shared layers between the two gradient blocks.")
    shapes = {tuple(v.shape) for v in per_layer.values()}
    if len(shapes) > 1:
        raise ValueError(
            "Layers disagree on the token axis, so their per-token contributions cannot be "
            f"summed: {sorted(shapes)}.  Use reduce='none'.",
        )
    return torch.stack(list(per_layer.values())).sum(0)


def effective_dims(f, layer_type: str) -> tuple[int, int, int, int]:
    """Cheap post-preprocess ``(B, S, K, D)`` read from the raw factor shapes
    (per-group widths for grouped convolutions)."""
    bf = f.as_batch_first()
    a, g = bf.activation, bf.pre_activation_grad
    mk = bf.module_kwargs
    if mk is None:
        if a.ndim == 4:
            return a.shape[0], a.shape[1], a.shape[-1], g.shape[-1]
        return a.shape[0], math.prod(a.shape[1:-1]), a.shape[-1], g.shape[-1]
    groups = mk.get("groups", 1)
    kprod = math.prod(mk["kernel_size"]) if "kernel_size" in mk else 1
    if is_conv(layer_type):
        return a.shape[0], math.prod(g.shape[2:]), a.shape[1] // groups * kprod, g.shape[1] // groups
    if is_conv_transpose(layer_type):
        return a.shape[0], math.prod(a.shape[2:]), a.shape[1] // groups, g.shape[1] // groups * kprod
    return a.shape[0], math.prod(a.shape[1:-1]), a.shape[-1], g.shape[-1]


def maybe_use_materialized_gram(B1: int, B2: int, S: int, K: int, D: int, kappa: float = 1.0) -> bool:
    """``True`` when materialize-then-GEMM is cheaper than the ghost route, by flop count:
    ``kappa * B1 B2 S^2 (D+K) >= (B1+B2) S D K + B1 B2 D K``."""
    return kappa * B1 * B2 * S * S * (D + K) >= (B1 + B2) * S * D * K + B1 * B2 * D * K


def maybe_use_materialized_norm(S: int, K: int, D: int) -> bool:
    """``True`` when materializing is cheaper for per-sample norms: ``S (D+K) >= D K``."""
    return S * (D + K) >= D * K
