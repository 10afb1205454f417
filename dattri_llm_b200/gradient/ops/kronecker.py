"""K-FAC / EK-FAC factors, inverses, preconditioning and streaming accumulators.

Parity: reference ``dattri_llm/gradient/ops/kronecker.py:33-748`` (same
definitions: ``A = E[a a^T]``, ``G = E[g g^T]`` over gradient-carrying token rows,
``F = E[dW dW^T]``; eigenbasis rotation ``U_G^T dW U_A``; damped inverses).

B200 differences: the covariance updates ``A += a^T a`` run as split-K tcgen05
Gram GEMMs that accumulate straight into the fp32 running sums (no bf16 round
trip of the update, no extra add kernel); gradient-free rows are masked on the
device instead of boolean-indexed, so an update never synchronizes the host; and
the row count is a device tensor until :meth:`result` reads it.  The cross-rank
reduction can go through the fused NVLink kernel in
:mod:`dattri_llm_b200.parallel.covariance`.
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass, field

import torch

from dattri_llm_b200.gradient.ops import dtypes
from dattri_llm_b200.gradient.ops.dot import cross_gram
from dattri_llm_b200.gradient.ops.materialize import materialize, materialize_factors
from dattri_llm_b200.gradient.ops.preprocess import preprocess_factors
from dattri_llm_b200.gradient.ops.types import is_conv, is_conv_transpose, is_embedding, is_norm
from dattri_llm_b200.utils.distributed import all_reduce_sum


def _flatten_for_kfac(a: torch.Tensor, g: torch.Tensor, layer_type: str):
    if is_norm(layer_type):
        raise NotImplementedError("K-FAC is not defined for normalization layers")
    if is_embedding(layer_type):
        raise NotImplementedError("K-FAC is not defined for embedding layers")
    a, g = dtypes.align(a, g)
    if a.ndim == 4:  # grouped: (G, N, w) per group
        groups = a.shape[2]
        return (a.permute(2, 0, 1, 3).reshape(groups, -1, a.shape[-1]),
                g.permute(2, 0, 1, 3).reshape(groups, -1, g.shape[-1]))
    return a.reshape(-1, a.shape[-1]), g.reshape(-1, g.shape[-1])


def _right_multiply(x: torch.Tensor, matrix: torch.Tensor) -> torch.Tensor:
    """``x @ matrix`` over the last axis (grouped per-group matrices for 3-D *matrix*).  Dense
    fp32 products run as the bf16x3 tcgen05 GEMM on sm_100 (``ops.matmul_f32``)."""
    if matrix.ndim == 3:
        return torch.einsum("...gk,gkj->...gj", x, matrix)
    from dattri_llm_b200.ops.gemm import matmul_f32

    if x.dtype == torch.float32 and matrix.dtype == torch.float32 and x.is_cuda:
        flat = x.reshape(-1, x.shape[-1])
        return matmul_f32(flat, matrix).reshape(*x.shape[:-1], matrix.shape[-1])
    return x @ matrix


def _row_mask(a_f, g_f, layer_type):
    """(masked a, g, number of gradient-carrying rows as a 0-d tensor)."""
    if is_conv(layer_type) or is_conv_transpose(layer_type):
        return a_f, g_f, torch.tensor(a_f.shape[-2], device=a_f.device)
    keep = (g_f != 0).any(dim=-1)
    a_f = a_f * keep.unsqueeze(-1).to(a_f.dtype)
    return a_f, g_f, keep.sum(dim=-1).reshape(-1)[0] if keep.ndim > 1 else keep.sum()


def gram_accumulate(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``out += x^T x`` (fp32 *out*) for ``x (N, w)`` or grouped ``(G, N, w)``.

    On sm_100 with bf16 rows this is one tcgen05 launch on CTA pairs that computes only
    the tiles on and above the diagonal (mirroring each off-diagonal one), splits the row
    sum over pairs along the samples, and adds into *out* with fp32 atomics.
    """
    from dattri_llm_b200 import ops as native_ops

    if (native_ops.use_native(x, out) and x.dtype == torch.bfloat16 and x.ndim == 2 and out.dtype == torch.float32
            and out.is_contiguous() and x.shape[0] > 0):
        xt = native_ops.gemm._k_aligned(native_ops.gemm.transpose_last2(x))  # (w, N): contraction axis contiguous
        native_ops.count_launch()
        native_ops.native().gram_acc(xt, out, 1.0, native_ops.error_word(x.device))
        return out
    out += (x.transpose(-1, -2) @ x).float()
    return out


def kfac_factors(a, g, layer_type: str, module_kwargs: dict | None = None,
                 include_bias: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """``(A, G)`` K-FAC covariances of one batch (fp32, gradient-free rows dropped).

    Raises:
        ValueError: if every row carries a zero gradient.
    """
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    a_f, g_f = _flatten_for_kfac(a, g, layer_type)
    a_f, g_f, n = _row_mask(a_f, g_f, layer_type)
    n = int(n)
    if n == 0:
        raise ValueError("K-FAC factors are undefined: every token row carries a zero gradient.")
    lead = a_f.shape[:-2]
    A = torch.zeros(*lead, a_f.shape[-1], a_f.shape[-1], device=a_f.device)
    G = torch.zeros(*lead, g_f.shape[-1], g_f.shape[-1], device=g_f.device)
    return gram_accumulate(a_f, A) / n, gram_accumulate(g_f, G) / n


def fim_factors(a, g, layer_type: str, module_kwargs: dict | None = None,
                include_bias: bool = True) -> torch.Tensor:
    """``(d, d)`` empirical Fisher of one batch's per-sample gradients (the same Gram
    accumulation as the K-FAC covariances: a tcgen05 split-K GEMM for bf16 rows on sm_100)."""
    grad = materialize_factors(a, g, layer_type, module_kwargs, include_bias)
    grad = grad.reshape(grad.shape[0], -1)
    fisher = torch.zeros(grad.shape[1], grad.shape[1], device=grad.device)
    return gram_accumulate(grad, fisher) / grad.shape[0]


def sym_inverse(matrix: torch.Tensor, damping: float = 0.0) -> torch.Tensor:
    """Damped symmetric inverse ``(M + damping I)^-1`` through ``eigh``."""
    evals, evecs = torch.linalg.eigh(matrix.float())
    return (evecs / (evals + damping).unsqueeze(-2)) @ evecs.transpose(-1, -2)


def dense_inverse(matrix: torch.Tensor, damping: float = 0.0) -> torch.Tensor:
    """Damped inverse through Cholesky, falling back to :func:`sym_inverse`."""
    m = matrix.float()
    damped = m + damping * torch.eye(m.shape[-1], device=m.device, dtype=m.dtype)
    try:
        return torch.cholesky_inverse(torch.linalg.cholesky(damped))
    except RuntimeError:
        return sym_inverse(matrix, damping)


def kfac_cross_factors(a1, g1, a2, g2, layer_type: str, A_inv, G_inv, module_kwargs1=None,
                       module_kwargs2=None, include_bias: bool = True) -> torch.Tensor:
    """K-FAC preconditioned cross-gram ``<G^-1 dW1 A^-1, dW2>``."""
    a1, g1 = preprocess_factors(a1, g1, layer_type, module_kwargs1, include_bias)
    a2, g2 = preprocess_factors(a2, g2, layer_type, module_kwargs2, include_bias)
    a1 = _right_multiply(a1.float(), A_inv.float())
    g1 = _right_multiply(g1.float(), G_inv.float())
    return cross_gram(a1, g1, a2, g2, layer_type)


def kfac_eigh(A: torch.Tensor, G: torch.Tensor):
    """Eigendecompose both factors: ``(s_A, U_A, s_G, U_G)``."""
    s_a, u_a = torch.linalg.eigh(A.float())
    s_g, u_g = torch.linalg.eigh(G.float())
    return s_a, u_a, s_g, u_g


def ekfac_materialize_factors(a, g, layer_type: str, U_A, U_G, module_kwargs=None,
                              include_bias: bool = True) -> torch.Tensor:
    """Per-sample weight gradient rotated into the K-FAC eigenbasis: ``U_G^T dW U_A``."""
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    a = _right_multiply(a.float(), U_A.float())
    g = _right_multiply(g.float(), U_G.float())
    return materialize_factors(a, g, layer_type)


def ekfac_lambda_accumulate(f, layer_type: str, U_A, U_G, lam: torch.Tensor | None,
                            include_bias: bool = True) -> tuple[torch.Tensor, int]:
    """``lam += sum_i (U_G^T dW_i U_A)^2`` over one batch; returns ``(lam, batch size)``.

    Factorized linear layers on sm_100 take the fused path: the factors are rotated into
    the eigenbasis (``a U_A``, ``g U_G``), then ONE batched tcgen05 GEMM forms every
    sample's rotated gradient and squares it into *lam* in its epilogue -- the per-sample
    ``(B, d_out * d_in)`` coordinates never reach HBM.  Everything else materializes the
    coordinates and sums their squares.  Reference:
    ``dattri_llm/attribution/algorithm/kronecker.py:1530-1563``."""
    from dattri_llm_b200 import ops as native_ops

    if not isinstance(f, torch.Tensor) and U_A.ndim == 2 and not is_conv_transpose(layer_type):
        bf = f.as_batch_first()
        a, g = preprocess_factors(bf.activation, bf.pre_activation_grad, layer_type, bf.module_kwargs,
                                  include_bias)
        if (a.ndim == 3 and g.ndim == 3 and native_ops.use_native(a, g) and a.dtype == torch.bfloat16
                and g.dtype == torch.bfloat16 and a.shape[-1] == U_A.shape[0] and g.shape[-1] == U_G.shape[0]):
            b, t = a.shape[:2]
            ka, kg = U_A.shape[-1], U_G.shape[-1]
            # eigenbasis factors stored token-major, (B, k, T): the operands of the next GEMM
            ar_t = torch.empty(b, ka, t, dtype=torch.bfloat16, device=a.device)
            gr_t = torch.empty(b, kg, t, dtype=torch.bfloat16, device=a.device)
            native_ops.gemm_tn(a.contiguous(), U_A.t().contiguous().bfloat16(), ar_t, mode=native_ops.STORE_BF16_T)
            native_ops.gemm_tn(g.contiguous(), U_G.t().contiguous().bfloat16(), gr_t, mode=native_ops.STORE_BF16_T)
            if lam is None:
                lam = torch.zeros(kg * ka, dtype=torch.float32, device=a.device)
            native_ops.gemm_tn(gr_t, ar_t, lam.view(kg, ka), mode=native_ops.STORE_SQ_SUM_F32)
            return lam, b
    m = ekfac_materialize(f, layer_type, U_A, U_G, include_bias)
    sq = (m * m).sum(0)
    return (sq if lam is None else lam.add_(sq)), m.shape[0]


def kfac(f, layer_type: str, include_bias: bool = True):
    """:func:`kfac_factors` on a :class:`Factorized` (batch-first-safe)."""
    bf = f.as_batch_first()
    return kfac_factors(bf.activation, bf.pre_activation_grad, layer_type, bf.module_kwargs,
                        include_bias)


def fim(f, layer_type: str, include_bias: bool = True):
    """:func:`fim_factors` on a :class:`Factorized` (batch-first-safe)."""
    bf = f.as_batch_first()
    return fim_factors(bf.activation, bf.pre_activation_grad, layer_type, bf.module_kwargs,
                       include_bias)


def kfac_cross(f1, f2, layer_type: str, A_inv, G_inv, include_bias: bool = True):
    """:func:`kfac_cross_factors` on two :class:`Factorized` (batch-first-safe)."""
    b1, b2 = f1.as_batch_first(), f2.as_batch_first()
    return kfac_cross_factors(b1.activation, b1.pre_activation_grad, b2.activation,
                              b2.pre_activation_grad, layer_type, A_inv, G_inv, b1.module_kwargs,
                              b2.module_kwargs, include_bias)


def _rotate_block(block, layer_type, U_A, U_G, transpose=False):
    """``U_G^T dW U_A`` (or ``U_G dW U_A^T`` with *transpose*) of a dense block."""
    batch = block.shape[0]
    ua, ug = U_A.float(), U_G.float()
    if transpose:
        ua, ug = ua.transpose(-1, -2), ug.transpose(-1, -2)
    if U_A.ndim == 3:
        groups, ka, kg = U_A.shape[0], U_A.shape[-1], U_G.shape[-1]
        if is_conv_transpose(layer_type):
            dw = block.reshape(batch, groups, ka, kg).float()
            return torch.einsum("gce,bgcp,gpf->bgef", ua, dw, ug).reshape(batch, -1)
        dw = block.reshape(batch, groups, kg, ka).float()
        return torch.einsum("goe,bgoi,gif->bgef", ug, dw, ua).reshape(batch, -1)
    if is_conv_transpose(layer_type):
        c_in, p = U_A.shape[0], U_G.shape[0]
        dw = block.reshape(batch, c_in, p).float()
        return (ua.transpose(0, 1) @ dw @ ug).reshape(batch, c_in * p)
    d_out, d_in = U_G.shape[0], U_A.shape[0]
    dw = block.reshape(batch, d_out, d_in).float()
    return (ug.transpose(0, 1) @ dw @ ua).reshape(batch, d_out * d_in)


def ekfac_materialize(f, layer_type: str, U_A, U_G, include_bias: bool = True) -> torch.Tensor:
    """Eigenbasis coordinates of a :class:`Factorized` layer, or of a dense block."""
    if isinstance(f, torch.Tensor):
        return _rotate_block(f, layer_type, U_A, U_G)
    bf = f.as_batch_first()
    return ekfac_materialize_factors(bf.activation, bf.pre_activation_grad, layer_type, U_A, U_G,
                                     bf.module_kwargs, include_bias)


def kfac_precondition(f, layer_type: str, A_inv, G_inv, include_bias: bool = True):
    """Preprocess and whiten one side's factors: ``(a A^-1, g G^-1)``."""
    bf = f.as_batch_first()
    a, g = preprocess_factors(bf.activation, bf.pre_activation_grad, layer_type,
                              bf.module_kwargs, include_bias)
    return _right_multiply(a.float(), A_inv.float()), _right_multiply(g.float(), G_inv.float())


def kfac_precondition_materialized(block: torch.Tensor, A_inv, G_inv) -> torch.Tensor:
    """Two-sided ``G^-1 dW A^-1`` of a compact dense block ``(B, k_g * k_a)``."""
    batch = block.shape[0]
    kg, ka = G_inv.shape[-1], A_inv.shape[-1]
    if A_inv.ndim == 3:
        dw = block.reshape(batch, A_inv.shape[0], kg, ka).float()
        return torch.einsum("gde,bgek,gkj->bgdj", G_inv.float(), dw, A_inv.float()).reshape(batch, -1)
    dw = block.reshape(batch, kg, ka).float()
    return (G_inv.float() @ dw @ A_inv.float()).reshape(batch, kg * ka)


def ekfac_precondition(M: torch.Tensor, U_A, U_G, lam: torch.Tensor, layer_type: str) -> torch.Tensor:
    """Apply the damped EK-FAC inverse to eigenbasis coordinates *M* and rotate back:
    ``U_G (M / lam) U_A^T``."""
    return _rotate_block(M / lam, layer_type, U_A, U_G, transpose=True)


@dataclass
class LayerKroneckerAccumulator:
    """Streaming fp32 ``(A, G)`` sums and gradient-carrying row count of one layer."""

    _A: torch.Tensor | None = field(default=None, init=False, repr=False)
    _G: torch.Tensor | None = field(default=None, init=False, repr=False)
    _count: torch.Tensor | int = field(default=0, init=False, repr=False)
    # Multi-GPU accumulation: the Gram GEMMs add into symmetric buffers that are reduced
    # over NVLink without a packing copy (parallel.covariance.SymmetricGram); None otherwise.
    _symm: tuple | None = field(default=None, init=False, repr=False)
    fused_reduce: bool | None = None

    @property
    def _n(self) -> int:
        return int(self._count)

    def _use_symm(self, a_f: torch.Tensor, g_f: torch.Tensor) -> bool:
        if self.fused_reduce is False or a_f.ndim != 2 or not a_f.is_cuda or a_f.dtype != torch.bfloat16:
            return False
        from dattri_llm_b200.ops import use_native
        from dattri_llm_b200.parallel import symm

        return use_native(a_f, g_f) and g_f.dtype == torch.bfloat16 and symm.available(a_f.device)

    def update(self, a, g, layer_type: str, module_kwargs: dict | None = None,
               include_bias: bool = True) -> None:
        """Add one batch's raw (or final) factors."""
        a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
        a_f, g_f = _flatten_for_kfac(a, g, layer_type)
        a_f, g_f, n = _row_mask(a_f, g_f, layer_type)
        if self._A is None and self._symm is None:
            if self._use_symm(a_f, g_f):
                from dattri_llm_b200.parallel.covariance import SymmetricGram

                self._symm = (SymmetricGram(a_f.shape[-1], a_f.device), SymmetricGram(g_f.shape[-1], g_f.device))
            else:
                lead = a_f.shape[:-2]
                self._A = torch.zeros(*lead, a_f.shape[-1], a_f.shape[-1], device=a_f.device)
                self._G = torch.zeros(*lead, g_f.shape[-1], g_f.shape[-1], device=g_f.device)
        if self._symm is not None:
            self._symm[0].add(a_f)
            self._symm[1].add(g_f)
        else:
            gram_accumulate(a_f, self._A)
            gram_accumulate(g_f, self._G)
        self._count = self._count + n

    def grouped_ok(self, a_f: torch.Tensor, g_f: torch.Tensor) -> bool:
        """Whether this layer's flattened ``(N, w)`` factors may join a step's grouped update
        (:func:`kfac_accumulate_grouped`): plain (not symmetric-memory) sums, 2-D rows."""
        return self._symm is None and a_f.ndim == 2 and g_f.ndim == 2 and not self._use_symm(a_f, g_f)

    def all_reduce(self) -> None:
        """Sum the accumulators and counts over ranks (collective)."""
        if self._symm is not None:
            self._A, self._G = self._symm[0].reduced(), self._symm[1].reduced()
            self._symm = None
            n = torch.tensor([self._n], dtype=torch.int64)
            self._count = int(all_reduce_sum(n).item())
            return
        if self._A is None:
            raise RuntimeError("No gradient-carrying data has been accumulated")
        all_reduce_sum(self._A)
        all_reduce_sum(self._G)
        n = torch.tensor([self._n], dtype=torch.int64)
        self._count = int(all_reduce_sum(n).item())

    def result(self, *, consume: bool = False):
        """``(A, G)`` means; with *consume* the sums are divided in place and released."""
        n = self._n
        if self._symm is not None:
            raise RuntimeError("This accumulator reduces across ranks: call all_reduce() on every rank first")
        if self._A is None or n == 0:
            raise RuntimeError("No gradient-carrying data has been accumulated")
        if not consume:
            return self._A / n, self._G / n
        A, G = self._A.div_(n), self._G.div_(n)
        self.reset()
        return A, G

    def reset(self) -> None:
        """Drop the accumulated state."""
        self._A, self._G, self._count, self._symm = None, None, 0, None


@dataclass
class LayerFisherAccumulator:
    """Streaming empirical Fisher ``sum_i dW_i dW_i^T`` of one layer."""

    _F: torch.Tensor | None = field(default=None, init=False, repr=False)
    _n: int = field(default=0, init=False, repr=False)

    def update(self, a, g, layer_type: str, module_kwargs: dict | None = None,
               include_bias: bool = True) -> None:
        """Add one batch from raw factors."""
        self.update_from_grad(materialize_factors(a, g, layer_type, module_kwargs, include_bias))

    def update_from_grad(self, grad: torch.Tensor) -> None:
        """Add one batch of dense per-sample gradients ``(B, d)`` (the Gram accumulation of
        :func:`gram_accumulate`: fp32 sums, one tcgen05 launch for bf16 rows on sm_100)."""
        grad = grad.reshape(grad.shape[0], -1)
        wide = grad.dtype == torch.float64
        if self._F is None:
            self._F = torch.zeros(grad.shape[-1], grad.shape[-1], dtype=torch.float64 if wide else torch.float32,
                                  device=grad.device)
        if wide:
            self._F += grad.T @ grad
        else:
            gram_accumulate(grad if grad.dtype == torch.bfloat16 else grad.float(), self._F)
        self._n += grad.shape[0]

    def all_reduce(self) -> None:
        """Sum over ranks."""
        if self._F is None:
            raise RuntimeError("No data has been accumulated")
        all_reduce_sum(self._F)
        self._n = int(all_reduce_sum(torch.tensor([self._n], dtype=torch.int64)).item())

    def result(self) -> torch.Tensor:
        """The mean Fisher."""
        if self._F is None:
            raise RuntimeError("No data has been accumulated")
        return self._F / self._n

    def reset(self) -> None:
        """Drop the accumulated state."""
        self._F, self._n = None, 0


class KroneckerAccumulator:
    """Per-layer :class:`LayerKroneckerAccumulator` over whole gradient blocks."""

    def __init__(self) -> None:
        self._layers: dict[str, LayerKroneckerAccumulator] = {}

    def update(self, gradient, layers: Iterable[str]) -> None:
        """Add the named factorized layers of *gradient*."""
        for name in layers:
            value = gradient.data[name]
            if isinstance(value, torch.Tensor):
                raise TypeError(
                    f"K-FAC covariances need factorized (activation, output-gradient) factors, "
                    f"but layer {name!r} holds a materialized tensor; exclude it from the K-FAC "
                    "layer set.",
                )
            bf = value.as_batch_first()
            self._layers.setdefault(name, LayerKroneckerAccumulator()).update(
                bf.activation, bf.pre_activation_grad, gradient.layer_types[name], bf.module_kwargs)

    def all_reduce(self) -> None:
        """Sum every layer over ranks (sorted order: identical on every rank)."""
        for name in sorted(self._layers):
            self._layers[name].all_reduce()

    def result(self, *, consume: bool = False) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """``{layer: (A, G)}``."""
        out = {n: acc.result(consume=consume) for n, acc in self._layers.items()}
        if consume:
            self._layers = {}
        return out


class FisherAccumulator:
    """Per-layer dense empirical Fishers; layers wider than *max_params* are skipped."""

    def __init__(self, max_params: int | None = None) -> None:
        self._max_params = max_params
        self._layers: dict[str, LayerFisherAccumulator] = {}
        self._skipped: dict[str, int] = {}

    def update(self, gradient, layers: Iterable[str]) -> None:
        """Add the named layers of *gradient* (any form)."""
        for name in layers:
            if name in self._skipped:
                continue
            value = gradient.data[name]
            g = (value.reshape(value.shape[0], -1).float() if isinstance(value, torch.Tensor)
                 else materialize(value, gradient.layer_types[name]))
            if self._max_params is not None and g.shape[-1] > self._max_params:
                self._skipped[name] = g.shape[-1]
                self._layers.pop(name, None)
                continue
            self._layers.setdefault(name, LayerFisherAccumulator()).update_from_grad(g)

    def all_reduce(self) -> None:
        """Sum every layer over ranks."""
        for name in sorted(self._layers):
            self._layers[name].all_reduce()

    def result(self) -> dict[str, torch.Tensor]:
        """``{layer: F}``."""
        return {n: acc.result() for n, acc in self._layers.items()}

    @property
    def skipped(self) -> dict[str, int]:
        """Layers left out for width, with their width."""
        return dict(self._skipped)


def kfac_accumulate_grouped(accs: list[LayerKroneckerAccumulator], a_fs: list[torch.Tensor],
                            g_fs: list[torch.Tensor]) -> None:
    """One step's flattened ``(N, w_a)`` / ``(N, w_g)`` factors of many layers of one shape added
    to their accumulators together: the row masks, both Gram products (one batched GEMM each;
    tcgen05 on sm_100 with bf16 rows) and the sums run once for all layers, instead of a
    handful of small launches per layer (capture-time projections make every layer's factors
    the same ``k``-wide shape)."""
    from dattri_llm_b200 import ops as native_ops

    a = torch.stack(a_fs)                            # (L, N, w_a)
    g = torch.stack(g_fs)                            # (L, N, w_g)
    keep = (g != 0).any(dim=-1)                      # rows that carry a gradient
    a = a * keep.unsqueeze(-1).to(a.dtype)
    counts = keep.sum(dim=-1)                        # (L,)
    grams = []
    for x in (a, g):
        out = torch.zeros(x.shape[0], x.shape[-1], x.shape[-1], dtype=torch.float32, device=x.device)
        if native_ops.use_native(x) and x.dtype == torch.bfloat16 and x.shape[1] > 0:
            xt = native_ops.gemm._k_aligned(native_ops.gemm.transpose_last2(x))  # (L, w, N)
            native_ops.gemm_tn(xt, xt, out, mode=native_ops.STORE_F32)
        else:  # layer by layer, the same products as gram_accumulate's
            for i in range(x.shape[0]):
                out[i] += (x[i].transpose(-1, -2) @ x[i]).float()
        grams.append(out)
    for acc, x_a, x_g in zip(accs, a_fs, g_fs, strict=True):
        if acc._A is None:
            acc._A = torch.zeros(x_a.shape[-1], x_a.shape[-1], device=x_a.device)
            acc._G = torch.zeros(x_g.shape[-1], x_g.shape[-1], device=x_g.device)
        if not isinstance(acc._count, torch.Tensor):
            acc._count = torch.tensor(acc._count, dtype=torch.int64, device=x_a.device)
    torch._foreach_add_([acc._A for acc in accs], list(grams[0].unbind(0)))
    torch._foreach_add_([acc._G for acc in accs], list(grams[1].unbind(0)))
    torch._foreach_add_([acc._count for acc in accs], list(counts.unbind(0)))


def flatten_kfac_factors(a, g, layer_type: str, module_kwargs: dict | None = None,
                         include_bias: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """The ``(N, w)`` rows a K-FAC accumulator sums (preprocessed, flattened over tokens)."""
    a, g = preprocess_factors(a, g, layer_type, module_kwargs, include_bias)
    return _flatten_for_kfac(a, g, layer_type)
