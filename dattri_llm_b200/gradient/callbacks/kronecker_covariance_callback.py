"""Accumulate per-layer K-FAC covariances ``(A, G)`` while capturing.

Pairs each layer's forward activation with its backward output gradient (LIFO per
layer) and feeds a :class:`LayerKroneckerAccumulator`; for pre-projected layers the
pair is the projected factors, so the covariances are ``k x k``.  The updates run
as split-K tcgen05 Gram GEMMs into fp32 sums; :meth:`all_reduce` sums them over
ranks -- through the fused NVLink covariance all-reduce when the process group is
NCCL over several GPUs of one node.  Parity: reference
``dattri_llm/gradient/callbacks/kronecker_covariance_callback.py``.
"""

from __future__ import annotations

import contextlib

import torch

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback


class KroneckerCovarianceCallback(HookManagerCallback):
    """Per-layer ``(A, G)`` accumulated over every captured step.

    Within a step the matched pairs of 2-D linear layers wait until the step ends and are
    then added together, grouped by shape (:func:`ops.kfac_accumulate_grouped`: one batched
    Gram product per side for all layers of a shape); other layers, and accumulators that
    reduce through symmetric memory across GPUs, update as their pair arrives."""

    def __init__(self, *, include_bias: bool = True) -> None:
        self._include_bias = include_bias
        self._accumulators: dict[str, ops.LayerKroneckerAccumulator] = {}
        self._pending: dict[str, list[torch.Tensor]] = {}
        self._step_rows: list[tuple[str, torch.Tensor, torch.Tensor]] = []  # (layer, a rows, g rows)

    def on_layer_forward(self, layer_name, activation, layer_type, module_kwargs) -> None:
        """Stack the activation until its backward."""
        if ops.is_kfac_eligible(layer_type):
            self._pending.setdefault(layer_name, []).append(activation)

    def on_layer_backward(self, layer_name, grad_output, layer_type, module_kwargs) -> None:
        """Accumulate the matched ``(a, g)`` pair."""
        if not ops.is_kfac_eligible(layer_type):
            return
        pending = self._pending.get(layer_name)
        if not pending:
            return
        acc = self._accumulators.setdefault(layer_name, ops.LayerKroneckerAccumulator())
        activation = pending.pop()
        if ops.is_linear(layer_type):
            a_f, g_f = ops.flatten_kfac_factors(activation, grad_output, layer_type, module_kwargs,
                                                include_bias=self._include_bias)
            if acc.grouped_ok(a_f, g_f):
                self._step_rows.append((layer_name, a_f, g_f))
                return
        acc.update(activation, grad_output, layer_type, module_kwargs, include_bias=self._include_bias)

    def on_step_end(self, record) -> None:
        """Add the step's waiting pairs, grouped by shape."""
        self._flush()

    def _flush(self) -> None:
        rows, self._step_rows = self._step_rows, []
        groups: dict[tuple, list[tuple[str, torch.Tensor, torch.Tensor]]] = {}
        for name, a_f, g_f in rows:
            key = (tuple(a_f.shape), tuple(g_f.shape), a_f.dtype, g_f.dtype, a_f.device)
            groups.setdefault(key, []).append((name, a_f, g_f))
        for items in groups.values():
            ops.kfac_accumulate_grouped([self._accumulators[n] for n, _, _ in items],
                                        [a for _, a, _ in items], [g for _, _, g in items])

    def all_reduce(self) -> None:
        """Sum every layer's accumulators over ranks (sorted order on every rank)."""
        self._flush()
        from dattri_llm_b200.parallel.covariance import all_reduce_accumulators

        all_reduce_accumulators([self._accumulators[n] for n in sorted(self._accumulators)])

    def result(self) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """``{layer: (A, G)}`` means (layers without gradient-carrying rows omitted)."""
        self._flush()
        out = {}
        for name, acc in self._accumulators.items():
            with contextlib.suppress(RuntimeError):
                out[name] = acc.result()
        return out

    def reset(self) -> None:
        """Drop every accumulator."""
        self._accumulators.clear()
        self._pending.clear()
        self._step_rows = []
