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
    """Per-layer ``(A, G)`` accumulated over every captured step."""

    def __init__(self, *, include_bias: bool = True) -> None:
        self._include_bias = include_bias
        self._accumulators: dict[str, ops.LayerKroneckerAccumulator] = {}
        self._pending: dict[str, list[torch.Tensor]] = {}

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
        self._accumulators.setdefault(layer_name, ops.LayerKroneckerAccumulator()).update(
            pending.pop(), grad_output, layer_type, module_kwargs, include_bias=self._include_bias)

    def all_reduce(self) -> None:
        """Sum every layer's accumulators over ranks (sorted order on every rank)."""
        from dattri_llm_b200.parallel.covariance import all_reduce_accumulators

        all_reduce_accumulators([self._accumulators[n] for n in sorted(self._accumulators)])

    def result(self) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """``{layer: (A, G)}`` means (layers without gradient-carrying rows omitted)."""
        out = {}
        for name, acc in self._accumulators.items():
            with contextlib.suppress(RuntimeError):
                out[name] = acc.result()
        return out

    def reset(self) -> None:
        """Drop every accumulator."""
        self._accumulators.clear()
        self._pending.clear()
