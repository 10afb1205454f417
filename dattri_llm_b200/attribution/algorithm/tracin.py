"""TracIn / Grad-Dot / Grad-Cos attribution.

Score = ``<g_train, g_test>`` (``"dot"``), or the cosine ``<g_train, g_test> /
(|g_train| |g_test|)`` with ``normalized_grad=True`` (GradCos), summed over the
task's checkpoints (TracIn's ensemble).  Norms are the full-model norms over the
shared layers.  Parity: reference ``dattri_llm/attribution/algorithm/tracin.py``.
The dot-product form of fully dense (projected / materialized) blocks is scored as
one packed tcgen05 GEMM per train block.
"""

from __future__ import annotations

from typing import ClassVar

import torch

from dattri_llm_b200.attribution.base import BaseInnerProductAttributor
from dattri_llm_b200.gradient import ops


class TracInAttributor(BaseInnerProductAttributor):
    """TracIn / GradCos attributor."""

    algorithm: ClassVar[str] = "TracIn"

    def __init__(self, args, *, task=None) -> None:
        super().__init__(args, task=task)
        self._metric = "dot"

    def _set_metric(self, normalized_grad: bool) -> None:
        self._metric = "cosine" if normalized_grad else "dot"
        self.algorithm = "GradCos" if normalized_grad else "TracIn"

    def uses_plain_inner_product(self) -> bool:
        """The dot-product form is the plain layerwise inner product."""
        return self._metric == "dot"

    def inner_product(self, train_rep, test_rep, *, dense_cache=None) -> torch.Tensor:
        """Dot product, or cosine of the full-model gradients over the shared layers."""
        dot = super().inner_product(train_rep, test_rep, dense_cache=dense_cache)
        if self._metric == "dot":
            return dot
        shared = [n for n in train_rep.data if n in test_rep.data]
        if not shared:
            return dot
        return dot / (self._norm(train_rep, shared, dense_cache)[:, None]
                      * self._norm(test_rep, shared, None)[None, :] + 1e-8)

    def inner_product_per_token(self, train_rep, test_rep) -> torch.Tensor:
        """Per-token decomposition (cosine normalised by the whole-sample norms)."""
        dot = super().inner_product_per_token(train_rep, test_rep)
        if self._metric == "dot":
            return dot
        shared = [n for n in train_rep.data if n in test_rep.data]
        if not shared:
            return dot
        return dot / (self._norm(train_rep, shared, None)[:, None, None]
                      * self._norm(test_rep, shared, None)[None, None, :] + 1e-8)

    @staticmethod
    def _norm(rep, layers, dense_cache) -> torch.Tensor:
        rows = rep.batch_size
        total = torch.zeros(rows, device=rep.device)
        for name in layers:
            v = rep.data[name]
            if dense_cache is not None and name in dense_cache:
                v = dense_cache.get(name)
            sq = ops.grad_norm_sq(v, rep.layer_types[name]).float()
            total += sq.expand(rows) if sq.shape[0] == 1 else sq
        return total.clamp_min(0).sqrt()

    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, enable_update: bool = False, gradient_cache_residency=None,
                  attribution_granularity: str = "instance", normalized_grad: bool = False):
        """Live TracIn (``normalized_grad=True``: GradCos)."""
        self._set_metric(normalized_grad)
        return super().attribute(train_dataset, test_dataset, hook_config=hook_config, verbose=verbose,
                                 loop_over_test=loop_over_test, enable_update=enable_update,
                                 gradient_cache_residency=gradient_cache_residency,
                                 attribution_granularity=attribution_granularity, normalized_grad=normalized_grad)

    def attribute_from_cache(self, train_source, test_source, *, selected_training_steps=None, layer_name=None,
                             verbose: bool = False, loop_over_test: bool = False, algorithm_meta=None,
                             attribution_granularity: str = "instance", normalized_grad: bool = False):
        """TracIn over stored gradients."""
        self._set_metric(normalized_grad)
        return super().attribute_from_cache(
            train_source, test_source, selected_training_steps=selected_training_steps, layer_name=layer_name,
            verbose=verbose, loop_over_test=loop_over_test, algorithm_meta=algorithm_meta,
            attribution_granularity=attribution_granularity, normalized_grad=normalized_grad)
