"""Option vocabularies: ``Literal`` aliases of every enumerated string option.

The aliases are for annotations; each option is still validated at runtime by
the function that takes it.  Same vocabulary as the reference's
``dattri_llm/options.py:152-189``.
"""

from __future__ import annotations

from typing import Literal

#: One score row per training sample (``"instance"``) or per training token position.
AttributionGranularity = Literal["instance", "token"]
#: How the training loss was reduced over each batch.
LossReduction = Literal["mean", "sum"]
#: Which side of a trajectory sweep carries the propagation.
Propagation = Literal["train", "test"]
#: DVEmb's per-step Hessian (Fisher) approximation.
HessianMode = Literal["full", "diagonal"]
#: The representation a captured layer is buffered in.
CaptureStyle = Literal["factorized", "materialized", "auto"]
#: How an inner-product kernel forms its result; ``"auto"`` applies the cost rule.
RoutingMode = Literal["factorized", "materialized", "auto"]
#: Sum layerwise cross-grams over layers, or keep them per layer.
DotReduce = Literal["sum", "none"]
#: Where a cache or gradient store keeps its entries.
CacheResidency = Literal["disk", "memory", "tiered"]
#: On-disk format of a gradient store.
DiskFormat = Literal["pickle", "memmap"]
#: Granularity an ``OffloadCallback`` records at.
RecordingType = Literal["per_sample", "per_batch"]
#: How a layer is projected.
ProjectionStyle = Literal["logra", "dense", "mask"]
#: One score row per training sample, or one per ``(sample, step)`` pair.
ScoreTrajectory = Literal["aware", "agnostic"]
#: EK-FAC's eigenvalue estimate.
EKFACMode = Literal["exact", "approx"]

__all__ = [
    "AttributionGranularity",
    "CacheResidency",
    "CaptureStyle",
    "DiskFormat",
    "DotReduce",
    "EKFACMode",
    "HessianMode",
    "LossReduction",
    "ProjectionStyle",
    "Propagation",
    "RecordingType",
    "RoutingMode",
    "ScoreTrajectory",
]
