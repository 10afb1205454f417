"""dattri_llm_b200: training-data attribution for LLMs, built for NVIDIA B200 (sm_100a).

The advertised surface matches dattri-llm's::

    from dattri_llm_b200 import HookManager, HookManagerConfig, OffloadCallback

    with HookManager(model, callbacks=[...]).collect(deregister_on_exit=True):
        trainer.train()

The capture core is imported eagerly with torch alone; the attribution layer and
the live streamer resolve lazily on first access.  Hot contractions run on the
sm_100a kernels of :mod:`dattri_llm_b200.ops` when tensors live on a B200.
"""

from importlib import import_module

from dattri_llm_b200.gradient import (
    REGISTER_ALL,
    CaptureCallback,
    DataSelectionCallback,
    GradientRecord,
    GradientStorageManager,
    HookManager,
    HookManagerCallback,
    HookManagerConfig,
    KroneckerCovarianceCallback,
    OffloadCallback,
    OptimizerStateCallback,
    ParameterSnapshotCallback,
    TrajectorySnapshots,
    default_hook_assignment,
)
from dattri_llm_b200.gradient.gradient import Factorized, Gradient
from dattri_llm_b200.utils.hashing import hash_batch, hash_sample

__version__ = "0.1.0"

_LAZY_EXPORTS = {
    "GradientStreamer": "dattri_llm_b200.gradient.streaming",
    "DiskGradientSource": "dattri_llm_b200.gradient.streaming",
    "ReplayGradientSource": "dattri_llm_b200.gradient.streaming",
    "AttributionArguments": "dattri_llm_b200.attribution.arguments",
    "AttributionTask": "dattri_llm_b200.task",
    "AttributionScore": "dattri_llm_b200.attribution.score",
    "BaseAttributor": "dattri_llm_b200.attribution",
    "BaseInnerProductAttributor": "dattri_llm_b200.attribution",
    "KroneckerAttributor": "dattri_llm_b200.attribution",
    "TracInAttributor": "dattri_llm_b200.attribution",
    "KFACAttributor": "dattri_llm_b200.attribution",
    "EKFACAttributor": "dattri_llm_b200.attribution",
    "DVEmbAttributor": "dattri_llm_b200.attribution",
    "LESSAttributor": "dattri_llm_b200.attribution",
    "AdamWInfluenceAttributor": "dattri_llm_b200.attribution",
    "TrajectoryAttributor": "dattri_llm_b200.attribution",
}

__all__ = sorted([
    "REGISTER_ALL", "CaptureCallback", "DataSelectionCallback", "Factorized", "Gradient",
    "GradientRecord", "GradientStorageManager", "HookManager", "HookManagerCallback",
    "HookManagerConfig", "KroneckerCovarianceCallback", "OffloadCallback", "OptimizerStateCallback",
    "ParameterSnapshotCallback", "TrajectorySnapshots", "default_hook_assignment", "hash_batch",
    "hash_sample", *_LAZY_EXPORTS,
])


def __getattr__(name: str) -> object:
    module = _LAZY_EXPORTS.get(name)
    if module is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    return getattr(import_module(module), name)


def __dir__() -> list[str]:
    return sorted(set(globals()) | set(_LAZY_EXPORTS))
