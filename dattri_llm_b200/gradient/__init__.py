"""Gradient capture: ``HookManager``, its callbacks, the on-disk store and the core ops."""

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.async_writer import AsyncGradientWriter
from dattri_llm_b200.gradient.callbacks import (
    CaptureCallback,
    DataSelectionCallback,
    HookManagerCallback,
    KroneckerCovarianceCallback,
    OffloadCallback,
    OptimizerStateCallback,
    ParameterSnapshotCallback,
)
from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
from dattri_llm_b200.gradient.hooks import (
    REGISTER_ALL,
    HookManager,
    HookManagerConfig,
    default_hook_assignment,
    register_linear_io_hooks,
    register_linear_param_hooks,
    register_param_grad_hooks,
    remove_hooks,
)
from dattri_llm_b200.gradient.ops import (
    FisherAccumulator,
    KroneckerAccumulator,
    LayerFisherAccumulator,
    LayerKroneckerAccumulator,
    canonical_class_name,
    dot,
    fim,
    grad_norm_sq,
    kfac,
    materialize,
    pairwise_dot,
)
from dattri_llm_b200.gradient.snapshots import TrajectorySnapshots
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager

__all__ = [
    "REGISTER_ALL",
    "AsyncGradientWriter",
    "CaptureCallback",
    "DataSelectionCallback",
    "Factorized",
    "FisherAccumulator",
    "Gradient",
    "GradientRecord",
    "GradientStorageManager",
    "HookManager",
    "HookManagerCallback",
    "HookManagerConfig",
    "KroneckerAccumulator",
    "KroneckerCovarianceCallback",
    "LayerFisherAccumulator",
    "LayerKroneckerAccumulator",
    "OffloadCallback",
    "OptimizerStateCallback",
    "ParameterSnapshotCallback",
    "TrajectorySnapshots",
    "canonical_class_name",
    "default_hook_assignment",
    "dot",
    "fim",
    "grad_norm_sq",
    "kfac",
    "materialize",
    "ops",
    "pairwise_dot",
    "register_linear_io_hooks",
    "register_linear_param_hooks",
    "register_param_grad_hooks",
    "remove_hooks",
]
