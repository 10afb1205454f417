"""Callbacks that act on each captured step."""

from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.callbacks.capture_callback import CaptureCallback
from dattri_llm_b200.gradient.callbacks.data_selection_callback import DataSelectionCallback
from dattri_llm_b200.gradient.callbacks.kronecker_covariance_callback import KroneckerCovarianceCallback
from dattri_llm_b200.gradient.callbacks.offload_callback import OffloadCallback
from dattri_llm_b200.gradient.callbacks.optimizer_state_callback import OptimizerStateCallback
from dattri_llm_b200.gradient.callbacks.parameter_snapshot_callback import ParameterSnapshotCallback

__all__ = [
    "CaptureCallback",
    "DataSelectionCallback",
    "HookManagerCallback",
    "KroneckerCovarianceCallback",
    "OffloadCallback",
    "OptimizerStateCallback",
    "ParameterSnapshotCallback",
]
