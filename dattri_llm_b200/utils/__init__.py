"""Utilities: content hashing, distributed and autograd helpers, the tensor cache, tracing."""

from dattri_llm_b200.utils.autograd import (
    queue_after_backward_finalization,
    queue_backward_end_callback,
)
from dattri_llm_b200.utils.cache import CACHE_RESIDENCIES, CacheBudget, TensorCache, tensor_nbytes
from dattri_llm_b200.utils.distributed import dist_rank, dist_world_size, is_dist_initialized
from dattri_llm_b200.utils.hashing import hash_batch, hash_sample
from dattri_llm_b200.utils.tracing import (
    DeviceTimer,
    MetricsLogger,
    set_tracing,
    throughput_row,
    trace_range,
    tracing_enabled,
)

__all__ = [
    "CACHE_RESIDENCIES",
    "CacheBudget",
    "DeviceTimer",
    "MetricsLogger",
    "TensorCache",
    "dist_rank",
    "dist_world_size",
    "hash_batch",
    "hash_sample",
    "is_dist_initialized",
    "queue_after_backward_finalization",
    "queue_backward_end_callback",
    "set_tracing",
    "tensor_nbytes",
    "throughput_row",
    "trace_range",
    "tracing_enabled",
]
