"""Guarded ``torch.distributed`` probes and the generic cross-rank reductions.

Parity: reference ``dattri_llm/utils/distributed.py:248-310`` (probes and the
SUM all-reduce).  Added here: a MAX reduction used for device-timed benchmarks
(max over ranks), and a barrier that is a no-op outside a process group.
"""

from __future__ import annotations

import torch


def is_dist_initialized() -> bool:
    """``True`` when a ``torch.distributed`` process group is active."""
    try:
        import torch.distributed as dist

        return dist.is_available() and dist.is_initialized()
    except Exception:  # noqa: BLE001 - the probe must never raise
        return False


def dist_rank() -> int | None:
    """The current rank, or ``None`` outside a distributed context."""
    if is_dist_initialized():
        import torch.distributed as dist

        return dist.get_rank()
    return None


def dist_world_size() -> int:
    """The process-group size, or ``1`` outside a distributed context."""
    if is_dist_initialized():
        import torch.distributed as dist

        return dist.get_world_size()
    return 1


def _collective_device() -> torch.device:
    import torch.distributed as dist

    if "nccl" in str(dist.get_backend()).lower():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def all_reduce_sum(tensor: torch.Tensor) -> torch.Tensor:
    """Sum *tensor* over ranks in place (moved to the backend's device if needed)."""
    return _all_reduce(tensor, "sum")


def all_reduce_max(tensor: torch.Tensor) -> torch.Tensor:
    """Elementwise max of *tensor* over ranks, in place."""
    return _all_reduce(tensor, "max")


def _all_reduce(tensor: torch.Tensor, op: str) -> torch.Tensor:
    if dist_world_size() == 1:
        return tensor
    import torch.distributed as dist

    buf = tensor.to(_collective_device())
    dist.all_reduce(buf, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX)
    if buf is not tensor:
        tensor.copy_(buf)
    return tensor


def barrier() -> None:
    """``dist.barrier()`` inside a process group, else nothing."""
    if dist_world_size() > 1:
        import torch.distributed as dist

        dist.barrier()
