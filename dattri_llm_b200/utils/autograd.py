"""Scheduling work at the end of the in-flight backward pass.

Parity: reference ``dattri_llm/utils/autograd.py:331-379``.  Both helpers use the
autograd engine's final-callback queue, the one hook that runs after every
gradient of a backward -- including DDP's bucketed all-reduce write-back and
FSDP's reduce-scatter, which themselves queue final callbacks.
"""

from __future__ import annotations

from collections.abc import Callable

import torch


def queue_backward_end_callback(fn: Callable[[], None]) -> bool:
    """Run *fn* once the in-flight backward completes; ``False`` outside a backward."""
    try:
        torch.autograd.Variable._execution_engine.queue_callback(fn)
    except Exception:  # noqa: BLE001 - no backward in flight
        return False
    return True


def queue_after_backward_finalization(fn: Callable[[], None]) -> bool:
    """Run *fn* after everything else queued during the backward (e.g. DDP's
    write-back of averaged gradients), by re-queueing from the final callback."""

    def _requeue() -> None:
        if not queue_backward_end_callback(fn):
            fn()

    return queue_backward_end_callback(_requeue)
