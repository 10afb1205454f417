"""Peer-memory building blocks over NVLink 5 / NVSwitch (one process per GPU, one node).

Buffers live in PyTorch symmetric memory (``torch.distributed._symmetric_memory``),
which maps every rank's buffer into every other rank's address space.  The library's
own kernels then read peer memory directly -- TMA tile loads without cluster multicast,
or plain loads/stores -- and ranks meet at :class:`PeerBarrier`, a one-CTA kernel whose
wait is bounded (a lost peer sets the device error word instead of hanging the GPU).

:func:`available` says whether this path applies (NCCL process group, CUDA tensors on
sm_100, world size > 1, symmetric memory importable); callers fall back to
``torch.distributed`` collectives otherwise.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def available(device: torch.device | None = None) -> bool:
    """Whether peer-memory kernels can run for the default process group."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() < 2:
        return False
    if dist.get_backend() != "nccl" or not torch.cuda.is_available():
        return False
    import importlib.util

    if importlib.util.find_spec("torch.distributed._symmetric_memory") is None:
        return False
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    return torch.cuda.get_device_capability(dev)[0] == 10


def _group_name(group) -> str:
    group = group if group is not None else dist.group.WORLD
    return group.group_name


class SymmetricBuffer:
    """One tensor in symmetric memory plus every peer's view of it."""

    def __init__(self, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device, group=None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.local = symm_mem.empty(*shape, dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.local, _group_name(group))
        self.world = self.handle.world_size
        self.rank = self.handle.rank
        self.peers = [self.handle.get_buffer(r, tuple(shape), dtype) for r in range(self.world)]


class PeerBarrier:
    """Epoch barrier across the group's GPUs on peer-mapped int32 flags (bounded wait).

    ``wait()`` enqueues the barrier on the current stream: everything this rank enqueued
    before it is visible to peers once they pass it, and this rank's later work starts
    after every peer arrived.  Create it on every rank, collectively."""

    def __init__(self, device: torch.device, group=None) -> None:
        self._flags = SymmetricBuffer((_world(group),), torch.int32, device, group)
        self._flags.local.zero_()
        self._ptrs = torch.tensor([int(p.data_ptr()) for p in self._flags.peers], dtype=torch.int64, device=device)
        self._epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def wait(self) -> None:
        from dattri_llm_b200.ops import count_launch, error_word, native

        self._epoch += 1
        count_launch()
        native().peer_barrier(self._ptrs, self._flags.rank, self._flags.world, self._epoch,
                              error_word(self._ptrs.device))


def _world(group) -> int:
    return dist.get_world_size(group) if group is not None else dist.get_world_size()


_ONESHOT_BYTES = 1 << 20
_STAGING: dict = {}


class _Staging:
    """A growable symmetric fp32 staging buffer and its barrier, per device."""

    def __init__(self, device: torch.device, n: int) -> None:
        self.buf = SymmetricBuffer((n,), torch.float32, device)
        self.barrier = PeerBarrier(device)
        self.capacity = n


def _staging(device: torch.device, n: int) -> _Staging:
    st = _STAGING.get(device)
    if st is None or st.capacity < n:
        # Every rank reduces the same size, so every rank grows here together (collective).
        st = _Staging(device, max(n, 1 << 20, 2 * (st.capacity if st else 0)))
        _STAGING[device] = st
    return st


def all_reduce_sum_(t: torch.Tensor) -> bool:
    """In-place SUM of an fp32 CUDA tensor over the default group through NVLink peer
    memory; ``False`` when the path does not apply (the caller then uses
    ``dist.all_reduce``).  Up to 1 MiB one shot (every rank reads every peer's buffer);
    above, reduce-scatter + all-gather (each rank reduces its slice, then copies the
    others' from their owners).  Bounded barriers separate the phases."""
    if t.dtype != torch.float32 or not t.is_cuda or not available(t.device):
        return False
    world = dist.get_world_size()
    if world > 16:
        return False
    from dattri_llm_b200.ops import count_launch, native

    n = t.numel()
    n4 = (n + 3) // 4 * 4
    st = _staging(t.device, n4)
    local = st.buf.local
    local[:n].copy_(t.reshape(-1))
    if n4 > n:
        local[n:n4].zero_()
    rank = st.buf.rank
    out = torch.empty(n4, dtype=torch.float32, device=t.device)
    st.barrier.wait()
    if n4 * 4 <= _ONESHOT_BYTES:
        count_launch()
        native().allreduce_phase(st.buf.peers, out, n4, 0, rank)
    else:
        count_launch(2)
        native().allreduce_phase(st.buf.peers, local, n4, 1, rank)
        st.barrier.wait()
        native().allreduce_phase(st.buf.peers, out, n4, 2, rank)
    st.barrier.wait()  # no rank refills its staging buffer while a peer still reads it
    t.copy_(out[:n].view_as(t))
    return True
