"""Failure detection without a GPU fault.

GPU: a cross-GPU barrier whose peer never arrives (a flag nothing sets) gives up after
its bounded wait, records the timeout in the device error word, and the host raises on
the next check -- the context stays usable.  CPU (gloo): a rank that fails between steps
is seen by the others as a collective error within the process-group timeout."""

from __future__ import annotations

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@pytest.mark.gpu
def test_barrier_timeout_sets_error_word():
    from dattri_llm_b200 import ops

    dev = torch.device("cuda", 0)
    ops.check_device_errors(dev)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    # Both "ranks" map to this GPU's own array; slot 1 (the absent peer) is never written.
    ptrs = torch.tensor([flags.data_ptr(), flags.data_ptr()], dtype=torch.int64, device=dev)
    t0 = time.time()
    ops.native().peer_barrier(ptrs, 0, 2, 1, ops.error_word(dev))
    torch.cuda.synchronize(dev)
    assert time.time() - t0 < 30
    with pytest.raises(RuntimeError, match="error 4"):
        ops.check_device_errors(dev)
    # The context is still usable.
    x = torch.ones(4, device=dev)
    assert float((x * 2).sum()) == 8.0
    ops.check_device_errors(dev)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(2)
    dist.all_reduce(t)  # step 0 completes on every rank
    if rank == 1:
        out[rank] = "left"
        os._exit(0)  # leaves between steps, with nothing in flight
    try:
        dist.all_reduce(t)  # step 1: the peer is gone
        out[rank] = "completed"
    except Exception as e:  # noqa: BLE001
        out[rank] = type(e).__name__
    os._exit(0)


def test_lost_rank_surfaces_as_collective_error():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        res = dict(out)
    assert res.get(1) == "left"
    assert res.get(0) not in (None, "completed"), res

