"""Host-side multi-process logic on CPU (gloo, world size 2)."""

from __future__ import annotations

import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world: int = 2, *args):
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_entry, args=(world, port, fn, out, args), nprocs=world, join=True)
        return dict(out)


def _entry(rank, world, port, fn, out, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        out[rank] = fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def _symm_unavailable_on_gloo(rank, world):
    from dattri_llm_b200.parallel import symm

    return symm.available()


def test_peer_path_is_off_under_gloo():
    res = _run(_symm_unavailable_on_gloo)
    assert res == {0: False, 1: False}


def _all_reduce(rank, world):
    from dattri_llm_b200.utils.distributed import all_reduce_sum

    t = torch.full((3,), float(rank + 1))
    return all_reduce_sum(t).tolist()


def test_all_reduce_sum_gloo():
    res = _run(_all_reduce)
    assert res[0] == res[1] == [3.0, 3.0, 3.0]
