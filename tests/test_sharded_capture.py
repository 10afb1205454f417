"""Per-sample capture through data-parallel wrappers (two gloo ranks on CPU): under DDP,
FSDP1 (full shard, ``use_orig_params``) and FSDP2 (``fully_shard``) the hooks sit on the
unwrapped layers and see full activations and output gradients, so each rank's captured
per-sample gradients equal those of the unsharded model on that rank's batch."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

B, T, D = 3, 4, 6
LAYERS = ["blk.fc1", "blk.fc2", "head"]


class Block(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(D, 8)
        self.fc2 = nn.Linear(8, D)

    def forward(self, x):
        return x + self.fc2(torch.relu(self.fc1(x)))


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.blk = Block()
        self.head = nn.Linear(D, 1)

    def forward(self, x):
        return self.head(self.blk(x)).sum(dim=(1, 2))


def _batch(rank):
    return torch.randn(B, T, D, generator=torch.Generator().manual_seed(100 + rank))


def _oracle(x):
    """Per-sample ``[dW | db]`` of every layer, one sample at a time."""
    torch.manual_seed(0)
    model = Net()
    out = {n: [] for n in LAYERS}
    for i in range(x.shape[0]):
        model.zero_grad()
        model(x[i : i + 1]).sum().backward()
        for n in LAYERS:
            m = model.get_submodule(n)
            out[n].append(torch.cat([m.weight.grad, m.bias.grad[:, None]], 1).reshape(-1))
    return {n: torch.stack(v) for n, v in out.items()}


def _worker(rank, world, port, kind, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from dattri_llm_b200.gradient.callbacks import CaptureCallback
        from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig

        torch.manual_seed(0)
        model = Net()
        if kind == "ddp":
            wrapped = nn.parallel.DistributedDataParallel(model)
        elif kind == "fsdp1":
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

            wrapped = FSDP(model, use_orig_params=True, device_id=torch.device("cpu"))
        else:
            from torch.distributed.device_mesh import init_device_mesh
            from torch.distributed.fsdp import fully_shard

            mesh = init_device_mesh("cpu", (world,))
            for m in (model.blk.fc1, model.blk.fc2, model.head):
                fully_shard(m, mesh=mesh)
            wrapped = fully_shard(model, mesh=mesh)
        cap = CaptureCallback()
        hm = HookManager(wrapped, HookManagerConfig(linear_io=[r"^(blk\.fc[12]|head)$"]), callbacks=[cap])
        x = _batch(rank)
        with hm.collect():
            wrapped(x).sum().backward()
        dense = cap.record.gradient.materialize()
        out[rank] = {n: dense.data[n].reshape(B, -1).clone() for n in LAYERS}
    except Exception as e:  # surfaced in the parent
        out[rank] = repr(e)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["ddp", "fsdp1", "fsdp2"])
def test_captured_per_sample_grads_equal_unsharded(kind):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, kind, out), nprocs=2, join=True)
        res = dict(out)
    for rank in range(2):
        got = res[rank]
        assert not isinstance(got, str), got
        want = _oracle(_batch(rank))
        for n in LAYERS:
            torch.testing.assert_close(got[n], want[n], rtol=1e-5, atol=1e-6, msg=f"{kind} rank {rank} {n}")
