"""Optimizer moments of hooked layers read through :class:`OptimizerSnapshot` when the
parameters are sharded (two gloo ranks on CPU): FSDP1 with ``use_orig_params=True`` (each
rank holds a slice of every flat parameter) and FSDP2 ``fully_shard`` (DTensor
parameters).  Both ranks train on the same batches, so the moments must equal those of an
unsharded model trained on that batch in one process."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

LAYERS = ["fc1", "fc2"]


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(6, 5)
        self.fc2 = nn.Linear(5, 3)

    def forward(self, x):
        return self.fc2(torch.tanh(self.fc1(x)))


def _batches():
    g = torch.Generator().manual_seed(4)
    return [torch.randn(4, 6, generator=g) for _ in range(3)]


def _train(model, opt):
    for x in _batches():
        opt.zero_grad()
        model(x).pow(2).sum().backward()
        opt.step()


def _reference_states():
    from dattri_llm_b200.gradient.optimizer_state import OptimizerSnapshot

    torch.manual_seed(0)
    model = Net()
    opt = torch.optim.AdamW(model.parameters(), lr=0.01)
    _train(model, opt)
    snap = OptimizerSnapshot(model, opt)
    return {layer: {k: v for k, v in snap.states(layer).items() if v is not None} for layer in LAYERS}


def _worker(rank, world, port, kind, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from dattri_llm_b200.gradient.optimizer_state import OptimizerSnapshot

        torch.manual_seed(0)
        model = Net()
        if kind == "fsdp1":
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

            wrapped = FSDP(model, use_orig_params=True, device_id=torch.device("cpu"))
            opt = torch.optim.AdamW(wrapped.parameters(), lr=0.01)
            snap = OptimizerSnapshot(wrapped, opt)
            # FSDP1 slices are discovered while the layer's parameters are unsharded: bind
            # from inside each layer's backward (as the capture hooks do)
            for layer in LAYERS:
                model.get_submodule(layer).register_full_backward_hook(
                    lambda _m, _gi, _go, layer=layer: snap.bind(layer))
            _train(wrapped, opt)
        else:
            from torch.distributed.device_mesh import init_device_mesh
            from torch.distributed.fsdp import fully_shard

            mesh = init_device_mesh("cpu", (world,))
            fully_shard(model.fc1, mesh=mesh)
            fully_shard(model.fc2, mesh=mesh)
            fully_shard(model, mesh=mesh)
            opt = torch.optim.AdamW(model.parameters(), lr=0.01)
            _train(model, opt)
            snap = OptimizerSnapshot(model, opt)
        out[rank] = {layer: {k: v for k, v in snap.states(layer).items() if v is not None} for layer in LAYERS}
    except Exception as e:  # reported to the parent (FSDP2 on CPU may be unavailable)
        out[rank] = repr(e)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["fsdp1", "fsdp2"])
def test_sharded_moments_equal_unsharded(kind):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, kind, out), nprocs=2, join=True)
        res = dict(out)
    want = _reference_states()
    for rank in range(2):
        got = res[rank]
        assert not isinstance(got, str), got
        for layer in LAYERS:
            assert set(got[layer]) == set(want[layer]), (layer, sorted(got[layer]), sorted(want[layer]))
            for k, v in want[layer].items():
                torch.testing.assert_close(got[layer][k], v, rtol=1e-5, atol=1e-7, msg=f"{layer}.{k}")
