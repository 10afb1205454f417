"""DataSelectionCallback under DDP and FSDP (two gloo ranks on CPU).

After the callback drops samples, the gradients the optimizer would see must equal
the averaged gradient of the surviving samples only: ``(1/W) sum_r G_r^kept``.  For
FSDP the sharded gradients are gathered with ``summon_full_params(with_grads=True)``.
Modes: nothing dropped (a no-op that must not deadlock), the bottom half of every rank
dropped, and a hard threshold at 0 (drop counts differ per rank)."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from dattri_llm_b200.gradient.callbacks import DataSelectionCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig

VOCAB, EMB, HID, SEQ, BATCH = 32, 8, 16, 5, 6


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.emb = nn.Embedding(VOCAB, EMB)
        self.fc1 = nn.Linear(EMB, HID)
        self.fc2 = nn.Linear(HID, 1)

    def forward(self, ids):
        return self.fc2(torch.tanh(self.fc1(self.emb(ids)))).sum(dim=(1, 2))


def _kwargs(mode: str) -> dict:
    if mode == "none":
        return {"selection_kwargs": {"threshold_mode": "hard", "threshold": -1e30}}
    if mode == "half":
        return {"selection_kwargs": {"threshold_mode": "bottom_fraction", "threshold": 0.5}}
    return {"selection_kwargs": {"threshold_mode": "hard", "threshold": 0.0}}


def _grads(model: nn.Module) -> dict[str, torch.Tensor]:
    return {n: (p.grad if p.grad is not None else torch.zeros_like(p)).detach().clone().float()
            for n, p in model.named_parameters() if n.startswith(("fc1", "fc2"))}


def _worker(rank, world, port, wrap, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        model = Net()
        init = {k: v.clone() for k, v in model.state_dict().items()}
        ids = torch.randint(0, VOCAB, (BATCH, SEQ), generator=torch.Generator().manual_seed(100 + rank))
        hm = HookManager(model, config=HookManagerConfig(linear_io=[r"^fc[12]$"]))
        if wrap == "ddp":
            wrapped = nn.parallel.DistributedDataParallel(model)
        else:
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
            from torch.distributed.fsdp import ShardingStrategy

            wrapped = FSDP(model, device_id=torch.device("cpu"), sharding_strategy=ShardingStrategy.FULL_SHARD,
                           use_orig_params=True)
        cb = DataSelectionCallback(model=wrapped, target="batch", scoring_kwargs={"score_mode": "ghost"},
                                   **_kwargs(mode))
        hm.add_callback(cb)
        wrapped.zero_grad()
        with hm.collect():
            wrapped(ids).sum().backward()
        dropped = list(cb.last_dropped)
        if wrap == "ddp":
            got = _grads(model)
        else:
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

            with FSDP.summon_full_params(wrapped, with_grads=True):
                got = _grads(model)
        ref = Net()
        ref.load_state_dict(init)
        keep = [i for i in range(BATCH) if i not in set(dropped)]
        if keep:
            ref(ids[keep]).sum().backward()
        want = _grads(ref)
        for t in want.values():
            dist.all_reduce(t)
            t /= world
        err = max(float((got[n] - want[n]).abs().max()) for n in want)
        scale = max(float(want[n].abs().max()) for n in want) or 1.0
        out[rank] = (len(dropped), err / scale)
    finally:
        dist.destroy_process_group()


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("wrap", ["ddp", "fsdp"])
@pytest.mark.parametrize("mode", ["none", "half", "hard0"])
def test_corrected_gradients_equal_surviving_samples(wrap, mode):
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, _port(), wrap, mode, out), nprocs=2, join=True)
        res = dict(out)
    assert len(res) == 2
    for n_dropped, err in res.values():
        assert err < 1e-4, res
        if mode == "none":
            assert n_dropped == 0
        if mode == "half":
            assert n_dropped == BATCH // 2
