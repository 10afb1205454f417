"""The streamer's own data-parallel wrapping (two gloo ranks on CPU): with ``args.fsdp``
set (full shard, with a class-based or size-based auto-wrap policy) or unset (DDP), live
TracIn over the rank shards gives the single-process scores; the auto-wrap policy is built
from ``fsdp_config`` and rejects conflicting or unknown options."""

from __future__ import annotations

import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from dattri_llm_b200.gradient.streaming import _auto_wrap_policy
from tests import tiny


def _scores(fsdp, fsdp_config):
    import dattri_llm_b200 as bw

    x, y, xt, yt = tiny.make_data(seed=12, n_train=10, n_test=3)
    model = tiny.make_model(seed=13)
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=2,
                                   per_device_eval_batch_size=3, fsdp=fsdp, fsdp_config=fsdp_config)
    att = bw.TracInAttributor(args, task=bw.AttributionTask(tiny.sq_loss, model))
    score = att.attribute(tiny.as_dataset(x, y), tiny.as_dataset(xt, yt),
                          hook_config=bw.HookManagerConfig(linear_io=tiny.LAYERS))
    return {h: score.trajectory_agnostic(h) for h in score.train_ids}


def _worker(rank, world, port, fsdp, fsdp_config, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        out[rank] = _scores(fsdp, fsdp_config)
    except Exception as e:  # surfaced in the parent
        out[rank] = repr(e)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize(("fsdp", "fsdp_config"), [
    ("", None),
    ("full_shard", {"min_num_params": 1}),
    ("full_shard", {"transformer_layer_cls_to_wrap": ["Linear"]}),
])
def test_wrapped_live_scores_equal_single_process(fsdp, fsdp_config):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, fsdp, fsdp_config, out), nprocs=2, join=True)
        res = dict(out)
    want = _scores("", None)
    merged = {}
    for rank in range(2):
        assert not isinstance(res[rank], str), res[rank]
        merged.update(res[rank])
    assert set(merged) == set(want)
    for h, row in want.items():
        torch.testing.assert_close(merged[h], row, rtol=1e-5, atol=1e-6)


def test_auto_wrap_policy_options():
    model = nn.Sequential(nn.Linear(3, 4), nn.ReLU(), nn.Linear(4, 2))
    assert _auto_wrap_policy(model, {}) is None
    assert _auto_wrap_policy(model, {"auto_wrap_policy": object()}) is None
    assert _auto_wrap_policy(model, {"min_num_params": 10}) is not None
    assert _auto_wrap_policy(model, {"transformer_layer_cls_to_wrap": "Linear"}) is not None
    with pytest.raises(ValueError, match="not both"):
        _auto_wrap_policy(model, {"min_num_params": 10, "transformer_layer_cls_to_wrap": "Linear"})
    with pytest.raises(ValueError, match="no module of class"):
        _auto_wrap_policy(model, {"transformer_layer_cls_to_wrap": ["Conv2d"]})
