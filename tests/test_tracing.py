"""Tracing utilities (CPU): NVTX ranges are off by default and balanced when on, the
device timer accumulates and reports the MAX over gloo ranks, the metrics logger writes
JSON lines on rank 0 only, and the instrumented phases (stream batch, capture step, store
write, score block) open their ranges during a live attribution."""

from __future__ import annotations

import datetime
import json
import os
import socket
import tempfile
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dattri_llm_b200.utils import tracing
from dattri_llm_b200.utils.tracing import DeviceTimer, MetricsLogger, set_tracing, throughput_row, trace_range
from tests import tiny


@pytest.fixture
def nvtx_log(monkeypatch):
    """Record NVTX pushes/pops as if CUDA were present."""
    events = []
    monkeypatch.setattr(tracing, "_nvtx_available", lambda: True)
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: events.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: events.append(("pop", None)))
    yield events
    set_tracing(False)


def test_off_by_default_emits_nothing(nvtx_log, monkeypatch):
    monkeypatch.delenv("DATTRI_B200_NVTX", raising=False)
    monkeypatch.setattr(tracing, "_enabled", None)
    assert not tracing.tracing_enabled()
    with trace_range("x"):
        pass
    assert nvtx_log == []


def test_env_turns_tracing_on(monkeypatch):
    monkeypatch.setenv("DATTRI_B200_NVTX", "1")
    monkeypatch.setattr(tracing, "_enabled", None)
    assert tracing.tracing_enabled()
    set_tracing(False)


def test_ranges_stay_balanced_on_error(nvtx_log):
    set_tracing(True)
    with pytest.raises(RuntimeError), trace_range("outer"):
        with trace_range("inner"):
            raise RuntimeError("boom")
    assert nvtx_log == [("push", "outer"), ("push", "inner"), ("pop", None), ("pop", None)]


def test_host_timer_accumulates():
    t = DeviceTimer("cpu")
    for _ in range(2):
        with t:
            time.sleep(0.01)
    assert t.elapsed_ms() >= 20.0
    t.reset()
    assert t.elapsed_ms() == 0.0


def _timer_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        t = DeviceTimer("cpu")
        t._host_ms = 10.0 * (rank + 1)  # a known per-rank time
        out[rank] = t.elapsed_ms()
        log = MetricsLogger(os.path.join(out["dir"], "m.jsonl"))
        log.log(rank=rank, value=torch.tensor([1.5, 2.0]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_timer_max_over_ranks_and_rank0_logger():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    d = tempfile.mkdtemp()
    with mp.Manager() as m:
        out = m.dict()
        out["dir"] = d
        mp.spawn(_timer_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    assert res[0] == res[1] == 20.0
    rows = [json.loads(x) for x in open(os.path.join(d, "m.jsonl"))]
    assert len(rows) == 1 and rows[0]["rank"] == 0 and rows[0]["world_size"] == 2
    assert rows[0]["value"] == [1.5, 2.0]


def test_throughput_row_fraction():
    row = throughput_row("score", 1000, 500.0, unit="samples/s", peak=4000.0, n_gpus=1)
    assert row["value"] == 2000.0 and row["fraction_of_peak"] == 0.5 and row["n_gpus"] == 1
    log = MetricsLogger(os.path.join(tempfile.mkdtemp(), "sub", "x.jsonl"))
    log.log(**row)
    assert log.read()[0]["name"] == "score"


def test_pipeline_phases_open_ranges(nvtx_log, tmp_path):
    import dattri_llm_b200 as bw

    set_tracing(True)
    x, y, xt, yt = tiny.make_data(seed=12, n_train=6, n_test=2)
    model = tiny.make_model(seed=13)
    args = bw.AttributionArguments(output_dir=str(tmp_path), per_device_train_batch_size=3,
                                   per_device_eval_batch_size=2)
    att = bw.TracInAttributor(args, task=bw.AttributionTask(tiny.sq_loss, model))
    att.attribute(tiny.as_dataset(x, y), tiny.as_dataset(xt, yt), hook_config=bw.HookManagerConfig(linear_io=tiny.LAYERS),
                  gradient_cache_residency="disk")
    names = [n for k, n in nvtx_log if k == "push"]
    assert sum(1 for n in names if n.startswith("dattri.stream.batch[")) >= 2
    assert sum(1 for n in names if n.startswith("dattri.capture.step[")) >= 2
    assert "dattri.score.block" in names
    assert "dattri.store.write" in names
    assert sum(1 for k, _ in nvtx_log if k == "push") == sum(1 for k, _ in nvtx_log if k == "pop")


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_device_timer_and_nvtx_on_gpu():
    """CUDA-event timing of queued work (no profiler attached: the NVTX calls are no-ops
    that must still balance)."""
    a = torch.randn(4096, 4096, device="cuda")
    timer = DeviceTimer()
    assert timer.device.type == "cuda"
    set_tracing(True)
    try:
        with trace_range("gpu.matmul"), timer:
            for _ in range(4):
                a = a @ a / 64.0
    finally:
        set_tracing(False)
    ms = timer.elapsed_ms()
    assert 0.0 < ms < 10_000.0
    row = throughput_row("matmul", 4 * 2 * 4096**3, ms, unit="flop/s")
    assert row["value"] > 0
