"""The small end-to-end configuration on CPU: the GPT-2-style model of
:mod:`dattri_llm_b200.models` (2 layers, d 128, 4 heads, MLP 512, vocab 1024, seq 64,
random init, fp32), 256 train and 16 test sequences of uniform token ids, LoGra capture
with a 16×16 projection per block linear, GradDot (TracIn at one checkpoint) to a 16×256
score matrix.  Two gloo ranks under the streamer's DDP wrapping give the single-device
matrix; without projection, a corner of the matrix equals per-sample autograd; on a GPU
(marked ``gpu``) the native bf16 path gives the CPU fp32 matrix within bf16 error."""

from __future__ import annotations

import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

import dattri_llm_b200 as bw
from dattri_llm_b200.models import GPT2Config, GPT2LMHeadModel

N_TRAIN, N_TEST, SEQ, VOCAB = 256, 16, 64, 1024
LINEARS = [r"^h\.\d+\.(attn\.(q|k|v|o)_proj|fc_in|fc_out)$"]


def _model():
    torch.manual_seed(0)
    return GPT2LMHeadModel(GPT2Config()).eval()


def _data(n_train=N_TRAIN, n_test=N_TEST):
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, VOCAB, (n_train + n_test, SEQ), generator=g)
    return [{"input_ids": r} for r in ids[:n_train]], [{"input_ids": r} for r in ids[n_train:]]


def _loss(model, batch):
    ids = batch["input_ids"]
    logits = model(input_ids=ids).logits
    return F.cross_entropy(logits[:, :-1].reshape(-1, VOCAB), ids[:, 1:].reshape(-1), reduction="sum")


def _scores(project: bool = True, n_train=N_TRAIN, n_test=N_TEST):
    train, test = _data(n_train, n_test)
    proj = {"__default__": {"style": "logra", "proj_dim": 16}} if project else None
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=16,
                                   per_device_eval_batch_size=16)
    att = bw.TracInAttributor(args, task=bw.AttributionTask(_loss, _model()))
    score = att.attribute(train, test, hook_config=bw.HookManagerConfig(linear_io=LINEARS, projection_kwargs=proj))
    return {h: score.trajectory_agnostic(h) for h in score.train_ids}


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        out[rank] = _scores()
    except Exception as e:  # surfaced in the parent
        out[rank] = repr(e)
    finally:
        dist.destroy_process_group()


def test_ddp_two_ranks_equal_single_device():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    merged = {**res[0], **res[1]}
    want = _scores()
    assert len(want) == N_TRAIN and set(merged) == set(want)
    mat = torch.stack([want[h] for h in sorted(want)])
    assert mat.shape == (N_TRAIN, N_TEST)
    scale = float(mat.abs().max())
    for h, row in want.items():
        torch.testing.assert_close(merged[h], row, rtol=1e-4, atol=1e-5 * scale)


def test_unprojected_corner_matches_autograd():
    from dattri_llm_b200.utils.hashing import hash_sample

    n_train, n_test = 6, 3
    got = _scores(project=False, n_train=n_train, n_test=n_test)
    train, test = _data(n_train, n_test)
    model = _model()
    names = [n for n, m in model.named_modules() if isinstance(m, torch.nn.Linear) and n != "lm_head"]
    params = [p for n in names for p in model.get_submodule(n).parameters()]

    def flat(batch):
        gs = torch.autograd.grad(_loss(model, {"input_ids": batch["input_ids"][None]}), params)
        return torch.cat([g.reshape(-1) for g in gs])

    tr = torch.stack([flat(b) for b in train])
    te = torch.stack([flat(b) for b in test])
    want = tr @ te.T
    for i, b in enumerate(train):
        h = hash_sample({"input_ids": b["input_ids"]})
        torch.testing.assert_close(got[h], want[i], rtol=1e-4, atol=1e-5 * float(want.abs().max()))


def _scores_on(device: str, dtype: torch.dtype):
    train, test = _data()
    proj = {"__default__": {"style": "logra", "proj_dim": 16}}
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=16,
                                   per_device_eval_batch_size=16, use_cpu=device == "cpu")
    model = _model().to(device=device, dtype=dtype)
    att = bw.TracInAttributor(args, task=bw.AttributionTask(_loss, model))
    score = att.attribute(train, test, hook_config=bw.HookManagerConfig(linear_io=LINEARS, projection_kwargs=proj))
    return {h: score.trajectory_agnostic(h).float().cpu() for h in score.train_ids}


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_native_bf16_matrix_matches_cpu_fp32():
    """The same 16×256 matrix through the native capture and score kernels in bf16 on one
    GPU against the CPU fp32 run (identical counter-based projections on both)."""
    from dattri_llm_b200 import ops

    launches = ops.launch_count()
    got = _scores_on("cuda", torch.bfloat16)
    assert ops.launch_count() > launches, "the native kernels did not run"
    want = _scores_on("cpu", torch.float32)
    keys = sorted(want)
    a = torch.stack([got[h] for h in keys])
    b = torch.stack([want[h] for h in keys])
    assert float((a - b).norm() / b.norm()) < 5e-2
    assert float(torch.corrcoef(torch.stack([a.flatten(), b.flatten()]))[0, 1]) > 0.995
