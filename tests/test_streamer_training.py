"""The training side of :class:`GradientStreamer` (a trajectory, ``enable_update=True``)
against an independent hand-written loop: the same shuffled batches, AdamW with the
decay / no-decay parameter groups, transformers' linear warm-up schedule, loss scaled by
the accumulation factor, global-norm clipping once per update and an update at every
window end including a ragged tail.  Final parameters must match, and every captured
step must hold the per-sample gradients at the parameters of that micro-step."""

from __future__ import annotations

import copy
import tempfile

import pytest
import torch
from torch.utils.data import DataLoader

import dattri_llm_b200 as bw
from tests import tiny

N, BATCH, LR, SEED = 11, 2, 0.05, 5


def _dataset():
    x, y, _, _ = tiny.make_data(seed=7, n_train=N)
    return tiny.as_dataset(x, y)


def _reference_run(model, ds, accum, clip):
    from transformers import get_scheduler

    decay = [p for n, p in model.named_parameters() if p.ndim >= 2 and not n.endswith(".bias")]
    rest = [p for n, p in model.named_parameters() if not (p.ndim >= 2 and not n.endswith(".bias"))]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.01}, {"params": rest, "weight_decay": 0.0}], lr=LR)
    loader = DataLoader(ds, batch_size=BATCH, shuffle=True, generator=torch.Generator().manual_seed(SEED))
    updates = -(-len(loader) // accum)
    sched = get_scheduler("linear", opt, num_warmup_steps=1, num_training_steps=updates)
    snapshots = []
    opt.zero_grad()
    for i, batch in enumerate(loader):
        snapshots.append((copy.deepcopy(model.state_dict()), batch))
        (tiny.sq_loss(model, batch) / accum).backward()
        if (i + 1) % accum == 0 or i + 1 == len(loader):
            if clip is not None:
                torch.nn.utils.clip_grad_norm_(model.parameters(), clip)
            opt.step()
            sched.step()
            opt.zero_grad()
    return snapshots


@pytest.mark.parametrize("accum", [1, 3])
@pytest.mark.parametrize("clip", [None, 0.3])
def test_trajectory_matches_hand_written_loop(accum, clip):
    ds = _dataset()
    ref_model = tiny.make_model(seed=1).train()
    snaps = _reference_run(ref_model, ds, accum, clip)

    model = tiny.make_model(seed=1).train()
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), learning_rate=LR, weight_decay=0.01,
                                   optim="adamw_torch", lr_scheduler_type="linear", warmup_steps=1,
                                   gradient_accumulation_steps=accum, max_grad_norm=clip, seed=SEED,
                                   per_device_train_batch_size=BATCH)
    cfg = bw.HookManagerConfig(linear_io=[r"^mlp\.fc[12]$"])
    streamer = bw.GradientStreamer(model, ds, args, batch_size=BATCH, enable_update=True, loss_fn=tiny.sq_loss,
                                   config=cfg)
    steps = 0
    with streamer:
        for i, (_step, grad, _hashes) in enumerate(streamer):
            state, batch = snaps[i]
            oracle_model = tiny.make_model()
            oracle_model.load_state_dict(state)
            want = tiny.per_sample_grads(oracle_model, batch["x"], batch["y"]) / accum
            got = torch.cat([grad.materialize().data[n].reshape(want.shape[0], -1) for n in tiny.LAYERS], 1)
            torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
            steps += 1
    assert steps == len(snaps) == -(-N // BATCH)
    for (name, p), (_, q) in zip(model.named_parameters(), ref_model.named_parameters(), strict=True):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6, msg=name)


def test_frozen_probe_leaves_parameters_and_grads_alone():
    ds = _dataset()
    model = tiny.make_model(seed=2)
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=BATCH)
    streamer = bw.GradientStreamer(model, ds, args, batch_size=BATCH, loss_fn=tiny.sq_loss,
                                   config=bw.HookManagerConfig(linear_io=[r"^mlp\.fc[12]$"]))
    with streamer:
        n = sum(1 for _ in streamer)
    assert n == -(-N // BATCH)
    for name, p in model.named_parameters():
        torch.testing.assert_close(p, before[name], msg=name)
        assert p.grad is None


def test_sample_hashes_come_from_host_copies(monkeypatch):
    """When the model is fed fields of the batch under other names too (``labels=input_ids``),
    the step's content hash is still computed from the host copies of the moved tensors
    (no device read-back), and equals the hash of the model's inputs."""
    import dattri_llm_b200.gradient.hooks.manager as manager
    import dattri_llm_b200.gradient.streaming as streaming
    from dattri_llm_b200.utils.hashing import hash_batch

    moved = []

    def fake_move(batch, device, non_blocking=False):  # a "device" copy distinct from the host batch
        out = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in batch.items()}
        moved.append((batch, out))
        return out

    seen = []
    real_hash = manager.hash_batch

    def spy(inputs, b):
        seen.append(inputs)
        return real_hash(inputs, b)

    monkeypatch.setattr(streaming, "move_batch", fake_move)
    monkeypatch.setattr(manager, "hash_batch", spy)
    ds = _dataset()

    class Alias(torch.nn.Module):  # the model also takes y under a second name
        def __init__(self):
            super().__init__()
            self.inner = tiny.make_model(seed=2)

        def forward(self, x, y, labels):
            return self.inner(x=x, y=y)

    model = Alias()

    def loss(m, batch):
        return ((m(x=batch["x"], y=batch["y"], labels=batch["y"]) - batch["y"]) ** 2).sum()

    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=BATCH)
    streamer = bw.GradientStreamer(model, ds, args, batch_size=BATCH, loss_fn=loss,
                                   config=bw.HookManagerConfig(linear_io=[r"^inner\.mlp\.fc[12]$"]))
    with streamer:
        got = [hashes for _, _, hashes in streamer]
    assert streamer.host_hash_trusted is False  # the host batch's hash is not the model inputs' hash
    assert len(seen) == len(moved), "every step is hashed by the manager"
    host_ids = {id(t) for host, _ in moved for t in host.values()}
    for inputs in seen:
        assert all(id(v) in host_ids for v in inputs.values() if isinstance(v, torch.Tensor))
    want = [hash_batch({"x": host["x"], "y": host["y"], "labels": host["y"]}, host["x"].shape[0])
            for host, _ in moved]
    assert got == want
