"""Data selection on one process (CPU) against per-sample autograd: the ``val_loader``
target (a secondary backward through the same hooks, with the manager's state and the
training gradients restored around it), the ``fixed`` target, the selection rules
(``hard``, ``bottom_fraction``, ``negative_bottom_fraction``, per-layer), and the
renormalized removal.  The training step's own record is untouched by the val pass;
as in the reference, sibling callbacks also observe the val pass's record (one extra,
smaller record per secondary backward)."""

from __future__ import annotations

import pytest
import torch

import dattri_llm_b200 as bw
from dattri_llm_b200.gradient.callbacks import DataSelectionCallback
from tests import tiny

N = 6


def _data(seed=0):
    x, y, xv, yv = tiny.make_data(seed=seed, n_train=N, n_test=2)
    return x, y, xv, yv


def _split(flat: torch.Tensor) -> dict[str, torch.Tensor]:
    """A flat per-sample gradient over tiny.WEIGHTS as ``{layer: (n, out*in)}``."""
    model = tiny.make_model()
    out, at = {}, 0
    for layer, w in zip(tiny.LAYERS, tiny.WEIGHTS, strict=True):
        size = dict(model.named_parameters())[w].numel()
        out[layer] = flat[:, at:at + size]
        at += size
    return out


def _val_loss(model, batch):
    return tiny.sq_loss(model, batch)


class _AllRecords(bw.CaptureCallback):
    """Keeps every record the manager dispatches."""

    def __init__(self) -> None:
        super().__init__()
        self.records = []

    def on_step_end(self, record) -> None:
        super().on_step_end(record)
        self.records.append(record)


def _run(cb, x, y, *, steps=1):
    """Records the sibling callback saw: the training steps' and the val passes'."""
    model = cb._root
    cap = _AllRecords()
    hm = bw.HookManager(model, bw.HookManagerConfig(linear_io=tiny.LAYERS), callbacks=[cap, cb])
    for _ in range(steps):
        model.zero_grad(set_to_none=True)
        with hm.collect():
            tiny.sq_loss(model, {"x": x, "y": y}).backward()
    hm.remove()
    return cap.records


def test_val_loader_target_scores_and_removal():
    x, y, xv, yv = _data()
    model = tiny.make_model(seed=1)
    per = tiny.per_sample_grads(model, x, y)  # (N, p)
    val = tiny.per_sample_grads(model, xv, yv).sum(0)  # the val batch's gradient
    want_scores = per @ val
    cb = DataSelectionCallback(model, target="val_loader", val_loader=[{"x": xv, "y": yv}], val_loss_fn=_val_loss)
    records = _run(cb, x, y)
    assert [r.gradient.batch_size for r in records] == [N, 2]  # the train step, then the val pass
    rec = records[0]
    torch.testing.assert_close(cb.last_scores.double(), want_scores.double(), rtol=1e-5, atol=1e-6)
    dropped = (want_scores < 0).nonzero().flatten().tolist()
    assert cb.last_dropped == dropped and 0 < len(dropped) < N
    keep = [i for i in range(N) if i not in dropped]
    grads = _split(per[keep].sum(0, keepdim=True))
    for layer, w in zip(tiny.LAYERS, tiny.WEIGHTS, strict=True):
        got = dict(model.named_parameters())[w].grad.reshape(1, -1)
        torch.testing.assert_close(got, grads[layer], rtol=1e-5, atol=1e-6)
    # the training step's record is the train batch, not the val pass
    assert rec.gradient.batch_size == N
    cat = torch.cat([rec.gradient.materialize().data[n].reshape(N, -1) for n in tiny.LAYERS], 1)
    torch.testing.assert_close(cat, per, rtol=1e-5, atol=1e-6)


def test_val_loader_cycles_over_steps():
    x, y, xv, yv = _data(seed=2)
    model = tiny.make_model(seed=3)
    batches = [{"x": xv[:1], "y": yv[:1]}, {"x": xv[1:], "y": yv[1:]}]
    cb = DataSelectionCallback(model, target="val_loader", val_loader=batches, val_loss_fn=_val_loss,
                               selection_kwargs={"threshold": -1e30})
    per = tiny.per_sample_grads(model, x, y)
    seen = []
    cap = _AllRecords()
    hm = bw.HookManager(model, bw.HookManagerConfig(linear_io=tiny.LAYERS), callbacks=[cap, cb])
    for _ in range(3):  # the loader restarts after two targets
        model.zero_grad(set_to_none=True)
        with hm.collect():
            tiny.sq_loss(model, {"x": x, "y": y}).backward()
        seen.append(cb.last_scores.clone())
    hm.remove()
    assert [r.gradient.batch_size for r in cap.records] == [N, 1] * 3
    assert [r.step for r in cap.records[::2]] == sorted({r.step for r in cap.records[::2]})  # train steps advance
    for k, batch in enumerate([batches[0], batches[1], batches[0]]):
        v = tiny.per_sample_grads(model, batch["x"], batch["y"]).sum(0)
        torch.testing.assert_close(seen[k].double(), (per @ v).double(), rtol=1e-5, atol=1e-6)


def test_fixed_target_equals_val_target():
    x, y, xv, yv = _data(seed=4)
    model = tiny.make_model(seed=5)
    cap = bw.CaptureCallback()
    hm = bw.HookManager(model, bw.HookManagerConfig(linear_io=tiny.LAYERS), callbacks=[cap])
    with hm.collect():
        tiny.sq_loss(model, {"x": xv, "y": yv}).backward()
    hm.remove()
    model.zero_grad(set_to_none=True)
    target = cap.record.gradient
    cb = DataSelectionCallback(model, target="fixed", target_gradient=target,
                               selection_kwargs={"threshold": -1e30})
    _run(cb, x, y)
    want = tiny.per_sample_grads(model, x, y) @ tiny.per_sample_grads(model, xv, yv).sum(0)
    torch.testing.assert_close(cb.last_scores.double(), want.double(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("mode", ["bottom_fraction", "negative_bottom_fraction"])
def test_fraction_rules(mode):
    scores = torch.tensor([0.5, -2.0, 3.0, -0.1, 1.0, -0.5])
    kw = {"threshold": 0.5, "threshold_mode": mode}
    got = DataSelectionCallback.select_samples(scores, selection_kwargs=kw)
    assert got == [1, 5, 3]  # the lowest round(6 * 0.5) = 3, all negative here
    scores2 = torch.tensor([0.5, -2.0, 3.0, 0.1, 1.0, 0.2])
    got2 = DataSelectionCallback.select_samples(scores2, selection_kwargs=kw)
    assert got2 == ([1, 3, 5] if mode == "bottom_fraction" else [1])
    with pytest.raises(ValueError):
        DataSelectionCallback(tiny.make_model(), selection_kwargs={"threshold": 1.5, "threshold_mode": mode})


def test_layer_wise_selection_and_renormalized_removal():
    x, y, _, _ = _data(seed=6)
    model = tiny.make_model(seed=7)
    per = _split(tiny.per_sample_grads(model, x, y))
    cb = DataSelectionCallback(model, target="batch", renormalize=True,
                               selection_kwargs={"threshold": 0.0, "layer_wise": True})
    _run(cb, x, y)
    params = dict(model.named_parameters())
    dropped_any = False
    for layer, w in zip(tiny.LAYERS, tiny.WEIGHTS, strict=True):
        g = per[layer]
        scores = g @ g.sum(0)  # this layer's alignment with the batch gradient
        drop = (scores < 0).nonzero().flatten().tolist()
        keep = [i for i in range(N) if i not in drop]
        dropped_any |= bool(drop)
        want = g[keep].sum(0) * (N / len(keep))  # kept samples rescaled to the batch's scale
        torch.testing.assert_close(params[w].grad.reshape(-1), want, rtol=1e-5, atol=1e-6, msg=layer)
    assert dropped_any
