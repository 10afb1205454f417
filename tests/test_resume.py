"""Resuming an interrupted gradient collection (CPU): a run that stopped mid-store and is
restarted with ``resume=True`` skips the batches it already stored (checked against the
stored hashes) and ends with the same stores and scores as an uninterrupted run; a group
whose index line was cut off is redone; a changed loader order and a trajectory stream
are refused."""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

import dattri_llm_b200 as bw
from tests import tiny


class _Crash(RuntimeError):
    pass


def _crashing_loss(after: int):
    calls = [0]

    def loss(model, batch):
        calls[0] += 1
        if calls[0] > after:
            raise _Crash("simulated interruption")
        return tiny.sq_loss(model, batch)

    return loss


def _att(cls, loss, tmp, model=None):
    args = bw.AttributionArguments(output_dir=str(tmp), per_device_train_batch_size=3,
                                   per_device_eval_batch_size=2)
    return cls(args, task=bw.AttributionTask(loss, model if model is not None else tiny.make_model(seed=3)))


def _data():
    x, y, xt, yt = tiny.make_data(seed=4)
    return tiny.as_dataset(x, y), tiny.as_dataset(xt, yt)


def _scores(cls, pairs, tmp, **kw):
    (tr, te), = pairs
    att = _att(cls, tiny.sq_loss, tmp)
    return att.attribute_from_cache(tr, te, **kw)


def _n_records(store_dir):
    return len(bw.GradientStorageManager(store_dir).own_records())


@pytest.mark.parametrize(("cls", "kw"), [(bw.TracInAttributor, {}), (bw.KFACAttributor, {"damping": 0.1})])
def test_interrupted_then_resumed_equals_uninterrupted(tmp_path, cls, kw):
    train, test = _data()
    cfg = bw.HookManagerConfig(linear_io=tiny.LAYERS)
    want_pairs = _att(cls, tiny.sq_loss, tmp_path / "a").cache(train, test, cache_dir=str(tmp_path / "full"),
                                                               hook_config=cfg)
    want = _scores(cls, want_pairs, tmp_path / "s1", **kw)
    # 2 test batches, then the first train batch, then the interruption
    with pytest.raises(_Crash):
        _att(cls, _crashing_loss(3), tmp_path / "b").cache(train, test, cache_dir=str(tmp_path / "part"),
                                                           hook_config=cfg)
    (tr, te), = [(str(tmp_path / "part/ckpt_0/train_grads"), str(tmp_path / "part/ckpt_0/test_grads"))]
    assert _n_records(tr) == 1 and _n_records(te) == 2
    pairs = _att(cls, tiny.sq_loss, tmp_path / "c").cache(train, test, cache_dir=str(tmp_path / "part"),
                                                          hook_config=cfg, resume=True)
    assert _n_records(tr) == 3 and _n_records(te) == 2  # nothing stored twice
    got = _scores(cls, pairs, tmp_path / "s2", **kw)
    torch.testing.assert_close(got.scores, want.scores, rtol=1e-5, atol=1e-6)
    assert got.row_train_ids == want.row_train_ids


def test_cut_off_index_line_is_redone(tmp_path):
    train, test = _data()
    cfg = bw.HookManagerConfig(linear_io=tiny.LAYERS)
    att = _att(bw.TracInAttributor, tiny.sq_loss, tmp_path / "a")
    (tr, te), = att.cache(train, test, cache_dir=str(tmp_path / "c"), hook_config=cfg)
    log = Path(tr) / "index.jsonl"
    lines = log.read_text().splitlines()
    log.write_text("\n".join(lines[:-1]) + "\n" + lines[-1][: len(lines[-1]) // 2])  # crash mid-line
    with pytest.warns(UserWarning, match="truncated"):
        assert _n_records(tr) == 2
    _att(bw.TracInAttributor, tiny.sq_loss, tmp_path / "b").cache(train, test, cache_dir=str(tmp_path / "c"),
                                                                  hook_config=cfg, resume=True)
    records = bw.GradientStorageManager(tr).own_records()
    assert len(records) == 3
    x, y, _, _ = tiny.make_data(seed=4)
    assert sorted(h for _, hs in records for h in hs) == sorted(tiny.hashes(x, y))


def test_changed_order_is_refused(tmp_path):
    train, test = _data()
    cfg = bw.HookManagerConfig(linear_io=tiny.LAYERS)
    with pytest.raises(_Crash):
        _att(bw.TracInAttributor, _crashing_loss(3), tmp_path / "a").cache(
            train, test, cache_dir=str(tmp_path / "c"), hook_config=cfg)
    with pytest.raises(RuntimeError, match="Cannot resume"):
        _att(bw.TracInAttributor, tiny.sq_loss, tmp_path / "b").cache(
            train[::-1], test, cache_dir=str(tmp_path / "c"), hook_config=cfg, resume=True)


def test_trajectory_cannot_resume(tmp_path):
    train, test = _data()
    att = _att(bw.TracInAttributor, tiny.sq_loss, tmp_path)
    with pytest.raises(ValueError, match="frozen probe"):
        att.cache(train, test, cache_dir=str(tmp_path / "c"), enable_update=True, resume=True)
    s = bw.GradientStreamer(tiny.make_model(), train, att.args, batch_size=3, enable_update=True,
                            loss_fn=tiny.sq_loss, config=bw.HookManagerConfig(linear_io=tiny.LAYERS))
    with pytest.raises(ValueError, match="frozen probe"):
        s.skip_batches(1)


def test_own_records_lists_this_directory_in_write_order(tmp_path):
    from dattri_llm_b200.gradient.gradient import Gradient, GradientRecord

    store = bw.GradientStorageManager(str(tmp_path / "s"))
    for step, ids in ((0, ["a", "b"]), (0, ["c"]), (1, ["d"])):
        g = Gradient({"w": "materialized"}, {"w": torch.zeros(len(ids), 2)}, {"w": "nn.Linear"}, {"w": "batch"})
        store.save_bulk([GradientRecord(step=step, input_hash=ids, gradient=g)])
    assert store.own_records() == [(0, ["a", "b"]), (0, ["c"]), (1, ["d"])]
    assert json.loads((tmp_path / "s" / "index_meta.json").read_text())["format"] == 2
