"""Multi-rank behaviour on CPU (two gloo ranks via ``torch.multiprocessing.spawn``):

* K-FAC covariance and Fisher accumulators reduced over ranks equal one process that
  saw all the data (including rows whose gradient is zero, which both must drop);
* the packed reduction of many layers' accumulators (one collective) equals reducing them
  one by one;
* live TracIn attribution with the train set sharded over ranks (each rank scores its
  shard against the whole test set) gives, once the rows are merged, the single-process
  scores;
* live K-FAC / EK-FAC on sharded data fit the global factors (covariances and EK-FAC's
  eigenvalue sweep reduced over ranks) and reproduce the single-process scores.
"""

from __future__ import annotations

import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests import tiny


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, *args, world: int = 2) -> dict:
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_entry, args=(world, _port(), fn, out, args), nprocs=world, join=True)
        return dict(out)


def _entry(rank, world, port, fn, out, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        out[rank] = fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def _factors(seed, n=12, t=3, k=5, d=4):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(n, t, k, generator=g)
    gr = torch.randn(n, t, d, generator=g)
    gr[::4, 1] = 0.0  # gradient-free rows: dropped by the covariance and the count
    return a, gr


def _accumulate(a, g):
    from dattri_llm_b200.gradient.ops.kronecker import LayerFisherAccumulator, LayerKroneckerAccumulator

    kron, fisher = LayerKroneckerAccumulator(), LayerFisherAccumulator()
    for i in range(0, a.shape[0], 3):
        kron.update(a[i : i + 3], g[i : i + 3], "nn.Linear", {"has_bias": True})
        fisher.update(a[i : i + 3], g[i : i + 3], "nn.Linear", {"has_bias": True})
    return kron, fisher


def _kron_worker(rank, world):
    a, g = _factors(0)
    half = a.shape[0] // world
    kron, fisher = _accumulate(a[rank * half : (rank + 1) * half], g[rank * half : (rank + 1) * half])
    kron.all_reduce()
    fisher.all_reduce()
    A, G = kron.result()
    return A, G, kron._n, fisher.result()


def test_reduced_accumulators_equal_single_process_fit():
    res = _spawn(_kron_worker)
    a, g = _factors(0)
    kron, fisher = _accumulate(a, g)
    A, G = kron.result()
    for rank in range(2):
        A_r, G_r, n_r, F_r = res[rank]
        assert n_r == kron._n
        torch.testing.assert_close(A_r, A)
        torch.testing.assert_close(G_r, G)
        torch.testing.assert_close(F_r, fisher.result(), rtol=1e-5, atol=1e-6)


def _packed_worker(rank, world):
    from dattri_llm_b200.gradient.ops.kronecker import LayerKroneckerAccumulator
    from dattri_llm_b200.parallel.covariance import all_reduce_accumulators

    packed, single = [], []
    for layer in range(3):
        a, g = _factors(10 + layer + 100 * rank, k=3 + layer, d=2 + layer)
        p, s = LayerKroneckerAccumulator(), LayerKroneckerAccumulator()
        p.update(a, g, "nn.Linear", None)
        s.update(a, g, "nn.Linear", None)
        packed.append(p)
        single.append(s)
    all_reduce_accumulators(packed)
    for s in single:
        s.all_reduce()
    return [(p._A, p._G, p._n, s._A, s._G, s._n) for p, s in zip(packed, single, strict=True)]


def test_packed_accumulator_reduction_equals_one_by_one():
    res = _spawn(_packed_worker)
    for rank in range(2):
        for A_p, G_p, n_p, A_s, G_s, n_s in res[rank]:
            torch.testing.assert_close(A_p, A_s)
            torch.testing.assert_close(G_p, G_s)
            assert n_p == n_s


def _scores():
    import dattri_llm_b200 as bw

    x, y, xt, yt = tiny.make_data(seed=3, n_train=10, n_test=4)
    model = tiny.make_model(seed=4)
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=3,
                                   per_device_eval_batch_size=2)
    task = bw.AttributionTask(tiny.sq_loss, model)
    att = bw.TracInAttributor(args, task=task)
    cfg = bw.HookManagerConfig(linear_io=tiny.LAYERS)
    score = att.attribute(tiny.as_dataset(x, y), tiny.as_dataset(xt, yt), hook_config=cfg)
    return {h: score.trajectory_agnostic(h) for h in score.train_ids}, list(score.test_ids)


def _score_worker(rank, world):
    return _scores()


def test_sharded_live_scores_merge_to_single_process_scores():
    res = _spawn(_score_worker)
    want, want_tests = _scores()
    merged = {}
    for rank in range(2):
        rows, tests = res[rank]
        assert tests == want_tests
        assert not (set(rows) & set(merged)), "a train sample was scored on both ranks"
        merged.update(rows)
    assert set(merged) == set(want)
    for h, row in want.items():
        torch.testing.assert_close(merged[h], row, rtol=1e-5, atol=1e-6)


def _kron_scores(cls_name, damping):
    import dattri_llm_b200 as bw

    x, y, xt, yt = tiny.make_data(seed=8, n_train=12, n_test=3)
    model = tiny.make_model(seed=9)
    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=2,
                                   per_device_eval_batch_size=3)
    att = getattr(bw, cls_name)(args, task=bw.AttributionTask(tiny.sq_loss, model))
    score = att.attribute(tiny.as_dataset(x, y), tiny.as_dataset(xt, yt),
                          hook_config=bw.HookManagerConfig(linear_io=tiny.LAYERS), damping=damping)
    return {h: score.trajectory_agnostic(h) for h in score.train_ids}


def _kron_worker_scores(rank, world, cls_name, damping):
    return _kron_scores(cls_name, damping)


@pytest.mark.parametrize("cls_name", ["KFACAttributor", "EKFACAttributor"])
def test_sharded_kronecker_fit_and_scores_equal_single_process(cls_name):
    """The covariance fit (and EK-FAC's eigenvalue sweep) run on both ranks' shards and are
    reduced, so every rank preconditions with the global factors."""
    res = _spawn(_kron_worker_scores, cls_name, 0.05)
    want = _kron_scores(cls_name, 0.05)
    merged = {}
    for rank in range(2):
        assert not (set(res[rank]) & set(merged))
        merged.update(res[rank])
    assert set(merged) == set(want)
    for h, row in want.items():
        torch.testing.assert_close(merged[h], row, rtol=1e-4, atol=1e-5)
