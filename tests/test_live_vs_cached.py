"""Live attribution equals attribution from stores, for the Kronecker family (CPU):
``attribute`` (streaming the model, fitting the covariances at capture time or in a
separate sweep, with or without a gradient cache) and ``attribute_from_cache`` over stores
collected from the same model give the same scores, which equal the dense K-FAC / EK-FAC
oracles of the attribution-oracle tests."""

from __future__ import annotations

import pytest
import torch

from dattri_llm_b200 import (
    AttributionArguments,
    AttributionTask,
    EKFACAttributor,
    HookManagerConfig,
    KFACAttributor,
)
from tests import tiny


def _args(path, **kw):
    return AttributionArguments(output_dir=str(path), use_cpu=True, per_device_train_batch_size=3,
                                per_device_eval_batch_size=2, **kw)


@pytest.mark.parametrize("cls", [KFACAttributor, EKFACAttributor])
@pytest.mark.parametrize(("residency", "at_capture"), [(None, True), (None, False), ("memory", True), ("disk", True)])
def test_live_equals_cached(tmp_path, cls, residency, at_capture):
    model = tiny.make_model(seed=3)
    xtr, ytr, xte, yte = tiny.make_data(seed=4)
    sd = tiny.checkpoints(model, 1)
    tiny.collect_to_disk(model, sd, xtr, ytr, tmp_path / "tr")
    tiny.collect_to_disk(model, sd, xte, yte, tmp_path / "te")
    cached = cls(_args(tmp_path / "c")).attribute_from_cache(str(tmp_path / "tr"), str(tmp_path / "te"), damping=0.1)
    model.load_state_dict(sd[0])
    task = AttributionTask(tiny.sq_loss, model, checkpoints=sd)
    live = cls(_args(tmp_path / "l"), task=task).attribute(
        tiny.as_dataset(xtr, ytr), tiny.as_dataset(xte, yte), hook_config=HookManagerConfig(linear_io=tiny.LAYERS),
        damping=0.1, gradient_cache_residency=residency, covariances_at_capture=at_capture)
    trh, teh = tiny.hashes(xtr, ytr), tiny.hashes(xte, yte)
    a = cached.query(trh, teh, trajectory="agnostic")
    b = live.query(trh, teh, trajectory="agnostic")
    torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-5 * float(a.abs().max()))
