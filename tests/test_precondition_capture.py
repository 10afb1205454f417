"""Capture-time preconditioning (LESS's Adam directions) on CPU: with
``HookManager(optimizer=...)`` and ``precondition`` on, each captured per-sample gradient
is the direction the optimizer's next step would take from that sample's gradient given
its current state, in the layer's materialized layout; the ``mask`` projection keeps exact
coordinates of that direction; LoGra (which mixes coordinates) is refused."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from dattri_llm_b200.gradient.callbacks import CaptureCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig
from dattri_llm_b200.gradient.ops.optimizer import precondition
from dattri_llm_b200.gradient.ops.projection import DattriProjector


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(5, 4)
        self.fc2 = nn.Linear(4, 2)

    def forward(self, x):
        return self.fc2(torch.tanh(self.fc1(x))).pow(2).sum(dim=-1)


def _trained():
    torch.manual_seed(0)
    model = Net()
    opt = torch.optim.AdamW(model.parameters(), lr=0.01)
    g = torch.Generator().manual_seed(1)
    for _ in range(3):
        opt.zero_grad()
        model(torch.randn(6, 5, generator=g)).sum().backward()
        opt.step()
    opt.zero_grad()
    return model, opt


def _layer_state(opt, layer):
    """Adam state of *layer* in the materialized layout ``[W | b]`` row-major."""
    st_w, st_b = opt.state[layer.weight], opt.state[layer.bias]
    return {k: torch.cat([st_w[k], st_b[k][:, None]], 1).reshape(-1) for k in ("exp_avg", "exp_avg_sq")}, \
        int(st_w["step"]) + 1


def _per_sample(model, x, layer):
    rows = []
    for i in range(x.shape[0]):
        model.zero_grad()
        model(x[i : i + 1]).sum().backward()
        rows.append(torch.cat([layer.weight.grad, layer.bias.grad[:, None]], 1).reshape(-1))
    model.zero_grad()
    return torch.stack(rows)


def test_captures_are_adam_directions():
    model, opt = _trained()
    x = torch.randn(3, 5, generator=torch.Generator().manual_seed(2))
    want = {}
    for name in ("fc1", "fc2"):
        layer = getattr(model, name)
        state, step = _layer_state(opt, layer)
        want[name] = precondition(_per_sample(model, x, layer), state, optimizer_type="AdamW", step=step)
    cap = CaptureCallback()
    hm = HookManager(model, HookManagerConfig(linear_io=[r"^fc[12]$"]), callbacks=[cap], optimizer=opt)
    assert hm.supports_preconditioning
    hm.precondition = True
    with hm.collect():
        model(x).sum().backward()
    hm.remove()
    for name, w in want.items():
        got = cap.record.gradient.data[name]
        torch.testing.assert_close(got.reshape(3, -1), w, rtol=1e-4, atol=1e-6)


def test_mask_keeps_coordinates_of_the_direction():
    model, opt = _trained()
    x = torch.randn(3, 5, generator=torch.Generator().manual_seed(3))
    layer = model.fc1
    state, step = _layer_state(opt, layer)
    full = precondition(_per_sample(model, x, layer), state, optimizer_type="AdamW", step=step)
    proj = {"fc1": {"style": "mask", "proj_dim": 7, "proj_seed": 5}}
    cap = CaptureCallback()
    hm = HookManager(model, HookManagerConfig(linear_io=[r"^fc1$"], projection_kwargs=proj), callbacks=[cap],
                     optimizer=opt)
    hm.precondition = True
    with hm.collect():
        model(x).sum().backward()
    hm.remove()
    idx = DattriProjector().mask_indices(full.shape[-1], proj_dim=7, proj_seed=5, device=torch.device("cpu"))
    torch.testing.assert_close(cap.record.gradient.data["fc1"].reshape(3, -1), full[:, idx], rtol=1e-4, atol=1e-6)


def test_logra_projection_cannot_be_preconditioned():
    model, opt = _trained()
    with pytest.raises(ValueError, match="logra"):
        HookManager(model, HookManagerConfig(linear_io=[r"^fc1$"],
                                             projection_kwargs={"fc1": {"style": "logra", "proj_dim": 2}}),
                    optimizer=opt)
