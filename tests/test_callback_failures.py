"""A failing callback does not poison the capture engine (CPU): the exception reaches the
caller, and the next step through the same manager records exactly what a fresh manager
records; a failing layer-level callback is bounded the same way."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from dattri_llm_b200.gradient.callbacks import CaptureCallback
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(4, 5)
        self.fc2 = nn.Linear(5, 2)

    def forward(self, x):
        return self.fc2(torch.relu(self.fc1(x))).sum(dim=-1)


class Boom(HookManagerCallback):
    def __init__(self, where: str, times: int = 1) -> None:
        self.where, self.left = where, times

    def _maybe(self, where):
        if where == self.where and self.left > 0:
            self.left -= 1
            raise RuntimeError(f"boom in {where}")

    def on_step_end(self, record) -> None:
        self._maybe("step")

    def on_layer_backward(self, *args, **kwargs) -> None:
        self._maybe("layer")


def _x(seed):
    return torch.randn(3, 4, generator=torch.Generator().manual_seed(seed))


def _fresh_record(x):
    torch.manual_seed(0)
    net = Net()
    cap = CaptureCallback()
    hm = HookManager(net, HookManagerConfig(linear_io=[r"^fc[12]$"]), callbacks=[cap])
    with hm.collect():
        net(x).sum().backward()
    hm.remove()
    return cap.record


@pytest.mark.parametrize("where", ["step", "layer"])
def test_manager_recovers_after_a_failing_callback(where):
    torch.manual_seed(0)
    net = Net()
    cap = CaptureCallback()
    hm = HookManager(net, HookManagerConfig(linear_io=[r"^fc[12]$"]), callbacks=[Boom(where), cap])
    with pytest.raises(RuntimeError, match="boom"), hm.collect():
        net(_x(1)).sum().backward()
    net.zero_grad(set_to_none=True)
    # no manual reset: leaving collect() with an error must leave the manager clean
    with hm.collect():
        net(_x(2)).sum().backward()
    hm.remove()
    want = _fresh_record(_x(2))
    got = cap.record
    assert set(got.gradient.data) == set(want.gradient.data)
    for name in want.gradient.data:
        torch.testing.assert_close(got.gradient.materialize().data[name], want.gradient.materialize().data[name])
    assert list(got.input_hash) == list(want.input_hash)
