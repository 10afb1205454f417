"""``invasive_linear_io`` on CPU: the layer's backward skips the weight-gradient GEMM, yet
the captured per-sample gradients equal the autograd oracle, the input gradient still
reaches the layers below, ``weight.grad`` of the invasive layer stays empty, and the
original forward is back once collection ends."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from dattri_llm_b200.gradient.callbacks import CaptureCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(5, 6)
        self.fc2 = nn.Linear(6, 3)

    def forward(self, x):
        return self.fc2(torch.tanh(self.fc1(x))).pow(2).sum(dim=(1, 2))


def _x():
    return torch.randn(4, 3, 5, generator=torch.Generator().manual_seed(1))


def test_invasive_layer_captures_without_weight_grad():
    torch.manual_seed(0)
    model = Net()
    ref = Net()
    ref.load_state_dict(model.state_dict())
    x = _x()
    cap = CaptureCallback()
    hm = HookManager(model, HookManagerConfig(invasive_linear_io=[r"^fc2$"], linear_io=[r"^fc1$"]), callbacks=[cap])
    with hm.collect():
        model(x).sum().backward()
    assert model.fc2.weight.grad is None and model.fc2.bias.grad is None
    # fc1 still receives its parameter gradient (the input gradient of fc2 flowed)
    ref(x).sum().backward()
    torch.testing.assert_close(model.fc1.weight.grad, ref.fc1.weight.grad)
    dense = cap.record.gradient.materialize()
    for i in range(x.shape[0]):
        ref.zero_grad()
        ref(x[i : i + 1]).sum().backward()
        want = torch.cat([ref.fc2.weight.grad, ref.fc2.bias.grad[:, None]], 1).reshape(-1)
        torch.testing.assert_close(dense.data["fc2"][i].reshape(-1), want, rtol=1e-5, atol=1e-6)
    hm.remove()
    assert "forward" not in vars(model.fc2)  # the original forward is back


def test_invasive_assignment_of_a_non_linear_layer_raises():
    class WithNorm(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.norm = nn.LayerNorm(5)

        def forward(self, x):
            return self.norm(x).sum()

    # a selector only picks capable layers (here: none); an explicit assignment is checked
    with pytest.warns(UserWarning, match="zero layers"):
        HookManager(WithNorm(), HookManagerConfig(invasive_linear_io=[r"^norm$"])).remove()
    with pytest.raises(ValueError, match="nn.Linear"):
        HookManager(WithNorm(), HookManagerConfig(hook_types={"norm": "invasive_linear_io"}))
