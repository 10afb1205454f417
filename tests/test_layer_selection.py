"""Which layers get which hook family (CPU): the default (every linear-IO-capable layer
``linear_io``, every other module with trainable parameters ``param_grad``), regex and
``REGISTER_ALL`` selectors per family, explicit ``hook_types`` with their checks, conflicts
between families, ``layer_types`` relabelling, frozen layers, and the probe-based default
that keeps only layers firing on a sample input."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from dattri_llm_b200.gradient.hooks import HookManagerConfig
from dattri_llm_b200.gradient.hooks.config import (
    REGISTER_ALL,
    default_hook_assignment,
    resolve_hook_assignments,
)


class Custom(nn.Module):
    """A module with its own parameter and no linear-IO structure."""

    def __init__(self) -> None:
        super().__init__()
        self.scale = nn.Parameter(torch.ones(4))

    def forward(self, x):
        return x * self.scale


class Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.emb = nn.Embedding(10, 4)
        self.proj = nn.Linear(4, 4)
        self.norm = nn.LayerNorm(4)
        self.custom = Custom()
        self.head = nn.Linear(4, 2)
        self.unused = nn.Linear(4, 4)

    def forward(self, ids):
        h = self.custom(self.norm(self.proj(self.emb(ids))))
        return self.head(h).sum()


def test_default_assignment_covers_every_family():
    got = resolve_hook_assignments(Net(), HookManagerConfig())
    assert got["proj"] == got["head"] == got["emb"] == got["norm"] == "linear_io"
    assert got["custom"] == "param_grad"
    assert "" not in got  # the root has no parameters of its own


def test_regex_and_register_all_selectors():
    got = resolve_hook_assignments(Net(), HookManagerConfig(linear_io=[r"^(proj|head)$"], param_grad=[r"custom"]))
    assert got == {"proj": "linear_io", "head": "linear_io", "custom": "param_grad"}
    everything = resolve_hook_assignments(Net(), HookManagerConfig(linear_io=REGISTER_ALL))
    assert {"proj", "head", "emb", "norm", "unused"} <= set(everything)
    assert all(v == "linear_io" for v in everything.values())


def test_conflicting_families_raise():
    with pytest.raises(ValueError, match="conflicting"):
        resolve_hook_assignments(Net(), HookManagerConfig(linear_io=[r"^proj$"], invasive_linear_io=[r"^proj$"]))


def test_explicit_hook_types_are_checked():
    with pytest.raises(ValueError, match="does not exist"):
        resolve_hook_assignments(Net(), HookManagerConfig(hook_types={"nope": "linear_io"}))
    with pytest.raises(ValueError, match="linear_io"):
        resolve_hook_assignments(Net(), HookManagerConfig(hook_types={"custom": "linear_io"}))
    with pytest.raises(ValueError):
        HookManagerConfig(hook_types={"proj": "sideways"})


def test_layer_types_relabel_a_custom_module():
    got = resolve_hook_assignments(Net(), HookManagerConfig(hook_types={"custom": "linear_io"},
                                                            layer_types={"custom": "nn.RMSNorm"}))
    assert got == {"custom": "linear_io"}


def test_frozen_layers_need_include_frozen():
    net = Net()
    net.head.requires_grad_(False)
    from dattri_llm_b200.gradient.callbacks import CaptureCallback
    from dattri_llm_b200.gradient.hooks import HookManager

    ids = torch.tensor([[1, 2, 3], [4, 5, 6]])
    cap = CaptureCallback()
    hm = HookManager(net, HookManagerConfig(linear_io=[r"^(proj|head)$"]), callbacks=[cap])
    with hm.collect():
        net(ids).backward()
    hm.remove()
    assert set(cap.record.gradient.data) == {"proj"}  # the frozen head is skipped
    cap2 = CaptureCallback()
    with pytest.warns(UserWarning, match="no trainable parameter"):
        hm2 = HookManager(net, HookManagerConfig(linear_io=[r"^(proj|head)$"], include_frozen=True),
                          callbacks=[cap2])
    with hm2.collect():
        net(ids).backward()
    hm2.remove()
    assert set(cap2.record.gradient.data) == {"proj", "head"}


def test_probe_default_keeps_only_layers_that_fire():
    net = Net()
    with pytest.warns(UserWarning, match="did not fire"):
        got = default_hook_assignment(net, torch.tensor([[1, 2, 3]]))
    assert "unused" not in got
    assert got["proj"] == "linear_io" and got["custom"] == "param_grad"
    assert all(p.grad is None for p in net.parameters())  # the probe leaves no gradients behind


def test_selected_layers_capture_and_others_do_not():
    from dattri_llm_b200.gradient.callbacks import CaptureCallback
    from dattri_llm_b200.gradient.hooks import HookManager

    net = Net()
    cap = CaptureCallback()
    hm = HookManager(net, HookManagerConfig(linear_io=[r"^(proj|head)$"], param_grad=[r"^custom$"]), callbacks=[cap])
    with hm.collect():
        net(torch.tensor([[1, 2, 3], [4, 5, 6]])).backward()
    hm.remove()
    assert set(cap.record.gradient.data) == {"proj", "head", "custom.scale"}
