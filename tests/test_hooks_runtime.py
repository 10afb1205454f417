"""Capture-engine behaviour on CPU: activation checkpointing, a module invoked twice per
forward, branches that never reach the loss, sample identifiers from a model input,
callbacks that re-enter the manager, and the capture-style choice.  Each check compares
against a plain autograd oracle (per-sample ``param.grad`` from running one sample)."""

from __future__ import annotations

import threading

import pytest
import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

from dattri_llm_b200.gradient.callbacks import CaptureCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig

B, T, D = 3, 4, 6


class Block(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(D, D)
        self.fc2 = nn.Linear(D, D)

    def forward(self, x):
        return self.fc2(torch.tanh(self.fc1(x)))


class Net(nn.Module):
    def __init__(self, ckpt: bool | None = None) -> None:
        super().__init__()
        self.block = Block()
        self.head = nn.Linear(D, 1)
        self.ckpt = ckpt  # None: no checkpointing; else use_reentrant

    def forward(self, x):
        h = checkpoint(self.block, x, use_reentrant=self.ckpt) if self.ckpt is not None else self.block(x)
        return self.head(h).sum(dim=(1, 2))


def _data(seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, T, D, generator=g)


def _capture(model, x, cfg=None, **kw):
    cap = CaptureCallback()
    hm = HookManager(model, cfg or HookManagerConfig(linear_io=[r"^(block\.fc[12]|head)$"]), callbacks=[cap], **kw)
    with hm.collect():
        model(x).sum().backward()
    hm.remove()
    return cap.record


def _per_sample_weight_grads(model, x, names):
    out = {n: [] for n in names}
    for i in range(x.shape[0]):
        model.zero_grad()
        model(x[i : i + 1]).sum().backward()
        params = dict(model.named_parameters())
        for n in names:
            out[n].append(params[n].grad.detach().clone())
    return {n: torch.stack(v) for n, v in out.items()}


def _dense(grad, layer):
    m = grad.materialize().data[layer]
    return m.reshape(m.shape[0], -1)


@pytest.mark.parametrize("use_reentrant", [True, False])
def test_checkpointed_block_matches_plain_run(use_reentrant):
    x = _data()
    torch.manual_seed(0)
    plain = Net()
    torch.manual_seed(0)
    ck = Net(ckpt=use_reentrant)
    x_ck = x.clone().requires_grad_(use_reentrant)  # the reentrant form needs an input that requires grad
    rec_plain = _capture(plain, x)
    rec_ck = _capture(ck, x_ck)
    assert set(rec_ck.gradient.data) == set(rec_plain.gradient.data)
    for layer in rec_plain.gradient.data:
        torch.testing.assert_close(_dense(rec_ck.gradient, layer), _dense(rec_plain.gradient, layer))
    # and both equal the per-sample autograd oracle (weight and bias blocks)
    want = _per_sample_weight_grads(plain, x, ["block.fc1.weight", "block.fc1.bias"])
    got = _dense(rec_ck.gradient, "block.fc1")
    oracle = torch.cat([want["block.fc1.weight"], want["block.fc1.bias"][..., None]], -1).reshape(B, -1)
    torch.testing.assert_close(got, oracle, rtol=1e-5, atol=1e-6)


def test_param_grads_unchanged_by_capture():
    x = _data(1)
    torch.manual_seed(0)
    a = Net()
    torch.manual_seed(0)
    b = Net()
    a(x).sum().backward()
    _capture(b, x)
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters(), strict=True):
        torch.testing.assert_close(pa.grad, pb.grad, msg=n)


class Twice(nn.Module):
    """``fc`` applied twice: its weight gradient is the sum over both invocations."""

    def __init__(self) -> None:
        super().__init__()
        self.fc = nn.Linear(D, D, bias=False)

    def forward(self, x):
        return self.fc(torch.tanh(self.fc(x))).sum(dim=(1, 2))


def test_invocations_are_virtual_layers_summing_to_the_weight_grad():
    torch.manual_seed(3)
    model = Twice()
    x = _data(2)
    rec = _capture(model, x, HookManagerConfig(linear_io=[r"^fc$"]))
    assert {"fc", "fc@2"} <= set(rec.gradient.data)
    total = _dense(rec.gradient, "fc") + _dense(rec.gradient, "fc@2")
    want = _per_sample_weight_grads(model, x, ["fc.weight"])["fc.weight"].reshape(B, -1)
    torch.testing.assert_close(total, want, rtol=1e-5, atol=1e-6)


class Side(nn.Module):
    """A hooked layer whose output never reaches the loss."""

    def __init__(self) -> None:
        super().__init__()
        self.fc = nn.Linear(D, 1)
        self.side = nn.Linear(D, D)

    def forward(self, x):
        _ = self.side(x).detach()
        return self.fc(x).sum(dim=(1, 2))


def test_branch_without_backward_does_not_stall():
    model = Side()
    with pytest.warns(UserWarning):
        rec = _capture(model, _data(3), HookManagerConfig(linear_io=[r"^(fc|side)$"]))
    assert "fc" in rec.gradient.data and "side" not in rec.gradient.data


class Keyed(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc = nn.Linear(D, 1)

    def forward(self, x, idx=None):
        return self.fc(x).sum(dim=(1, 2))


def test_sample_id_key_names_the_samples():
    model = Keyed()
    cap = CaptureCallback()
    hm = HookManager(model, HookManagerConfig(linear_io=[r"^fc$"]), callbacks=[cap], sample_id_key="idx")
    with hm.collect():
        model(_data(4), idx=torch.tensor([10, 11, 12])).sum().backward()
    assert list(cap.record.input_hash) == ["10", "11", "12"]
    with pytest.raises(KeyError), hm.collect():
        model(_data(4)).sum().backward()
    hm.remove()


def test_sample_id_key_with_wrong_length_raises():
    model = Keyed()
    hm = HookManager(model, HookManagerConfig(linear_io=[r"^fc$"]), callbacks=[CaptureCallback()],
                     sample_id_key="idx")
    with pytest.raises(ValueError), hm.collect():
        model(_data(4), idx=torch.tensor([1, 2])).sum().backward()
    hm.remove()


def test_alternative_identifier_schemes_are_exclusive():
    with pytest.raises(ValueError):
        HookManager(Keyed(), HookManagerConfig(linear_io=[r"^fc$"]), sample_id_key="idx",
                    sample_hash_fields=["x"])


def test_step_lock_is_free_during_on_step_end():
    """A callback that calls back into the manager from ``on_step_end`` must not deadlock."""
    model = Keyed()

    class Reenter(CaptureCallback):
        def __init__(self):
            super().__init__()
            self.saw = None

        def on_step_end(self, record):
            super().on_step_end(record)
            state = self.hm.save_state()  # takes the step lock
            self.hm.clear_state()
            self.hm.load_state(state)
            self.saw = sorted(state)

    cb = Reenter()
    hm = HookManager(model, HookManagerConfig(linear_io=[r"^fc$"]), callbacks=[cb])
    cb.hm = hm
    err = []

    def run():
        try:
            with hm.collect():
                model(_data(5)).sum().backward()
        except Exception as e:  # pragma: no cover - surfaced below
            err.append(e)

    th = threading.Thread(target=run, daemon=True)
    th.start()
    th.join(timeout=60)
    assert not th.is_alive(), "on_step_end deadlocked on the manager's lock"
    assert not err, err
    assert cb.record is not None and cb.saw
    hm.remove()


@pytest.mark.parametrize("tokens", [1, 5])
def test_materialized_style_equals_materialized_factors(tokens):
    g = torch.Generator().manual_seed(6)
    x = torch.randn(B, tokens, D, generator=g)
    torch.manual_seed(0)
    m1 = Net()
    torch.manual_seed(0)
    m2 = Net()
    fac = _capture(m1, x, HookManagerConfig(linear_io=[r"^(block\.fc[12]|head)$"], capture_style="factorized"))
    mat = _capture(m2, x, HookManagerConfig(linear_io=[r"^(block\.fc[12]|head)$"], capture_style="materialized"))
    for layer in fac.gradient.data:
        assert mat.gradient.representation[layer] == "materialized"
        torch.testing.assert_close(mat.gradient.data[layer].reshape(B, -1), _dense(fac.gradient, layer),
                                   rtol=1e-5, atol=1e-6)


def test_auto_style_follows_the_cost_rule():
    """``auto`` materializes a layer when its factors are larger than its gradient:
    ``T (D_out + D_in) >= D_out D_in`` (with the bias column)."""
    from dattri_llm_b200.gradient.ops.dot import maybe_use_materialized_norm

    for tokens in (1, 2, 40):
        x = torch.randn(B, tokens, D)
        torch.manual_seed(0)
        rec = _capture(Net(), x, HookManagerConfig(linear_io=[r"^block\.fc1$"], capture_style="auto"))
        rep = rec.gradient.representation["block.fc1"]
        want = maybe_use_materialized_norm(tokens, D + 1, D)
        assert rep == ("materialized" if want else "factorized"), (tokens, rep)


class InPlaceAfter(nn.Module):
    """Layer outputs modified in place right after the layer (inplace ReLU, ``mul_``)."""

    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(D, D)
        self.act = nn.ReLU(inplace=True)
        self.fc2 = nn.Linear(D, 1)

    def forward(self, x):
        h = self.act(self.fc1(x))
        y = self.fc2(h)
        y.mul_(3.0)
        return y.sum(dim=(1, 2))


def test_in_place_ops_after_a_layer_do_not_change_its_capture():
    torch.manual_seed(5)
    model = InPlaceAfter()
    x = _data(7)
    rec = _capture(model, x, HookManagerConfig(linear_io=[r"^fc[12]$"]))
    want = _per_sample_weight_grads(model, x, ["fc1.weight", "fc1.bias", "fc2.weight", "fc2.bias"])
    for layer in ("fc1", "fc2"):
        oracle = torch.cat([want[f"{layer}.weight"], want[f"{layer}.bias"][..., None]], -1).reshape(B, -1)
        torch.testing.assert_close(_dense(rec.gradient, layer), oracle, rtol=1e-5, atol=1e-6)
