"""Captured per-sample gradients against autograd, one sample at a time (CPU).

Each case wraps one layer type in a tiny model, captures a step with
:class:`HookManager` (raw factorized capture), materializes the layer's per-sample
gradient and compares it, plus the derived norms and pairwise dots, with the gradient
autograd gives for each sample's own loss.  Layout of the materialized rows (part of
the store format): linear / conv ``(out, in [+ bias column])`` row-major; norm
``[dW, db]``; embedding ``(vocab, E)``.
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks import CaptureCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig

B = 5


class Wrap(nn.Module):
    def __init__(self, layer: nn.Module, head_in: int) -> None:
        super().__init__()
        self.layer = layer
        torch.manual_seed(7)
        self.register_buffer("head", torch.randn(head_in))

    def forward(self, x):
        y = self.layer(x)
        return (y.reshape(y.shape[0], -1) * self.head).sum(1)  # one scalar per sample


def _cases():
    return {
        "linear2d": (lambda: nn.Linear(6, 4), lambda: torch.randn(B, 6), 4),
        "linear2d_nobias": (lambda: nn.Linear(6, 4, bias=False), lambda: torch.randn(B, 6), 4),
        "linear3d": (lambda: nn.Linear(6, 4), lambda: torch.randn(B, 3, 6), 12),
        "conv1d": (lambda: nn.Conv1d(3, 4, 3), lambda: torch.randn(B, 3, 9), 28),
        "conv1d_nobias": (lambda: nn.Conv1d(3, 4, 3, bias=False), lambda: torch.randn(B, 3, 9), 28),
        "conv2d": (lambda: nn.Conv2d(2, 3, 3, padding=1), lambda: torch.randn(B, 2, 5, 5), 75),
        "conv3d": (lambda: nn.Conv3d(2, 3, 2), lambda: torch.randn(B, 2, 3, 3, 3), 24),
        "layernorm": (lambda: nn.LayerNorm(6), lambda: torch.randn(B, 4, 6), 24),
        "layernorm_nobias": (lambda: nn.LayerNorm(6, bias=False), lambda: torch.randn(B, 4, 6), 24),
        "rmsnorm": (lambda: nn.RMSNorm(6), lambda: torch.randn(B, 4, 6), 24),
        "embedding": (lambda: nn.Embedding(11, 4), lambda: torch.randint(0, 11, (B, 7)), 28),
        "embedding_padding": (lambda: nn.Embedding(11, 4, padding_idx=0), lambda: torch.randint(0, 3, (B, 7)), 28),
        "linear4d": (lambda: nn.Linear(6, 4), lambda: torch.randn(B, 2, 3, 6), 24),
        "conv2d_grouped": (lambda: nn.Conv2d(4, 6, 3, groups=2), lambda: torch.randn(B, 4, 5, 5), 54),
        "conv2d_strided_dilated": (lambda: nn.Conv2d(2, 3, 3, stride=2, padding=2, dilation=2),
                                   lambda: torch.randn(B, 2, 7, 7), 48),
        "conv1d_depthwise": (lambda: nn.Conv1d(4, 4, 3, groups=4, padding=1), lambda: torch.randn(B, 4, 6), 24),
        "conv_transpose1d": (lambda: nn.ConvTranspose1d(3, 2, 3), lambda: torch.randn(B, 3, 5), 14),
        "conv_transpose2d": (lambda: nn.ConvTranspose2d(2, 3, 2, stride=2), lambda: torch.randn(B, 2, 3, 3), 108),
        "embedding_bag_sum": (lambda: nn.EmbeddingBag(11, 4, mode="sum"), lambda: torch.randint(0, 11, (B, 5)), 4),
        "embedding_bag_mean_padding": (lambda: nn.EmbeddingBag(11, 4, mode="mean", padding_idx=1),
                                       lambda: torch.randint(0, 4, (B, 6)), 4),
        "groupnorm": (lambda: nn.GroupNorm(2, 4), lambda: torch.randn(B, 4, 5), 20),
        "instancenorm_affine": (lambda: nn.InstanceNorm1d(4, affine=True), lambda: torch.randn(B, 4, 5), 20),
    }


def _reference(model: Wrap, x: torch.Tensor) -> torch.Tensor:
    """``(B, d)`` per-sample gradients in the store layout, from autograd."""
    layer = model.layer
    rows = []
    for i in range(x.shape[0]):
        layer.zero_grad(set_to_none=True)
        model(x[i:i + 1]).sum().backward()
        w = layer.weight.grad
        b = layer.bias.grad if getattr(layer, "bias", None) is not None else None
        if isinstance(layer, nn.Embedding):
            rows.append(w.reshape(-1))
        elif isinstance(layer, (nn.LayerNorm, nn.RMSNorm, nn.GroupNorm, nn.InstanceNorm1d)):
            rows.append(torch.cat([w.reshape(-1)] + ([b.reshape(-1)] if b is not None else [])))
        elif isinstance(layer, nn.modules.conv._ConvTransposeNd):
            # weight (c_in, c_out, k...): rows are input channels; the bias sits in an extra
            # row, in a padded block of c_out columns after the weight's c_out * k columns
            w2 = w.reshape(w.shape[0], -1)
            if b is not None:
                full = torch.zeros(w2.shape[0] + 1, w2.shape[1] + b.numel())
                full[:-1, : w2.shape[1]] = w2
                full[-1, w2.shape[1]:] = b
                w2 = full
            rows.append(w2.reshape(-1))
        else:
            w2 = w.reshape(w.shape[0], -1)
            if b is not None:
                w2 = torch.cat([w2, b[:, None]], 1)
            rows.append(w2.reshape(-1))
    layer.zero_grad(set_to_none=True)
    return torch.stack(rows)


def _capture(model: Wrap, x: torch.Tensor):
    cap = CaptureCallback()
    cfg = HookManagerConfig(linear_io=[r"^layer$"])
    hm = HookManager(model, cfg, callbacks=[cap])
    with hm.collect():
        model(x).sum().backward()
    hm.remove()
    g = cap.record.gradient
    (name,) = list(g.data)
    return g, name


@pytest.mark.parametrize("case", list(_cases()))
def test_materialize_matches_autograd(case):
    make_layer, make_x, head = _cases()[case]
    torch.manual_seed(0)
    model = Wrap(make_layer(), head)
    x = make_x()
    want = _reference(model, x)
    g, name = _capture(model, x)
    got = ops.materialize(g.data[name], g.layer_types[name])
    assert got.shape == want.shape, (got.shape, want.shape)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("case", ["linear3d", "conv2d", "layernorm", "embedding", "linear2d"])
def test_norms_and_pairwise_dots_match_autograd(case):
    make_layer, make_x, head = _cases()[case]
    torch.manual_seed(1)
    model = Wrap(make_layer(), head)
    x = make_x()
    want = _reference(model, x)
    g, name = _capture(model, x)
    f, lt = g.data[name], g.layer_types[name]
    torch.testing.assert_close(ops.grad_norm_sq(f, lt), (want * want).sum(1), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(ops.cross_dot(f, f, lt), want @ want.T, rtol=1e-4, atol=1e-5)
