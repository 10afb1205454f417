"""Fused model-path kernels (RMSNorm, SwiGLU, cross-entropy) vs fp32 PyTorch."""

import pytest
import torch

from dattri_llm_b200 import ops
from dattri_llm_b200.ops import fused

pytestmark = pytest.mark.gpu


def test_rms_norm_forward_backward():
    x = torch.randn(37, 2048, device="cuda").bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(2048, device="cuda")).bfloat16().requires_grad_()
    y = fused.rms_norm(x, w, 1e-5)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = torch.nn.functional.rms_norm(xr, (2048,), wr, 1e-5)
    yr.backward(gy.float())
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad.float(), wr.grad, rtol=3e-2, atol=0.5)


def test_swiglu_forward_backward():
    g = torch.randn(64, 8192, device="cuda").bfloat16().requires_grad_()
    u = torch.randn(64, 8192, device="cuda").bfloat16().requires_grad_()
    h = fused.swiglu(g, u)
    dh = torch.randn_like(h)
    h.backward(dh)
    gr, ur = g.detach().float().requires_grad_(), u.detach().float().requires_grad_()
    hr = torch.nn.functional.silu(gr) * ur
    hr.backward(dh.float())
    torch.testing.assert_close(h.float(), hr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(g.grad.float(), gr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(u.grad.float(), ur.grad, rtol=3e-2, atol=3e-2)


def test_linear_cross_entropy_matches_fp32():
    n, d, v = 300, 256, 5000
    h = (0.5 * torch.randn(n, d, device="cuda")).bfloat16().requires_grad_()
    w = (0.5 * torch.randn(v, d, device="cuda")).bfloat16().requires_grad_()
    tgt = torch.randint(0, v, (n,), device="cuda")
    tgt[::7] = -100
    loss = fused.linear_cross_entropy(h, w, tgt)
    loss.backward()
    hr, wr = h.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    ref = torch.nn.functional.cross_entropy(hr @ wr.T, tgt, ignore_index=-100, reduction="sum")
    ref.backward()
    torch.testing.assert_close(loss.float(), ref, rtol=1e-2, atol=1e-1)
    torch.testing.assert_close(h.grad.float(), hr.grad, rtol=5e-2, atol=5e-2)
    torch.testing.assert_close(w.grad.float(), wr.grad, rtol=5e-2, atol=5e-2)
    ops.check_device_errors(h.device)
