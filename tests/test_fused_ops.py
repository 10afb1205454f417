"""Fused model-path kernels (RMSNorm, SwiGLU, cross-entropy) vs fp32 PyTorch."""

import pytest
import torch
import torch.nn.functional as F

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


@pytest.mark.parametrize("cols", [2048, 4096, 520])
def test_add_rms_norm_forward_backward(cols):
    x = torch.randn(45, cols, device="cuda").bfloat16().requires_grad_()
    d = torch.randn(45, cols, device="cuda").bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(cols, device="cuda")).bfloat16().requires_grad_()
    y, h = fused.add_rms_norm(x, d, w, 1e-5)
    gy, gh = torch.randn_like(y), torch.randn_like(h)
    (y.float() * gy.float()).sum().add_((h.float() * gh.float()).sum()).backward()
    xr, dr, wr = (t.detach().float().requires_grad_() for t in (x, d, w))
    hr = (xr + dr).bfloat16().float()  # the residual stream is bf16
    hr.retain_grad()
    yr = torch.nn.functional.rms_norm(hr, (cols,), wr, 1e-5)
    (yr * gy.float()).sum().add_((hr * gh.float()).sum()).backward()
    torch.testing.assert_close(h.float(), (xr + dr).detach(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(d.grad.float(), dr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad.float(), wr.grad, rtol=3e-2, atol=0.5)


def _rope_ref(x, cos, sin):
    """Rotate-half RoPE in fp32 on ``x (B, T, H, D)``."""
    c = torch.cat([cos, cos], -1)[None, :, None, :]
    s = torch.cat([sin, sin], -1)[None, :, None, :]
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * c + rot * s


@pytest.mark.parametrize("head_dim", [64, 128])
def test_rope_forward_backward(head_dim):
    b, t, hq, hk = 3, 77, 8, 2
    ang = torch.outer(torch.arange(t, device="cuda", dtype=torch.float32),
                      1.0 / (10000 ** (torch.arange(0, head_dim, 2, device="cuda") / head_dim)))
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q = torch.randn(b, t, hq, head_dim, device="cuda").bfloat16().requires_grad_()
    k = torch.randn(b, t, hk, head_dim, device="cuda").bfloat16().requires_grad_()
    qo, ko = fused.rope(q, k, cos, sin)
    # Gradients arrive strided, as from attention over (B, H, T, D) views.
    gq = torch.randn(b, hq, t, head_dim, device="cuda").bfloat16().transpose(1, 2)
    gk = torch.randn(b, hk, t, head_dim, device="cuda").bfloat16().transpose(1, 2)
    torch.autograd.backward([qo, ko], [gq, gk])
    qr, kr = q.detach().float().requires_grad_(), k.detach().float().requires_grad_()
    qor, kor = _rope_ref(qr, cos, sin), _rope_ref(kr, cos, sin)
    torch.autograd.backward([qor, kor], [gq.float(), gk.float()])
    torch.testing.assert_close(qo.float(), qor, rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(ko.float(), kor, rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(q.grad.float(), qr.grad, rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(k.grad.float(), kr.grad, rtol=1e-2, atol=2e-2)


def test_adam_direction_matches_formula():
    g = torch.randn(6, 1000, device="cuda")
    m0 = 0.1 * torch.randn(1000, device="cuda")
    v0 = 0.01 * torch.rand(1000, device="cuda")
    out = ops.adam_direction(g, m0, v0, step=3, beta1=0.9, beta2=0.999, eps=1e-8)
    m = 0.9 * m0.double() + 0.1 * g.double()
    v = 0.999 * v0.double() + 0.001 * g.double() ** 2
    want = (m / (1 - 0.9**3)) / ((v / (1 - 0.999**3)).sqrt() + 1e-8)
    torch.testing.assert_close(out.double(), want, rtol=1e-4, atol=1e-5)


def test_llama_fused_blocks_match_unfused():
    from dattri_llm_b200.models.llama import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig.tiny(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2)
    model = LlamaForCausalLM(cfg, frozen_probe=True)
    model.reset_parameters(seed=0)
    model = model.cuda().bfloat16().requires_grad_(False)
    ids = torch.randint(0, cfg.vocab_size, (2, 96), device="cuda")
    outs = []
    for fused_on in (True, False):
        model._fused_blocks = (lambda _x: True) if fused_on else (lambda _x: False)
        loss = model(input_ids=ids, labels=ids, loss_reduction="sum", return_logits=False).loss
        emb = model.model.embed_tokens.weight
        h = model.hidden_states(ids)
        outs.append((float(loss), h.float()))
        del emb
    del model._fused_blocks
    assert abs(outs[0][0] - outs[1][0]) / abs(outs[1][0]) < 2e-2
    torch.testing.assert_close(outs[0][1], outs[1][1], rtol=5e-2, atol=5e-2)
    ops.check_device_errors()


@pytest.mark.parametrize("kind", ["nn.RMSNorm", "nn.LayerNorm"])
@pytest.mark.parametrize("bias", [False, True])
def test_norm_per_sample_grad_matches_torch(kind, bias):
    from dattri_llm_b200.gradient.ops.materialize import materialize_factors

    b, t, d = 5, 77, 1024
    x = torch.randn(b, t, d, device="cuda").bfloat16()
    g = torch.randn(b, t, d, device="cuda").bfloat16()
    mk = {"has_bias": bias, "eps": 1e-5, "normalized_shape": (d,)}
    got = materialize_factors(x, g, kind, mk)
    xf, gf = x.float(), g.float()
    if kind == "nn.LayerNorm":
        xh = (xf - xf.mean(-1, keepdim=True)) / (xf.var(-1, unbiased=False, keepdim=True) + 1e-5).sqrt()
    else:
        xh = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)
    want = (xh * gf).sum(1)
    if bias:
        want = torch.cat([want, gf.sum(1)], 1)
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-2)
    ops.check_device_errors()


def test_swiglu_split_forward_backward():
    """SwiGLU over ``[gate | up]`` rows with the valid-row count read from the device."""
    rows, inter, valid = 300, 256, 217
    h = torch.randn(rows, 2 * inter, device="cuda").bfloat16()
    out = torch.zeros(rows, inter, device="cuda", dtype=torch.bfloat16)
    n = torch.tensor([valid], dtype=torch.int32, device="cuda")
    ops.native().swiglu_split(h, out, n)
    hr = h.float().requires_grad_(True)
    ref = F.silu(hr[:, :inter]) * hr[:, inter:]
    torch.testing.assert_close(out[:valid].float(), ref[:valid].detach(), rtol=1e-2, atol=2e-2)
    assert not out[valid:].any()
    da = torch.randn(rows, inter, device="cuda").bfloat16()
    dh = torch.zeros_like(h)
    ops.native().swiglu_split_bwd(da, h, dh, n)
    ref.backward(da.float())
    torch.testing.assert_close(dh[:valid].float(), hr.grad[:valid], rtol=1e-2, atol=3e-2)
    assert not dh[valid:].any()


def test_moe_dispatch_and_combine_with_emulated_ranks():
    """Dispatch, combine and the fused combine-backward-dispatch with three "ranks" whose
    receive buffers are separate allocations on this GPU (the kernels take peer pointers;
    local ones exercise the same code)."""
    world, t, k, h = 3, 37, 2, 136
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(t, h, device="cuda", generator=g).bfloat16()
    rows = t * k
    dest = torch.randint(0, world, (rows,), device="cuda", generator=g)
    order = torch.argsort(dest, stable=True)
    per = torch.bincount(dest, minlength=world)
    start = torch.cumsum(per, 0) - per
    row = torch.empty_like(dest)
    row[order] = torch.arange(rows, device="cuda") - start[dest[order]]
    recv = [torch.zeros(rows, h, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    meta = [torch.full((rows, 2), -1, device="cuda", dtype=torch.int32) for _ in range(world)]
    d32, r32 = dest.int().contiguous(), row.int().contiguous()
    ops.native().moe_dispatch(x, k, d32, r32, recv, meta, 1)
    for r in range(rows):
        dr, rr = int(dest[r]), int(row[r])
        assert torch.equal(recv[dr][rr], x[r // k])
        assert meta[dr][rr].tolist() == [1, r]
    # combine: y[t] = sum_j w[t, j] * slots[t * k + j]
    slots = torch.randn(rows, h, device="cuda", generator=g).bfloat16()
    w = torch.rand(t, k, device="cuda", generator=g)
    y = torch.empty(t, h, device="cuda", dtype=torch.bfloat16)
    ops.native().moe_combine(slots, w, y)
    want = (slots.float().view(t, k, h) * w[..., None]).sum(1)
    torch.testing.assert_close(y.float(), want, rtol=1e-2, atol=2e-2)
    # backward: dw = <slots, dy>, and w * dy dispatched to the owners
    dy = torch.randn(t, h, device="cuda", generator=g).bfloat16()
    dw = torch.empty(t, k, device="cuda")
    for buf in recv:
        buf.zero_()
    ops.native().moe_combine_bwd_dispatch(dy, slots, w, dw, d32, r32, recv, meta, 2)
    torch.testing.assert_close(dw, (slots.float().view(t, k, h) * dy.float()[:, None]).sum(-1), rtol=1e-3, atol=1e-2)
    for r in range(rows):
        dr, rr = int(dest[r]), int(row[r])
        torch.testing.assert_close(recv[dr][rr].float(), (w.reshape(-1)[r] * dy[r // k].float()).bfloat16().float())
        assert meta[dr][rr].tolist() == [2, r]
    ops.check_device_errors()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_embedding_dense_grad_matches_index_add(dtype):
    from dattri_llm_b200.gradient.ops.materialize import materialize_factors

    b, t, e, vocab = 3, 257, 192, 1000
    gen = torch.Generator(device="cuda").manual_seed(0)
    ids = torch.randint(0, 40, (b, t), device="cuda", generator=gen)  # many repeats per sample
    ids[1, :5] = vocab - 1  # the last row
    ids[2, 7] = 0
    g = torch.randn(b, t, e, device="cuda", generator=gen).to(dtype)
    n0 = ops.launch_count()
    out = ops.embedding_dense_grad(ids, g, vocab)
    assert ops.launch_count() == n0 + 1
    ref = torch.zeros(b * vocab, e, device="cuda")
    ref.index_add_(0, (ids + torch.arange(b, device="cuda")[:, None] * vocab).reshape(-1), g.float().reshape(-1, e))
    assert out.dtype == dtype and out.shape == (b, vocab * e)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    torch.testing.assert_close(out.float(), ref.reshape(b, vocab * e), rtol=tol, atol=tol)
    via = materialize_factors(ids, g, "nn.Embedding", module_kwargs={"num_embeddings": vocab})
    torch.testing.assert_close(via.float(), out.float(), rtol=0, atol=0)


def test_gated_rms_norm_matches_the_mamba2_module():
    from transformers.models.mamba2.modeling_mamba2 import MambaRMSNormGated

    rows, d = 300, 5120
    gen = torch.Generator(device="cuda").manual_seed(3)
    y = torch.randn(rows, d, device="cuda", generator=gen).requires_grad_()
    proj = torch.randn(rows, d + 64, device="cuda", generator=gen).bfloat16()
    g = proj[:, 32:32 + d].detach().requires_grad_()  # a column slice, as the mixer's gate is
    norm = MambaRMSNormGated(d, eps=1e-5).cuda()
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(d, device="cuda", generator=gen))
    w = norm.weight.detach().bfloat16().requires_grad_()
    out = fused.gated_rms_norm(y, g, w, 1e-5)
    dout = torch.randn(rows, d, device="cuda", generator=gen).bfloat16()
    out.backward(dout)
    yr, gr = y.detach().clone().requires_grad_(), g.detach().float().requires_grad_()
    norm.weight.data.copy_(w.detach().float())
    ref = norm(yr, gr)
    ref.backward(dout.float())
    assert out.dtype == torch.bfloat16
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(y.grad, yr.grad, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(g.grad.float(), gr.grad, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(w.grad.float(), norm.weight.grad, rtol=1e-2, atol=1e-1)


@pytest.mark.parametrize(("b", "c", "s", "h", "g"), [(2, 3, 128, 6, 2), (1, 2, 256, 4, 1)])
def test_ssd_intra_matches_torch(b, c, s, h, g):
    gen = torch.Generator(device="cuda").manual_seed(5)
    cb = torch.randn(b, g, c, s, s, device="cuda", generator=gen).requires_grad_()
    cum = (-0.05 * torch.rand(b, h, c, s, device="cuda", generator=gen)).cumsum(-1).requires_grad_()
    x = torch.randn(b, c, s, h, 64, device="cuda", generator=gen).requires_grad_()
    y = fused.ssd_intra(cb, cum, x)
    dy = torch.randn_like(y)
    y.backward(dy)
    refs = [t.detach().double().requires_grad_() for t in (cb, cum, x)]
    cb_r, cum_r, x_r = refs
    causal = torch.ones(s, s, dtype=torch.bool, device="cuda").tril()
    decay = (cum_r[..., :, None] - cum_r[..., None, :]).masked_fill(~causal, float("-inf")).exp()
    mix = cb_r.repeat_interleave(h // g, dim=1) * decay  # (b, h, c, s, t)
    y_r = torch.einsum("bhcst,bcthp->bcshp", mix, x_r)
    y_r.backward(dy.double())

    def rel(a, want):
        return float((a.double() - want).norm() / want.norm())

    assert rel(y, y_r) < 1e-5
    assert rel(x.grad, x_r.grad) < 1e-5
    assert rel(cb.grad, cb_r.grad) < 1e-5
    assert rel(cum.grad, cum_r.grad) < 1e-4


@pytest.mark.parametrize(("b", "length", "bias"), [(2, 77, True), (1, 2048, False)])
def test_causal_conv_silu_matches_conv1d(b, length, bias):
    c = 96
    gen = torch.Generator(device="cuda").manual_seed(7)
    proj = torch.randn(b, length, c + 40, device="cuda", generator=gen).bfloat16()
    x = proj[..., 20:20 + c].detach().requires_grad_()  # a channel slice of a wider projection
    conv = torch.nn.Conv1d(c, c, 4, groups=c, padding=3, bias=bias).cuda().bfloat16()
    assert fused.causal_conv_silu_enabled(x, conv)
    out = fused.causal_conv_silu(x, conv.weight, conv.bias)
    dout = torch.randn(b, length, c, device="cuda", generator=gen).bfloat16()
    out.backward(dout)
    xr = x.detach().float().requires_grad_()
    wr = conv.weight.detach().float().requires_grad_()
    br = conv.bias.detach().float().requires_grad_() if bias else None
    ref = F.silu(F.conv1d(xr.transpose(1, 2), wr, br, padding=3, groups=c)[..., :length]).transpose(1, 2)
    ref.backward(dout.float())
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=1e-2, atol=1e-2)
    tol = 2e-2 * float(wr.grad.abs().max())
    torch.testing.assert_close(conv.weight.grad.float(), wr.grad, rtol=2e-2, atol=tol)
    if bias:
        torch.testing.assert_close(conv.bias.grad.float(), br.grad, rtol=2e-2, atol=2e-2 * float(br.grad.abs().max()))


def test_ssd_chunked_on_gpu_matches_fp64_cpu():
    """The whole chunked scan on the GPU (fused intra-chunk kernels, TF32 chunk-state
    products) against the same code in fp64 on the CPU: outputs and input gradients."""
    from dattri_llm_b200.models.mamba2 import ssd_chunked

    bsz, length, heads, hd, groups, state, chunk = 2, 300, 8, 64, 2, 32, 64
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(bsz, length, heads, hd, generator=gen)
    dt = 0.1 * torch.rand(bsz, length, heads, generator=gen)
    a = -1.0 - torch.rand(heads, generator=gen)
    b = torch.randn(bsz, length, groups, state, generator=gen)
    c = torch.randn(bsz, length, groups, state, generator=gen)
    dy = torch.randn(bsz, length, heads, hd, generator=gen)
    cpu = [t.double().requires_grad_() for t in (x, dt, a, b, c)]
    gpu = [t.cuda().requires_grad_() for t in (x, dt, a, b, c)]
    want = ssd_chunked(*cpu, chunk)
    want.backward(dy.double())
    got = ssd_chunked(*gpu, chunk)
    got.backward(dy.cuda())

    def rel(u, v):
        return float((u.double().cpu() - v).norm() / v.norm())

    assert rel(got, want) < 5e-3
    for g_, w_, name in zip(gpu, cpu, ("x", "dt", "a", "b", "c"), strict=True):
        assert rel(g_.grad, w_.grad) < 1e-2, name
