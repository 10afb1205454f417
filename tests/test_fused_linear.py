"""Dense layers on the tcgen05 CTA-pair GEMM and the capture projections fused into them.

* the pair kernel's narrow last column tile (N not a multiple of 256) against fp32;
* one launch producing a layer's output and its token-major projected input against
  two separate fp32 products;
* :class:`TcLinear` forward / input gradient against ``F.linear`` in fp32;
* a LoGra capture of a Llama decoder with the projections computed inside the layers'
  GEMMs equals the capture with the hooks' own projection launches.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(("m", "n", "k"), [(1024, 2112, 512), (600, 320, 256), (512, 64 + 256 * 3, 128),
                                           (2048, 4000, 1024)])
def test_pair_gemm_narrow_last_tile(m, n, k):
    from dattri_llm_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(m + n)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    b = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    ops.gemm_tn(a, b, out, mode=ops.STORE_BF16)
    want = a.float() @ b.float().T
    torch.testing.assert_close(out.float(), want, rtol=1.6e-2, atol=1e-2 * float(want.abs().max()))
    ops.check_device_errors()


@pytest.mark.parametrize(("segs", "t", "d_in", "n", "k"), [(4, 256, 512, 1024, 64), (2, 512, 2048, 512, 64),
                                                          (3, 128, 256, 256, 192)])
def test_gemm_with_projection_tail(segs, t, d_in, n, k):
    from dattri_llm_b200 import ops
    from dattri_llm_b200.ops.linear import gemm_with_tail

    g = torch.Generator(device="cuda").manual_seed(n + k)
    x = torch.randn(segs * t, d_in, device="cuda", generator=g).bfloat16()
    w = torch.randn(n, d_in, device="cuda", generator=g).bfloat16()
    p_t = torch.randn(k, d_in, device="cuda", generator=g).bfloat16()
    y, a_pt = gemm_with_tail(x, w, p_t, t)
    want_y = x.float() @ w.float().T
    want_a = (x.float() @ p_t.float().T).view(segs, t, k).transpose(1, 2)
    torch.testing.assert_close(y.float(), want_y, rtol=1.6e-2, atol=1e-2 * float(want_y.abs().max()))
    torch.testing.assert_close(a_pt.float(), want_a, rtol=1.6e-2, atol=1e-2 * float(want_a.abs().max()))
    ops.check_device_errors()


def test_tc_linear_forward_and_input_gradient():
    from dattri_llm_b200 import ops
    from dattri_llm_b200.models.layers import TcLinear

    torch.manual_seed(0)
    lin = TcLinear(512, 768, bias=False).cuda().bfloat16()
    for _ in range(2):  # the second pass reuses the cached transposed weight
        x = torch.randn(4, 100, 512, device="cuda").bfloat16().requires_grad_(True)
        y = lin(x)
        dy = torch.randn_like(y)
        y.backward(dy)
    xf = x.detach().float().requires_grad_(True)
    yf = torch.nn.functional.linear(xf, lin.weight.float())
    yf.backward(dy.float())
    torch.testing.assert_close(y.detach().float(), yf.detach(), rtol=1.6e-2, atol=1e-2 * float(yf.abs().max()))
    torch.testing.assert_close(x.grad.float(), xf.grad, rtol=1.6e-2, atol=1e-2 * float(xf.grad.abs().max()))
    ops.check_device_errors()


def _capture_llama(fused: bool):
    from dattri_llm_b200 import CaptureCallback, HookManager, HookManagerConfig
    from dattri_llm_b200.models.llama import LlamaConfig, LlamaForCausalLM, token_sum_loss
    from dattri_llm_b200.ops import linear as tc

    cfg = LlamaConfig.tiny(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                           vocab_size=1024)
    model = LlamaForCausalLM(cfg, frozen_probe=True)
    model.reset_parameters(seed=0)
    model = model.cuda().bfloat16().requires_grad_(False)
    proj = {"__default__": {"style": "logra", "proj_dim": 64}}
    cb = CaptureCallback()
    hm = HookManager(model, HookManagerConfig(linear_io=[r"\.(q_proj|k_proj|v_proj|o_proj|gate_proj|up_proj|down_proj)$"],
                                              projection_kwargs=proj, include_frozen=True, capture_style="auto"),
                     callbacks=[cb])
    ids = torch.randint(0, cfg.vocab_size, (3, 128), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    old = tc.set_fused_capture(fused)
    try:
        for _ in range(2):  # two steps: shared projections and cached transposes are reused
            with hm.collect():
                token_sum_loss(model, {"input_ids": ids}).backward()
    finally:
        tc.set_fused_capture(old)
        hm.remove()
    return cb.record.gradient


def test_fused_capture_equals_hook_projections():
    from dattri_llm_b200 import ops

    fused, plain = _capture_llama(True), _capture_llama(False)
    assert sorted(fused.data) == sorted(plain.data) and len(fused.data) == 14
    for name in plain.data:
        got, want = fused.data[name], plain.data[name]
        assert isinstance(got, torch.Tensor) and got.shape == want.shape, name
        scale = float(want.float().abs().max())
        torch.testing.assert_close(got.float(), want.float(), rtol=3e-2, atol=3e-2 * scale, msg=name)
    ops.check_device_errors()


@pytest.mark.parametrize(("m", "n", "k", "tail"), [(8192, 2048, 2048, 0), (8192, 2048, 1024, 64),
                                                   (4096, 4096, 512, 0)])
def test_pair_gemm_stream_k_last_wave(m, n, k, tail):
    """Shapes whose last wave of 256 x 256 tiles is under half full (e.g. 256 tiles on 74 CTA
    pairs): those tiles run as two K halves whose partials meet through a workspace.  Two
    launches in a row (the second reuses the workspace under a new epoch) against fp32."""
    from dattri_llm_b200 import ops
    from dattri_llm_b200.ops.linear import gemm_with_tail

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    for _ in range(2):
        a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
        b = torch.randn(n, k, device="cuda", generator=g).bfloat16()
        want = a.float() @ b.float().T
        if tail:
            p_t = torch.randn(tail, k, device="cuda", generator=g).bfloat16()
            out, a_pt = gemm_with_tail(a, b, p_t, 1024)
            want_t = (a.float() @ p_t.float().T).view(m // 1024, 1024, tail).transpose(1, 2)
            torch.testing.assert_close(a_pt.float(), want_t, rtol=1.6e-2, atol=1e-2 * float(want_t.abs().max()))
        else:
            out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            ops.gemm_tn(a, b, out, mode=ops.STORE_BF16)
        torch.testing.assert_close(out.float(), want, rtol=1.6e-2, atol=1e-2 * float(want.abs().max()))
    ops.check_device_errors()


@pytest.mark.parametrize(("n", "w"), [(16384, 2048), (8192, 64), (1000, 300), (3000, 520)])
def test_symmetric_gram_accumulate(n, w):
    """K-FAC covariance accumulation ``out += x^T x``: upper-triangle tiles mirrored, the
    sample sum split over CTA pairs with atomic fp32 epilogues; two accumulating calls
    against fp64."""
    from dattri_llm_b200 import ops
    from dattri_llm_b200.gradient.ops.kronecker import gram_accumulate

    g = torch.Generator(device="cuda").manual_seed(n + w)
    out = torch.zeros(w, w, device="cuda")
    want = torch.zeros(w, w, device="cuda", dtype=torch.float64)
    for _ in range(2):
        x = torch.randn(n, w, device="cuda", generator=g).bfloat16()
        gram_accumulate(x, out)
        want += x.double().T @ x.double()
    torch.testing.assert_close(out.double(), want, rtol=1e-3, atol=1e-3 * float(want.abs().max()))
    # mirrored entries are summed in a different order: symmetric to fp32 rounding
    torch.testing.assert_close(out, out.T, rtol=1e-5, atol=1e-6 * float(out.abs().max()))
    ops.check_device_errors()


@pytest.mark.parametrize("shape", [(16384, 2048), (3, 200, 136), (1000, 64)])
def test_transpose_kernel(shape):
    from dattri_llm_b200 import ops
    from dattri_llm_b200.ops.gemm import transpose_last2

    x = torch.randn(*shape, device="cuda").bfloat16()
    torch.testing.assert_close(transpose_last2(x), x.transpose(-1, -2).contiguous(), rtol=0, atol=0)
    sl = x[..., 8:]  # a strided source (row stride kept, 16-byte aligned start)
    torch.testing.assert_close(transpose_last2(sl), sl.transpose(-1, -2).contiguous(), rtol=0, atol=0)
    ops.check_device_errors()


@pytest.mark.parametrize(("m", "n", "k", "bt"), [(512, 768, 1024, False), (300, 200, 4100, True), (2048, 64, 512, True)])
def test_matmul_f32_bf16x3(m, n, k, bt):
    """fp32 products on the tensor cores through the bf16x3 split: relative error of a few
    1e-5 against fp64 (the split's 2^-17 per product, growing like sqrt(K) over the sum),
    far below a plain bf16 (2^-8) or TF32 (2^-11) product."""
    from dattri_llm_b200 import ops
    from dattri_llm_b200.ops.gemm import matmul_f32

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(n, k, device="cuda", generator=g) if bt else torch.randn(k, n, device="cuda", generator=g)
    got = matmul_f32(a, b, b_transposed=bt)
    want = a.double() @ (b.double().T if bt else b.double())
    rel = float((got.double() - want).abs().max() / want.abs().max())
    assert rel < 5e-5, rel
    ops.check_device_errors()


@pytest.mark.gpu
def test_data_selection_token_contraction_on_tensor_cores():
    """The dropped samples' linear-layer contribution is one tcgen05 contraction over their
    tokens; it equals the fp32 sum of per-sample weight gradients."""
    from dattri_llm_b200.gradient.callbacks.data_selection_callback import DataSelectionCallback

    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(3, 96, 256, device="cuda", generator=g).bfloat16()
    d = torch.randn(3, 96, 128, device="cuda", generator=g).bfloat16()
    got = DataSelectionCallback._weight_contribution("nn.Linear", None, a, d, (128, 256))
    want = torch.einsum("bto,bti->oi", d.float(), a.float()).reshape(-1)
    torch.testing.assert_close(got, want, rtol=2e-3, atol=2e-3)


@pytest.mark.gpu
def test_direct_fisher_accumulates_on_the_gram_kernel():
    """The direct empirical Fisher of bf16 per-sample gradients (K-FAC's non-Kronecker
    layers) accumulates through the symmetric tcgen05 Gram kernel: equal to fp32 G^T G."""
    from dattri_llm_b200.gradient.ops.kronecker import LayerFisherAccumulator

    g = torch.Generator(device="cuda").manual_seed(4)
    acc = LayerFisherAccumulator()
    batches = [torch.randn(16, 384, device="cuda", generator=g).bfloat16() for _ in range(3)]
    for b in batches:
        acc.update_from_grad(b)
    want = sum(b.float().T @ b.float() for b in batches) / 48
    torch.testing.assert_close(acc.result(), want, rtol=2e-3, atol=2e-3)
