"""Capture on Hugging Face model families against per-sample autograd (CPU, tiny
random configs): OLMoE (fused experts with a router, regrouped per sample), Mamba2
(selective-scan mixer with a functional depthwise conv) and GPT-2 (``Conv1D`` layers).

Per-sample oracle: each sample's token-summed next-token loss, one sample per forward
(MoE routing and the scan are per token / per sequence, so a batch of one sees the same
computation)."""

from __future__ import annotations

import warnings

import pytest
import torch
import torch.nn.functional as F

import dattri_llm_b200 as bw
from dattri_llm_b200.gradient import ops

transformers = pytest.importorskip("transformers")
warnings.filterwarnings("ignore")


def _loss(model, ids):
    logits = model(input_ids=ids).logits
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1),
                           reduction="sum")


def _capture(model, ids, cfg, **hm_kw):
    cap = bw.CaptureCallback()
    hm = bw.HookManager(model, cfg, callbacks=[cap], **hm_kw)
    with hm.collect():
        _loss(model, ids).backward()
    hm.remove()
    model.zero_grad(set_to_none=True)
    return cap.record.gradient


def _per_sample(model, ids, params: dict) -> dict[str, torch.Tensor]:
    """``{name: (B, ...)}``: autograd gradient of each named parameter view per sample."""
    out = {n: [] for n in params}
    for i in range(ids.shape[0]):
        model.zero_grad(set_to_none=True)
        _loss(model, ids[i:i + 1]).backward()
        for n, fn in params.items():
            out[n].append(fn().detach().clone())
    model.zero_grad(set_to_none=True)
    return {n: torch.stack(v) for n, v in out.items()}


def _check(grad, name, want):
    got = ops.materialize(grad.data[name], grad.layer_types[name])
    want = want.reshape(want.shape[0], -1)
    assert got.shape == want.shape, (name, got.shape, want.shape)
    scale = float(want.abs().max()) or 1.0
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-4 * scale)


def test_olmoe_router_and_experts():
    cfg = transformers.OlmoeConfig(vocab_size=64, hidden_size=32, intermediate_size=16, num_hidden_layers=1,
                                   num_attention_heads=4, num_key_value_heads=4, num_experts=4,
                                   num_experts_per_tok=2, max_position_embeddings=64)
    torch.manual_seed(0)
    model = transformers.OlmoeForCausalLM(cfg).eval()
    ids = torch.randint(0, 64, (3, 8))
    grad = _capture(model, ids, bw.HookManagerConfig(linear_io=[r"mlp"]), moe_routed_layers=["model.layers.0.mlp"])
    mlp = model.model.layers[0].mlp
    views = {"router": lambda: mlp.gate.weight.grad}
    for e in range(4):
        views[f"gu{e}"] = lambda e=e: mlp.experts.gate_up_proj.grad[e]
        views[f"dn{e}"] = lambda e=e: mlp.experts.down_proj.grad[e]
    want = _per_sample(model, ids, views)
    _check(grad, "model.layers.0.mlp.gate.dattri_router", want["router"])
    for e in range(4):
        _check(grad, f"model.layers.0.mlp.experts.dattri_experts.{e}.gate_up", want[f"gu{e}"])
        _check(grad, f"model.layers.0.mlp.experts.dattri_experts.{e}.down", want[f"dn{e}"])


def test_mamba2_mixer():
    cfg = transformers.Mamba2Config(vocab_size=64, hidden_size=32, state_size=8, num_hidden_layers=1, head_dim=8,
                                    num_heads=8, expand=2, n_groups=1, chunk_size=8, conv_kernel=4)
    torch.manual_seed(0)
    model = transformers.Mamba2ForCausalLM(cfg).eval()
    ids = torch.randint(0, 64, (3, 16))
    grad = _capture(model, ids, bw.HookManagerConfig(linear_io=[r"mixer"]))
    mixer = model.backbone.layers[0].mixer
    want = _per_sample(model, ids, {
        "in": lambda: mixer.in_proj.weight.grad,
        "out": lambda: mixer.out_proj.weight.grad,
        "conv": lambda: torch.cat([mixer.conv1d.weight.grad.reshape(mixer.conv1d.weight.shape[0], -1),
                                   mixer.conv1d.bias.grad[:, None]], 1),
    })
    _check(grad, "backbone.layers.0.mixer.in_proj", want["in"])
    _check(grad, "backbone.layers.0.mixer.out_proj", want["out"])
    _check(grad, "backbone.layers.0.mixer.conv1d", want["conv"])


def test_gpt2_conv1d_layers():
    cfg = transformers.GPT2Config(vocab_size=64, n_positions=32, n_embd=32, n_layer=1, n_head=4)
    torch.manual_seed(0)
    model = transformers.GPT2LMHeadModel(cfg).eval()
    ids = torch.randint(0, 64, (3, 10))
    grad = _capture(model, ids, bw.HookManagerConfig(linear_io=[r"c_attn$", r"c_fc$"]))
    blk = model.transformer.h[0]

    def conv1d(mod):
        # HF Conv1D computes x @ W + b with W (in, out): its per-sample gradient in the
        # linear layout (out, in | bias).
        return lambda: torch.cat([mod.weight.grad.T, mod.bias.grad[:, None]], 1)

    want = _per_sample(model, ids, {"attn": conv1d(blk.attn.c_attn), "fc": conv1d(blk.mlp.c_fc)})
    _check(grad, "transformer.h.0.attn.c_attn", want["attn"])
    _check(grad, "transformer.h.0.mlp.c_fc", want["fc"])
