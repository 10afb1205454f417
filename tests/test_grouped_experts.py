"""Grouped capture of fused-expert MoE blocks equals the per-expert capture.

A frozen-expert OLMoE probe with LoGra-projected, materialized expert captures runs once
through the grouped path (one function per block) and once through the per-expert proxy
loop; every expert projection's per-sample block, the router's capture and the trainable
embedding's gradient must agree, experts no token reached must hold zero rows, and the
grouped path must not have run the proxies.  On the CPU the grouped path runs its PyTorch
steps; the GPU test runs the sm_100a kernels (ragged tcgen05 GEMMs, fused combine) on the
same comparison in bf16.
"""

from __future__ import annotations

import warnings

import pytest
import torch
import torch.nn.functional as F

transformers = pytest.importorskip("transformers")

import dattri_llm_b200 as bw  # noqa: E402
from dattri_llm_b200.gradient.hooks.override_layers.grouped_experts import set_grouped_experts  # noqa: E402

E = 8


def _model(device, dtype, layers=2):
    cfg = transformers.OlmoeConfig(vocab_size=96, hidden_size=64, intermediate_size=32, num_hidden_layers=layers,
                                   num_attention_heads=4, num_key_value_heads=4, num_experts=E,
                                   num_experts_per_tok=2, max_position_embeddings=64)
    torch.manual_seed(0)
    model = transformers.OlmoeForCausalLM(cfg).to(device=device, dtype=dtype).eval()
    model.requires_grad_(False)
    model.get_input_embeddings().requires_grad_(True)
    return model


def _loss(model, ids):
    logits = model(input_ids=ids).logits
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1),
                           reduction="sum")


def _capture(model, ids, grouped: bool, proj_dim: int = 4):
    blocks = [f"model.layers.{i}.mlp" for i in range(len(model.model.layers))]
    proj = {"__default__": {"style": "logra", "proj_dim": proj_dim, "proj_type": "rademacher", "proj_seed": 0}}
    cfg = bw.HookManagerConfig(linear_io=[r"\.mlp\.(experts|gate)$"], projection_kwargs=proj, capture_style="auto",
                               include_frozen=True)
    cap = bw.CaptureCallback()
    previous = set_grouped_experts(grouped)
    calls = {"n": 0}
    try:
        hm = bw.HookManager(model, cfg, callbacks=[cap], moe_routed_layers=blocks)
        proxies = [m for n, m in model.named_modules() if ".dattri_experts." in n and n.endswith("gate_up")]
        handles = [m.register_forward_hook(lambda *_: calls.__setitem__("n", calls["n"] + 1)) for m in proxies]
        model.get_input_embeddings().weight.grad = None
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            with hm.collect():
                _loss(model, ids).backward()
        for h in handles:
            h.remove()
        hm.remove()
    finally:
        set_grouped_experts(previous)
    grad = cap.record.gradient
    data = {n: v.float() for n, v in grad.data.items()}
    return data, model.get_input_embeddings().weight.grad.float().clone(), calls["n"]


def _compare(device, dtype, rtol, atol, proj_dim=4, layers=2):
    model = _model(device, dtype, layers)
    ids = torch.randint(0, 96, (3, 16), generator=torch.Generator().manual_seed(5)).to(device)
    grouped, emb_g, proxy_calls = _capture(model, ids, grouped=True, proj_dim=proj_dim)
    looped, emb_l, loop_calls = _capture(model, ids, grouped=False, proj_dim=proj_dim)
    assert proxy_calls == 0 and loop_calls > 0
    experts = [n for n in grouped if ".dattri_experts." in n]
    assert len(experts) == 2 * E * layers
    for name, want in looped.items():
        _close(grouped[name], want, rtol, atol, name)
    for name in set(experts) - set(looped):  # experts no token reached: zero rows
        assert not grouped[name].any(), name
    _close(emb_g, emb_l, rtol, atol, "embedding")


def _close(got, want, rtol, atol, name):
    if rtol is None:  # bf16: the two paths round differently; compare whole blocks
        err = (got - want).norm() / want.norm().clamp_min(1e-6)
        assert err < atol, f"{name}: relative error {float(err):.3g}"
    else:
        torch.testing.assert_close(got, want, rtol=rtol, atol=atol, msg=name)


def test_grouped_expert_capture_matches_per_expert_capture_cpu():
    _compare("cpu", torch.float32, rtol=1e-4, atol=1e-5)


def test_grouped_path_steps_aside_for_trainable_experts():
    model = _model("cpu", torch.float32)
    model.model.layers[0].mlp.experts.requires_grad_(True)
    ids = torch.randint(0, 96, (2, 16), generator=torch.Generator().manual_seed(6))
    _data, _emb, proxy_calls = _capture(model, ids, grouped=True)
    assert proxy_calls > 0  # layer 0 took the per-expert loop


@pytest.mark.gpu
def test_grouped_expert_capture_matches_per_expert_capture_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    # one block: in bf16 a second block's routing can flip on near-tied router scores, since
    # the two paths round the first block's output differently (fp32 vs bf16 combine sums)
    _compare("cuda", torch.bfloat16, rtol=None, atol=3e-2, proj_dim=16, layers=1)


def test_exact_row_positions_pair_repeated_rows_in_order():
    from dattri_llm_b200.gradient.hooks.routing import _exact_positions

    grid = torch.tensor([[1.0, 2.0], [0.0, 0.0], [3.0, 4.0], [0.0, 0.0], [5.0, 6.0]])
    picks = torch.tensor([4, 1, 0, 3])  # two identical zero rows among them
    got = _exact_positions(grid[picks], grid)
    assert got.tolist() == [4, 1, 0, 3]
    assert _exact_positions(torch.tensor([[9.0, 9.0]]), grid) is None  # a row the grid does not hold
    three_zeros = torch.zeros(3, 2)
    assert _exact_positions(three_zeros, grid) is None  # more copies than the grid has
