"""Capture on state-space and linear-attention model families (CPU, float64, tiny random
configs of every family the installed Transformers provides): while the manager collects,
the sequence-mixer overrides leave the model's output unchanged, and every ``nn.Linear``
the default configuration captures (the mixers' projections included) holds each
sample's exact gradient, against per-sample autograd; layers that share one weight (an
embedding and the head tied to it) sum to that weight's per-sample gradient."""

from __future__ import annotations

import warnings

import pytest
import torch
import torch.nn.functional as F
from torch import nn

import dattri_llm_b200 as bw
from dattri_llm_b200.gradient import ops

transformers = pytest.importorskip("transformers")
warnings.filterwarnings("ignore")

VOCAB, B, T = 48, 3, 12


def _build(name: str):
    t = transformers
    common = {"vocab_size": VOCAB, "use_cache": False}
    if name == "mamba":
        cfg = t.MambaConfig(hidden_size=16, state_size=4, num_hidden_layers=2, expand=2, conv_kernel=3,
                            time_step_rank=2, use_mambapy=False, **common)
        return t.MambaForCausalLM(cfg)
    if name == "falcon_mamba":
        cfg = t.FalconMambaConfig(hidden_size=16, state_size=4, num_hidden_layers=2, expand=2, conv_kernel=3,
                                  time_step_rank=2, **common)
        return t.FalconMambaForCausalLM(cfg)
    if name == "rwkv":
        cfg = t.RwkvConfig(hidden_size=16, attention_hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                           context_length=32, **common)
        return t.RwkvForCausalLM(cfg)
    if name == "lfm2":
        cfg = t.Lfm2Config(hidden_size=32, intermediate_size=32, num_hidden_layers=2, num_attention_heads=2,
                           num_key_value_heads=2, layer_types=["conv", "full_attention"], conv_L_cache=3, **common)
        return t.Lfm2ForCausalLM(cfg)
    if name == "zamba":
        cfg = t.ZambaConfig(hidden_size=16, intermediate_size=32, num_hidden_layers=4,
                            layers_block_type=["mamba", "hybrid", "mamba", "hybrid"], num_attention_heads=2,
                            num_key_value_heads=2, mamba_d_state=4, mamba_d_conv=4, mamba_expand=2,
                            mamba_dt_rank=2, n_mamba_heads=1, use_mamba_kernels=False, **common)
        return t.ZambaForCausalLM(cfg)
    if name == "jamba":
        cfg = t.JambaConfig(hidden_size=16, intermediate_size=32, num_hidden_layers=2, num_attention_heads=2,
                            num_key_value_heads=2, num_experts=2, num_experts_per_tok=1, expert_layer_period=2,
                            expert_layer_offset=1, attn_layer_period=2, attn_layer_offset=1, mamba_d_state=4,
                            mamba_d_conv=3, mamba_expand=2, mamba_dt_rank=2, use_mamba_kernels=False, **common)
        return t.JambaForCausalLM(cfg)
    if name == "bamba":
        cfg = t.BambaConfig(hidden_size=16, intermediate_size=32, num_hidden_layers=2, num_attention_heads=2,
                            num_key_value_heads=2, attn_layer_indices=[1], mamba_n_heads=4, mamba_d_head=8,
                            mamba_n_groups=1, mamba_d_state=4, mamba_d_conv=3, mamba_expand=2, mamba_chunk_size=4,
                            **common)
        return t.BambaForCausalLM(cfg)
    if name == "zamba2":
        cfg = t.Zamba2Config(hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                             layers_block_type=["mamba", "hybrid"], num_attention_heads=2, num_key_value_heads=2,
                             mamba_d_state=4, mamba_d_conv=3, mamba_expand=2, mamba_headdim=8, mamba_ngroups=1,
                             n_mamba_heads=4, chunk_size=4, use_mem_rope=False, **common)
        return t.Zamba2ForCausalLM(cfg)
    if name == "falcon_h1":
        cfg = t.FalconH1Config(hidden_size=16, intermediate_size=32, num_hidden_layers=2, num_attention_heads=2,
                               num_key_value_heads=2, mamba_d_ssm=32, mamba_n_heads=4, mamba_d_head=8,
                               mamba_n_groups=1, mamba_d_state=4, mamba_d_conv=3, mamba_expand=2,
                               mamba_chunk_size=4, **common)
        return t.FalconH1ForCausalLM(cfg)
    if name == "qwen3_next":
        cfg = t.Qwen3NextConfig(hidden_size=16, intermediate_size=32, num_hidden_layers=2, num_attention_heads=2,
                                num_key_value_heads=2, head_dim=8, linear_num_value_heads=2, linear_num_key_heads=2,
                                linear_key_head_dim=8, linear_value_head_dim=8, linear_conv_kernel_dim=3,
                                num_experts=2, num_experts_per_tok=1, moe_intermediate_size=16,
                                shared_expert_intermediate_size=16,
                                layer_types=["linear_attention", "full_attention"], **common)
        return t.Qwen3NextForCausalLM(cfg)
    if name == "nemotron_h":
        cfg = t.NemotronHConfig(hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                                hybrid_override_pattern="M*", num_attention_heads=2, num_key_value_heads=2,
                                head_dim=8, mamba_num_heads=4, mamba_head_dim=8, n_groups=1, ssm_state_size=4,
                                conv_kernel=3, expand=2, chunk_size=4, **common)
        return t.NemotronHForCausalLM(cfg)
    if name == "granitemoehybrid":
        cfg = t.GraniteMoeHybridConfig(hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                                       num_attention_heads=2, num_key_value_heads=2, layer_types=["mamba", "attention"],
                                       mamba_n_heads=4, mamba_d_head=8, mamba_n_groups=1, mamba_d_state=4,
                                       mamba_d_conv=3, mamba_expand=2, mamba_chunk_size=4, num_local_experts=2,
                                       num_experts_per_tok=1, shared_intermediate_size=16, **common)
        return t.GraniteMoeHybridForCausalLM(cfg)
    raise ValueError(name)


FAMILIES = ["mamba", "falcon_mamba", "rwkv", "lfm2", "zamba", "jamba", "bamba", "zamba2", "falcon_h1", "qwen3_next",
            "nemotron_h", "granitemoehybrid"]


def _model(name: str) -> nn.Module:
    torch.manual_seed(0)
    try:
        model = _build(name)
    except (AttributeError, TypeError, ValueError) as exc:  # not in this Transformers version
        pytest.skip(f"{name}: {exc}")
    if hasattr(model.config, "_experts_implementation"):
        model.config._experts_implementation = "eager"  # the grouped-GEMM experts take no float64
    return model.double().eval()


def _loss(model, ids):
    logits = model(input_ids=ids).logits
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1), reduction="sum")


def _linear_layout(m: nn.Linear) -> torch.Tensor:
    w = m.weight.grad
    return torch.cat([w, m.bias.grad[:, None]], 1) if m.bias is not None else w


@pytest.mark.parametrize("name", FAMILIES)
def test_family_capture_matches_per_sample_autograd(name):
    model = _model(name)
    ids = torch.randint(0, VOCAB, (B, T), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want_out = model(input_ids=ids).logits
    from dattri_llm_b200.gradient.hooks.override_layers.fused_experts import find_fused_experts

    # MoE blocks (Jamba, Qwen3-Next, GraniteMoeHybrid) are declared so their rows regroup per
    # sample; Granite's parallel experts (3-D weights) are batch-level parameter captures
    moe = {n.rpartition(".")[0] for n in find_fused_experts(model)}
    moe = sorted(moe | {n for n, _ in model.named_modules() if n.endswith("block_sparse_moe")})
    cap = bw.CaptureCallback()
    hm = bw.HookManager(model, bw.HookManagerConfig(), callbacks=[cap], moe_routed_layers=moe or None)
    with hm.collect():
        out = model(input_ids=ids).logits
        torch.testing.assert_close(out, want_out, rtol=1e-10, atol=1e-10)  # the overrides keep the math
        F.cross_entropy(out[:, :-1].reshape(-1, VOCAB), ids[:, 1:].reshape(-1), reduction="sum").backward()
    hm.remove()
    model.zero_grad(set_to_none=True)
    grad = cap.record.gradient
    owners: dict[int, list[str]] = {}
    for n, m in model.named_modules(remove_duplicate=False):
        w = getattr(m, "weight", None)
        if isinstance(w, nn.Parameter):
            owners.setdefault(id(w), []).append(n)
    # a weight shared with another module (a tied head) is checked through the tied sum below
    linears = {n: m for n, m in model.named_modules()
               if isinstance(m, nn.Linear) and n in grad.data and len(owners[id(m.weight)]) == 1}
    tied = [names for names in owners.values() if len(names) > 1 and all(n in grad.data for n in names)]
    assert linears, f"{name}: no linear layer captured"
    per = {n: [] for n in linears}
    per_tied = [[] for _ in tied]
    modules = dict(model.named_modules(remove_duplicate=False))
    for i in range(B):
        model.zero_grad(set_to_none=True)
        _loss(model, ids[i:i + 1]).backward()
        for n, m in linears.items():
            per[n].append(_linear_layout(m).detach().clone())
        for j, names in enumerate(tied):
            per_tied[j].append(modules[names[0]].weight.grad.detach().clone())
    model.zero_grad(set_to_none=True)
    for names, rows in zip(tied, per_tied, strict=True):
        # e.g. an embedding and the head tied to it: the two captures sum to the weight's gradient
        want = torch.stack(rows).reshape(B, -1)
        got = sum(ops.materialize(grad.data[n], grad.layer_types[n], include_bias=False).reshape(B, -1)
                  for n in names)
        torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-8 * float(want.abs().max()), msg=str(names))
    for n in linears:
        want = torch.stack(per[n]).reshape(B, -1)
        got = ops.materialize(grad.data[n], grad.layer_types[n]).reshape(B, -1)
        scale = float(want.abs().max()) or 1.0
        torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-8 * scale, msg=f"{name}: {n}")
