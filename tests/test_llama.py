"""Llama implementation vs Hugging Face's on identical weights; frozen-probe capture."""

import pytest
import torch

from dattri_llm_b200.models.llama import LlamaConfig, LlamaForCausalLM


def _hf_pair(tied=True):
    transformers = pytest.importorskip("transformers")
    cfg = LlamaConfig.tiny(tie_word_embeddings=tied, rope_scaling={
        "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 64})
    hfc = transformers.LlamaConfig(
        vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
        num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
        num_key_value_heads=cfg.num_key_value_heads, rope_theta=cfg.rope_theta,
        max_position_embeddings=cfg.max_position_embeddings, tie_word_embeddings=tied,
        rope_scaling=cfg.rope_scaling, rms_norm_eps=cfg.rms_norm_eps, attn_implementation="eager")
    torch.manual_seed(0)
    hf = transformers.LlamaForCausalLM(hfc).eval()
    ours = LlamaForCausalLM(cfg).eval()
    ours.load_hf_state_dict(hf.state_dict())
    return hf, ours


@pytest.mark.parametrize("tied", [True, False])
def test_logits_match_hf(tied):
    hf, ours = _hf_pair(tied)
    ids = torch.randint(0, 512, (2, 40))
    with torch.no_grad():
        a = hf(input_ids=ids).logits
        b = ours(input_ids=ids).logits
    torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-4)


def test_frozen_probe_reaches_every_layer():
    from dattri_llm_b200 import CaptureCallback, HookManager, HookManagerConfig
    from dattri_llm_b200.models.llama import token_sum_loss

    cfg = LlamaConfig.tiny()
    m = LlamaForCausalLM(cfg, frozen_probe=True)
    m.requires_grad_(False)
    cb = CaptureCallback()
    hm = HookManager(m, HookManagerConfig(linear_io=[r"proj$"], include_frozen=True), callbacks=[cb])
    ids = torch.randint(0, 512, (3, 16))
    with hm.collect():
        token_sum_loss(m, {"input_ids": ids}).backward()
    names = cb.record.gradient.layer_names
    assert len(names) == 7 * cfg.num_hidden_layers
    assert all(p.grad is None for p in m.parameters())
