"""Model families with B200-tuned implementations: GPT-2-style, Llama, OLMoE (MoE with
expert parallelism) and Mamba2.  Every projection is an ``nn.Linear`` (and norms are
``nn.LayerNorm`` / ``nn.RMSNorm``), so the capture hooks see them like any user model."""

from dattri_llm_b200.models.gpt2 import GPT2Config, GPT2LMHeadModel

__all__ = ["GPT2Config", "GPT2LMHeadModel"]
