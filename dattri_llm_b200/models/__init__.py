"""Model families with B200-tuned implementations: a GPT-2-style decoder and Llama
(``models.llama``).  Every projection is an ``nn.Linear`` and every norm an
``nn.LayerNorm`` / ``nn.RMSNorm``-shaped module, so the capture hooks see them like
any user model."""

from dattri_llm_b200.models.gpt2 import GPT2Config, GPT2LMHeadModel

__all__ = ["GPT2Config", "GPT2LMHeadModel"]
