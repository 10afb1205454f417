"""Model families with B200-tuned implementations: a GPT-2-style decoder (``models.gpt2``)
and Llama (``models.llama``), both built from :class:`TcLinear` projections (tcgen05 GEMMs
with an optional fused LoGra projection tail) and ``nn.LayerNorm`` / ``nn.RMSNorm``-shaped
norms, so the capture hooks see them like any user model.  ``models.mamba2`` accelerates
Hugging Face Mamba2 models in place (a memory-bounded SSD forward, linears on the tcgen05
kernels); :func:`tc_linearize` does the latter for any model."""

from dattri_llm_b200.models.gpt2 import GPT2Config, GPT2LMHeadModel
from dattri_llm_b200.models.layers import TcLinear, tc_linearize
from dattri_llm_b200.models.llama import LlamaConfig, LlamaForCausalLM, LlamaModel, token_sum_loss
from dattri_llm_b200.models.mamba2 import accelerate_mamba2, ssd_chunked

__all__ = ["GPT2Config", "accelerate_mamba2", "ssd_chunked", "GPT2LMHeadModel", "LlamaConfig", "LlamaForCausalLM", "LlamaModel", "TcLinear",
           "tc_linearize", "token_sum_loss"]
