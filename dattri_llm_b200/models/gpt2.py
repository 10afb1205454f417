"""A GPT-2-style causal LM (learned positions, pre-LayerNorm blocks, GELU MLP, tied head).

Used for the small end-to-end configuration (2 layers, d 128, 4 heads, MLP 512,
vocab 1024).  Attention is ``scaled_dot_product_attention`` (flash / cuDNN kernels
on the GPU).  ``forward(input_ids, attention_mask=None, labels=None)`` returns an
object with ``.logits`` and, given labels, the mean next-token ``.loss``.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class GPT2Config:
    """Hyperparameters of :class:`GPT2LMHeadModel`."""

    vocab_size: int = 1024
    n_positions: int = 256
    n_embd: int = 128
    n_layer: int = 2
    n_head: int = 4
    n_inner: int = 512
    layer_norm_epsilon: float = 1e-5
    tie_word_embeddings: bool = True


class GPT2Attention(nn.Module):
    """Causal multi-head self-attention with separate q/k/v projections."""

    def __init__(self, cfg: GPT2Config) -> None:
        super().__init__()
        self.n_head = cfg.n_head
        self.q_proj = nn.Linear(cfg.n_embd, cfg.n_embd)
        self.k_proj = nn.Linear(cfg.n_embd, cfg.n_embd)
        self.v_proj = nn.Linear(cfg.n_embd, cfg.n_embd)
        self.o_proj = nn.Linear(cfg.n_embd, cfg.n_embd)

    def forward(self, x: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        b, t, d = x.shape
        h = self.n_head
        q = self.q_proj(x).view(b, t, h, d // h).transpose(1, 2)
        k = self.k_proj(x).view(b, t, h, d // h).transpose(1, 2)
        v = self.v_proj(x).view(b, t, h, d // h).transpose(1, 2)
        if attention_mask is None:
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            causal = torch.ones(t, t, dtype=torch.bool, device=x.device).tril()
            mask = causal[None, None] & attention_mask[:, None, None, :].bool()
            y = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return self.o_proj(y.transpose(1, 2).reshape(b, t, d))


class GPT2Block(nn.Module):
    """Pre-LN transformer block."""

    def __init__(self, cfg: GPT2Config) -> None:
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_epsilon)
        self.attn = GPT2Attention(cfg)
        self.ln_2 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_epsilon)
        self.fc_in = nn.Linear(cfg.n_embd, cfg.n_inner)
        self.fc_out = nn.Linear(cfg.n_inner, cfg.n_embd)

    def forward(self, x: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        x = x + self.attn(self.ln_1(x), attention_mask)
        return x + self.fc_out(F.gelu(self.fc_in(self.ln_2(x)), approximate="tanh"))


class GPT2LMHeadModel(nn.Module):
    """GPT-2-style causal language model."""

    def __init__(self, cfg: GPT2Config) -> None:
        super().__init__()
        self.config = cfg
        self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.wpe = nn.Embedding(cfg.n_positions, cfg.n_embd)
        self.h = nn.ModuleList([GPT2Block(cfg) for _ in range(cfg.n_layer)])
        self.ln_f = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_epsilon)
        self.lm_head = nn.Linear(cfg.n_embd, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.wte.weight
        self.apply(self._init)

    @staticmethod
    def _init(m: nn.Module) -> None:
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, std=0.02)
        if isinstance(m, nn.Linear) and m.bias is not None:
            nn.init.zeros_(m.bias)

    def forward(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                labels: torch.Tensor | None = None, **_unused) -> SimpleNamespace:
        t = input_ids.shape[1]
        pos = torch.arange(t, device=input_ids.device)
        x = self.wte(input_ids) + self.wpe(pos)[None]
        for block in self.h:
            x = block(x, attention_mask)
        logits = self.lm_head(self.ln_f(x))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[:, :-1].float().reshape(-1, logits.shape[-1]),
                                   labels[:, 1:].reshape(-1), ignore_index=-100)
        return SimpleNamespace(logits=logits, loss=loss)
