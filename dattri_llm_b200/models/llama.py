"""Llama-architecture decoder (Llama 3 / 3.2 shapes) for attribution on B200.

Module names follow Hugging Face's ``LlamaForCausalLM``
(``model.layers.<i>.self_attn.{q,k,v,o}_proj``, ``mlp.{gate,up,down}_proj``,
``input_layernorm``, ``post_attention_layernorm``, ``model.norm``, ``lm_head``), so a
Hugging Face state dict loads with :meth:`LlamaForCausalLM.load_hf_state_dict`
and every projection is an ``nn.Linear`` the capture hooks see.

B200 execution choices:

* every projection is a :class:`~dattri_llm_b200.models.layers.TcLinear`: its forward and
  input-gradient GEMMs run on the library's tcgen05 CTA-pair kernel, and a LoGra capture
  computes its projections inside those GEMMs;
* attention is ``scaled_dot_product_attention`` with grouped KV heads (no K/V
  repetition in memory);
* RMSNorm and SwiGLU use the library's fused elementwise kernels on sm_100;
* the LM loss never materializes fp32 logits: bf16 logits from one GEMM, then a
  fused kernel computes per-row log-sum-exp and the loss, and in the backward the
  same bf16 buffer is turned into ``dlogits`` in place;
* ``frozen_probe=True`` (attribution at a fixed checkpoint) makes the token
  embeddings the only leaf that requires grad -- the backward then reaches every
  layer's output without computing or all-reducing any parameter gradient.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from torch import nn

from dattri_llm_b200.models.layers import TcLinear


@dataclass
class LlamaConfig:
    """Hyperparameters (Hugging Face field names)."""

    vocab_size: int = 128256
    hidden_size: int = 2048
    intermediate_size: int = 8192
    num_hidden_layers: int = 16
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int | None = None
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = field(default_factory=lambda: {
        "rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192})
    max_position_embeddings: int = 131072
    tie_word_embeddings: bool = True
    initializer_range: float = 0.02

    @property
    def dim_per_head(self) -> int:
        """Head dimension."""
        return self.head_dim or self.hidden_size // self.num_attention_heads

    @classmethod
    def llama_3_2_1b(cls) -> LlamaConfig:
        """Llama-3.2-1B: 16 layers, d 2048, 32 / 8 heads, FFN 8192, vocab 128256, tied head."""
        return cls()

    @classmethod
    def llama_3_8b(cls) -> LlamaConfig:
        """Llama-3-8B: 32 layers, d 4096, 32 / 8 heads, FFN 14336, vocab 128256."""
        return cls(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, rope_scaling=None,
                   max_position_embeddings=8192, tie_word_embeddings=False)

    @classmethod
    def tiny(cls, **kw) -> LlamaConfig:
        """A small configuration for tests."""
        base = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                    num_attention_heads=4, num_key_value_heads=2, rope_scaling=None, max_position_embeddings=512)
        base.update(kw)
        return cls(**base)


def _rope_inv_freq(cfg: LlamaConfig) -> torch.Tensor:
    d = cfg.dim_per_head
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    rs = cfg.rope_scaling
    if rs and rs.get("rope_type", rs.get("type")) == "llama3":
        factor, lo, hi = rs["factor"], rs["low_freq_factor"], rs["high_freq_factor"]
        old = rs["original_max_position_embeddings"]
        lo_wl, hi_wl = old / lo, old / hi
        wl = 2 * math.pi / inv
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        smooth = (old / wl - lo) / (hi - lo)
        mid = (1 - smooth) * scaled / factor + smooth * scaled
        is_mid = (wl >= hi_wl) & (wl <= lo_wl)
        inv = torch.where(is_mid, mid, scaled)
    return inv.float()


class RotaryEmbedding(nn.Module):
    """``cos``/``sin`` tables of the rotate-half RoPE convention."""

    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.register_buffer("inv_freq", _rope_inv_freq(cfg), persistent=False)
        self._cache: dict = {}

    def forward(self, seq_len: int, device, dtype):
        key = (seq_len, str(device), dtype)
        hit = self._cache.get(key)
        if hit is None:
            t = torch.arange(seq_len, device=device, dtype=torch.float32)
            freqs = torch.outer(t, self.inv_freq.to(device))
            emb = torch.cat([freqs, freqs], dim=-1)
            hit = (emb.cos().to(dtype), emb.sin().to(dtype))
            self._cache = {k: v for k, v in self._cache.items() if k[0] == "half"}
            self._cache[key] = hit
        return hit

    def half_tables(self, seq_len: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 ``cos``/``sin`` of the ``(T, d/2)`` distinct angles (the fused RoPE kernel's
        tables; rotate-half repeats each angle in both halves)."""
        key = ("half", seq_len, str(device))
        hit = self._cache.get(key)
        if hit is None:
            t = torch.arange(seq_len, device=device, dtype=torch.float32)
            freqs = torch.outer(t, self.inv_freq.to(device))
            hit = (freqs.cos().contiguous(), freqs.sin().contiguous())
            self._cache[key] = hit
        return hit


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Rotate ``q, k (B, H, T, d)`` by position."""
    cos, sin = cos[None, None], sin[None, None]
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


class RMSNorm(nn.RMSNorm):
    """``nn.RMSNorm`` (so the capture engine recognises it) running the fused sm_100
    kernel on bf16 CUDA inputs."""

    __bw_layer_type__ = "nn.RMSNorm"

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from dattri_llm_b200.ops import fused

        if fused.enabled(x):
            return fused.rms_norm(x, self.weight, self.eps)
        return super().forward(x)


class LlamaAttention(nn.Module):
    """Grouped-query causal self-attention."""

    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        d, hd = cfg.hidden_size, cfg.dim_per_head
        self.n_heads, self.n_kv, self.head_dim = cfg.num_attention_heads, cfg.num_key_value_heads, hd
        self.q_proj = TcLinear(d, self.n_heads * hd, bias=False)
        self.k_proj = TcLinear(d, self.n_kv * hd, bias=False)
        self.v_proj = TcLinear(d, self.n_kv * hd, bias=False)
        self.o_proj = TcLinear(self.n_heads * hd, d, bias=False)

    def forward(self, x: torch.Tensor, cos, sin, attention_mask: torch.Tensor | None = None,
                half_tables: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
        from dattri_llm_b200.ops import fused

        b, t, _ = x.shape
        q = self.q_proj(x).view(b, t, self.n_heads, self.head_dim)
        k = self.k_proj(x).view(b, t, self.n_kv, self.head_dim)
        v = self.v_proj(x).view(b, t, self.n_kv, self.head_dim).transpose(1, 2)
        if (half_tables is not None and fused.rope_enabled(q) and fused.rope_enabled(k)
                and (self.n_heads + self.n_kv) * self.head_dim // 16 <= 1024):
            q, k = fused.rope(q, k, *half_tables)
            q, k = q.transpose(1, 2), k.transpose(1, 2)
        else:
            q, k = apply_rope(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
        gqa = self.n_kv != self.n_heads
        if attention_mask is None:
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=gqa)
        else:
            causal = torch.ones(t, t, dtype=torch.bool, device=x.device).tril()
            mask = causal[None, None] & attention_mask[:, None, None, :].bool()
            y = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, enable_gqa=gqa)
        return self.o_proj(y.transpose(1, 2).reshape(b, t, -1))


class LlamaMLP(nn.Module):
    """SwiGLU feed-forward ``down(silu(gate(x)) * up(x))``."""

    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.gate_proj = TcLinear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = TcLinear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = TcLinear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from dattri_llm_b200.ops import fused

        g, u = self.gate_proj(x), self.up_proj(x)
        h = fused.swiglu(g, u) if fused.enabled(g) else F.silu(g) * u
        return self.down_proj(h)


class LlamaDecoderLayer(nn.Module):
    """Pre-norm attention + MLP block."""

    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.self_attn = LlamaAttention(cfg)
        self.mlp = LlamaMLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)

    def forward(self, x, cos, sin, attention_mask=None):
        x = x + self.self_attn(self.input_layernorm(x), cos, sin, attention_mask)
        return x + self.mlp(self.post_attention_layernorm(x))

    def forward_fused(self, x, pending, cos, sin, attention_mask=None, half_tables=None):
        """The block with each residual add fused into the RMSNorm that reads it: returns
        ``(h, m)`` whose sum is the block's output (the next block, or the final norm, adds
        them).  *pending* is the previous block's ``m`` (``None`` for the first block)."""
        from dattri_llm_b200.ops import fused

        ln1, ln2 = self.input_layernorm, self.post_attention_layernorm
        if pending is None:
            n1, h0 = ln1(x), x
        else:
            n1, h0 = fused.add_rms_norm(x, pending, ln1.weight, ln1.eps)
        a = self.self_attn(n1, cos, sin, attention_mask, half_tables)
        n2, h = fused.add_rms_norm(h0, a, ln2.weight, ln2.eps)
        return h, self.mlp(n2)


class LlamaModel(nn.Module):
    """Embeddings, decoder stack and final norm."""

    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([LlamaDecoderLayer(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)
        self.rotary_emb = RotaryEmbedding(cfg)


class LlamaForCausalLM(nn.Module):
    """Llama causal LM.

    Args:
        cfg: :class:`LlamaConfig`.
        frozen_probe: With every parameter frozen, start the autograd graph at the
            token embeddings so the backward still reaches every layer (attribution
            at a fixed checkpoint needs layer output gradients, not weight gradients).
    """

    def __init__(self, cfg: LlamaConfig, *, frozen_probe: bool = False) -> None:
        super().__init__()
        self.config = cfg
        self.frozen_probe = frozen_probe
        self.model = LlamaModel(cfg)
        self.lm_head = TcLinear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, seed: int | None = None) -> None:
        """Random init (normal, std ``initializer_range``), optionally seeded.  The values are
        drawn on the device the weights live on (a seeded draw is reproducible per device
        type: CPU-built and CUDA-built models differ)."""
        gens: dict = {}
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                dev = m.weight.device
                if seed is not None and dev not in gens:
                    gens[dev] = torch.Generator(device=dev).manual_seed(seed)
                w = torch.empty(m.weight.shape, dtype=torch.float32, device=dev)
                w.normal_(0.0, self.config.initializer_range, generator=gens.get(dev))
                m.weight.copy_(w)
            elif isinstance(m, nn.RMSNorm):
                m.weight.fill_(1.0)

    def get_input_embeddings(self) -> nn.Embedding:
        """The token embedding (Hugging Face name)."""
        return self.model.embed_tokens

    def get_output_embeddings(self) -> nn.Linear:
        """The LM head (Hugging Face name)."""
        return self.lm_head

    def load_hf_state_dict(self, state_dict: dict) -> None:
        """Load a Hugging Face ``LlamaForCausalLM`` state dict (same key names)."""
        sd = {k: v for k, v in state_dict.items() if "rotary_emb" not in k}
        if self.config.tie_word_embeddings:
            sd.pop("lm_head.weight", None)
        missing, unexpected = self.load_state_dict(sd, strict=False)
        missing = [m for m in missing if not (self.config.tie_word_embeddings and m == "lm_head.weight")]
        if missing or unexpected:
            raise KeyError(f"state dict mismatch: missing {missing[:5]}, unexpected {unexpected[:5]}")

    def hidden_states(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        """Final-norm hidden states ``(B, T, d)``."""
        x = self.model.embed_tokens(input_ids)
        if self.frozen_probe and torch.is_grad_enabled() and not x.requires_grad:
            x = x.detach().requires_grad_(True)
        cos, sin = self.model.rotary_emb(input_ids.shape[1], x.device, x.dtype)
        if not self._fused_blocks(x):
            for layer in self.model.layers:
                x = layer(x, cos, sin, attention_mask)
            return self.model.norm(x)
        half = self.model.rotary_emb.half_tables(input_ids.shape[1], x.device)
        pending = None
        for layer in self.model.layers:
            x, pending = layer.forward_fused(x, pending, cos, sin, attention_mask, half)
        if pending is None:
            return self.model.norm(x)
        from dattri_llm_b200.ops import fused

        norm = self.model.norm
        return fused.add_rms_norm(x, pending, norm.weight, norm.eps)[0]

    def _fused_blocks(self, x: torch.Tensor) -> bool:
        """Fused residual/norm blocks apply to bf16 sm_100 activations when no hook watches
        a norm module or a decoder block (a capture of those layers needs their calls)."""
        from dattri_llm_b200.ops import fused

        if not fused.enabled(x) or x.shape[-1] > 4096:
            return False
        watched = (self.model.norm, *(m for layer in self.model.layers
                                      for m in (layer, layer.input_layernorm, layer.post_attention_layernorm)))
        return not any(m._forward_hooks or m._forward_pre_hooks or m._backward_hooks or m._backward_pre_hooks
                       for m in watched)

    def forward(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                labels: torch.Tensor | None = None, *, loss_reduction: str = "mean",
                return_logits: bool = True, **_unused) -> SimpleNamespace:
        """``.logits`` (unless ``return_logits=False``) and, with labels, the next-token
        ``.loss`` (``loss_reduction`` ``"mean"`` or ``"sum"``; ``-100`` labels ignored)."""
        h = self.hidden_states(input_ids, attention_mask)
        if labels is not None and not return_logits:
            return SimpleNamespace(logits=None, loss=self.lm_loss(h, labels, loss_reduction))
        logits = self.lm_head(h)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[:, :-1].float().reshape(-1, logits.shape[-1]),
                                   labels[:, 1:].reshape(-1), ignore_index=-100, reduction=loss_reduction)
        return SimpleNamespace(logits=logits, loss=loss)

    def lm_loss(self, h: torch.Tensor, labels: torch.Tensor, reduction: str = "sum") -> torch.Tensor:
        """Next-token cross-entropy of hidden states *h* without fp32 logits."""
        from dattri_llm_b200.ops import fused

        hs = h[:, :-1].reshape(-1, h.shape[-1])
        tgt = labels[:, 1:].reshape(-1)
        if fused.enabled(hs):
            total = fused.linear_cross_entropy(hs, self.lm_head.weight, tgt)
        else:
            total = F.cross_entropy(self.lm_head(hs).float(), tgt, ignore_index=-100, reduction="sum")
        if reduction == "sum":
            return total
        return total / (tgt != -100).sum().clamp_min(1)


def token_sum_loss(model: nn.Module, batch: dict) -> torch.Tensor:
    """Token-summed next-token loss of a batch ``{"input_ids", ["attention_mask"]}`` (the
    attribution loss: per-sample gradients of a sum are each sample's own gradient)."""
    ids = batch["input_ids"]
    mask = batch.get("attention_mask")
    labels = ids if mask is None else ids.masked_fill(mask == 0, -100)
    inner = getattr(model, "module", model)
    if isinstance(inner, LlamaForCausalLM):
        return model(input_ids=ids, attention_mask=mask, labels=labels, loss_reduction="sum",
                     return_logits=False).loss
    out = model(input_ids=ids, attention_mask=mask)
    logits = out.logits if hasattr(out, "logits") else out
    return F.cross_entropy(logits[:, :-1].float().reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1),
                           ignore_index=-100, reduction="sum")
