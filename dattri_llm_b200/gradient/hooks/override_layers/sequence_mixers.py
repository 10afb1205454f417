"""Route state-space mixers' functional projections through their modules while collecting.

Mamba-family mixers in Transformers call fused kernels (``causal_conv1d_fn``, the
``*inner_fn`` / ``split_conv1d_scan_combined`` scans) that read the convolution
and projection weights directly, so hooks on ``conv1d`` / ``in_proj`` /
``out_proj`` never fire.  While collecting:

* Mamba-1 mixers (``MambaMixer``, ``FalconMambaMixer``, ``JambaMambaMixer``) run
  :func:`mamba1_reference_forward`, a module-by-module forward;
* other mixers with a depthwise ``nn.Conv1d`` and a functional conv path (Mamba2
  and its hybrids, gated delta-nets) get their modelling module's fast-path flag
  off, the fused scans disabled, and ``causal_conv1d_fn`` redirected to the
  mixer's own ``conv1d`` module.

Decoding steps (a cache with previous state) keep the original forward.
Parity: reference ``dattri_llm/gradient/hooks/override_layers/sequence_mixers.py``.
"""

from __future__ import annotations

import sys
from collections.abc import Callable

import torch
from torch import nn
from torch.nn import functional as F

from dattri_llm_b200.gradient.hooks.override_layers._forward_slot import swap_forward

MAMBA1_MIXER_CLASSES: set[str] = {"MambaMixer", "FalconMambaMixer", "JambaMambaMixer"}
_MAMBA1_ATTRS = ("in_proj", "conv1d", "x_proj", "dt_proj", "out_proj", "A_log", "D", "act",
                 "time_step_rank", "ssm_state_size")
_CONV_FN = "causal_conv1d_fn"
_FUSED_SUFFIXES = ("inner_fn", "split_conv1d_scan_combined")
_FAST_FLAG = "is_fast_path_available"


def _modeling(module: nn.Module):
    return sys.modules.get(type(module).__module__)


def is_mamba1_mixer(module: nn.Module) -> bool:
    """A Mamba-1 style mixer with every attribute the reference forward uses."""
    return type(module).__name__ in MAMBA1_MIXER_CLASSES and all(hasattr(module, a) for a in _MAMBA1_ATTRS)


def _depthwise(module: nn.Module) -> dict[int, nn.Conv1d]:
    return {c.weight.data_ptr(): c for c in module.children()
            if isinstance(c, nn.Conv1d) and c.groups == c.in_channels}


def is_functional_conv_mixer(module: nn.Module) -> bool:
    """A mixer with a depthwise conv whose modelling module has a functional conv path."""
    if is_mamba1_mixer(module) or not _depthwise(module):
        return False
    mod = _modeling(module)
    return mod is not None and (callable(getattr(mod, _CONV_FN, None)) or hasattr(mod, _FAST_FLAG))


def find_sequence_mixers(root: nn.Module) -> dict[str, nn.Module]:
    """Every mixer under *root* an override serves."""
    return {n: m for n, m in root.named_modules() if is_mamba1_mixer(m) or is_functional_conv_mixer(m)}


def mamba1_reference_forward(mixer: nn.Module, hidden_states: torch.Tensor,
                             attention_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Module-by-module Mamba-1 forward (sequential selective scan)."""
    b, length, _ = hidden_states.shape
    dtype = hidden_states.dtype
    if attention_mask is not None:
        hidden_states = hidden_states * attention_mask.unsqueeze(-1).to(dtype)
    x, gate = mixer.in_proj(hidden_states).transpose(1, 2).chunk(2, dim=1)
    if attention_mask is not None:
        x = x * attention_mask.unsqueeze(1).to(dtype)
    x = mixer.act(mixer.conv1d(x)[..., :length])
    if attention_mask is not None:
        x = x * attention_mask.unsqueeze(1).to(dtype)
    ts, bm, cm = torch.split(mixer.x_proj(x.transpose(1, 2)),
                             [mixer.time_step_rank, mixer.ssm_state_size, mixer.ssm_state_size], dim=-1)
    if hasattr(mixer, "dt_layernorm"):
        ts, bm, cm = mixer.dt_layernorm(ts), mixer.b_layernorm(bm), mixer.c_layernorm(cm)
    elif hasattr(mixer, "rms_eps"):
        rms = _modeling(mixer).rms_forward
        ts, bm, cm = (rms(t, variance_epsilon=mixer.rms_eps) for t in (ts, bm, cm))
    dt = F.softplus(mixer.dt_proj(ts)).transpose(1, 2)
    a = -torch.exp(mixer.A_log.float())
    da = torch.exp(a[None, :, None, :] * dt[:, :, :, None])
    dbu = dt[:, :, :, None] * bm[:, None, :, :].float() * x[:, :, :, None].float()
    state = torch.zeros(b, x.shape[1], mixer.ssm_state_size, device=x.device, dtype=dtype)
    ys = []
    for i in range(length):
        state = da[:, :, i, :] * state + dbu[:, :, i, :]
        ys.append(torch.matmul(state.to(dtype), cm[:, i, :].unsqueeze(-1))[:, :, 0])
    y = (torch.stack(ys, dim=-1) + x * mixer.D[None, :, None]) * mixer.act(gate)
    return mixer.out_proj(y.transpose(1, 2))


def _conv_through_module(mixer: nn.Module, original: Callable) -> Callable:
    convs = _depthwise(mixer)

    def conv_fn(x, weight, bias=None, activation=None, **kwargs):
        conv = convs.get(weight.data_ptr())
        if conv is None or x.ndim != 3:
            return original(x, weight, bias, activation, **kwargs)
        out = conv(x.to(conv.weight.dtype))[..., : x.shape[-1]]
        if activation is not None:
            act = getattr(mixer, "act", None) or _modeling(mixer).ACT2FN[activation]
            out = act(out)
        return out.to(x.dtype)

    return conv_fn


_HIDDEN_KWARGS = ("hidden_states", "input_states", "x")


def _hidden(args: tuple, kwargs: dict) -> tuple[torch.Tensor, tuple]:
    """The mixer's input, passed first positionally or by keyword, and the positional
    arguments after it."""
    if args:
        return args[0], args[1:]
    for key in _HIDDEN_KWARGS:
        if key in kwargs:
            return kwargs[key], ()
    raise TypeError(f"sequence mixer called without its input (positional or one of {_HIDDEN_KWARGS})")


def _decoding(mixer, rest, kwargs) -> bool:
    cache = kwargs.get("cache_params", rest[0] if rest else None)
    if cache is None:
        return False
    prev = getattr(cache, "has_previous_state", None)
    if prev is None:
        return True
    if callable(prev):
        try:
            return bool(prev(getattr(mixer, "layer_idx", 0)))
        except TypeError:
            return bool(prev())
    return bool(prev)


def install_sequence_mixer_forward(root: nn.Module, mixer_names: list[str],
                                   should_intervene: Callable[[], bool]) -> list[Callable[[], None]]:
    """Override the named mixers' forwards while *should_intervene()*; returns reverts.

    Raises:
        ValueError: for a module no override serves.
    """
    modules = dict(root.named_modules())
    reverts = []
    for name in mixer_names:
        mixer = modules[name]
        original = mixer.forward
        if is_mamba1_mixer(mixer):
            def forward(*args, _m=mixer, _o=original, **kwargs):
                h, rest = _hidden(args, kwargs)
                if not should_intervene() or _decoding(_m, rest, kwargs):
                    return _o(*args, **kwargs)
                return mamba1_reference_forward(_m, h, kwargs.get("attention_mask"))
        elif is_functional_conv_mixer(mixer):
            def forward(*args, _m=mixer, _o=original, _mod=_modeling(mixer), **kwargs):
                _h, rest = _hidden(args, kwargs)
                if not should_intervene() or _decoding(_m, rest, kwargs):
                    return _o(*args, **kwargs)
                saved = {}
                for attr, value in list(vars(_mod).items()):
                    if attr == _CONV_FN:
                        saved[attr] = value
                        setattr(_mod, attr, _conv_through_module(_m, value))
                    elif callable(value) and attr.endswith(_FUSED_SUFFIXES):
                        saved[attr] = value
                        setattr(_mod, attr, lambda *a, **k: None)
                    elif attr == _FAST_FLAG:
                        saved[attr] = value
                        setattr(_mod, attr, False)
                try:
                    return _o(*args, **kwargs)
                finally:
                    for attr, value in saved.items():
                        setattr(_mod, attr, value)
        else:
            raise ValueError(f"{name} is not a sequence mixer an override serves.")
        reverts.append(swap_forward(mixer, forward))
    return reverts
