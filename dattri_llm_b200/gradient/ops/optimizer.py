"""Per-sample optimizer update directions and AdamW-influence Jacobian pieces.

:func:`precondition` returns the direction ``torch.optim`` would take from a
per-sample gradient given the optimizer's state before the step (LESS's
``Gamma``); the update rules are those of ``torch.optim`` and the state keys are
its state-dict keys (parity: reference ``dattri_llm/gradient/ops/optimizer.py``).
On an sm_100 device the Adam/AdamW rule -- the one LESS-style capture uses on
every hooked layer and sample -- is one fused elementwise kernel over the
``(B, k)`` block (:func:`dattri_llm_b200.ops.adam_direction`).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Mapping

import torch

#: Per ``torch.optim`` optimizer, the state keys its preconditioning reads.
OPTIMIZER_STATE_KEYS: dict[str, tuple[str, ...]] = {
    "SGD": ("momentum_buffer",),
    "Adam": ("exp_avg", "exp_avg_sq", "max_exp_avg_sq"),
    "AdamW": ("exp_avg", "exp_avg_sq", "max_exp_avg_sq"),
    "Adamax": ("exp_avg", "exp_inf"),
    "NAdam": ("exp_avg", "exp_avg_sq", "mu_product"),
    "RAdam": ("exp_avg", "exp_avg_sq"),
    "RMSprop": ("square_avg", "grad_avg", "momentum_buffer"),
    "Adagrad": ("sum",),
    "Adadelta": ("square_avg", "acc_delta"),
    "Lion": ("exp_avg",),
}

_DEFAULTS: dict[str, dict[str, object]] = {
    "SGD": {"momentum": 0.0, "dampening": 0.0, "nesterov": False},
    "Adam": {"betas": (0.9, 0.999), "eps": 1e-8, "amsgrad": False},
    "AdamW": {"betas": (0.9, 0.999), "eps": 1e-8, "amsgrad": False},
    "Adamax": {"betas": (0.9, 0.999), "eps": 1e-8},
    "NAdam": {"betas": (0.9, 0.999), "eps": 1e-8, "momentum_decay": 4e-3},
    "RAdam": {"betas": (0.9, 0.999), "eps": 1e-8},
    "RMSprop": {"alpha": 0.99, "eps": 1e-8, "momentum": 0.0, "centered": False},
    "Adagrad": {"eps": 1e-10, "lr_decay": 0.0},
    "Adadelta": {"rho": 0.9, "eps": 1e-6},
    "Lion": {"betas": (0.9, 0.99)},
}


def _state(g: torch.Tensor, state: Mapping, key: str) -> torch.Tensor:
    v = state.get(key)
    if v is None:
        return torch.zeros(g.shape[-1], device=g.device, dtype=g.dtype)
    return v.to(g.device, g.dtype)


def _ema(prev, x, beta):
    return beta * prev + (1.0 - beta) * x


def _sgd(g, state, step, hp):
    mu = float(hp["momentum"])
    if not mu:
        return g
    buf = state.get("momentum_buffer")
    new = g if buf is None else mu * buf.to(g.device, g.dtype) + (1.0 - hp["dampening"]) * g
    return g + mu * new if hp["nesterov"] else new


def _adam(g, state, step, hp):
    b1, b2 = hp["betas"]
    from dattri_llm_b200 import ops as native_ops

    if (native_ops.use_native(g) and not hp["amsgrad"] and state.get("exp_avg") is not None
            and state.get("exp_avg_sq") is not None and g.shape[-1] % 4 == 0
            and state["exp_avg"].numel() == g.shape[-1] == state["exp_avg_sq"].numel()):
        return native_ops.adam_direction(g, state["exp_avg"], state["exp_avg_sq"], step=step,
                                         beta1=b1, beta2=b2, eps=hp["eps"])
    m = _ema(_state(g, state, "exp_avg"), g, b1)
    v = _ema(_state(g, state, "exp_avg_sq"), g * g, b2)
    if hp["amsgrad"]:
        v = torch.maximum(_state(g, state, "max_exp_avg_sq"), v)
    return m / (1.0 - b1**step) / (v.sqrt() / math.sqrt(1.0 - b2**step) + hp["eps"])


def _adamax(g, state, step, hp):
    b1, b2 = hp["betas"]
    m = _ema(_state(g, state, "exp_avg"), g, b1)
    u = torch.maximum(b2 * _state(g, state, "exp_inf"), g.abs() + hp["eps"])
    return m / ((1.0 - b1**step) * u)


def _nadam(g, state, step, hp):
    b1, b2 = hp["betas"]
    decay = float(hp["momentum_decay"])
    mu = b1 * (1.0 - 0.5 * 0.96 ** (step * decay))
    mu_next = b1 * (1.0 - 0.5 * 0.96 ** ((step + 1) * decay))
    prod = state.get("mu_product")
    prod = (1.0 if prod is None else float(prod)) * mu
    m = _ema(_state(g, state, "exp_avg"), g, b1)
    v = _ema(_state(g, state, "exp_avg_sq"), g * g, b2)
    denom = (v / (1.0 - b2**step)).sqrt() + hp["eps"]
    return ((1.0 - mu) / (1.0 - prod)) * g / denom + (mu_next / (1.0 - prod * mu_next)) * m / denom


def _radam(g, state, step, hp):
    b1, b2 = hp["betas"]
    m = _ema(_state(g, state, "exp_avg"), g, b1)
    v = _ema(_state(g, state, "exp_avg_sq"), g * g, b2)
    bc2 = 1.0 - b2**step
    m_hat = m / (1.0 - b1**step)
    rho_inf = 2.0 / (1.0 - b2) - 1.0
    rho_t = rho_inf - 2.0 * step * b2**step / bc2
    if rho_t <= 5.0:
        return m_hat
    rect = math.sqrt((rho_t - 4.0) * (rho_t - 2.0) * rho_inf / ((rho_inf - 4.0) * (rho_inf - 2.0) * rho_t))
    return m_hat * rect * math.sqrt(bc2) / (v.sqrt() + hp["eps"])


def _rmsprop(g, state, step, hp):
    alpha = float(hp["alpha"])
    v = _ema(_state(g, state, "square_avg"), g * g, alpha)
    if hp["centered"]:
        ga = _ema(_state(g, state, "grad_avg"), g, alpha)
        avg = (v - ga * ga).sqrt() + hp["eps"]
    else:
        avg = v.sqrt() + hp["eps"]
    direction = g / avg
    mu = float(hp["momentum"])
    return mu * _state(g, state, "momentum_buffer") + direction if mu > 0.0 else direction


def _adagrad(g, state, step, hp):
    total = _state(g, state, "sum") + g * g
    return g / (total.sqrt() + hp["eps"]) / (1.0 + (step - 1) * hp["lr_decay"])


def _adadelta(g, state, step, hp):
    rho, eps = float(hp["rho"]), float(hp["eps"])
    v = _ema(_state(g, state, "square_avg"), g * g, rho)
    return (_state(g, state, "acc_delta") + eps).sqrt() / (v + eps).sqrt() * g


def _lion(g, state, step, hp):
    return torch.sign(_ema(_state(g, state, "exp_avg"), g, hp["betas"][0]))


_RULES: dict[str, Callable] = {
    "SGD": _sgd, "Adam": _adam, "AdamW": _adam, "Adamax": _adamax, "NAdam": _nadam,
    "RAdam": _radam, "RMSprop": _rmsprop, "Adagrad": _adagrad, "Adadelta": _adadelta,
    "Lion": _lion,
}


def precondition(g: torch.Tensor, state: Mapping, *, optimizer_type: str, step: int,
                 **hyperparameters: object) -> torch.Tensor:
    """The per-sample update direction ``torch.optim`` would take from *g* (rows of
    ``(B, k)``) at *step* (the update about to run, >= 1), given the pre-step state.

    Raises:
        NotImplementedError: for an optimizer without a rule.
        ValueError: for ``step < 1``.
    """
    rule = _RULES.get(optimizer_type)
    if rule is None:
        raise NotImplementedError(
            f"precondition has no rule for optimizer type {optimizer_type!r}; supported: "
            f"{sorted(_RULES)}.",
        )
    if step < 1:
        raise ValueError(f"step must be >= 1 (the update about to run), got {step}.")
    hp = {**_DEFAULTS[optimizer_type], **hyperparameters}
    return rule(g.float(), state, int(step), hp)


def adam_preconditioner(m_hat: torch.Tensor, v_hat: torch.Tensor, *, eps: float = 1e-8):
    """Diagonals ``D = 1/(sqrt(v) + eps)`` and ``S = m / (2 sqrt(v) (sqrt(v) + eps)^2)`` of
    AdamW-influence's transition (``S = 0`` where ``v = 0``)."""
    root = torch.sqrt(v_hat.double())
    d = 1.0 / (root + eps)
    denom = 2.0 * root * (root + eps) ** 2
    s = torch.where(root > 0, m_hat.double() / denom.clamp_min(1e-300), 0.0)
    return d.float(), s.float()


def adamw_influence_push(g_z, g_t, d, s, *, lr: float, step: int, beta1: float = 0.9,
                         beta2: float = 0.999) -> torch.Tensor:
    """``Z_push(z) = (theta_dot, m_dot, v_dot)`` for per-sample gradients *g_z* ``(B, p)``."""
    g_z = g_z.float()
    m_dot = -(1.0 - beta1) * g_z
    v_dot = -2.0 * (1.0 - beta2) * g_t.float() * g_z
    theta_dot = -lr * (d * m_dot / (1.0 - beta1**step) - s * v_dot / (1.0 - beta2**step))
    return torch.cat([theta_dot, m_dot, v_dot], dim=-1)


def adamw_influence_transition(w_theta, w_m, w_v, d, s, *, lr: float, step: int,
                               beta1: float = 0.9, beta2: float = 0.999,
                               weight_decay: float = 0.0):
    """``W M_t`` for the block-diagonal AdamW transition ``M_t`` (rows of *W* are test sides)."""
    c1 = beta1 / (1.0 - beta1**step)
    c2 = beta2 / (1.0 - beta2**step)
    new_theta = (1.0 - lr * weight_decay) * w_theta
    new_m = w_theta * (-lr * c1 * d)[None, :] + beta1 * w_m
    new_v = w_theta * (lr * c2 * s)[None, :] + beta2 * w_v
    return new_theta, new_m, new_v


def adamw_influence_coupling(w_theta, w_m, w_v, g_z, g_t, d, s, *, lr: float, step: int,
                             beta1: float = 0.9, beta2: float = 0.999) -> torch.Tensor:
    """``W R_t g_z`` for every sample of a batch: ``(B, p)`` against the ``(n, p)`` rows of W."""
    g_z = g_z.float()
    scale = (-lr * (1.0 - beta1) / (1.0 - beta1**step) * d
             + (2.0 * lr * (1.0 - beta2) / (1.0 - beta2**step)) * s * g_t.float())
    r_theta = scale[None, :] * g_z
    r_m = (1.0 - beta1) * g_z
    r_v = 2.0 * (1.0 - beta2) * g_t.float()[None, :] * g_z
    # the three products are one GEMM over the concatenated (theta, m, v) coordinates
    from dattri_llm_b200.ops.gemm import matmul_f32

    return matmul_f32(torch.cat([r_theta, r_m, r_v], dim=1), torch.cat([w_theta, w_m, w_v], dim=1).float(),
                      b_transposed=True)
