"""Per-expert proxies for MoE blocks whose experts are fused 3-D parameters.

Transformers-5 style MoE blocks hold every expert in two stacked parameters
(``gate_up_proj (E, ., .)``, ``down_proj (E, ., .)``) and apply them with batched
kernels, so no per-expert ``nn.Linear`` exists to hook.  While collecting, the
block's forward is replaced by an explicit per-expert loop through
:class:`SliceLinear` proxies (views of expert ``e``'s slice), which the capture
hooks see as ordinary linear layers; a router applied with a functional
``F.linear`` gets a :class:`RouterLinear` proxy the same way.  Gradients still
accumulate into the fused parameters.  Proxy names (``<block>.dattri_experts.<e>.
gate_up`` / ``.down``, ``<router>.dattri_router``) are layer names in the stored
records and match the reference's
(``dattri_llm/gradient/hooks/override_layers/fused_experts.py:59-382``).
"""

from __future__ import annotations

from collections.abc import Callable, Iterator

import torch
from torch import nn
from torch.nn import functional as F

_linear = F.linear
GATE_UP = "gate_up_proj"
DOWN = "down_proj"
PROXY_EXPERTS = "dattri_experts"
PROXY_ROUTER = "dattri_router"
_INDEX_KWARGS = ("top_k_index", "router_indices", "selected_experts", "topk_indices")
_WEIGHT_KWARGS = ("top_k_weights", "routing_weights", "router_scores", "topk_weights")


class SliceLinear(nn.Module):
    """A linear layer whose weight is slice *index* of a fused 3-D parameter."""

    def __init__(self, owner: nn.Module, weight_name: str, index: int, bias_name: str | None = None,
                 *, transposed: bool = False) -> None:
        super().__init__()
        object.__setattr__(self, "_owner", owner)  # not a submodule: no parameter duplication
        self._weight_name, self._bias_name = weight_name, bias_name
        self._index, self._transposed = index, transposed

    @property
    def weight(self) -> torch.Tensor:
        """Expert *index*'s ``(out, in)`` weight view."""
        w = getattr(self._owner, self._weight_name)[self._index]
        return w.transpose(0, 1) if self._transposed else w

    @property
    def bias(self) -> torch.Tensor | None:
        """Expert *index*'s bias view (``None`` without biases)."""
        return None if self._bias_name is None else getattr(self._owner, self._bias_name)[self._index]

    def proxied_parameters(self) -> Iterator[nn.Parameter]:
        """The fused parameters this proxy reads."""
        yield getattr(self._owner, self._weight_name)
        if self._bias_name is not None:
            yield getattr(self._owner, self._bias_name)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _linear(x, self.weight, self.bias)


class RouterLinear(nn.Module):
    """Hookable stand-in for a router applied with ``F.linear`` on its own weight."""

    def __init__(self, router: nn.Module) -> None:
        super().__init__()
        object.__setattr__(self, "_router", router)

    @property
    def weight(self) -> torch.Tensor:
        """The router's weight."""
        return self._router.weight

    @property
    def bias(self) -> torch.Tensor | None:
        """The router's bias, if any."""
        return getattr(self._router, "bias", None)

    def proxied_parameters(self) -> Iterator[nn.Parameter]:
        """The router parameters this proxy reads."""
        yield self._router.weight
        if self.bias is not None:
            yield self.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b = self.bias
        return _linear(x, self.weight.to(x.dtype), None if b is None else b.to(x.dtype))


def is_fused_experts(module: nn.Module) -> bool:
    """Whether *module* holds experts as fused ``gate_up_proj`` / ``down_proj`` 3-D tensors."""
    gu, dn = getattr(module, GATE_UP, None), getattr(module, DOWN, None)
    return (isinstance(gu, torch.Tensor) and isinstance(dn, torch.Tensor) and gu.ndim == 3
            and dn.ndim == 3 and gu.shape[0] == dn.shape[0])


def is_fused_router(module: nn.Module, num_experts: int) -> bool:
    """A leaf module with an ``(E, d)`` weight that is not an ``nn.Linear``."""
    w = getattr(module, "weight", None)
    return (isinstance(w, nn.Parameter) and w.ndim == 2 and w.shape[0] == num_experts
            and not isinstance(module, nn.Linear) and not any(True for _ in module.children()))


def find_fused_experts(root: nn.Module) -> dict[str, nn.Module]:
    """Every fused-experts module under *root*."""
    return {n: m for n, m in root.named_modules() if is_fused_experts(m)}


def _routing_args(args: tuple, kwargs: dict):
    if len(args) >= 2:
        return args[0], args[1]
    index = next((kwargs[k] for k in _INDEX_KWARGS if k in kwargs), None)
    weights = next((kwargs[k] for k in _WEIGHT_KWARGS if k in kwargs), None)
    if len(args) == 1:
        if index is None:
            index = args[0]
        else:
            weights = args[0]
    if index is None or weights is None:
        raise TypeError(
            f"fused experts forward called without recognisable routing arguments: positional "
            f"{len(args)}, keywords {sorted(kwargs)}.",
        )
    return index, weights


def _experts_loop(experts, proxies, x, top_k_index, top_k_weights) -> torch.Tensor:
    """Reference per-expert loop: gather routed rows, gate_up -> model gate -> down, weight,
    scatter-add back."""
    n_exp = len(proxies)
    out = torch.zeros_like(x)
    with torch.no_grad():
        hit = torch.zeros(n_exp + 1, dtype=torch.bool, device=x.device)
        hit[top_k_index.reshape(-1).clamp(max=n_exp)] = True
        experts_hit = hit[:n_exp].nonzero().flatten().tolist()
    for e in experts_hit:
        tok, pos = torch.where(top_k_index == e)
        h = proxies[e]["down"](experts._apply_gate(proxies[e]["gate_up"](x[tok])))
        out.index_add_(0, tok, (h * top_k_weights[tok, pos, None]).to(out.dtype))
    return out


def _override_router(router: nn.Module, proxy: RouterLinear, should_intervene) -> Callable[[], None]:
    original = router.forward

    def patched(x, weight, bias=None):
        return proxy(x) if weight.shape == router.weight.shape else _linear(x, weight, bias)

    def forward(*args, **kwargs):
        if not should_intervene():
            return original(*args, **kwargs)
        F.linear = patched
        try:
            return original(*args, **kwargs)
        finally:
            F.linear = _linear

    router.forward = forward

    def revert():
        del router.forward
        delattr(router, PROXY_ROUTER)

    return revert


def install_fused_experts(root: nn.Module, experts_names: list[str],
                          should_intervene: Callable[[], bool], grouped: Callable | None = None):
    """Attach per-expert proxies and override the forwards while *should_intervene()*.

    *grouped*: ``(experts_name, experts) -> capture`` with a ``try_forward(x, index, weights)``
    that runs the whole block (returning ``None`` when it does not apply); the per-expert
    loop runs otherwise.  Returns ``(proxy_types, reverts)``: ``{proxy_layer_name:
    "nn.Linear"}`` and undo callables.
    """
    modules = dict(root.named_modules())
    types: dict[str, str] = {}
    reverts: list[Callable[[], None]] = []
    for name in experts_names:
        experts = modules[name]
        if not is_fused_experts(experts):
            raise ValueError(f"{name} is not a fused experts module.")
        if hasattr(experts, PROXY_EXPERTS):
            raise RuntimeError(f"{name} already carries fused-expert proxies.")
        n_exp = getattr(experts, GATE_UP).shape[0]
        transposed = bool(getattr(experts, "is_transposed", False))
        has_bias = bool(getattr(experts, "has_bias", False)) and hasattr(experts, GATE_UP + "_bias")
        proxies = nn.ModuleList([nn.ModuleDict({
            "gate_up": SliceLinear(experts, GATE_UP, e, GATE_UP + "_bias" if has_bias else None,
                                   transposed=transposed),
            "down": SliceLinear(experts, DOWN, e, DOWN + "_bias" if has_bias else None,
                                transposed=transposed),
        }) for e in range(n_exp)])
        experts.add_module(PROXY_EXPERTS, proxies)
        for e in range(n_exp):
            types[f"{name}.{PROXY_EXPERTS}.{e}.gate_up"] = "nn.Linear"
            types[f"{name}.{PROXY_EXPERTS}.{e}.down"] = "nn.Linear"
        original = experts.forward
        bulk = grouped(name, experts) if grouped is not None else None

        def forward(*args, _e=experts, _p=proxies, _o=original, _g=bulk, **kwargs):
            if not should_intervene():
                return _o(*args, **kwargs)
            index, weights = _routing_args(args[1:], kwargs)
            if _g is not None:
                out = _g.try_forward(args[0], index, weights)
                if out is not None:
                    return out
            return _experts_loop(_e, _p, args[0], index, weights)

        experts.forward = forward

        def revert(_e=experts):
            del _e.forward
            delattr(_e, PROXY_EXPERTS)

        reverts.append(revert)
        parent_name = name.rpartition(".")[0]
        parent = modules.get(parent_name, root if not parent_name else None)
        if parent is None:
            continue
        for child_name, child in parent.named_children():
            if not is_fused_router(child, n_exp) or hasattr(child, PROXY_ROUTER):
                continue
            proxy = RouterLinear(child)
            child.add_module(PROXY_ROUTER, proxy)
            full = f"{parent_name}.{child_name}" if parent_name else child_name
            types[f"{full}.{PROXY_ROUTER}"] = "nn.Linear"
            reverts.append(_override_router(child, proxy, should_intervene))
            break
    return types, reverts
