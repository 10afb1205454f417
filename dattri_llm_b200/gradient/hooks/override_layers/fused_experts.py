"""Hookable stand-ins for MoE blocks whose experts are fused 3-D parameters.

Transformers-5 MoE blocks keep every expert in two stacked parameters
(``gate_up_proj (E, 2I, H)``, ``down_proj (E, H, I)``) and apply them in bulk, so there is
no per-expert ``nn.Linear`` a capture hook could sit on; the router, too, is often an
``F.linear`` on a bare weight.  While a capture collects, such a block gets:

* per expert, two :class:`SliceLinear` stand-ins (``gate_up`` / ``down``) that read slice
  ``e`` of the fused parameters -- gradients still land in the fused parameters;
* for the router, a :class:`RouterLinear` stand-in that the router's own forward calls in
  place of ``F.linear``;
* a forward that either hands the whole block to a grouped capture (one function for all
  experts, :mod:`.grouped_experts`) or loops over the experts that received tokens,
  feeding each stand-in the rows routed to it and telling the row tracker where those rows
  came from.

Stand-in names -- ``<experts>.dattri_experts.<e>.gate_up`` / ``.down`` and
``<router>.dattri_router`` -- are layer names in stored records, the same as the
reference's (``dattri_llm/gradient/hooks/override_layers/fused_experts.py``), so stores
are interchangeable.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator

import torch
from torch import nn
from torch.nn import functional as F

from dattri_llm_b200.gradient.hooks.override_layers._forward_slot import swap_forward

_F_LINEAR = F.linear
GATE_UP = "gate_up_proj"
DOWN = "down_proj"
PROXY_EXPERTS = "dattri_experts"
PROXY_ROUTER = "dattri_router"
# keyword spellings of the routing arguments across model families
_INDEX_NAMES = ("top_k_index", "router_indices", "selected_experts", "topk_indices")
_WEIGHT_NAMES = ("top_k_weights", "routing_weights", "router_scores", "topk_weights")


class SliceLinear(nn.Module):
    """A bias-optional linear map whose weight is slice *index* of a fused 3-D parameter of
    *owner* (held by reference, not as a submodule, so no parameter is registered twice)."""

    def __init__(self, owner: nn.Module, weight_name: str, index: int, bias_name: str | None = None,
                 *, transposed: bool = False) -> None:
        super().__init__()
        self.__dict__["_owner"] = owner
        self._names = (weight_name, bias_name)
        self._index, self._transposed = index, transposed

    @property
    def weight(self) -> torch.Tensor:
        """This expert's ``(out, in)`` weight view."""
        w = getattr(self._owner, self._names[0])[self._index]
        return w.t() if self._transposed else w

    @property
    def bias(self) -> torch.Tensor | None:
        """This expert's bias view (``None`` without biases)."""
        name = self._names[1]
        return None if name is None else getattr(self._owner, name)[self._index]

    def proxied_parameters(self) -> Iterator[nn.Parameter]:
        """The fused parameters this stand-in reads."""
        for name in self._names:
            if name is not None:
                yield getattr(self._owner, name)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _F_LINEAR(x, self.weight, self.bias)


class RouterLinear(nn.Module):
    """The router's ``F.linear`` on its own weight, as a hookable module."""

    def __init__(self, router: nn.Module) -> None:
        super().__init__()
        self.__dict__["_router"] = router

    @property
    def weight(self) -> torch.Tensor:
        """The router's weight."""
        return self._router.weight

    @property
    def bias(self) -> torch.Tensor | None:
        """The router's bias, if it has one."""
        return getattr(self._router, "bias", None)

    def proxied_parameters(self) -> Iterator[nn.Parameter]:
        """The router parameters this stand-in reads."""
        yield self._router.weight
        if self.bias is not None:
            yield self.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bias = self.bias
        return _F_LINEAR(x, self.weight.to(x.dtype), None if bias is None else bias.to(x.dtype))


def is_fused_experts(module: nn.Module) -> bool:
    """Whether *module* keeps its experts as fused ``gate_up_proj`` / ``down_proj`` 3-D tensors."""
    up, down = getattr(module, GATE_UP, None), getattr(module, DOWN, None)
    return (isinstance(up, torch.Tensor) and isinstance(down, torch.Tensor) and up.ndim == down.ndim == 3
            and up.shape[0] == down.shape[0])


def is_fused_router(module: nn.Module, num_experts: int) -> bool:
    """A childless, non-``nn.Linear`` module holding an ``(E, d)`` weight parameter."""
    w = getattr(module, "weight", None)
    return (isinstance(w, nn.Parameter) and w.ndim == 2 and w.shape[0] == num_experts
            and not isinstance(module, nn.Linear) and next(module.children(), None) is None)


def find_fused_experts(root: nn.Module) -> dict[str, nn.Module]:
    """Every fused-experts module under *root*."""
    return {n: m for n, m in root.named_modules() if is_fused_experts(m)}


def _routing_arguments(args: tuple, kwargs: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """``(expert index, routing weights)`` from an experts forward's arguments after the
    hidden states (positional, or under any of the families' keyword names)."""
    found = {"index": next((kwargs[k] for k in _INDEX_NAMES if k in kwargs), None),
             "weights": next((kwargs[k] for k in _WEIGHT_NAMES if k in kwargs), None)}
    positional = list(args[:2])
    for slot in ("index", "weights"):
        if found[slot] is None and positional:
            found[slot] = positional.pop(0)
    if found["index"] is None or found["weights"] is None:
        raise TypeError(f"a fused-experts forward was called without recognisable routing arguments "
                        f"({len(args)} positional, keywords {sorted(kwargs)}).")
    return found["index"], found["weights"]


def _loop_over_experts(experts: nn.Module, stand_ins: nn.ModuleList, x: torch.Tensor, index: torch.Tensor,
                       weights: torch.Tensor, place: Callable | None) -> torch.Tensor:
    """The block through the stand-ins: per expert with tokens, its rows through
    ``gate_up`` -> the model's gate -> ``down``, weighted and added back at their tokens."""
    n_experts = len(stand_ins)
    out = torch.zeros_like(x)
    with torch.no_grad():
        used = torch.bincount(index.reshape(-1).clamp(max=n_experts), minlength=n_experts + 1)[:n_experts]
        active = used.nonzero().flatten().tolist()  # one host read per block
    for e in active:
        tokens, slots = torch.where(index == e)
        rows = x.index_select(0, tokens)
        if place is not None:
            place(rows, tokens)
        pair = stand_ins[e]
        hidden = pair["down"](experts._apply_gate(pair["gate_up"](rows)))
        out.index_add_(0, tokens, (hidden * weights[tokens, slots, None]).to(out.dtype))
    return out


def _patch_router(router: nn.Module, stand_in: RouterLinear, should_intervene: Callable[[], bool]):
    """Make the router's forward call *stand_in* where it applies ``F.linear`` to its own
    weight (while collecting); returns the undo."""
    original = router.forward

    def linear(x, weight, bias=None):
        return stand_in(x) if weight.shape == router.weight.shape else _F_LINEAR(x, weight, bias)

    def forward(*args, **kwargs):
        if not should_intervene():
            return original(*args, **kwargs)
        F.linear = linear
        try:
            return original(*args, **kwargs)
        finally:
            F.linear = _F_LINEAR

    restore = swap_forward(router, forward)

    def undo():
        restore()
        delattr(router, PROXY_ROUTER)

    return undo


def _attach_stand_ins(name: str, experts: nn.Module) -> tuple[nn.ModuleList, dict[str, str]]:
    n_experts = getattr(experts, GATE_UP).shape[0]
    transposed = bool(getattr(experts, "is_transposed", False))
    biased = bool(getattr(experts, "has_bias", False)) and hasattr(experts, GATE_UP + "_bias")
    stand_ins = nn.ModuleList()
    types = {}
    for e in range(n_experts):
        stand_ins.append(nn.ModuleDict({
            "gate_up": SliceLinear(experts, GATE_UP, e, GATE_UP + "_bias" if biased else None, transposed=transposed),
            "down": SliceLinear(experts, DOWN, e, DOWN + "_bias" if biased else None, transposed=transposed),
        }))
        for part in ("gate_up", "down"):
            types[f"{name}.{PROXY_EXPERTS}.{e}.{part}"] = "nn.Linear"
    experts.add_module(PROXY_EXPERTS, stand_ins)
    return stand_ins, types


def install_fused_experts(root: nn.Module, experts_names: list[str], should_intervene: Callable[[], bool],
                          grouped: Callable | None = None, place: Callable | None = None):
    """Attach the stand-ins to each named fused-experts module (and its sibling router) and
    override the forwards while *should_intervene()*.

    *grouped*: ``(experts_name, experts) -> capture`` whose ``try_forward(x, index, weights)``
    runs the whole block (``None`` when it does not apply).  *place*: ``(x) ->
    callable(rows, tokens) or None`` -- the row tracker's placement for a block input, used by
    the per-expert loop.  Returns ``(stand-in layer types, undo callables)``.
    """
    modules = dict(root.named_modules())
    types: dict[str, str] = {}
    undos: list[Callable[[], None]] = []
    for name in experts_names:
        experts = modules[name]
        if not is_fused_experts(experts):
            raise ValueError(f"{name} holds no fused expert parameters.")
        if hasattr(experts, PROXY_EXPERTS):
            raise RuntimeError(f"{name} already carries expert stand-ins.")
        stand_ins, block_types = _attach_stand_ins(name, experts)
        types.update(block_types)
        bulk = grouped(name, experts) if grouped is not None else None
        original = experts.forward

        def forward(*args, _experts=experts, _stand_ins=stand_ins, _original=original, _bulk=bulk, **kwargs):
            if not should_intervene():
                return _original(*args, **kwargs)
            x = args[0]
            index, weights = _routing_arguments(args[1:], kwargs)
            if _bulk is not None:
                out = _bulk.try_forward(x, index, weights)
                if out is not None:
                    return out
            placer = place(x) if place is not None else None
            return _loop_over_experts(_experts, _stand_ins, x, index, weights, placer)

        restore = swap_forward(experts, forward)

        def undo(_experts=experts, _restore=restore):
            _restore()
            delattr(_experts, PROXY_EXPERTS)

        undos.append(undo)
        parent_name = name.rpartition(".")[0]
        parent = modules.get(parent_name) if parent_name else root
        router = next(((n, m) for n, m in (parent.named_children() if parent is not None else ())
                       if is_fused_router(m, len(stand_ins)) and not hasattr(m, PROXY_ROUTER)), None)
        if router is not None:
            child_name, module = router
            stand_in = RouterLinear(module)
            module.add_module(PROXY_ROUTER, stand_in)
            full = f"{parent_name}.{child_name}" if parent_name else child_name
            types[f"{full}.{PROXY_ROUTER}"] = "nn.Linear"
            undos.append(_patch_router(module, stand_in, should_intervene))
    return types, undos
