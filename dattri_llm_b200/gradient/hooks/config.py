"""Capture configuration: which layers are hooked, with which family, and how.

Three hook families (parity: reference ``dattri_llm/gradient/hooks/config.py``):
``linear_io`` (factorized per-sample capture of input activations and output
gradients), ``invasive_linear_io`` (the same, for ``nn.Linear`` layers whose
weight-gradient GEMM is skipped during collection) and ``param_grad``
(batch-level parameter gradients of any module).  A selector is ``None``,
``REGISTER_ALL`` or a list of regexes searched in module names.  With no
selector at all every linear-IO-capable layer gets ``linear_io`` and every other
module with trainable parameters ``param_grad``.
"""

from __future__ import annotations

import re
import warnings
from collections.abc import Callable

import torch
from torch import nn

from dattri_llm_b200.gradient.hooks.hooks import (
    has_trainable_params,
    is_linear_io_capable,
    remove_hooks,
)
from dattri_llm_b200.gradient.hooks.override_layers import is_invasive_capable
from dattri_llm_b200.gradient.ops import ALL_LAYER_TYPES, canonical_class_name


class _RegisterAll:
    _instance: _RegisterAll | None = None

    def __new__(cls) -> _RegisterAll:
        if cls._instance is None:
            cls._instance = super().__new__(cls)
        return cls._instance

    def __repr__(self) -> str:
        return "REGISTER_ALL"

    def __reduce__(self):
        return (_RegisterAll, ())


#: Selector meaning "register every applicable layer" for a hook family.
REGISTER_ALL = _RegisterAll()
Selector = _RegisterAll | list[str] | None
LINEAR_IO = "linear_io"
PARAM_GRAD = "param_grad"
INVASIVE_LINEAR_IO = "invasive_linear_io"
_HOOK_TYPES = frozenset({LINEAR_IO, PARAM_GRAD, INVASIVE_LINEAR_IO})


class HookManagerConfig:
    """Configuration for :class:`HookManager`.

    Args:
        hook_types: Explicit ``{layer_name: hook_type}`` assignments.
        linear_io / param_grad / invasive_linear_io: Selectors per family.
        layer_types: Relabel layers (``{"model.norm": "nn.RMSNorm"}``); does not select.
        module_kwargs: Per-layer hyperparameters overriding what is read off the module.
        projection_kwargs: ``{layer_name or "__default__": {"style", "proj_dim", ...}}``.
        projector: A dattri-protocol projection factory (``None``: the library's
            counter-based projector).
        capture_style: ``"factorized"``, ``"materialized"`` or ``"auto"``.
        include_frozen: Also hook layers without trainable parameters.
    """

    def __init__(self, hook_types: dict[str, str] | None = None, linear_io: Selector = None,
                 param_grad: Selector = None, invasive_linear_io: Selector = None,
                 layer_types: dict[str, str] | None = None, module_kwargs: dict[str, dict] | None = None,
                 projection_kwargs: dict[str, dict] | None = None, projector: Callable | None = None,
                 capture_style: str = "factorized", include_frozen: bool = False) -> None:
        self.hook_types = self._check_assignment(hook_types)
        self.linear_io = self._check_selector(LINEAR_IO, linear_io)
        self.param_grad = self._check_selector(PARAM_GRAD, param_grad)
        self.invasive_linear_io = self._check_selector(INVASIVE_LINEAR_IO, invasive_linear_io)
        self.layer_types = self._check_layer_types(layer_types)
        self.module_kwargs = self._check_module_kwargs(module_kwargs)
        self.projection_kwargs = self._check_projection(projection_kwargs)
        self.capture_style = self._check_capture_style(capture_style)
        self.projector = projector
        self.include_frozen = bool(include_frozen)

    @staticmethod
    def _check_assignment(hook_types):
        if hook_types is None:
            return {}
        if not isinstance(hook_types, dict):
            raise TypeError(
                "hook_types must be a dict mapping layer name to hook type "
                f"({sorted(_HOOK_TYPES)}), got {type(hook_types).__name__}.",
            )
        for name, kind in hook_types.items():
            if kind not in _HOOK_TYPES:
                raise ValueError(
                    f"hook_types['{name}'] = '{kind}' is not a valid hook type. "
                    f"Valid types: {sorted(_HOOK_TYPES)}.",
                )
        return dict(hook_types)

    @staticmethod
    def _check_projection(projection):
        from dattri_llm_b200.gradient.ops import MASK_KEYS, PROJECTION_STYLES

        if projection is None:
            return None
        if not isinstance(projection, dict) or not all(isinstance(v, dict) for v in projection.values()):
            raise TypeError(
                "projection_kwargs must be a dict mapping layer name (or '__default__') to a "
                "proj_kwargs dict, e.g. {'__default__': {'style': 'logra', 'proj_dim': 512}}.",
            )
        for name, kw in projection.items():
            style = kw.get("style", "logra")
            if style not in PROJECTION_STYLES:
                raise ValueError(
                    f"projection_kwargs[{name!r}]['style'] = {style!r} is not a valid projection "
                    f"style. Valid styles: {list(PROJECTION_STYLES)}.",
                )
            if "seq_len" in kw:
                raise ValueError(
                    f"projection_kwargs[{name!r}] carries 'seq_len', which is not used: "
                    "capture_style='auto' decides from the actual shapes at capture.",
                )
            if style == "mask" and set(kw) - MASK_KEYS:
                raise ValueError(
                    f"projection_kwargs[{name!r}] is 'mask', which takes only "
                    f"{sorted(MASK_KEYS - {'style'})}; got unexpected {sorted(set(kw) - MASK_KEYS)}.",
                )
        return {k: dict(v) for k, v in projection.items()}

    @staticmethod
    def _check_capture_style(style):
        from dattri_llm_b200.gradient.ops import CAPTURE_STYLES

        if style not in CAPTURE_STYLES:
            raise ValueError(f"capture_style must be one of {list(CAPTURE_STYLES)}, got {style!r}.")
        return style

    @staticmethod
    def _check_layer_types(layer_types):
        if layer_types is None:
            return {}
        if not isinstance(layer_types, dict):
            raise TypeError(
                "layer_types must be a dict mapping layer name to a layer-type string, got "
                f"{type(layer_types).__name__}.",
            )
        for name, lt in layer_types.items():
            if not isinstance(name, str) or not isinstance(lt, str):
                raise TypeError(f"layer_types must map str layer names to str type names, got {name!r}: {lt!r}.")
        return dict(layer_types)

    @staticmethod
    def _check_module_kwargs(module_kwargs):
        if module_kwargs is None:
            return {}
        if not isinstance(module_kwargs, dict) or not all(
                isinstance(k, str) and isinstance(v, dict) for k, v in module_kwargs.items()):
            raise TypeError(
                "module_kwargs must be a dict mapping layer name to the layer's hyperparameter "
                "dict (see extract_module_kwargs).",
            )
        return {k: dict(v) for k, v in module_kwargs.items()}

    @staticmethod
    def _check_selector(name, selector):
        if selector is None or selector is REGISTER_ALL:
            return selector
        if isinstance(selector, (list, tuple)):
            if not all(isinstance(p, str) for p in selector):
                raise TypeError(f"{name} pattern list must contain only regex strings.")
            return list(selector)
        raise TypeError(
            f"{name} must be None, REGISTER_ALL, or a list of regex strings, got {type(selector).__name__}.",
        )

    @property
    def is_default(self) -> bool:
        """No hook selection at all (the default assignment applies)."""
        return (not self.hook_types and self.linear_io is None and self.param_grad is None
                and self.invasive_linear_io is None)


def _matches(selector: Selector, name: str) -> bool:
    if selector is None:
        return False
    if selector is REGISTER_ALL:
        return True
    return any(re.search(p, name) for p in selector)


def _warn_zero_layers() -> None:
    warnings.warn(
        "HookManager registered zero layers: no module matched the requested hook "
        "configuration. No gradients will be collected.",
        stacklevel=3,
    )


def _tap_covered(modules: dict[str, nn.Module]) -> set[str]:
    """Modules whose trainable parameters are all read by a capture tap (e.g. an
    expert-parallel router's weight, captured per sample through its ``dattri_router``):
    pattern and default selection give them no ``param_grad`` hook, which would count the
    same weight twice."""
    proxied: set[int] = set()
    for m in modules.values():
        if getattr(type(m), "__bw_capture_tap__", False) and hasattr(m, "proxied_parameters"):
            proxied.update(id(p) for p in m.proxied_parameters())
    if not proxied:
        return set()
    out = set()
    for name, m in modules.items():
        own = [p for _, p in m.named_parameters(recurse=False) if p.requires_grad]
        if own and all(id(p) in proxied for p in own):
            out.add(name)
    return out


def resolve_hook_assignments(root: nn.Module, config: HookManagerConfig) -> dict[str, str]:
    """The final ``{layer_name: hook_type}`` assignment of *config* on *root*.

    Raises:
        ValueError: for unknown names, families a layer cannot take, or a layer
            selected by two families.
    """
    modules = dict(root.named_modules())
    assignment: dict[str, str] = {}

    def assign(name: str, kind: str) -> None:
        prev = assignment.get(name)
        if prev is not None and prev != kind:
            raise ValueError(
                f"Layer '{name}' is assigned conflicting hook types: '{prev}' and '{kind}'. "
                "A layer may only be registered with one hook family.",
            )
        assignment[name] = kind

    covered = _tap_covered(modules)
    if config.is_default:
        for name, module in modules.items():
            if is_linear_io_capable(module):
                assignment[name] = LINEAR_IO
            elif has_trainable_params(module) and name not in covered:
                assignment[name] = PARAM_GRAD
        if not assignment:
            _warn_zero_layers()
        return assignment
    for name, kind in config.hook_types.items():
        module = modules.get(name)
        if module is None:
            raise ValueError(f"hook_types names layer '{name}', which does not exist in the model.")
        if (kind == LINEAR_IO and not is_linear_io_capable(module)
                and config.layer_types.get(name) not in ALL_LAYER_TYPES):
            raise ValueError(
                f"Layer '{name}' was assigned 'linear_io' but its type ({canonical_class_name(module)}) "
                "does not support factorized linear-IO hooks. If the layer computes the same math as "
                f"a supported type, declare it via layer_types (e.g. layer_types={{'{name}': 'nn.RMSNorm'}}).",
            )
        if kind == PARAM_GRAD and not has_trainable_params(module):
            raise ValueError(f"Layer '{name}' was assigned 'param_grad' but has no trainable parameters.")
        if kind == INVASIVE_LINEAR_IO and not is_invasive_capable(module):
            raise ValueError(
                f"Layer '{name}' was assigned 'invasive_linear_io' but its type "
                f"({canonical_class_name(module)}) is not nn.Linear.",
            )
        assign(name, kind)
    for name, module in modules.items():
        if is_linear_io_capable(module) and _matches(config.linear_io, name):
            assign(name, LINEAR_IO)
        if has_trainable_params(module) and name not in covered and _matches(config.param_grad, name):
            assign(name, PARAM_GRAD)
        if is_invasive_capable(module) and _matches(config.invasive_linear_io, name):
            assign(name, INVASIVE_LINEAR_IO)
    if not assignment:
        _warn_zero_layers()
    return assignment


def _invoke(model: nn.Module, sample_input: object) -> object:
    if isinstance(sample_input, dict):
        return model(**sample_input)
    if isinstance(sample_input, (list, tuple)):
        return model(*sample_input)
    return model(sample_input)


def _scalar_loss(output: object) -> torch.Tensor | None:
    loss = getattr(output, "loss", None)
    if isinstance(loss, torch.Tensor):
        return loss
    cand = output if isinstance(output, torch.Tensor) else getattr(output, "logits", None)
    if cand is None:
        values = output.values() if isinstance(output, dict) else output if isinstance(output, (list, tuple)) else ()
        cand = next((v for v in values if isinstance(v, torch.Tensor) and v.is_floating_point()), None)
    if isinstance(cand, torch.Tensor) and cand.is_floating_point():
        return cand.sum()
    return None


def default_hook_assignment(model: nn.Module, sample_input: object,
                            loss_fn: Callable[[object], torch.Tensor] | None = None) -> dict[str, str]:
    """The default assignment restricted to layers that actually fire on *sample_input*
    (linear-IO layers that run forward; param-grad layers whose parameters get a gradient)."""
    root = getattr(model, "module", model)
    modules = dict(root.named_modules())
    candidate = {}
    covered = _tap_covered(modules)
    for name, module in modules.items():
        if is_linear_io_capable(module):
            candidate[name] = LINEAR_IO
        elif has_trainable_params(module) and name not in covered:
            candidate[name] = PARAM_GRAD
    fired: set[str] = set()
    handles = []
    for name, module in modules.items():
        kind = candidate.get(name)
        if kind == LINEAR_IO:
            handles.append(module.register_forward_hook(lambda *_a, n=name: fired.add(n)))
        elif kind == PARAM_GRAD:
            for _, p in module.named_parameters(recurse=False):
                if p.requires_grad:
                    handles.append(p.register_hook(lambda _g, n=name: fired.add(n)))
    try:
        with torch.enable_grad():
            output = _invoke(model, sample_input)
            try:
                loss = loss_fn(output) if loss_fn is not None else _scalar_loss(output)
            except Exception as exc:  # noqa: BLE001 - a user loss may raise anything
                loss = None
                warnings.warn(f"default_hook_assignment could not compute a loss ({exc!r}); "
                              "param_grad layers may be missed. Pass loss_fn.", stacklevel=2)
            if isinstance(loss, torch.Tensor) and loss.requires_grad:
                model.zero_grad(set_to_none=True)
                loss.backward()
            elif any(k == PARAM_GRAD for k in candidate.values()):
                warnings.warn("default_hook_assignment could not derive a differentiable scalar "
                              "loss; param_grad layers may be missed. Pass loss_fn.", stacklevel=2)
    finally:
        remove_hooks(handles)
        model.zero_grad(set_to_none=True)
    assignment = {n: k for n, k in candidate.items() if n in fired}
    skipped = sorted(set(candidate) - set(assignment))
    if skipped:
        warnings.warn("default_hook_assignment skipped layers that did not fire during the sample "
                      f"pass (e.g. invoked functionally): {skipped}.", stacklevel=2)
    if not assignment:
        _warn_zero_layers()
    return assignment
