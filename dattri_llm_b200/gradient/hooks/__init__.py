"""Hook registration, :class:`HookManagerConfig` and layer selectors."""

from dattri_llm_b200.gradient.callbacks.offload_callback import OffloadCallback
from dattri_llm_b200.gradient.hooks.config import (
    INVASIVE_LINEAR_IO,
    LINEAR_IO,
    PARAM_GRAD,
    REGISTER_ALL,
    HookManagerConfig,
    Selector,
    default_hook_assignment,
    resolve_hook_assignments,
)
from dattri_llm_b200.gradient.hooks.hooks import (
    HF_Conv1D,
    LayerBuffer,
    ParamGradBuffer,
    register_linear_io_hooks,
    register_linear_param_hooks,
    register_param_grad_hooks,
    remove_hooks,
)
from dattri_llm_b200.gradient.hooks.manager import HookManager
from dattri_llm_b200.gradient.hooks.override_layers.fused_experts import (
    RouterLinear,
    SliceLinear,
    find_fused_experts,
)
from dattri_llm_b200.gradient.hooks.routing import RoutedTokenTracker, RowLayout
from dattri_llm_b200.gradient.hooks.override_layers import (
    install_fused_experts,
    install_invasive_forward,
    install_sequence_mixer_forward,
)
from dattri_llm_b200.gradient.callbacks.base import HookManagerCallback

__all__ = [
    "HF_Conv1D",
    "RoutedTokenTracker",
    "RouterLinear",
    "RowLayout",
    "SliceLinear",
    "find_fused_experts",
    "INVASIVE_LINEAR_IO",
    "LINEAR_IO",
    "PARAM_GRAD",
    "REGISTER_ALL",
    "HookManager",
    "HookManagerCallback",
    "HookManagerConfig",
    "LayerBuffer",
    "OffloadCallback",
    "ParamGradBuffer",
    "Selector",
    "default_hook_assignment",
    "install_fused_experts",
    "install_invasive_forward",
    "install_sequence_mixer_forward",
    "register_linear_io_hooks",
    "register_linear_param_hooks",
    "register_param_grad_hooks",
    "remove_hooks",
    "resolve_hook_assignments",
]
