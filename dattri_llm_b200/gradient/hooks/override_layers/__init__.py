"""Forward overrides that route fused / functional compute through hookable modules.

* ``invasive_linear``: capture ``nn.Linear`` layers without their weight-gradient GEMM.
* ``fused_experts``: per-expert proxy modules for MoE blocks whose experts are fused
  3-D parameters, and for routers applied functionally.
* ``sequence_mixers``: state-space / linear-attention mixers whose kernels apply
  projections functionally (Mamba, Mamba2 and hybrids).
"""

from dattri_llm_b200.gradient.hooks.override_layers.fused_experts import (
    RouterLinear,
    SliceLinear,
    find_fused_experts,
    install_fused_experts,
    is_fused_experts,
)
from dattri_llm_b200.gradient.hooks.override_layers.invasive_linear import (
    InvasiveLinearFunction,
    install_invasive_forward,
    is_invasive_capable,
)
from dattri_llm_b200.gradient.hooks.override_layers.sequence_mixers import (
    MAMBA1_MIXER_CLASSES,
    find_sequence_mixers,
    install_sequence_mixer_forward,
    is_functional_conv_mixer,
    is_mamba1_mixer,
    mamba1_reference_forward,
)

__all__ = [
    "MAMBA1_MIXER_CLASSES",
    "InvasiveLinearFunction",
    "RouterLinear",
    "SliceLinear",
    "find_fused_experts",
    "find_sequence_mixers",
    "install_fused_experts",
    "install_invasive_forward",
    "install_sequence_mixer_forward",
    "is_functional_conv_mixer",
    "is_fused_experts",
    "is_invasive_capable",
    "is_mamba1_mixer",
    "mamba1_reference_forward",
]
