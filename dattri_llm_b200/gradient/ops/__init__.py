"""Layer-type-aware operations on factorized or materialized per-sample gradients.

Dot products and their cost-based routing, projection, K-FAC / EK-FAC and
optimizer preconditioning.  Every function accepts CPU or CUDA tensors; on an
sm_100 device the hot contractions dispatch to the native kernels of
:mod:`dattri_llm_b200.ops`.
"""

from dattri_llm_b200.gradient.ops import dtypes, norm
from dattri_llm_b200.gradient.ops.dot import (
    cross_dot,
    cross_dot_factors,
    cross_dot_per_token,
    cross_gram,
    cross_gram_per_token,
    cross_gram_per_token_dense,
    dot,
    dot_factors,
    effective_dims,
    grad_norm_sq,
    grad_norm_sq_factors,
    layerwise_cross_dot,
    layerwise_cross_dot_per_token,
    maybe_use_materialized_gram,
    maybe_use_materialized_norm,
    pairwise_dot,
    pairwise_dot_factors,
)
from dattri_llm_b200.gradient.ops.dtypes import (
    align,
    as_float,
    compute_dtype,
    get_compute_dtype,
    set_compute_dtype,
)
from dattri_llm_b200.gradient.ops.kronecker import (
    FisherAccumulator,
    KroneckerAccumulator,
    LayerFisherAccumulator,
    LayerKroneckerAccumulator,
    dense_inverse,
    ekfac_lambda_accumulate,
    ekfac_materialize,
    ekfac_materialize_factors,
    ekfac_precondition,
    fim,
    fim_factors,
    flatten_kfac_factors,
    kfac,
    kfac_cross,
    kfac_accumulate_grouped,
    kfac_cross_factors,
    kfac_eigh,
    kfac_factors,
    kfac_precondition,
    kfac_precondition_materialized,
    sym_inverse,
)
from dattri_llm_b200.gradient.ops.materialize import materialize, materialize_factors
from dattri_llm_b200.gradient.ops.optimizer import (
    OPTIMIZER_STATE_KEYS,
    adam_preconditioner,
    adamw_influence_coupling,
    adamw_influence_push,
    adamw_influence_transition,
    precondition,
)
from dattri_llm_b200.gradient.ops.preprocess import (
    extract_module_kwargs,
    preprocess_factorized,
    preprocess_factors,
    to_3d,
)
from dattri_llm_b200.gradient.ops.projection import (
    CAPTURE_STYLES,
    MASK_KEYS,
    PROJECTION_STYLES,
    DattriProjector,
    ProjectionMatrix,
    apply_projection,
    counter_projector,
    mask_coordinates,
    mask_factorized,
    mask_factors,
    mask_materialized,
    maybe_materialize_projected,
    project_activation,
    project_factorized,
    project_factors,
    project_gradient,
    project_layer,
    project_materialized,
    project_materialized_factors,
    should_materialize,
)
from dattri_llm_b200.gradient.ops.types import (
    ALL_LAYER_TYPES,
    CONV_TRANSPOSE_TYPES,
    CONV_TYPES,
    EMBEDDING_TYPES,
    LINEAR_TYPES,
    NORM_TYPES,
    PARAM_GRAD_TYPES,
    canonical_class_name,
    is_conv,
    is_conv_transpose,
    is_embedding,
    is_kfac_eligible,
    is_linear,
    is_norm,
)

__all__ = [n for n in dir() if not n.startswith("_")]
