"""Projection styles on CPU against the dense per-sample gradient ``dW = g^T a``:

* ``logra`` keeps the structure: ``g_p^T a_p == P_g dW P_a^T`` with the projector's two
  matrices (gradient side seeded ``s``, activation side ``s + 1``), bias folded in as a
  column of ones on the activation side;
* ``dense`` (TRAK) projects the flattened gradient: ``P vec(dW)``;
* ``mask`` keeps exact coordinates: ``vec(dW)[idx]`` with the mask's indices, computed
  without forming ``dW`` (linear and embedding layers);
* a user projector given through the factory protocol (here: truncation) is honoured.
"""

from __future__ import annotations

import pytest
import torch

from dattri_llm_b200.gradient.ops import materialize_factors
from dattri_llm_b200.gradient.ops.projection import (
    DattriProjector,
    mask_factors,
    project_factors,
    project_layer,
    project_materialized_factors,
)

B, T, K, D = 3, 5, 6, 4


def _factors(seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, T, K, generator=g), torch.randn(B, T, D, generator=g)


def _with_bias(a):
    return torch.cat([a, torch.ones(*a.shape[:-1], 1)], -1)


def test_logra_projects_each_side():
    a, g = _factors(1)
    proj = DattriProjector()
    a_p, g_p = project_factors(a, g, "nn.Linear", proj, {"has_bias": True}, proj_dim=3, proj_seed=7)
    p_g = proj.matrix(D, proj_dim=3, proj_seed=7, device=torch.device("cpu"), dtype=torch.float32)
    p_a = proj.matrix(K + 1, proj_dim=3, proj_seed=8, device=torch.device("cpu"), dtype=torch.float32)
    dw = torch.einsum("btd,btk->bdk", g, _with_bias(a))
    want = torch.einsum("dp,bdk,kq->bpq", p_g, dw, p_a)
    got = torch.einsum("btp,btq->bpq", g_p, a_p)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)


def test_dense_style_projects_the_flattened_gradient():
    a, g = _factors(2)
    proj = DattriProjector()
    got = project_materialized_factors(a, g, "nn.Linear", proj, {"has_bias": False}, proj_dim=5, proj_seed=3)
    dense = materialize_factors(a, g, "nn.Linear", {"has_bias": False})
    p = proj.matrix(dense.shape[-1], proj_dim=5, proj_seed=3, device=torch.device("cpu"), dtype=torch.float32)
    torch.testing.assert_close(got, dense @ p, rtol=1e-4, atol=1e-5)


def test_mask_keeps_exact_coordinates_of_linear_and_embedding_grads():
    a, g = _factors(3)
    proj = DattriProjector()
    got = mask_factors(a, g, "nn.Linear", proj, {"has_bias": True}, proj_dim=9, proj_seed=4)
    dense = materialize_factors(a, g, "nn.Linear", {"has_bias": True})
    idx = proj.mask_indices(dense.shape[-1], proj_dim=9, proj_seed=4, device=torch.device("cpu"))
    torch.testing.assert_close(got, dense[:, idx], rtol=1e-5, atol=1e-6)
    vocab = 11
    ids = torch.randint(0, vocab, (B, T), generator=torch.Generator().manual_seed(5))
    kw = {"num_embeddings": vocab, "padding_idx": None}
    got_e = mask_factors(ids, g, "nn.Embedding", proj, kw, proj_dim=7, proj_seed=2)
    dense_e = materialize_factors(ids, g, "nn.Embedding", kw)
    idx_e = proj.mask_indices(dense_e.shape[-1], proj_dim=7, proj_seed=2, device=torch.device("cpu"))
    torch.testing.assert_close(got_e, dense_e[:, idx_e], rtol=1e-5, atol=1e-6)


def test_mask_indices_are_distinct_and_reproducible():
    proj = DattriProjector()
    i1 = proj.mask_indices(1000, proj_dim=64, proj_seed=9, device=torch.device("cpu"))
    i2 = DattriProjector().mask_indices(1000, proj_dim=64, proj_seed=9, device=torch.device("cpu"))
    assert torch.equal(i1, i2) and i1.unique().numel() == 64 and int(i1.max()) < 1000
    with pytest.raises(ValueError):
        proj.mask_indices(10, proj_dim=11, proj_seed=0, device=torch.device("cpu"))


def _truncate_factory(feature, batch_size, proj_dim, proj_seed=0, device="cpu", **_):
    """A dattri-protocol factory whose projector keeps the first ``proj_dim`` features."""
    return lambda x, ensemble_id=0: x[..., :proj_dim]


def test_user_projector_through_the_factory_protocol():
    a, g = _factors(6)
    a_p, g_p = project_factors(a, g, "nn.Linear", _truncate_factory, {"has_bias": False}, proj_dim=2, proj_seed=0)
    torch.testing.assert_close(a_p, a[..., :2])
    torch.testing.assert_close(g_p, g[..., :2])


@pytest.mark.parametrize(("capture_style", "tokens", "materialized"),
                         [("factorized", 50, False), ("materialized", 1, True), ("auto", 50, True), ("auto", 1, False)])
def test_project_layer_routes_logra_by_capture_style(capture_style, tokens, materialized):
    from dattri_llm_b200.gradient.gradient import Factorized

    g = torch.Generator().manual_seed(8)
    f = Factorized(torch.randn(B, tokens, K, generator=g), torch.randn(B, tokens, D, generator=g),
                   module_kwargs={"has_bias": False})
    payload, is_fac = project_layer(f, "nn.Linear", DattriProjector(), style="logra", capture_style=capture_style,
                                    proj_dim=3, proj_seed=0)
    assert is_fac == (not materialized)
    if materialized:
        assert payload.shape == (B, 9)
