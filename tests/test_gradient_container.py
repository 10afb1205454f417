"""The :class:`Gradient` container on CPU, each operation checked against the dense
per-sample gradients it stands for: batch concatenation of factorized layers with
unequal token lengths (zero padding must not change any gradient), token aggregation,
batch / token slicing, layer selection with derived ``@k`` names, and similarity as dot
products, cosines and per-token shares that sum back to the instance scores."""

from __future__ import annotations

import pytest
import torch

from dattri_llm_b200.gradient.gradient import Factorized, Gradient


def _block(b, t, seed, *, k=5, d=4):
    g = torch.Generator().manual_seed(seed)
    fac = Factorized(torch.randn(b, t, k, generator=g), torch.randn(b, t, d, generator=g))
    dense = torch.randn(b, 7, generator=g)
    return Gradient({"f": "factorized", "m": "materialized", "f@2": "factorized"},
                    {"f": fac, "m": dense,
                     "f@2": Factorized(torch.randn(b, t, k, generator=g), torch.randn(b, t, d, generator=g))},
                    {"f": "nn.Linear", "m": "nn.Linear", "f@2": "nn.Linear"},
                    {"f": "batch_token", "m": "batch", "f@2": "batch_token"})


def _dense(grad: Gradient) -> dict[str, torch.Tensor]:
    m = grad.materialize()
    return {n: v.reshape(v.shape[0], -1) for n, v in m.data.items()}


def _per_sample_flat(grad: Gradient) -> torch.Tensor:
    d = _dense(grad)
    return torch.cat([d[n] for n in sorted(d)], 1)


def test_concatenate_pads_unequal_token_lengths_without_changing_gradients():
    a, b = _block(2, 3, 0), _block(3, 5, 1)
    cat = a.concatenate(b, dim="batch")
    assert cat.batch_size == 5
    want = torch.cat([_per_sample_flat(a), _per_sample_flat(b)])
    torch.testing.assert_close(_per_sample_flat(cat), want)


def test_aggregate_sums_out_tokens():
    g = _block(3, 4, 2)
    agg = g.aggregate("token")
    assert all(v == "batch" for v in agg.indexing.values())
    torch.testing.assert_close(_per_sample_flat(agg), _per_sample_flat(g))


@pytest.mark.parametrize("index", [1, [2, 0], torch.tensor([1, 2])])
def test_batch_slice_selects_samples(index):
    g = _block(3, 4, 3)
    idx = [index] if isinstance(index, int) else [int(i) for i in index]
    torch.testing.assert_close(_per_sample_flat(g.slice("batch", index)), _per_sample_flat(g)[idx])


def test_token_slices_partition_the_gradient():
    fac_layers = ["f", "f@2"]
    g = _block(2, 5, 4).select_layers(fac_layers)
    parts = [g.slice("token", [0, 1]), g.slice("token", [2, 3, 4])]
    whole = _dense(g)
    summed = {n: sum(_dense(p)[n] for p in parts) for n in fac_layers}
    for n in fac_layers:
        torch.testing.assert_close(summed[n], whole[n])
    with pytest.raises(ValueError, match="batch_token"):  # a batch-indexed layer has no token axis
        _block(2, 5, 4).slice("token", [0])


def test_select_layers_with_derived_names():
    g = _block(2, 3, 5)
    assert set(g.select_layers(["f"]).data) == {"f"}
    assert set(g.select_layers(["f"], include_derived=True).data) == {"f", "f@2"}


@pytest.mark.parametrize("metric", ["dot", "cosine"])
def test_similarity_matches_dense_vectors(metric):
    a, b = _block(3, 4, 6), _block(2, 6, 7)
    got = a.similarity(b, metric=metric, reduce="all")
    va, vb = _per_sample_flat(a), _per_sample_flat(b)
    if metric == "cosine":
        va = va / va.norm(dim=1, keepdim=True)
        vb = vb / vb.norm(dim=1, keepdim=True)
    torch.testing.assert_close(got, va @ vb.T, rtol=1e-4, atol=1e-5)
    per_layer = a.similarity(b, metric="dot", reduce="none")
    da, db = _dense(a), _dense(b)
    for n, m in per_layer.items():
        torch.testing.assert_close(m, da[n] @ db[n].T, rtol=1e-4, atol=1e-5)


def test_per_token_similarity_sums_to_instance_similarity():
    fac_only = ["f", "f@2"]
    a, b = _block(2, 5, 8).select_layers(fac_only), _block(3, 4, 9).select_layers(fac_only)
    tok = a.similarity_per_token(b, reduce="all")
    assert tok.shape == (2, 5, 3)
    torch.testing.assert_close(tok.sum(1), a.similarity(b, metric="dot", reduce="all"), rtol=1e-4, atol=1e-5)
