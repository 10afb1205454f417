"""The scoring loop (``attribution.utils.score_sources``) on CPU: scores equal the dense
oracle ``G_train G_test^T``; rows and columns are keyed by the first time a hash is seen;
the result does not depend on how train blocks are rebatched, on looping over a re-iterable
test source instead of caching it, or on the packed one-GEMM path vs the layerwise path;
``rebatch_blocks`` concatenates dense blocks and passes factorized blocks through in order.
"""

from __future__ import annotations

import pytest
import torch

from dattri_llm_b200.attribution.utils import PackedDense, packed_cross_dot, score_sources
from dattri_llm_b200.gradient.gradient import Factorized, Gradient
from dattri_llm_b200.gradient.streaming import rebatch_blocks


def _dense_block(b, seed):
    g = torch.Generator().manual_seed(seed)
    return Gradient({"u": "materialized", "v": "materialized"},
                    {"u": torch.randn(b, 4, generator=g), "v": torch.randn(b, 3, generator=g)},
                    {"u": "nn.Linear", "v": "nn.Linear"}, {"u": "batch", "v": "batch"})


def _source(sizes, seed, prefix):
    out, k = [], 0
    for step, b in enumerate(sizes):
        out.append((step, _dense_block(b, seed + step), [f"{prefix}{k + i}" for i in range(b)]))
        k += b
    return out


class _Reusable(list):
    reusable = True


def _flat(src):
    return torch.cat([torch.cat([blk.data["u"], blk.data["v"]], 1) for _, blk, _ in src])


def _layerwise_dot(train_block, test_block, dense_cache=None):
    """The plain layerwise inner product (the loop passes a per-test-block dense cache)."""
    del dense_cache
    return sum(train_block.data[n] @ test_block.data[n].T for n in train_block.data)


@pytest.mark.parametrize("batch_size", [1, 2, 5, 100])
@pytest.mark.parametrize("loop_over_test", [False, True])
def test_scores_match_oracle_and_are_invariant(batch_size, loop_over_test):
    train = _source([2, 3, 1, 4], 0, "tr")
    test = _Reusable(_source([3, 2], 50, "te"))
    scores, rows, steps, tests, tokens = score_sources(
        train, test, torch.device("cpu"), inner_product=_layerwise_dot, batch_size=batch_size,
        loop_over_test=loop_over_test)
    assert tokens is None
    assert rows == [f"tr{i}" for i in range(10)] and tests == [f"te{i}" for i in range(5)]
    assert steps == [0, 0, 1, 1, 1, 2, 3, 3, 3, 3]
    torch.testing.assert_close(scores, _flat(train) @ _flat(test).T, rtol=1e-5, atol=1e-5)


def test_packed_path_equals_layerwise_path():
    train = _source([3, 2], 1, "tr")
    test = _Reusable(_source([4], 9, "te"))
    packed, *_ = score_sources(train, test, torch.device("cpu"), inner_product=_layerwise_dot,
                               packed_inner_product=True)
    plain, *_ = score_sources(train, test, torch.device("cpu"), inner_product=_layerwise_dot)
    torch.testing.assert_close(packed, plain, rtol=1e-5, atol=1e-5)
    a, b = PackedDense.pack(train[0][1]), PackedDense.pack(test[0][1])
    assert a.layout == b.layout
    torch.testing.assert_close(packed_cross_dot(a, b), _layerwise_dot(train[0][1], test[0][1]), rtol=1e-5, atol=1e-5)


def test_columns_follow_the_first_seen_order_across_test_blocks():
    train = _source([2], 3, "tr")
    t_a, t_b = _dense_block(2, 60), _dense_block(3, 61)
    test = [(0, t_b, ["b0", "b1", "b2"]), (0, t_a, ["a0", "a1"])]
    scores, _, _, tests, _ = score_sources(train, test, torch.device("cpu"), inner_product=_layerwise_dot)
    assert tests == ["b0", "b1", "b2", "a0", "a1"]
    g = _flat(train)
    torch.testing.assert_close(scores[:, :3], g @ _flat([(0, t_b, None)]).T, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(scores[:, 3:], g @ _flat([(0, t_a, None)]).T, rtol=1e-5, atol=1e-5)


def test_rebatch_concatenates_dense_and_passes_factorized_through():
    d1, d2, d3 = (_dense_block(2, 1), _dense_block(1, 2), _dense_block(2, 3))
    fac = Gradient({"f": "factorized"}, {"f": Factorized(torch.randn(2, 3, 4), torch.randn(2, 3, 5))},
                   {"f": "nn.Linear"}, {"f": "batch_token"})
    src = [(0, d1, ["a", "b"]), (1, d2, ["c"]), (2, fac, ["d", "e"]), (3, d3, ["f", "g"])]
    out = list(rebatch_blocks(src, batch_size=3))
    assert [ids for _, _, ids in out] == [["a", "b", "c"], ["d", "e"], ["f", "g"]]
    assert out[0][0] == [0, 0, 1] and out[1][0] == [2, 2] and out[2][0] == [3, 3]
    torch.testing.assert_close(out[0][1].data["u"], torch.cat([d1.data["u"], d2.data["u"]]))
    assert out[1][1] is fac
    with pytest.raises(ValueError):
        list(rebatch_blocks(src, batch_size=0))


def test_rebatch_zero_fills_a_layer_some_blocks_lack():
    """A routed expert no token of a block reached is absent from that block: its rows are zero."""
    d1, d2 = _dense_block(2, 1), _dense_block(1, 2)
    extra = torch.randn(1, 6)
    d2 = Gradient({**d2.representation, "e": "materialized"}, {**d2.data, "e": extra},
                  {**d2.layer_types, "e": "nn.Linear"}, {**d2.indexing, "e": "batch"})
    d3 = _dense_block(2, 3)
    (steps, merged, ids), = list(rebatch_blocks([(0, d1, ["a", "b"]), (1, d2, ["c"]), (2, d3, ["d", "e"])],
                                                batch_size=5))
    assert ids == ["a", "b", "c", "d", "e"] and steps == [0, 0, 1, 2, 2]
    want = torch.cat([torch.zeros(2, 6), extra, torch.zeros(2, 6)])
    torch.testing.assert_close(merged.data["e"], want)
    assert merged.data["u"].shape[0] == 5
