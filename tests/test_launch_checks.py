"""Launch-argument checks (CPU): each validator accepts the tables the library builds and
names the first index that would address memory outside its buffer; with checks on, the
extension wrapper runs the validator before the entry point, and with checks off it
hands out the module itself."""

from __future__ import annotations

import pytest
import torch

from dattri_llm_b200.ops import checks
from dattri_llm_b200.ops.checks import LaunchCheckError


def _peers(rows=(6, 4)):
    return [torch.zeros(r, 8) for r in rows]


def test_routed_rows():
    peers = _peers()
    checks.check_routed_rows("x", torch.tensor([0, 1, 1]), torch.tensor([5, 0, 3]), peers)
    with pytest.raises(LaunchCheckError, match=r"dst_row\[2\] = 4 outside \[0, 4\)"):
        checks.check_routed_rows("x", torch.tensor([0, 1, 1]), torch.tensor([5, 0, 4]), peers)
    with pytest.raises(LaunchCheckError, match=r"dst_rank\[0\] = 2"):
        checks.check_routed_rows("x", torch.tensor([2]), torch.tensor([0]), peers)
    with pytest.raises(LaunchCheckError, match="dst_row"):
        checks.check_routed_rows("x", torch.tensor([0]), torch.tensor([-1]), peers)


def _tables(lens, rows=None):
    lens = torch.tensor(lens)
    blocks = (lens + 255) // 256
    prefix = torch.cat([torch.zeros(1, dtype=torch.long), blocks.cumsum(0)])
    base = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)[:-1]])
    return prefix.int(), base.int(), lens.int(), int(lens.sum()) if rows is None else rows


def test_ragged_tables():
    prefix, base, lens, rows = _tables([300, 0, 17])
    checks.check_ragged_tables("g", rows, prefix, base, lens, int(prefix[-1]))
    with pytest.raises(LaunchCheckError, match="covers 2"):
        checks.check_ragged_tables("g", rows, prefix, base, lens, 2)
    with pytest.raises(LaunchCheckError, match="job 2 reads rows"):
        checks.check_ragged_tables("g", rows - 1, prefix, base, lens, 8)
    short = prefix.clone()
    short[1] = 1  # 300 rows in one 256-row block
    with pytest.raises(LaunchCheckError, match="job 0 has 1 blocks for 300 rows"):
        checks.check_ragged_tables("g", rows, short, base, lens, 8)
    bad0 = prefix.clone()
    bad0[0] = 1
    with pytest.raises(LaunchCheckError, match="tile_prefix\\[0\\]"):
        checks.check_ragged_tables("g", rows, bad0, base, lens, 8)


def test_scatter_expert_ids_and_mask_coords():
    meta = torch.tensor([[0, 5], [1, 3], [1, 9]])  # the third row is past `rows`
    checks.check_scatter("s", meta, _peers(), rows=2)
    with pytest.raises(LaunchCheckError):
        checks.check_scatter("s", meta, _peers(), rows=3)
    checks.check_expert_ids("c", torch.tensor([[0, 7]]), 8)
    with pytest.raises(LaunchCheckError, match="expert id"):
        checks.check_expert_ids("c", torch.tensor([[0, 8]]), 8)
    checks.check_mask_coords("m", torch.tensor([0, 15]), torch.tensor([7]), 16, 8)
    with pytest.raises(LaunchCheckError, match="column coordinate"):
        checks.check_mask_coords("m", torch.tensor([0]), torch.tensor([8]), 16, 8)


def test_wrapper_validates_before_the_call(monkeypatch):
    import dattri_llm_b200.ops as ops

    calls = []

    class Fake:
        @staticmethod
        def moe_count(topi, counts):
            calls.append("moe_count")

        @staticmethod
        def rope(*a):
            calls.append("rope")

    monkeypatch.setattr(ops, "_C", Fake)
    checks.set_checks(False)
    try:
        assert ops.native() is Fake
        checks.set_checks(True)
        nat = ops.native()
        assert isinstance(nat, checks.CheckedNative)
        nat.moe_count(torch.tensor([0, 3]), torch.zeros(4, dtype=torch.int32))
        with pytest.raises(LaunchCheckError):
            nat.moe_count(torch.tensor([0, 4]), torch.zeros(4, dtype=torch.int32))
        nat.rope(1, 2)  # no validator: passed straight through
        assert calls == ["moe_count", "rope"]
    finally:
        checks.set_checks(False)
        ops._checked = None


def test_env_switch(monkeypatch):
    monkeypatch.setenv("DATTRI_B200_CHECKS", "1")
    monkeypatch.setattr(checks, "_enabled", None)
    assert checks.checks_enabled()
    monkeypatch.setenv("DATTRI_B200_CHECKS", "0")
    monkeypatch.setattr(checks, "_enabled", None)
    assert not checks.checks_enabled()


def test_validators_cover_the_data_dependent_entry_points():
    assert {"moe_dispatch", "moe_combine_bwd_dispatch", "gemm_ragged", "moe_count", "moe_place",
            "mask_gather"} <= set(checks.VALIDATORS)
    # argument positions match the bindings' signatures
    peers = _peers()
    dr, drow = torch.tensor([0, 1]), torch.tensor([1, 2])
    checks.VALIDATORS["moe_dispatch"]((None, 1, dr, drow, peers, peers, 0), {})
    checks.VALIDATORS["moe_combine_bwd_dispatch"]((None, None, None, None, dr, drow, peers, peers, 0), {})
    prefix, base, lens, rows = _tables([5, 3])
    a = torch.zeros(rows, 8)
    meta = torch.tensor([[0, 1]] * rows)
    checks.VALIDATORS["gemm_ragged"]((a, None, None, prefix, base, lens, 2, peers, meta, None, 0), {})
    checks.VALIDATORS["moe_place"]((torch.tensor([3]), torch.zeros(2, 4, dtype=torch.int32), 0, 2), {})
    checks.VALIDATORS["mask_gather"]((torch.zeros(1, 2, 16), torch.zeros(1, 2, 8), torch.tensor([15]),
                                      torch.tensor([7]), None), {})
