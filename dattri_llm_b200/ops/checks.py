"""Launch-argument checks: a host-side bounds sanitizer for the native kernels.

``compute-sanitizer`` does not run on the deployment pool, and a kernel must never trap
the GPU on purpose, so out-of-bounds accesses are caught before the launch instead.  The
C++ bindings already check every static property of an operand (dtype, shape, contiguity,
the 16-byte rules of TMA).  What they cannot see without reading device memory is the
*content* of the index tensors that steer data-dependent stores: expert-parallel
destination rows and ranks, scatter metadata of the ragged GEMM's epilogue, the ragged
GEMM's job tables, expert ids and mask-projection coordinates.  With checks on
(:func:`set_checks` or ``DATTRI_B200_CHECKS=1``), :func:`dattri_llm_b200.ops.native`
returns a wrapper that runs the validator of each such entry point on its arguments
and raises :class:`LaunchCheckError` naming the first bad index before anything is
launched.  Validation reads the index tensors back (a device synchronization per
launch): a debugging mode, off by default.

Every validator is a plain function of tensors, so the rules are tested on CPU.
"""

from __future__ import annotations

import os
from collections.abc import Callable, Sequence

import torch

_ENV = "DATTRI_B200_CHECKS"
_enabled: bool | None = None
ROWS_PER_TILE = 256  # rows per block of the ragged GEMM's job tables


class LaunchCheckError(ValueError):
    """A native launch's index arguments would address memory outside its buffers."""


def checks_enabled() -> bool:
    """Whether native launches are validated."""
    global _enabled
    if _enabled is None:
        _enabled = os.environ.get(_ENV, "0").lower() not in ("", "0", "false", "no")
    return _enabled


def set_checks(enabled: bool) -> None:
    """Turn launch validation on or off for this process (overrides ``DATTRI_B200_CHECKS``)."""
    global _enabled
    _enabled = bool(enabled)


def _first_bad(mask: torch.Tensor) -> int | None:
    bad = mask.reshape(-1).nonzero()
    return int(bad[0]) if bad.numel() else None


def _in_range(name: str, values: torch.Tensor, lo: int, hi: torch.Tensor | int, what: str) -> None:
    """Raise unless ``lo <= values < hi`` elementwise (*hi* scalar or per element)."""
    v = values.reshape(-1).long().cpu()
    h = hi.reshape(-1).long().cpu() if isinstance(hi, torch.Tensor) else torch.full_like(v, int(hi))
    i = _first_bad((v < lo) | (v >= h))
    if i is not None:
        raise LaunchCheckError(f"{name}: {what}[{i}] = {int(v[i])} outside [{lo}, {int(h[i])})")


def check_routed_rows(name: str, dst_rank: torch.Tensor, dst_row: torch.Tensor,
                      peer_rows: Sequence[torch.Tensor]) -> None:
    """Every routed row goes to a rank of the group and a row inside that rank's buffer."""
    world = len(peer_rows)
    _in_range(name, dst_rank, 0, world, "dst_rank")
    caps = torch.tensor([int(p.shape[0]) for p in peer_rows], dtype=torch.long)
    _in_range(name, dst_row, 0, caps[dst_rank.reshape(-1).long().cpu()], "dst_row")


def check_ragged_tables(name: str, rows: int, tile_prefix: torch.Tensor, base: torch.Tensor, lens: torch.Tensor,
                        max_tiles: int) -> None:
    """Job ``j`` reads rows ``[base[j], base[j] + len[j])`` of A and owns blocks
    ``[tile_prefix[j], tile_prefix[j+1])`` of 256 rows; the launch covers ``max_tiles``."""
    p, b, n = tile_prefix.long().cpu(), base.long().cpu(), lens.long().cpu()
    if int(p[0]) != 0:
        raise LaunchCheckError(f"{name}: tile_prefix[0] = {int(p[0])}, expected 0")
    i = _first_bad(p[1:] < p[:-1])
    if i is not None:
        raise LaunchCheckError(f"{name}: tile_prefix decreases at job {i}")
    need = (n + ROWS_PER_TILE - 1) // ROWS_PER_TILE
    i = _first_bad(p[1:] - p[:-1] < need)
    if i is not None:
        raise LaunchCheckError(f"{name}: job {i} has {int(p[i + 1] - p[i])} blocks for {int(n[i])} rows")
    if int(p[-1]) > max_tiles:
        raise LaunchCheckError(f"{name}: the tables need {int(p[-1])} blocks, the launch covers {max_tiles}")
    i = _first_bad((b < 0) | (n < 0) | (b + n > rows))
    if i is not None:
        raise LaunchCheckError(f"{name}: job {i} reads rows [{int(b[i])}, {int(b[i] + n[i])}) of {rows}")


def check_scatter(name: str, meta: torch.Tensor, peers: Sequence[torch.Tensor], rows: int) -> None:
    """Each of the first *rows* ``(rank, row)`` pairs names a rank and a row of its output."""
    m = meta.reshape(-1, 2)[:rows]
    check_routed_rows(name, m[:, 0], m[:, 1], peers)


def check_expert_ids(name: str, topi: torch.Tensor, n_experts: int) -> None:
    """Expert ids index the routing histogram."""
    _in_range(name, topi, 0, n_experts, "expert id")


def check_mask_coords(name: str, rows: torch.Tensor, cols: torch.Tensor, k_rows: int, k_cols: int) -> None:
    """Mask-projection coordinates address the two factors' feature axes."""
    _in_range(name, rows, 0, k_rows, "row coordinate")
    _in_range(name, cols, 0, k_cols, "column coordinate")


def _opt(args: tuple, kwargs: dict, i: int, key: str, default=None):
    if len(args) > i:
        return args[i]
    return kwargs.get(key, default)


def _v_moe_dispatch(args, kwargs):
    # (src, rows_per_token, dst_rank, dst_row, peer_rows, peer_meta, self)
    check_routed_rows("moe_dispatch", args[2], args[3], args[4])


def _v_moe_combine_bwd_dispatch(args, kwargs):
    # (dy, slots, w, dw, dst_rank, dst_row, peer_rows, peer_meta, self)
    check_routed_rows("moe_combine_bwd_dispatch", args[4], args[5], args[6])


def _v_gemm_ragged(args, kwargs):
    # (A, B3, C, tile_prefix, base, len, max_tiles, peer_C, scatter, err, bn)
    a = args[0]
    check_ragged_tables("gemm_ragged", int(a.shape[0]), args[3], args[4], args[5], int(args[6]))
    scatter = _opt(args, kwargs, 8, "scatter")
    if scatter is not None and scatter.numel():
        check_scatter("gemm_ragged", scatter, args[7], int(a.shape[0]))


def _v_moe_count(args, kwargs):
    # (topi, counts)
    check_expert_ids("moe_count", args[0], int(args[1].numel()))


def _v_moe_place(args, kwargs):
    # (topi, all_counts, rank, e_l, ...)
    check_expert_ids("moe_place", args[0], int(args[1].shape[1]))


def _v_mask_gather(args, kwargs):
    # (R, C, rows, cols, out)
    check_mask_coords("mask_gather", args[2], args[3], int(args[0].shape[-1]), int(args[1].shape[-1]))


VALIDATORS: dict[str, Callable[[tuple, dict], None]] = {
    "moe_dispatch": _v_moe_dispatch,
    "moe_combine_bwd_dispatch": _v_moe_combine_bwd_dispatch,
    "gemm_ragged": _v_gemm_ragged,
    "moe_count": _v_moe_count,
    "moe_place": _v_moe_place,
    "mask_gather": _v_mask_gather,
}


class CheckedNative:
    """The extension module with :data:`VALIDATORS` run before the entry points they cover."""

    def __init__(self, module) -> None:
        self._module = module

    def __getattr__(self, name: str):
        fn = getattr(self._module, name)
        check = VALIDATORS.get(name)
        if check is None:
            return fn

        def checked(*args, **kwargs):
            check(args, kwargs)
            return fn(*args, **kwargs)

        checked.__name__ = name
        return checked
