"""Counter-based random numbers in plain PyTorch (the host twin of ``csrc/projector.cu``).

Entry ``(i, j)`` of a ``(d_in, k)`` projection is a pure function of
``(seed, d_in, k, i, j)`` -- a SplitMix64 finalizer (Steele, Lea & Flood, 2014)
of the counter ``key(seed, d_in, k) + i*k + j`` -- so any block of the matrix can
be produced independently, on any device, without materializing an identity.
Unsigned 64-bit arithmetic is emulated on ``torch.int64`` (multiplication wraps
in two's complement; right shifts are made logical with a mask).
"""

from __future__ import annotations

import math

import torch

_M64 = (1 << 64) - 1


def _s64(v: int) -> int:
    """A uint64 constant as the int64 with the same bits."""
    v &= _M64
    return v - (1 << 64) if v >= 1 << 63 else v


_GOLDEN = _s64(0x9E3779B97F4A7C15)
_MIX1 = _s64(0xBF58476D1CE4E5B9)
_MIX2 = _s64(0x94D049BB133111EB)
_FNV = 0x100000001B3


def splitmix64_int(x: int) -> int:
    """SplitMix64 finalizer on a Python int (uint64 semantics)."""
    x = (x + 0x9E3779B97F4A7C15) & _M64
    z = x
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def _lshr(x: torch.Tensor, s: int) -> torch.Tensor:
    return (x >> s) & ((1 << (64 - s)) - 1)


def splitmix64(x: torch.Tensor) -> torch.Tensor:
    """SplitMix64 finalizer on an int64 tensor holding uint64 bit patterns."""
    x = x + _GOLDEN
    z = (x ^ _lshr(x, 30)) * _MIX1
    z = (z ^ _lshr(z, 27)) * _MIX2
    return z ^ _lshr(z, 31)


def projection_key(seed: int, d_in: int, k: int) -> int:
    """Per-matrix counter offset (uint64 as a Python int)."""
    return splitmix64_int(splitmix64_int(seed & _M64) ^ ((d_in * _FNV) & _M64) ^ k)


def counter_projection_matrix(
    d_in: int,
    k: int,
    seed: int,
    *,
    kind: str = "rademacher",
    dtype: torch.dtype = torch.float32,
    device: torch.device | str = "cpu",
    rows: slice | None = None,
) -> torch.Tensor:
    """Rows *rows* (default all) of the ``(d_in, k)`` counter-based projection.

    Rademacher entries are ``+-1/sqrt(k)``; Gaussian entries are Box-Muller
    normals scaled by ``1/sqrt(k)``, so ``E[<xP, yP>] = <x, y>``.
    """
    start, stop = (0, d_in) if rows is None else (rows.start or 0, min(rows.stop, d_in))
    key = _s64(projection_key(seed, d_in, k))
    i = torch.arange(start, stop, dtype=torch.int64, device=device)
    j = torch.arange(k, dtype=torch.int64, device=device)
    h = splitmix64(key + i[:, None] * k + j[None, :])
    scale = 1.0 / math.sqrt(k)
    if kind == "rademacher":
        sign = torch.where(h < 0, -1.0, 1.0)  # bit 63 set <=> negative int64
        return (sign * scale).to(dtype)
    if kind in ("normal", "gaussian"):
        u1 = (_lshr(h, 40).double() + 0.5) / 16777216.0
        u2 = ((_lshr(h, 16) & 0xFFFFFF).double() + 0.5) / 16777216.0
        v = torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)
        return (v * scale).to(dtype)
    raise ValueError(f"unknown projection kind {kind!r}")
