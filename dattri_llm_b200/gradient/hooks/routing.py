"""Recover (sample, position) of the token rows an MoE router or expert receives.

An MoE block hands its router the block input flattened to ``(B*T, d)`` and each
expert only the rows routed to it, so those layers' captures have no batch axis.
For every block declared in ``moe_routed_layers`` the tracker records the
``(B, T, d)`` input of the enclosing module, and when a 2-D row matrix enters a
module under the declared block it locates every row in that input:

* the whole input flattened (router): a reshape;
* a gathered subset (expert): exact row matching -- each row is summarised by an
  int64 fingerprint of its raw bits, both sides are sorted by fingerprint, and
  repeated identical rows are paired by rank, then the gathered rows are checked
  bit-for-bit against their matches (any mismatch disables the layout).

:class:`RowLayout.regroup` scatters a layer's rows back into a zero ``(B, T, .)``
tensor, so unrouted positions carry an exactly-zero gradient (inert for every
downstream op; K-FAC drops them).  Parity: reference
``dattri_llm/gradient/hooks/routing.py:56-360``.  Under expert parallelism
(:mod:`dattri_llm_b200.models.olmoe`) the dispatch carries each token's
``(sample, position)`` explicitly and this matching is not needed.
"""

from __future__ import annotations

import threading
from collections.abc import Iterable
from dataclasses import dataclass

import torch
from torch import nn

_CHUNK_ELEMS = 8 * 1024 * 1024
_SEED = 0x5EED
_INT_VIEW = {2: torch.int16, 4: torch.int32, 8: torch.int64}


@dataclass(frozen=True)
class RowLayout:
    """Where each of ``rows`` routed rows sits in the ``(batch, tokens)`` grid
    (``sample`` / ``position`` ``None`` for the identity layout)."""

    batch: int
    tokens: int
    rows: int
    sample: torch.Tensor | None = None
    position: torch.Tensor | None = None

    def regroup(self, t: torch.Tensor) -> torch.Tensor:
        """``(rows, ...) -> (batch, tokens, ...)`` with zeros at unrouted positions.

        Raises:
            ValueError: when *t* does not have ``rows`` rows.
        """
        if t.shape[0] != self.rows:
            raise ValueError(f"routed capture has {t.shape[0]} rows but the layout holds {self.rows}.")
        if self.sample is None:
            return t.reshape(self.batch, self.tokens, *t.shape[1:])
        out = t.new_zeros((self.batch, self.tokens, *t.shape[1:]))
        out[self.sample.to(t.device), self.position.to(t.device)] = t
        return out


@dataclass
class _Source:
    flat: torch.Tensor
    batch: int
    tokens: int
    keys: torch.Tensor | None = None   # sorted fingerprints
    order: torch.Tensor | None = None  # row index of each sorted fingerprint


class RoutedTokenTracker:
    """Tracks routed row layouts for the hooked layers under the declared MoE blocks."""

    def __init__(self, root: nn.Module, module_names: Iterable[str]) -> None:
        modules = dict(root.named_modules())
        self._declared = tuple(sorted(set(module_names)))
        missing = [n for n in self._declared if n not in modules]
        if missing:
            raise ValueError(f"moe_routed_layers names modules that do not exist: {missing}.")
        self._root = root
        self.layers: set[str] = set()
        self._handles: list = []
        self._lock = threading.Lock()
        self._source: dict[int, _Source] = {}
        self._seen: dict[int, list] = {}
        self._latest: dict[int, RowLayout] = {}
        self._pending: dict[tuple[str, int], list[RowLayout]] = {}
        self._mult: dict = {}

    def covers(self, layer_name: str) -> bool:
        """Whether *layer_name* lies under a declared block."""
        return any(layer_name == d or layer_name.startswith(d + ".") for d in self._declared)

    def bind(self, hooked_layers: Iterable[str]) -> None:
        """Attach pre-hooks: the declared blocks' ancestors record the ``(B, T, d)``
        source, modules inside the blocks resolve 2-D row matrices against it."""
        self.layers = {n for n in hooked_layers if self.covers(n)}
        modules = dict(self._root.named_modules())
        context, subtree = set(), set()
        for d in self._declared:
            parts = d.split(".")
            context.update(".".join(parts[:i]) for i in range(len(parts)))
            subtree.update(n for n in modules if n == d or n.startswith(d + "."))
        for name in context - subtree:
            self._handles.append(modules[name].register_forward_pre_hook(self._on_context, with_kwargs=True))
        for name in subtree:
            self._handles.append(modules[name].register_forward_pre_hook(self._on_routed, with_kwargs=True))

    def remove(self) -> None:
        """Detach every hook and drop the state."""
        for h in self._handles:
            h.remove()
        self._handles = []
        self.reset()

    def reset(self) -> None:
        """Drop the per-step state."""
        with self._lock:
            self._source.clear()
            self._seen.clear()
            self._latest.clear()
            self._pending.clear()

    @staticmethod
    def _first_tensor(args, kwargs):
        for a in (*args, *kwargs.values()):
            if isinstance(a, torch.Tensor):
                return a
        return None

    @staticmethod
    def _dev(t: torch.Tensor) -> int:
        return t.device.index if t.is_cuda else 0

    def _record(self, x: torch.Tensor) -> None:
        x = x.detach()
        b, t, w = x.shape
        dev = self._dev(x)
        with self._lock:
            self._source[dev] = _Source(x.reshape(b * t, w), b, t)
            self._seen[dev] = []
            self._latest.pop(dev, None)

    def _on_context(self, _m, args, kwargs) -> None:
        if not torch.is_grad_enabled():
            return
        x = self._first_tensor(args, kwargs)
        if x is not None and x.ndim == 3 and x.is_floating_point():
            self._record(x)

    def _on_routed(self, _m, args, kwargs) -> None:
        if not torch.is_grad_enabled():
            return
        x = self._first_tensor(args, kwargs)
        if x is None or not x.is_floating_point():
            return
        if x.ndim == 3:
            self._record(x)
            return
        if x.ndim != 2:
            return
        x = x.detach()
        dev = self._dev(x)
        with self._lock:
            src = self._source.get(dev)
            if src is None or x.shape[1] != src.flat.shape[1]:
                return
            for seen, layout in self._seen.get(dev, ()):
                if seen is x or (seen.data_ptr() == x.data_ptr() and seen.shape == x.shape):
                    self._latest[dev] = layout
                    return
            layout = self._match(x, src)
            if layout is not None:
                self._seen.setdefault(dev, []).append((x, layout))
                self._latest[dev] = layout

    def push(self, layer_name: str, a: torch.Tensor, dev: int) -> RowLayout | None:
        """The layout of a 2-D capture entering *layer_name* (stacked for its backward).

        Raises:
            ValueError: when no layout with *a*'s row count exists in this forward.
        """
        if a.ndim != 2:
            return None
        with self._lock:
            layout = self._latest.get(dev)
            if layout is None or layout.rows != a.shape[0]:
                have = None if layout is None else layout.rows
                raise ValueError(
                    f"{layer_name} is declared in moe_routed_layers and received {a.shape[0]} token "
                    f"rows, but no routed layout with that row count was established in this forward "
                    f"(latest: {have}). The rows must be gathered from the (B, T, d) input of an "
                    "enclosing module, or be that input flattened to (B*T, d).",
                )
            self._pending.setdefault((layer_name, dev), []).append(layout)
        return layout

    def pop(self, layer_name: str, dev: int) -> RowLayout | None:
        """The layout pushed by the matching forward (LIFO)."""
        with self._lock:
            stack = self._pending.get((layer_name, dev))
            return stack.pop() if stack else None

    def identity_shape(self, x: torch.Tensor) -> tuple[int, int] | None:
        """``(batch, tokens)`` when *x* -- the 2-D input a module under a declared block just
        received -- is that block's whole ``(B, T, d)`` input flattened, else ``None``."""
        with self._lock:
            layout = self._latest.get(self._dev(x))
        if layout is None or layout.sample is not None or layout.rows != x.shape[0]:
            return None
        return layout.batch, layout.tokens

    def _match(self, x: torch.Tensor, src: _Source) -> RowLayout | None:
        n = x.shape[0]
        if n == src.batch * src.tokens:
            # the block's input flattened: a view of the recorded storage needs no comparison
            # (and no device read-back)
            same_view = x.data_ptr() == src.flat.data_ptr() and x.stride() == src.flat.stride()
            if same_view or torch.equal(x, src.flat):
                return RowLayout(src.batch, src.tokens, n)
        if src.keys is None:
            k = self._fingerprint(src.flat)
            src.order = torch.argsort(k, stable=True)
            src.keys = k[src.order]
        kx = self._fingerprint(x)
        lo = torch.searchsorted(src.keys, kx)
        hi = torch.searchsorted(src.keys, kx, right=True)
        # rank of each row among the gathered rows with the same fingerprint
        order_x = torch.argsort(kx, stable=True)
        sorted_x = kx[order_x]
        run_start = torch.searchsorted(sorted_x, sorted_x)
        rank = torch.empty_like(kx)
        rank[order_x] = torch.arange(n, device=x.device) - run_start
        pos = lo + rank
        if bool((pos >= hi).any()):
            return None
        token = src.order[pos]
        if not torch.equal(src.flat[token], x):
            return None
        sample = torch.div(token, src.tokens, rounding_mode="floor")
        return RowLayout(src.batch, src.tokens, n, sample, token - sample * src.tokens)

    def _fingerprint(self, t: torch.Tensor) -> torch.Tensor:
        """int64 fingerprint of each row's raw bits (random odd multipliers, summed)."""
        mult = self._multiplier(t.shape[1], t.device)
        view = _INT_VIEW[t.element_size()]
        step = max(1, _CHUNK_ELEMS // max(1, t.shape[1]))
        out = torch.empty(t.shape[0], dtype=torch.int64, device=t.device)
        for s in range(0, t.shape[0], step):
            out[s : s + step] = (t[s : s + step].contiguous().view(view).to(torch.int64) * mult).sum(-1)
        return out

    def _multiplier(self, width: int, device) -> torch.Tensor:
        key = (width, str(device))
        m = self._mult.get(key)
        if m is None:
            gen = torch.Generator().manual_seed(_SEED)
            m = (torch.randint(-(2**62), 2**62, (width,), generator=gen, dtype=torch.int64) | 1).to(device)
            self._mult[key] = m
        return m
