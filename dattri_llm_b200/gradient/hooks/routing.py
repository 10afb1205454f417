"""Where the token rows an MoE router or expert receives sit in the ``(batch, token)`` grid.

An MoE block hands its router the block input flattened to ``(B*T, d)`` and each expert
only the rows routed to it, so those layers' captures carry no batch axis.  For every
block named in ``moe_routed_layers`` the tracker keeps the ``(B, T, d)`` input of the
enclosing module (the *grid*), and when a 2-D row matrix enters a module inside the block
it decides where each row came from:

* placed: the library's own expert loop (:mod:`.override_layers.fused_experts`) gathers
  the rows itself and says which grid positions they are -- nothing is matched;
* the whole grid flattened (a router): recognised by storage, or by one comparison;
* any other gather from the grid (user-written experts): exact row matching.  The grid
  rows and the gathered rows are numbered together by ``torch.unique`` over their raw
  bits (identical rows share a number), the grid's positions are grouped per number, and
  the k-th gathered row with a number takes the k-th grid position with it -- repeated
  identical rows (padding, say) pair up in order, and no hash can collide.

:meth:`RowLayout.regroup` scatters a layer's rows back into a zero ``(B, T, .)`` tensor, so
positions not routed to the layer carry an exactly-zero gradient.  Reference behaviour:
``dattri_llm/gradient/hooks/routing.py``.  Under expert parallelism
(:mod:`dattri_llm_b200.parallel.moe`) every row carries its ``(sample, position)`` and no
matching is needed.
"""

from __future__ import annotations

import threading
from collections.abc import Iterable
from dataclasses import dataclass

import torch
from torch import nn

_BITS = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


@dataclass(frozen=True)
class RowLayout:
    """The grid positions (``b * tokens + t``) of ``rows`` routed rows; ``flat`` is
    ``None`` when the rows are the whole grid in order."""

    batch: int
    tokens: int
    rows: int
    flat: torch.Tensor | None = None

    @property
    def identity(self) -> bool:
        """Whether the rows are the whole grid, in order."""
        return self.flat is None

    def regroup(self, t: torch.Tensor) -> torch.Tensor:
        """``(rows, ...) -> (batch, tokens, ...)``, zero at positions no row came from.

        Raises:
            ValueError: when *t* does not have ``rows`` rows.
        """
        if t.shape[0] != self.rows:
            raise ValueError(f"a routed capture brought {t.shape[0]} rows to a layout of {self.rows}.")
        tail = t.shape[1:]
        if self.flat is None:
            return t.reshape(self.batch, self.tokens, *tail)
        grid = t.new_zeros((self.batch * self.tokens, *tail))
        grid.index_copy_(0, self.flat.to(t.device), t)
        return grid.view(self.batch, self.tokens, *tail)


def _exact_positions(gathered: torch.Tensor, grid: torch.Tensor) -> torch.Tensor | None:
    """Grid row of every gathered row (exact bitwise equality; repeated rows paired in
    order), or ``None`` when some gathered row is not in the grid."""
    n_grid = grid.shape[0]
    bits = _BITS[grid.element_size()]
    both = torch.cat([grid.contiguous().view(bits), gathered.contiguous().view(bits)])
    _, number = torch.unique(both, dim=0, return_inverse=True)
    grid_no, row_no = number[:n_grid], number[n_grid:]
    # grid positions grouped by number (stable: each group in position order)
    grid_sorted, grid_order = torch.sort(grid_no, stable=True)
    group_start = torch.searchsorted(grid_sorted, row_no)
    group_end = torch.searchsorted(grid_sorted, row_no, right=True)
    # the k-th gathered row of a number takes the group's k-th position
    rows_sorted, rows_order = torch.sort(row_no, stable=True)
    first_of_run = torch.searchsorted(rows_sorted, rows_sorted)
    rank = torch.empty_like(row_no)
    rank[rows_order] = torch.arange(row_no.numel(), device=row_no.device) - first_of_run
    slot = group_start + rank
    if bool((slot >= group_end).any()):
        return None
    return grid_order[slot]


@dataclass
class _Grid:
    flat: torch.Tensor
    batch: int
    tokens: int


class RoutedTokenTracker:
    """Row layouts of the hooked layers inside the declared MoE blocks (see the module
    docstring)."""

    def __init__(self, root: nn.Module, module_names: Iterable[str]) -> None:
        modules = dict(root.named_modules())
        self._blocks = tuple(sorted(set(module_names)))
        unknown = [n for n in self._blocks if n not in modules]
        if unknown:
            raise ValueError(f"moe_routed_layers names no module of the model: {unknown}.")
        self._root = root
        self.layers: set[str] = set()
        self._handles: list = []
        self._lock = threading.Lock()
        self._grid: dict[int, _Grid] = {}                   # device -> the block input in use
        self._known: dict[int, list] = {}                   # device -> [(rows tensor, layout)] this forward
        self._current: dict[int, RowLayout] = {}            # device -> layout of the last rows that entered
        self._stacks: dict[tuple[str, int], list[RowLayout]] = {}  # (layer, device) -> layouts awaiting backward

    def covers(self, layer_name: str) -> bool:
        """Whether *layer_name* lies inside a declared block."""
        return any(layer_name == b or layer_name.startswith(b + ".") for b in self._blocks)

    def bind(self, hooked_layers: Iterable[str]) -> None:
        """Install the pre-hooks: modules around a declared block record the grid, modules
        inside it resolve the 2-D rows they receive."""
        self.layers = {n for n in hooked_layers if self.covers(n)}
        modules = dict(self._root.named_modules())
        outer, inner = set(), set()
        for block in self._blocks:
            parts = block.split(".")
            outer.update(".".join(parts[:i]) for i in range(len(parts)))
            inner.update(n for n in modules if n == block or n.startswith(block + "."))
        for name in outer - inner:
            self._handles.append(modules[name].register_forward_pre_hook(self._grid_input, with_kwargs=True))
        for name in inner:
            self._handles.append(modules[name].register_forward_pre_hook(self._row_input, with_kwargs=True))

    def remove(self) -> None:
        """Detach every hook and drop the state."""
        for handle in self._handles:
            handle.remove()
        self._handles = []
        self.reset()

    def reset(self) -> None:
        """Forget the step's grids and layouts."""
        with self._lock:
            self._grid.clear()
            self._known.clear()
            self._current.clear()
            self._stacks.clear()

    @staticmethod
    def _tensor_arg(args: tuple, kwargs: dict) -> torch.Tensor | None:
        return next((a for a in (*args, *kwargs.values()) if isinstance(a, torch.Tensor)), None)

    @staticmethod
    def _device(t: torch.Tensor) -> int:
        return t.device.index if t.is_cuda else 0

    def _set_grid(self, x: torch.Tensor) -> None:
        b, t, width = x.shape
        dev = self._device(x)
        with self._lock:
            self._grid[dev] = _Grid(x.detach().reshape(b * t, width), b, t)
            self._known[dev] = []
            self._current.pop(dev, None)

    def _grid_input(self, _module, args, kwargs) -> None:
        x = self._tensor_arg(args, kwargs)
        if torch.is_grad_enabled() and x is not None and x.ndim == 3 and x.is_floating_point():
            self._set_grid(x)

    def _row_input(self, _module, args, kwargs) -> None:
        x = self._tensor_arg(args, kwargs)
        if not torch.is_grad_enabled() or x is None or not x.is_floating_point():
            return
        if x.ndim == 3:
            self._set_grid(x)
            return
        if x.ndim != 2:
            return
        dev = self._device(x)
        with self._lock:
            grid = self._grid.get(dev)
            if grid is None or x.shape[1] != grid.flat.shape[1]:
                return  # not rows of the grid (e.g. an expert's hidden activation): keep the current layout
            for rows, layout in self._known.get(dev, ()):
                if rows is x:
                    self._current[dev] = layout
                    return
            layout = self._resolve(x.detach(), grid)
            if layout is not None:
                self._known.setdefault(dev, []).append((x, layout))
                self._current[dev] = layout

    @staticmethod
    def _resolve(x: torch.Tensor, grid: _Grid) -> RowLayout | None:
        n = x.shape[0]
        if n == grid.batch * grid.tokens:
            same_storage = x.data_ptr() == grid.flat.data_ptr() and x.stride() == grid.flat.stride()
            if same_storage or torch.equal(x, grid.flat):
                return RowLayout(grid.batch, grid.tokens, n)
        flat = _exact_positions(x, grid.flat)
        return None if flat is None else RowLayout(grid.batch, grid.tokens, n, flat)

    def place(self, rows: torch.Tensor, flat_positions: torch.Tensor) -> None:
        """Declare that *rows* are the grid rows at *flat_positions* (``b * T + t``): the
        layout of the next layers that receive them, with no matching."""
        dev = self._device(rows)
        with self._lock:
            grid = self._grid.get(dev)
            if grid is None:
                return
            layout = RowLayout(grid.batch, grid.tokens, rows.shape[0], flat_positions)
            self._known.setdefault(dev, []).append((rows, layout))
            self._current[dev] = layout

    def identity_shape(self, x: torch.Tensor) -> tuple[int, int] | None:
        """``(batch, tokens)`` when *x* -- the 2-D input a module inside a declared block just
        received -- is that block's whole grid in order, else ``None``."""
        with self._lock:
            layout = self._current.get(self._device(x))
        if layout is None or not layout.identity or layout.rows != x.shape[0]:
            return None
        return layout.batch, layout.tokens

    def push(self, layer_name: str, a: torch.Tensor, dev: int) -> RowLayout | None:
        """The layout of a 2-D capture entering *layer_name*, kept for its backward.

        Raises:
            ValueError: when no layout with *a*'s row count was established in this forward.
        """
        if a.ndim != 2:
            return None
        with self._lock:
            layout = self._current.get(dev)
            if layout is None or layout.rows != a.shape[0]:
                seen = None if layout is None else layout.rows
                raise ValueError(
                    f"{layer_name} lies in a moe_routed_layers block and received {a.shape[0]} token rows, but "
                    f"this forward established no row layout of that size (last one: {seen} rows). Rows must be "
                    "gathered from the (B, T, d) input of an enclosing module, or be that input flattened.")
            self._stacks.setdefault((layer_name, dev), []).append(layout)
        return layout

    def pop(self, layer_name: str, dev: int) -> RowLayout | None:
        """The layout pushed by the matching forward (last in, first out)."""
        with self._lock:
            stack = self._stacks.get((layer_name, dev))
            return stack.pop() if stack else None
