"""The shared scoring loop and collection helpers of the inner-product attributors.

:func:`score_sources` pairs every train block with every test block through an
``inner_product`` (parity: reference ``dattri_llm/attribution/utils.py:239-447``:
test set cached once or looped per train block, dense test blocks merged, train
blocks re-batched to the train batch size, dense materialization of a factorized
train layer reused across test blocks, instance or token granularity).

B200 execution differences:

* scores stay on the device in fp32 and come back to the host once at the end
  (the reference copies every ``(B_train, B_test)`` block to the host as it goes,
  a synchronization per pair);
* when both sides of a pair are entirely dense with the same layers and widths --
  the common case of projected / materialized captures -- the layers are packed
  into one contiguous ``(B, sum_l d_l)`` matrix per side (the test side once) and
  the whole layerwise sum is ONE split-K tcgen05 GEMM instead of one GEMM per layer.
"""

from __future__ import annotations

from dattri_llm_b200.options import AttributionGranularity  # noqa: F401  (re-exported option types)
import json
import pathlib
from collections.abc import Callable, Iterable, Mapping

import torch

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
from dattri_llm_b200.gradient.streaming import rebatch_blocks
from dattri_llm_b200.utils.cache import CacheBudget, TensorCache
from dattri_llm_b200.utils.tracing import trace_range

InnerProduct = Callable[..., torch.Tensor]
Transform = Callable[[Gradient], Gradient]


def normalize_layer_names(layer_name: str | list[str] | None) -> list[str] | None:
    """``None`` / one name / a list -> ``None`` or a list."""
    if layer_name is None:
        return None
    return [layer_name] if isinstance(layer_name, str) else list(layer_name)


def collect_gradients(streamer, store, *, offload_interval: int = 1, on_block=None,
                      async_write: bool | None = None, resume: bool = False):
    """Run *streamer* to completion into *store* (groups of *offload_interval* steps;
    asynchronous writes per ``args.async_disk_write``).

    With *resume*, a collection that was interrupted picks up where it stopped: the
    batches whose records this rank already wrote for the streamer's checkpoint (whole
    groups; a group whose index line was cut off is redone) are skipped, checked against
    the stored hashes, and the rest are appended.  Frozen probes only.
    """
    if offload_interval < 1:
        raise ValueError(f"offload_interval must be >= 1, got {offload_interval}.")
    if resume:
        done = [h for step, h in store.own_records() if step == streamer.checkpoint_step]
        if done:
            streamer.skip_batches(len(done), expected_hashes=done)
    if async_write is None:
        async_write = getattr(getattr(streamer, "args", None), "async_disk_write", False)
    writer = None
    if async_write:
        from dattri_llm_b200.gradient.async_writer import AsyncGradientWriter

        writer = AsyncGradientWriter(store)
    save = writer.submit if writer is not None else store.save_bulk
    id_key = streamer.hook_manager.sample_id_key
    staged: list[GradientRecord] = []
    try:
        with streamer:
            for step, grad, hashes in streamer:
                if on_block is not None:
                    on_block(step, grad, hashes)
                staged.append(GradientRecord(step, hashes, grad, id_key))
                if len(staged) >= offload_interval:
                    save(staged)
                    staged = []
            if staged:
                save(staged)
    finally:
        if writer is not None:
            writer.close()
    return store


def _identity(block: Gradient) -> Gradient:
    return block


def finalize_factors(rep: Gradient, *, budget: CacheBudget | None = None, held: int = 0) -> Gradient:
    """Apply preprocessing once (im2col, x_hat, bias columns) to every raw factorized
    layer, within the budget, so pairing a block with many others does not redo it."""
    names = [n for n, v in rep.data.items()
             if isinstance(v, Factorized) and v.module_kwargs is not None and not ops.is_embedding(rep.layer_types[n])]
    if not names:
        return rep
    charged = held

    def finalize(_n, value: Factorized, lt: str):
        nonlocal charged
        a, g = ops.preprocess_factorized(value, lt)
        final = Factorized(a, g, module_kwargs=None)
        growth = max(final.nbytes - value.nbytes, 0)
        if budget is not None and not budget.fits(growth, charged):
            return value
        charged += growth
        return final

    return rep.map_layers(finalize, layers=names, consume=True)


class PackedDense:
    """A fully dense block packed into one contiguous ``(B, sum_l d_l)`` matrix
    (layers in sorted order) plus the layout needed to check a partner block."""

    __slots__ = ("layout", "matrix")

    def __init__(self, matrix: torch.Tensor, layout: tuple) -> None:
        self.matrix, self.layout = matrix, layout

    @staticmethod
    def layout_of(block: Gradient) -> tuple | None:
        if not block.data or not all(isinstance(v, torch.Tensor) for v in block.data.values()):
            return None
        if any(t == ops.PARAM_GRAD_TYPES for t in block.layer_types.values()):
            return None
        b = block.batch_size
        layout = []
        for name in sorted(block.data):
            v = block.data[name]
            if v.shape[0] != b:  # a broadcast layer: keep the general path
                return None
            layout.append((name, v[0].numel()))
        return tuple(layout)

    @classmethod
    def pack(cls, block: Gradient, dtype: torch.dtype | None = None) -> PackedDense | None:
        layout = cls.layout_of(block)
        if layout is None:
            return None
        rows = block.batch_size  # a scan over every layer: once, not per layer
        parts = [block.data[n].reshape(rows, -1) for n, _ in layout]
        dtype = dtype or parts[0].dtype
        return cls(torch.cat([p.to(dtype) for p in parts], dim=1), layout)


def packed_cross_dot(train: PackedDense, test: PackedDense) -> torch.Tensor:
    """``(B_train, B_test)`` fp32 sum over layers as one GEMM."""
    a, b = train.matrix, test.matrix
    from dattri_llm_b200 import ops as native_ops

    if native_ops.use_native(a, b) and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
        return native_ops.matmul_tn(a, b)
    return a.float() @ b.float().T


def score_sources(train_source: Iterable, test_source: Iterable, device, *, inner_product: InnerProduct,
                  transform_train: Transform | None = None, transform_test: Transform | None = None,
                  batch_size: int = 1, loop_over_test: bool = False, cache_budget: CacheBudget | None = None,
                  granularity: str = "instance", inner_product_per_token: InnerProduct | None = None,
                  packed_inner_product: bool = False):
    """Score every train block against every test block.

    Returns ``(scores (rows, num_test) fp32 on the host, row_train_ids, row_steps,
    test_ids, row_token_ids or None)``.  *packed_inner_product* declares that
    *inner_product* is the plain layerwise dot product, which lets fully dense
    pairs take the one-GEMM packed path.
    """
    if loop_over_test and not getattr(test_source, "reusable", False):
        raise ValueError("loop_over_test=True requires a re-iterable test source (reusable=True); got a "
                         "single-shot source.")
    if granularity not in {"instance", "token"}:
        raise ValueError(f"granularity must be 'instance' or 'token', got {granularity!r}.")
    per_token = granularity == "token"
    if per_token and inner_product_per_token is None:
        raise ValueError("granularity='token' needs inner_product_per_token.")
    transform_train = transform_train or _identity
    transform_test = transform_test or _identity
    budget = cache_budget if cache_budget is not None else CacheBudget(device)

    test_ids: list[str] = []
    test_index: dict[str, int] = {}
    cached: list[tuple[Gradient, list[int]]] = []
    for _s, tg, th in test_source:
        cols = []
        for h in th:
            if h not in test_index:
                test_index[h] = len(test_ids)
                test_ids.append(h)
            cols.append(test_index[h])
        if not loop_over_test:
            cached.append((transform_test(tg.to(device)), cols))
    num_test = len(test_ids)
    if len(cached) > 1:
        merged = list(rebatch_blocks(((0, rep, cols) for rep, cols in cached),
                                     batch_size=sum(len(c) for _, c in cached)))
        cached = [(rep, cols) for _st, rep, cols in merged]
    packed_test = None
    if packed_inner_product and not per_token and len(cached) == 1:
        p = PackedDense.pack(cached[0][0])
        if p is not None:
            packed_test = (p, torch.tensor(cached[0][1], dtype=torch.long, device=p.matrix.device))

    def n_rows(rep: Gradient) -> int:
        if not per_token:
            return rep.batch_size
        toks = [t for t in rep.token_dim.values() if t is not None]
        return rep.batch_size * (max(toks) if toks else 1)

    def score_block(train_rep: Gradient, test_blocks, dense_cache) -> torch.Tensor:
        with trace_range("dattri.score.block"):
            return _score_block(train_rep, test_blocks, dense_cache)

    def _score_block(train_rep: Gradient, test_blocks, dense_cache) -> torch.Tensor:
        row = None
        if packed_test is not None:
            pk, cols = packed_test
            if PackedDense.layout_of(train_rep) == pk.layout:
                tp = PackedDense.pack(train_rep, pk.matrix.dtype)
                block = packed_cross_dot(tp, pk)
                row = torch.zeros(block.shape[0], num_test, dtype=torch.float32, device=block.device)
                row[:, cols] = block.float()
                return row
        for test_rep, cols in test_blocks:
            if per_token:
                b = inner_product_per_token(train_rep, test_rep)
                block = b.reshape(-1, b.shape[-1])
            else:
                block = inner_product(train_rep, test_rep, dense_cache=dense_cache)
            if row is None:
                row = torch.zeros(n_rows(train_rep), num_test, dtype=torch.float32, device=block.device)
            row[:, cols] = block.detach().float()
        if row is None:
            row = torch.zeros(n_rows(train_rep), num_test, dtype=torch.float32)
        return row

    chunks: list[torch.Tensor] = []
    row_ids: list[str] = []
    row_steps: list[int] = []
    row_toks: list[int] = []

    def stamp(ids, steps, chunk):
        if not per_token:
            row_ids.extend(ids)
            row_steps.extend(steps)
            return
        t = chunk.shape[0] // max(len(ids), 1)
        for h, s in zip(ids, steps, strict=True):
            row_ids.extend([h] * t)
            row_steps.extend([s] * t)
            row_toks.extend(range(t))

    if not loop_over_test:
        reuse = len(cached) > 1 and not per_token
        for steps, tg, ids in rebatch_blocks(train_source, batch_size):
            rep = transform_train(tg.to(device))
            if reuse:
                with TensorCache("memory", budget=budget) as dc:
                    chunk = score_block(rep, cached, dc)
            else:
                chunk = score_block(rep, cached, None)
            chunks.append(chunk)
            stamp(ids, steps, chunk)
    else:
        for step, tg, th in train_source:
            rep = transform_train(tg.to(device))

            def blocks():
                for _s, g2, h2 in test_source:
                    yield transform_test(g2.to(device)), [test_index[h] for h in h2]

            with TensorCache("memory", budget=budget) as dc:
                chunk = score_block(rep, blocks(), dc)
            chunks.append(chunk)
            stamp(list(th), [step] * rep.batch_size, chunk)
    if chunks:
        dev = chunks[0].device
        scores = torch.cat([c.to(dev) for c in chunks], dim=0).cpu()
    else:
        scores = torch.zeros(0, num_test, dtype=torch.float32)
    return scores, row_ids, row_steps, test_ids, (row_toks if per_token else None)


LR_SCHEDULE_FILE = "lr_schedule.json"


def write_lr_schedule(train_gradients_dir: str, lrs: Mapping[int, float]) -> None:
    """Store ``{step: lr}`` next to a train store."""
    root = pathlib.Path(train_gradients_dir)
    root.mkdir(exist_ok=True, parents=True)
    (root / LR_SCHEDULE_FILE).write_text(json.dumps({str(k): float(v) for k, v in lrs.items()}), encoding="utf-8")


def read_lr_schedule(train_gradients_dir: str) -> dict[int, float] | None:
    """The ``{step: lr}`` stored next to a train store, or ``None``."""
    path = pathlib.Path(train_gradients_dir) / LR_SCHEDULE_FILE
    if not path.exists():
        return None
    return {int(k): float(v) for k, v in json.loads(path.read_text(encoding="utf-8")).items()}
