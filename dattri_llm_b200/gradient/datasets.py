"""Readers of the on-disk store: per-file multi-step datasets and block iteration.

Each dataset item is one store file, yielding ``{step: (block, hashes)}`` with the
records of that file concatenated per step; a ``DataLoader`` over it prefetches
files in worker processes (disk residency).  Batch-level ``param_grad`` layers
are skipped with a warning.  Parity: reference ``dattri_llm/gradient/datasets.py``.
"""

from __future__ import annotations

import warnings
from collections.abc import Iterable, Iterator

from torch.utils.data import DataLoader, Dataset, get_worker_info

from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.gradient import Gradient, base_layer_name


def identity_collate(batch: list) -> object:
    """Unwrap a batch of one item."""
    (item,) = batch
    return item


def _records_to_block(records: list, idxs: list[int], layer_name: list[str] | None, *, file_rel: str,
                      step: int) -> tuple[Gradient, list[str]]:
    grads, hashes, skipped = [], [], set()
    for idx in idxs:
        rec = records[idx]
        g = rec.gradient
        selected = g.layer_names if layer_name is None else set(layer_name)
        missing = selected - g.layer_names
        if missing:
            raise KeyError(f"Unknown layers: {sorted(missing)}")
        if layer_name is not None:
            selected |= {n for n in g.layer_names if base_layer_name(n) in selected}
        skipped.update(n for n in selected if g.layer_types[n] == ops.PARAM_GRAD_TYPES)
        keep = selected - skipped
        if not keep:
            raise ValueError("No per-sample gradient layers remain after skipping batch-level param_grad "
                             f"layers in {file_rel!r} at step {step}.")
        grads.append(g.select_layers(keep))
        hashes.extend(rec.input_hash if isinstance(rec.input_hash, list) else [rec.input_hash])
    if skipped:
        warnings.warn(f"Skipping batch-level param_grad layers during per-sample attribution: {sorted(skipped)}.",
                      stacklevel=3)
    if not grads:
        raise RuntimeError(f"No records selected for file {file_rel!r} at step {step}.")
    block = grads[0]
    for g in grads[1:]:
        block = block.concatenate(g, dim="batch")
    if block.batch_size != len(hashes):
        raise RuntimeError(f"Block batch size ({block.batch_size}) disagrees with hash count ({len(hashes)}) "
                           f"for file {file_rel!r} at step {step}.")
    return block, hashes


class GradientFileMultiStepDataset(Dataset):
    """One item per store file holding any of *steps*: ``{step: (block, hashes)}``."""

    def __init__(self, file_manager, steps: list[int], layer_name: list[str] | None = None) -> None:
        self._fm = file_manager
        self._layer_name = list(layer_name) if layer_name is not None else None
        self._files = file_manager.iter_steps(list(steps))

    def __len__(self) -> int:
        return len(self._files)

    def __getitem__(self, i: int) -> dict:
        file_rel, by_step = self._files[i]
        records = self._fm.load_records(file_rel)
        blocks = {s: _records_to_block(records, idxs, self._layer_name, file_rel=file_rel, step=s)
                  for s, idxs in by_step.items()}
        if get_worker_info() is not None:  # detach from the worker's memmap before pickling back
            blocks = {s: (b.clone(), h) for s, (b, h) in blocks.items()}
        return blocks


def make_gradient_multistep_dataloader(file_manager, steps: list[int], args, layer_name=None) -> DataLoader:
    """A ``DataLoader`` of :class:`GradientFileMultiStepDataset` (workers only for disk stores)."""
    workers = args.dataloader_num_workers if file_manager.residency == "disk" else 0
    kw: dict = {"dataset": GradientFileMultiStepDataset(file_manager, steps, layer_name=layer_name),
                "batch_size": 1, "shuffle": False, "collate_fn": identity_collate, "num_workers": workers,
                "pin_memory": args.dataloader_pin_memory}
    if workers > 0:
        kw["persistent_workers"] = args.dataloader_persistent_workers
        if args.dataloader_prefetch_factor is not None:
            kw["prefetch_factor"] = args.dataloader_prefetch_factor
    return DataLoader(**kw)


def resolve_steps(file_manager, requested: Iterable[int] | None) -> list[int]:
    """The stored steps among *requested* (all when ``None``).

    Raises:
        ValueError: when none of the requested steps is stored.
    """
    available = file_manager.available_steps()
    if requested is None:
        return available
    wanted = set(requested)
    selected = [s for s in available if s in wanted]
    if not selected:
        raise ValueError(f"None of the requested steps {sorted(wanted)} are present in the gradients; "
                         f"available steps: {available}.")
    return selected


def iter_gradient_blocks(file_manager, steps: list[int], args, layer_name=None, desc=None,
                         verbose: bool = False) -> Iterator[tuple[int, Gradient, list[str]]]:
    """``(step, block, hashes)`` for every stored block of *steps*, file by file."""
    if not steps:
        return
    bar = None
    if verbose and desc is not None and args.should_log:
        from tqdm.auto import tqdm

        bar = tqdm(total=sum(len(b) for _, b in file_manager.iter_steps(list(steps))), desc=desc,
                   unit="block", leave=False)
    try:
        for by_step in make_gradient_multistep_dataloader(file_manager, list(steps), args, layer_name):
            for step, (block, hashes) in by_step.items():
                yield step, block, hashes
                if bar is not None:
                    bar.update(1)
    finally:
        if bar is not None:
            bar.close()
