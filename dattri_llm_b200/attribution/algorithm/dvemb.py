"""DVEmb: data value embeddings (trajectory-aware, first-order with Fisher propagation).

Sweeping the trajectory backwards from the final step, a sample's embedding at step
``t`` is ``lr_t * (g - g M_t^T)`` where ``M`` accumulates ``lr * s * sum_b e_b g_b^T``
over the later steps (``s = n_t`` for a mean-reduced loss, else 1): the effect of
the sample's step propagated through the later Fisher ``(I - lr H)`` factors --
``hessian_mode="full"`` keeps one ``d x d`` operator, ``"diagonal"`` a block per
layer.  Scores are ``<embedding, g_test>``.  ``propagation="test"`` instead carries
the query matrix backwards (``W <- W - lr s D^T g``), never forming the ``d x d``
operator.  Parity: reference ``dattri_llm/attribution/algorithm/dvemb.py:135-929``.
The per-step operator products are dense GEMMs (cuBLAS fp32 / tf32).
"""

from __future__ import annotations

import contextlib
import pathlib
import tempfile
import warnings
from collections.abc import Iterable, Iterator, Mapping
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.algorithm.trajectory import TrajectoryAttributor, dense_block
from dattri_llm_b200.ops.gemm import matmul_f32
from dattri_llm_b200.gradient.gradient import Gradient, GradientRecord
from dattri_llm_b200.gradient.snapshots import TrajectorySnapshots
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.utils.cache import CACHE_RESIDENCIES


class DVEmbAttributor(TrajectoryAttributor):
    """DVEmb (Data Value Embedding) attributor."""

    algorithm: ClassVar[str] = "DVEmb"

    def cache_dvemb(self, train_gradients_dir: str, dvemb_dir: str | None = None, *,
                    selected_training_steps: Iterable[int] | None = None, hessian_mode: str = "full",
                    final_step: int | None = None, loss_reduction: str = "mean", verbose: bool = False,
                    layer_name=None, learning_rate=1.0) -> str:
        """Compute the embeddings of a stored trajectory and store them (score later with
        ``TracInAttributor.attribute_from_cache``)."""
        dvemb_dir = dvemb_dir or str(pathlib.Path(self.args.output_dir) / "dvemb_grads")
        self._validate(loss_reduction, "train", hessian_mode, loop_over_test=False, dvemb_dir=None)
        train = self.open_train_source(train_gradients_dir, layer_name=layer_name)
        try:
            prop, out, _final, lr = self._resolve_sweep(train, self.recorded_lr_of(train), selected_training_steps,
                                                        final_step, learning_rate)
            emb = self.embed_trajectory(train.for_steps(prop), prop, out, learning_rate=lr,
                                        loss_reduction=loss_reduction, hessian_mode=hessian_mode, verbose=verbose)
            self.cache_representations(emb, GradientStorageManager(dvemb_dir), transform=lambda b: b,
                                       sample_id_key=self._sample_id_key(train))
        finally:
            self.close_source(train)
        return dvemb_dir

    @staticmethod
    def _sample_id_key(train):
        return getattr(getattr(train, "file_manager", None), "sample_id_key", None)

    @staticmethod
    def _normalize_lr(lr):
        if isinstance(lr, Mapping):
            return {int(k): float(v) for k, v in lr.items()}
        lr = float(lr)
        if lr < 0:
            raise ValueError(f"learning_rate must be non-negative, got {lr}.")
        return lr

    @staticmethod
    def _lr(lr, step: int) -> float:
        if isinstance(lr, dict):
            if step not in lr:
                raise ValueError(f"learning_rate mapping has no entry for step {step}; it must cover every "
                                 f"propagated step (step < final_step). Provided steps: {sorted(lr)}.")
            return lr[step]
        return lr

    def _warn_on_lr_mismatch(self, lr, recorded: Mapping[int, float], prop: list[int]) -> None:
        bad = []
        for s in sorted(prop):
            want = recorded.get(s)
            if want is None:
                continue
            try:
                got = self._lr(lr, s)
            except ValueError:
                continue
            if abs(got - want) > 1e-9 + 1e-6 * abs(want):
                bad.append((s, got, want))
        if bad:
            s0, g0, w0 = bad[0]
            warnings.warn(f"DVEmb learning_rate disagrees with the schedule recorded during training at "
                          f"{len(bad)}/{len(prop)} step(s) (e.g. step {s0}: configured {g0:g} vs recorded {w0:g}). "
                          "The configured schedule is used, but the Fisher factors (I - eta H) will not match the "
                          "trajectory -- set learning_rate to the recorded schedule.", stacklevel=2)

    def _resolve_sweep(self, train, recorded, selected, final_step, lr):
        prop, out, final_step = self.resolve_steps(self.available_steps(train), selected, final_step)
        lr = self._normalize_lr(lr)
        if recorded is not None:
            self._warn_on_lr_mismatch(lr, recorded, prop)
        return prop, out, final_step, lr

    @staticmethod
    def _validate(loss_reduction, propagation, hessian_mode, loop_over_test, dvemb_dir) -> None:
        if loss_reduction not in ("mean", "sum"):
            raise ValueError(f"loss_reduction must be 'mean' or 'sum', got {loss_reduction!r}.")
        TrajectoryAttributor.validate_propagation(propagation, loop_over_test)
        if hessian_mode not in ("full", "diagonal"):
            raise ValueError(f"hessian_mode must be 'full' or 'diagonal', got {hessian_mode!r}.")
        if dvemb_dir is not None and propagation != "train":
            raise ValueError("dvemb_dir requires propagation='train': data value embeddings only exist in the "
                             "train-side sweep.")

    def _layer_slices(self, train_source, step: int):
        for _s, g, _h in train_source.for_steps([step]):
            mat = dense_block(g.to(self.args.device))
            layers, slices, off = list(mat.data), {}, 0
            for n in layers:
                slices[n] = (off, off + mat.data[n].shape[1])
                off = slices[n][1]
            return layers, slices
        raise ValueError(f"No train gradients recorded at step {step}.")

    def embed_trajectory(self, train_source, prop_steps: list[int], output_steps: set, *, learning_rate,
                         loss_reduction: str = "mean", hessian_mode: str = "full",
                         verbose: bool = False) -> Iterator[tuple[int, Gradient, list[str]]]:
        """Yield ``(step, embeddings, hashes)`` for the output steps, sweeping backwards."""
        dev = self.args.device
        layers, slices = self._layer_slices(train_source, max(prop_steps))
        d = slices[layers[-1]][1] if layers else 0
        elems = d * d if hessian_mode == "full" else sum((e - s) ** 2 for s, e in slices.values())
        if elems * 4 / 2**30 > 2.0:
            warnings.warn(f"propagation='train' maintains a {'(%d, %d)' % (d, d) if hessian_mode == 'full' else 'block-diagonal'} "
                          f"float32 operator (~{elems * 4 / 2**30:.1f} GiB) on {dev}. Project the gradients at "
                          "collection time and/or restrict layer_name, or use propagation='test'.", stacklevel=3)
        op: torch.Tensor | None = None
        blocks: dict[str, torch.Tensor | None] = dict.fromkeys(layers)
        for ts in self.steps_bar(prop_steps, "DVEmb: embedding (train side)", verbose):
            lr = self._lr(learning_rate, ts)
            emit = ts in output_steps
            delta = None
            delta_blocks: dict[str, torch.Tensor] = {}
            n_t = 0
            for _s, g, hashes in train_source.for_steps([ts]):
                mat = dense_block(g.to(dev))
                shared = [n for n in layers if n in mat.data]
                if not shared:
                    continue
                b = mat.data[shared[0]].shape[0]
                n_t += b
                flat = torch.zeros(b, d, device=dev)
                for n in shared:
                    s, e = slices[n]
                    flat[:, s:e] = mat.data[n]
                if hessian_mode == "full":
                    e_raw = flat if op is None else flat - matmul_f32(flat, op, b_transposed=True)
                else:
                    e_raw = flat.clone()
                    for n in shared:
                        if blocks[n] is not None:
                            s, e = slices[n]
                            e_raw[:, s:e] = flat[:, s:e] - matmul_f32(flat[:, s:e], blocks[n], b_transposed=True)
                if emit:
                    emb = lr * e_raw
                    yield ts, Gradient(dict.fromkeys(shared, "materialized"),
                                       {n: emb[:, slices[n][0]:slices[n][1]].contiguous() for n in shared},
                                       {n: g.layer_types[n] for n in shared}), list(hashes)
                if hessian_mode == "full":
                    upd = matmul_f32(e_raw.t(), flat)
                    delta = upd if delta is None else delta + upd
                else:
                    for n in shared:
                        s, e = slices[n]
                        upd = matmul_f32(e_raw[:, s:e].t(), flat[:, s:e])
                        delta_blocks[n] = upd if n not in delta_blocks else delta_blocks[n] + upd
            scale = float(n_t) if loss_reduction == "mean" else 1.0
            if delta is not None:
                op = lr * scale * delta if op is None else op + lr * scale * delta
            for n, upd in delta_blocks.items():
                blocks[n] = lr * scale * upd if blocks[n] is None else blocks[n] + lr * scale * upd

    def _propagate_test_and_score(self, w: dict[str, torch.Tensor], n_cols: int, train_source, prop_steps,
                                  output_steps, *, learning_rate, loss_reduction: str, hessian_mode: str,
                                  verbose: bool, block_dtype: torch.dtype = torch.float32):
        dev = self.args.device
        layers = list(w)
        chunks, ids, steps = [], [], []
        for ts in self.steps_bar(prop_steps, "DVEmb: propagating (test side)", verbose):
            lr = self._lr(learning_rate, ts)
            emit = ts in output_steps
            delta = {n: torch.zeros_like(w[n]) for n in layers}
            n_t = 0
            for _s, g, hashes in train_source.for_steps([ts]):
                mat = dense_block(g.to(dev), block_dtype).data
                shared = [n for n in layers if n in mat]
                if not shared:
                    continue
                b = mat[shared[0]].shape[0]
                n_t += b
                per_layer = {n: matmul_f32(mat[n].float(), w[n], b_transposed=True) for n in shared}
                dmat = torch.zeros(b, n_cols, device=dev)
                for n in shared:
                    dmat += per_layer[n]
                if emit:
                    chunks.append(lr * dmat)
                    ids.extend(hashes)
                    steps.extend([ts] * b)
                for n in shared:
                    delta[n] += matmul_f32((dmat if hessian_mode == "full" else per_layer[n]).t(), mat[n].float())
            scale = float(n_t) if loss_reduction == "mean" else 1.0
            for n in layers:
                w[n] -= lr * scale * delta[n]
        scores = torch.cat(chunks).cpu() if chunks else torch.zeros(0, n_cols)
        return scores, ids, steps

    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False,
                  loop_over_test: bool = False, gradient_cache_residency: str = "disk", propagation: str = "train",
                  dvemb_dir: str | None = None, hessian_mode: str = "full", selected_training_steps=None,
                  loss_reduction: str = "mean", learning_rate=1.0):
        """Train from checkpoint 0 collecting the trajectory, then attribute over it."""
        self.require_task("attribute")
        if gradient_cache_residency not in CACHE_RESIDENCIES:
            raise ValueError(f"gradient_cache_residency must be one of {list(CACHE_RESIDENCIES)}, got "
                             f"{gradient_cache_residency!r}.")
        opts = {"propagation": propagation, "dvemb_dir": dvemb_dir, "hessian_mode": hessian_mode,
                "loop_over_test": loop_over_test, "selected_training_steps": selected_training_steps,
                "loss_reduction": loss_reduction, "verbose": verbose, "learning_rate": learning_rate}
        if gradient_cache_residency == "disk":
            ((train_dir, test_dir),) = self.cache(train_dataset, test_dataset, hook_config=hook_config)
            return self.attribute_from_cache(train_dir, test_dir, hook_config=hook_config, **opts)
        target = (TrajectorySnapshots(tempfile.mkdtemp(prefix="dvemb_snapshots_")) if self.recompute
                  else GradientStorageManager(tempfile.mkdtemp(prefix="dvemb_train_"),
                                              residency=gradient_cache_residency))
        with (target if isinstance(target, GradientStorageManager) else contextlib.nullcontext(),
              GradientStorageManager(tempfile.mkdtemp(prefix="dvemb_test_"), residency=gradient_cache_residency)
              as test_store):
            lrs = self.collect_trajectory(target, test_store, train_dataset, test_dataset, hook_config=hook_config)
            return self.attribute_from_cache(target, test_store, recorded_lr=lrs, hook_config=hook_config,
                                             algorithm_meta={"gradient_cache_residency": gradient_cache_residency},
                                             **opts)

    def attribute_from_cache(self, train_source, test_source, *, selected_training_steps=None, layer_name=None,
                             verbose: bool = False, loop_over_test: bool = False, algorithm_meta=None,
                             propagation: str = "train", dvemb_dir: str | None = None, hessian_mode: str = "full",
                             final_step: int | None = None, loss_reduction: str = "mean", learning_rate=1.0,
                             recorded_lr=None, hook_config=None, block_dtype: torch.dtype = torch.float32):
        """DVEmb over a stored (or snapshotted) trajectory."""
        self._validate(loss_reduction, propagation, hessian_mode, loop_over_test=loop_over_test, dvemb_dir=dvemb_dir)
        train = self.open_train_source(train_source, layer_name=layer_name, hook_config=hook_config, verbose=verbose)
        try:
            test_store = self.resolve_store(test_source)
            if recorded_lr is None:
                recorded_lr = self.recorded_lr_of(train)
            prop, out, final_step, lr = self._resolve_sweep(train, recorded_lr, selected_training_steps,
                                                            final_step, learning_rate)
            train = train.for_steps(prop)
            test = self.load_test_rep(test_store, layer_name=layer_name, verbose=verbose)
            sweep = {"learning_rate": lr, "loss_reduction": loss_reduction, "hessian_mode": hessian_mode,
                     "verbose": verbose}
            if propagation == "train":
                emb = self.embed_trajectory(train, prop, out, **sweep)
                if dvemb_dir is not None:
                    emb = self._tee_to_store(emb, GradientStorageManager(dvemb_dir), self._sample_id_key(train))
                scores, rids, rsteps, tids, _ = self.score_sources(emb, test, transform_test=dense_block)
            elif not loop_over_test:
                w, tids = self.collect_test_matrix(test)
                scores, rids, rsteps = self._propagate_test_and_score(w, len(tids), train, prop, out,
                                                                      block_dtype=block_dtype, **sweep)
            else:
                tids, index = self.test_column_order(test)
                scores, rids, rsteps = None, [], []
                for _s, tg, th in test:
                    wb = dense_block(tg.to(self.args.device)).data
                    cols = [index[h] for h in th]
                    bs, r_ids, r_steps = self._propagate_test_and_score(wb, len(cols), train, prop, out,
                                                                        block_dtype=block_dtype, **sweep)
                    if scores is None:
                        scores = torch.zeros(bs.shape[0], len(tids))
                        rids, rsteps = r_ids, r_steps
                    scores[:, cols] = bs
                if scores is None:
                    scores = torch.zeros(0, len(tids))
            meta = {"final_step": final_step, "selected_training_steps": sorted(out), "propagated_steps": sorted(prop),
                    "learning_rate": lr, "loss_reduction": loss_reduction, "propagation": propagation,
                    "loop_over_test": loop_over_test, "block_dtype": str(block_dtype), "dvemb_dir": dvemb_dir,
                    "hessian_mode": hessian_mode, **self.source_meta(train, test_store), **(algorithm_meta or {})}
            layer_name = train.layer_name
        finally:
            self.close_source(train)
        return self.build_score(scores, rids, rsteps, tids, algorithm_meta=meta, layer_name=layer_name)

    @staticmethod
    def _tee_to_store(blocks, store, sample_id_key):
        for step, block, hashes in blocks:
            store.save_bulk([GradientRecord(step, list(hashes), block.to("cpu"), sample_id_key)])
            yield step, block, hashes
