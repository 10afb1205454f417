"""AdamW-influence: trajectory influence through the AdamW update's full state.

AdamW carries ``(theta, m, v)``; a train sample ``z`` at step ``t`` perturbs that
state by ``Z_push(z)`` and every later step maps state perturbations through the
linearised update ``M_t`` (diagonal per coordinate: weight decay, the moment EMAs,
``D = 1/(sqrt(v_hat)+eps)`` and ``S = m_hat/(2 sqrt(v_hat)(sqrt(v_hat)+eps)^2)``)
plus the batch's Fisher coupling ``R_t``.  The influence on a query ``g_q`` is
``-g_q^T [W_theta W_m W_v] Z_push(z)`` where ``W`` is the accumulated backwards
product.  Per-step moments come from :class:`OptimizerStateCallback` (pre- and
post-update records); the step's mean gradient is recovered as
``(m_post - beta1 m_pre) / (1 - beta1)``.

``propagation="train"`` carries the ``(p, 3p)`` train-side operator (start ``W =
[I 0 0]``); ``"test"`` carries the ``(n_q, p)`` query rows per layer, chunked so a
step's push never exceeds a few GiB.  Parity: reference
``dattri_llm/attribution/algorithm/adamw_influence.py:76-560``.
"""

from __future__ import annotations

import pathlib
from collections.abc import Iterable, Mapping
from typing import ClassVar

import torch

from dattri_llm_b200.attribution.algorithm.trajectory import TrajectoryAttributor, dense_block
from dattri_llm_b200.ops.gemm import matmul_f32
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.callbacks.optimizer_state_callback import OptimizerStateCallback, assemble_dynamics
from dattri_llm_b200.gradient.snapshots import LazyDynamics
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.gradient.streaming import ReplayGradientSource

DYNAMICS_FILE = "adamw_dynamics.pt"
_CHUNK_BYTES = 3 << 30


def _flat(block, layers: list[str]) -> torch.Tensor:
    """``(B, p)`` fp32: the layers' dense per-sample gradients side by side."""
    cols = []
    for n in layers:
        v = block.data[n]
        e = v if isinstance(v, torch.Tensor) else ops.materialize(v, block.layer_types[n])
        cols.append(e.reshape(e.shape[0], -1).float())
    return torch.cat(cols, dim=1)


class _StepTerms:
    """One step's (or one layer's) linearisation: ``g_t``, ``D``, ``S`` and the scalars."""

    def __init__(self, dyn: dict, layers: list[str], device) -> None:
        b1, b2 = dyn["betas"]
        self.beta1, self.beta2 = float(b1), float(b2)
        self.count, self.lr, self.eps = int(dyn["step"]), float(dyn["lr"]), float(dyn["eps"])
        self.weight_decay = float(dyn["weight_decay"])

        def cat(side: str, which: int) -> torch.Tensor:
            return torch.cat([dyn[side][n][which].reshape(-1).float() for n in layers]).to(device)

        m_pre, m_post, v_post = cat("pre", 0), cat("post", 0), cat("post", 1)
        self.g_t = (m_post - self.beta1 * m_pre) / (1.0 - self.beta1)
        self.d, self.s = ops.adam_preconditioner(m_post / (1.0 - self.beta1**self.count),
                                                 v_post / (1.0 - self.beta2**self.count), eps=self.eps)

    @property
    def common(self) -> dict:
        return {"lr": self.lr, "step": self.count, "beta1": self.beta1, "beta2": self.beta2}

    def push(self, g):
        return ops.adamw_influence_push(g, self.g_t, self.d, self.s, **self.common)

    def coupling(self, w_theta, w_m, w_v, g):
        return ops.adamw_influence_coupling(w_theta, w_m, w_v, g, self.g_t, self.d, self.s, **self.common)

    def transition(self, w_theta, w_m, w_v):
        return ops.adamw_influence_transition(w_theta, w_m, w_v, self.d, self.s, weight_decay=self.weight_decay,
                                              **self.common)


class AdamWInfluenceAttributor(TrajectoryAttributor):
    """AdamW-influence attributor (needs one optimizer step per captured step)."""

    algorithm: ClassVar[str] = "AdamWInfluence"

    def __init__(self, args, *, task=None, projection_kwargs: dict[str, dict] | None = None) -> None:
        super().__init__(args, task=task)
        self._projection = projection_kwargs
        self._recorder: OptimizerStateCallback | None = None

    # -- trajectory hooks ---------------------------------------------------------
    def trajectory_callbacks(self, model, streamer, snapshots) -> list:
        """An :class:`OptimizerStateCallback` on the trajectory's optimizer.

        Raises:
            NotImplementedError: with gradient accumulation (one update per captured step is needed).
        """
        if self.args.gradient_accumulation_steps > 1:
            raise NotImplementedError(f"{type(self).__name__} needs one optimizer update per captured step; "
                                      f"gradient_accumulation_steps={self.args.gradient_accumulation_steps} is "
                                      "not supported.")
        if self._projection is None and self.trajectory_hook_config is not None:
            self._projection = self.trajectory_hook_config.projection_kwargs
        self._recorder = OptimizerStateCallback(model, lambda: streamer.optimizer,
                                                projection_kwargs=self._projection, snapshots=snapshots)
        return [self._recorder]

    def on_trajectory_block(self):
        """Record the post-update moments once the step's block is out."""
        rec = self._recorder
        if rec is None:
            raise RuntimeError("trajectory_callbacks() must run first.")
        return lambda step, _g, _h: rec.record_post(step)

    def finish_trajectory(self, train_target) -> None:
        """Store the dynamics beside a gradient store (snapshots keep their own)."""
        if isinstance(train_target, GradientStorageManager) and self._recorder is not None:
            torch.save(dict(self._recorder.dynamics()), pathlib.Path(train_target.save_dir) / DYNAMICS_FILE)

    @staticmethod
    def load_dynamics(train, dynamics) -> Mapping[int, dict]:
        """The per-step dynamics: given, from the snapshots, or from the store's file."""
        if isinstance(dynamics, Mapping):
            return dynamics
        if dynamics is None:
            if isinstance(train, ReplayGradientSource):
                return LazyDynamics(train.snapshots, assemble_dynamics)
            dynamics = pathlib.Path(train.file_manager.save_dir) / DYNAMICS_FILE
        return torch.load(dynamics, weights_only=False)

    # -- sweeps -------------------------------------------------------------------
    def _step_rows(self, train, step: int, layers: list[str], dtype=torch.float32):
        """``({layer: (B, w)}, hashes)`` of one step (blocks concatenated)."""
        parts: dict[str, list] = {n: [] for n in layers}
        ids: list[str] = []
        for _s, block, hashes in train.for_steps([step]):
            dense = dense_block(block.to(self.args.device), dtype).data
            for n in layers:
                parts[n].append(dense[n])
            ids.extend(hashes)
        if not ids:
            raise ValueError(f"No train gradients recorded at step {step}.")
        return {n: v[0] if len(v) == 1 else torch.cat(v) for n, v in parts.items()}, ids

    def sweep(self, train, dynamics, test_rep: torch.Tensor, *, layers, prop_steps, output_steps,
              loss_reduction: str = "mean", verbose: bool = False):
        """Train-side sweep: ``(scores, row ids, row steps)``."""
        dev = self.args.device
        p = test_rep.shape[1]
        test_rep = test_rep.to(dev)
        w_theta = torch.eye(p, device=dev)
        w_m = torch.zeros(p, p, device=dev)
        w_v = torch.zeros(p, p, device=dev)
        rows, rids, rsteps = [], [], []
        for step in self.steps_bar(prop_steps, "AdamW-influence: sweep (W)", verbose):
            blocks, ids = self._step_rows(train, step, layers)
            g = torch.cat([blocks[n] for n in layers], dim=1)
            t = _StepTerms(dynamics[step], layers, dev)
            if step in output_steps:
                z = t.push(g)
                infl = matmul_f32(z, torch.cat([w_theta, w_m, w_v], dim=1), b_transposed=True)
                rows.append((-matmul_f32(infl, test_rep, b_transposed=True)).cpu())
                rids.extend(ids)
                rsteps.extend([step] * len(ids))
            coup = t.coupling(w_theta, w_m, w_v, g)
            w_theta, w_m, w_v = t.transition(w_theta, w_m, w_v)
            scale = float(g.shape[0]) if loss_reduction == "mean" else 1.0
            w_theta += scale * matmul_f32(coup.t(), g)
        return (torch.cat(rows) if rows else torch.zeros(0, test_rep.shape[0])), rids, rsteps

    def sweep_queries(self, train, dynamics, queries: torch.Tensor, *, layers, prop_steps, output_steps,
                      loss_reduction: str = "mean", verbose: bool = False, block_dtype: torch.dtype = torch.float32):
        """Test-side sweep over the query rows, layer by layer: ``(scores, row ids, row steps)``.

        Raises:
            ValueError: when the query width disagrees with the train side.
        """
        dev = self.args.device
        n_q = queries.shape[0]
        widths = None
        for _s, block, _h in train.for_steps([max(prop_steps)]):
            dense = dense_block(block.to(dev)).data
            widths = {n: dense[n].shape[1] for n in layers}
            break
        if widths is None:
            raise ValueError(f"No train gradients recorded at step {max(prop_steps)}.")
        if sum(widths.values()) != queries.shape[1]:
            raise ValueError(f"query width {queries.shape[1]} does not match the train side's "
                             f"{sum(widths.values())} coordinates over {len(layers)} layers.")
        queries = queries.to(dev).float()
        u, off = {}, 0
        for n in layers:
            u[n] = [queries[:, off:off + widths[n]].clone(), None, None]
            u[n][1] = torch.zeros_like(u[n][0])
            u[n][2] = torch.zeros_like(u[n][0])
            off += widths[n]
        del queries
        rows, rids, rsteps = [], [], []
        for step in self.steps_bar(prop_steps, "AdamW-influence: sweep (U)", verbose):
            blocks, ids = self._step_rows(train, step, layers, block_dtype)
            b = len(ids)
            emit = step in output_steps
            scores = torch.zeros(b, n_q, device=dev)
            coup = torch.zeros(b, n_q, device=dev)
            terms = {n: _StepTerms(dynamics[step], [n], dev) for n in layers}
            for n in layers:
                w, t = widths[n], terms[n]
                chunk = max(1, _CHUNK_BYTES // (6 * w * 4))
                for c0 in range(0, b, chunk):
                    gc = blocks[n][c0:c0 + chunk].float()
                    if emit:
                        z = t.push(gc)
                        scores[c0:c0 + chunk] -= matmul_f32(z, torch.cat(list(u[n]), dim=1), b_transposed=True)
                        del z
                    coup[c0:c0 + chunk] += t.coupling(*u[n], gc)
            if emit:
                rows.append(scores.cpu())
                rids.extend(ids)
                rsteps.extend([step] * b)
            scale = float(b) if loss_reduction == "mean" else 1.0
            for n in layers:
                fisher = matmul_f32(coup.t(), blocks[n].float())
                u[n] = list(terms[n].transition(*u[n]))
                u[n][0] += scale * fisher
            del blocks, terms, coup, scores
        return (torch.cat(rows) if rows else torch.zeros(0, n_q)), rids, rsteps

    # -- entry points ---------------------------------------------------------------
    def attribute(self, train_dataset, test_dataset, *, hook_config=None, verbose: bool = False, **kwargs):
        """Run the trajectory into stores, then attribute from them."""
        ((train_dir, test_dir),) = self.cache(train_dataset, test_dataset, hook_config=hook_config)
        return self.attribute_from_cache(train_dir, test_dir, hook_config=hook_config, verbose=verbose, **kwargs)

    def attribute_from_cache(self, train_source, test_source, *, dynamics=None,
                             selected_training_steps: Iterable[int] | None = None, layer_name=None,
                             verbose: bool = False, loss_reduction: str = "mean", propagation: str = "train",
                             loop_over_test: bool = False, final_step: int | None = None, hook_config=None,
                             block_dtype: torch.dtype = torch.float32, **kwargs):
        """AdamW-influence over a stored (or snapshotted) trajectory.

        Raises:
            ValueError: for a bad ``loss_reduction`` / propagation, or steps without dynamics.
        """
        if loss_reduction not in ("mean", "sum"):
            raise ValueError(f"loss_reduction must be 'mean' or 'sum', got {loss_reduction!r}.")
        self.validate_propagation(propagation, loop_over_test)
        train = self.open_train_source(train_source, layer_name=layer_name, hook_config=hook_config, verbose=verbose)
        try:
            test_store = self.resolve_store(test_source)
            test = self.load_test_rep(test_store, layer_name=layer_name, verbose=verbose)
            dyn = self.load_dynamics(train, dynamics)
            prop, out, final_step = self.resolve_steps(self.available_steps(train), selected_training_steps,
                                                       final_step)
            missing = [s for s in prop if s not in dyn]
            if missing:
                raise ValueError(f"no optimizer dynamics recorded for steps {missing[:5]}...")
            layers = None
            for _s, block, _h in test:
                layers = sorted(block.data)
                break
            if layers is None:
                raise ValueError("the test source yielded no blocks.")
            kw = {"layers": layers, "prop_steps": prop, "output_steps": out, "loss_reduction": loss_reduction,
                  "verbose": verbose}
            if propagation == "test":
                kw["block_dtype"] = block_dtype
            if propagation == "train" or not loop_over_test:
                tids, parts = [], []
                for _s, block, hashes in test:
                    parts.append(_flat(block, layers))
                    tids.extend(hashes)
                run = self.sweep if propagation == "train" else self.sweep_queries
                scores, rids, rsteps = run(train, dyn, torch.cat(parts), **kw)
            else:
                tids, index = self.test_column_order(test)
                scores, rids, rsteps = None, [], []
                for _s, block, hashes in test:
                    bs, r_ids, r_steps = self.sweep_queries(train, dyn, _flat(block, layers), **kw)
                    if scores is None:
                        scores = torch.zeros(bs.shape[0], len(tids))
                        rids, rsteps = r_ids, r_steps
                    scores[:, [index[h] for h in hashes]] = bs
                if scores is None:
                    scores = torch.zeros(0, len(tids))
            meta = {"final_step": final_step, "selected_training_steps": sorted(out), "propagated_steps": sorted(prop),
                    "loss_reduction": loss_reduction, "propagation": propagation, "loop_over_test": loop_over_test,
                    "block_dtype": str(block_dtype), **self.source_meta(train, test_store), **kwargs}
        finally:
            self.close_source(train)
        return self.build_score(scores, rids, rsteps, tids, algorithm_meta=meta, layer_name=layers)
