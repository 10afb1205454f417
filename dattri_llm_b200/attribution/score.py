"""``AttributionScore``: trajectory-aware attribution scores keyed by sample identity.

Rows are ``(train sample, step)`` pairs (or ``(sample, step, token position)`` for
token granularity), columns are test samples.  Saved as ``scores.pt`` +
``metadata.json`` with the reference's field names
(``dattri_llm/attribution/score.py:50-470``), so a saved score loads in either
framework.  Every reduction over rows (per step, per sample, per token position) is one
``index_add_`` on whatever device holds the scores, and :meth:`topk` runs there too.
"""

from __future__ import annotations

from dattri_llm_b200.options import ScoreTrajectory  # noqa: F401  (re-exported option types)
import json
from collections.abc import Hashable, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

SCORES_FILE = "scores.pt"
METADATA_FILE = "metadata.json"


def _grouped_sum(scores: torch.Tensor, rows: Sequence[int], keys: Sequence[Hashable]) -> tuple[list, torch.Tensor]:
    """``(distinct keys in first-seen order, (n_keys, num_test))``: the *rows* of *scores*
    summed per key (``keys[i]`` labels ``rows[i]``)."""
    order: dict = {}
    slot = [order.setdefault(k, len(order)) for k in keys]
    out = scores.new_zeros(len(order), scores.shape[1])
    device = scores.device
    out.index_add_(0, torch.tensor(slot, dtype=torch.long, device=device),
                   scores.index_select(0, torch.tensor(list(rows), dtype=torch.long, device=device)))
    return list(order), out


@dataclass
class AttributionScore:
    """Scores ``(num_rows, num_test)`` with row and column identities."""

    scores: torch.Tensor
    row_train_ids: list[str]
    row_steps: list[int]
    test_ids: list[str]
    algorithm: str
    algorithm_meta: dict[str, Any]
    layer_name: list[str] | None
    row_token_ids: list[int] | None = None
    train_index: dict[str, list[tuple[int, int]]] = field(init=False, repr=False)
    test_index: dict[str, int] = field(init=False, repr=False)

    def __post_init__(self) -> None:
        rows, cols = self.scores.shape[0], self.scores.shape[1]
        lengths = {"row_train_ids": len(self.row_train_ids), "row_steps": len(self.row_steps)}
        if self.row_token_ids is not None:
            lengths["row_token_ids"] = len(self.row_token_ids)
        wrong = {k: n for k, n in lengths.items() if n != rows}
        if wrong:
            raise ValueError(f"the scores have {rows} rows but {wrong} (one entry per row is needed).")
        if len(self.test_ids) != cols:
            raise ValueError(f"the scores have {cols} columns but {len(self.test_ids)} test ids.")
        rows_of: dict[str, list[tuple[int, int]]] = {}
        for row, (sample, step) in enumerate(zip(self.row_train_ids, self.row_steps, strict=True)):
            rows_of.setdefault(sample, []).append((step, row))
        for entries in rows_of.values():
            entries.sort()
        self.train_index = rows_of  # sample -> [(step, row)] in step order
        self.test_index = {h: c for c, h in enumerate(self.test_ids)}

    # ------------------------------------------------------------------ shape
    @property
    def granularity(self) -> str:
        """``"instance"`` or ``"token"``."""
        return "instance" if self.row_token_ids is None else "token"

    @property
    def train_ids(self) -> list[str]:
        """Distinct train identities in first-row order."""
        return list(dict.fromkeys(self.row_train_ids))

    @property
    def num_rows(self) -> int:
        """Score rows."""
        return self.scores.shape[0]

    @property
    def num_train(self) -> int:
        """Distinct train samples."""
        return len(self.train_index)

    @property
    def num_test(self) -> int:
        """Test samples."""
        return self.scores.shape[1]

    def _rows_of(self, sample: str) -> list[tuple[int, int]]:
        try:
            return self.train_index[sample]
        except KeyError:
            raise KeyError(f"no score row belongs to train sample {sample[:16]}...") from None

    def _column_of(self, test: str) -> int:
        try:
            return self.test_index[test]
        except KeyError:
            raise KeyError(f"no score column belongs to test sample {test[:16]}...") from None

    def _missing_step(self, sample: str, step: int) -> KeyError:
        steps = sorted({s for s, _ in self._rows_of(sample)})
        return KeyError(f"train sample {sample[:16]}... has no score at step {step} (its steps: {steps}).")

    # ------------------------------------------------------------------ views
    def trajectory_aware(self, train_hash: str) -> tuple[list[int], torch.Tensor]:
        """``(steps, (n_steps, num_test))`` of one train sample (token rows summed per step)."""
        entries = self._rows_of(train_hash)
        if self.row_token_ids is None:
            return [s for s, _ in entries], self.scores[[r for _, r in entries]]
        steps, sums = _grouped_sum(self.scores, [r for _, r in entries], [s for s, _ in entries])
        return steps, sums

    def token_scores(self, train_hash: str, step: int | None = None) -> tuple[list[int], torch.Tensor]:
        """``(positions, (n_pos, num_test))`` per token position of one train sample."""
        if self.row_token_ids is None:
            raise ValueError("these are per-sample scores; token_scores() needs "
                             "attribution_granularity='token'.")
        rows = [r for s, r in self._rows_of(train_hash) if step is None or s == step]
        if not rows:
            raise self._missing_step(train_hash, step)
        positions = sorted({self.row_token_ids[r] for r in rows})
        rank = {p: i for i, p in enumerate(positions)}
        _keys, sums = _grouped_sum(self.scores, rows, [rank[self.row_token_ids[r]] for r in rows])
        order = sorted(range(len(_keys)), key=lambda i: _keys[i])
        return positions, sums[order]

    def trajectory_agnostic(self, train_hash: str) -> torch.Tensor:
        """One train sample's scores summed over steps."""
        return self.scores[[r for _, r in self._rows_of(train_hash)]].sum(0)

    def agnostic_matrix(self) -> tuple[list[str], torch.Tensor]:
        """``(train_ids, (num_train, num_test))`` summed over steps (one scatter-add)."""
        return _grouped_sum(self.scores, range(self.num_rows), self.row_train_ids)

    def column(self, test_hash: str) -> torch.Tensor:
        """Every row's score against one test sample."""
        return self.scores[:, self._column_of(test_hash)]

    def step_matrix(self, step: int) -> tuple[list[str], torch.Tensor]:
        """``(train_ids, rows)`` of one step (token rows summed per sample)."""
        rows = [i for i, s in enumerate(self.row_steps) if s == step]
        if not rows:
            raise KeyError(f"no score row was taken at step {step}.")
        if self.row_token_ids is None:
            return [self.row_train_ids[i] for i in rows], self.scores[rows]
        return _grouped_sum(self.scores, rows, [self.row_train_ids[i] for i in rows])

    def step_matrices(self) -> dict[int, tuple[list[str], torch.Tensor]]:
        """:meth:`step_matrix` for every step present."""
        return {s: self.step_matrix(s) for s in sorted(set(self.row_steps))}

    def score_at(self, train_hash: str, step: int, test_hash: str) -> torch.Tensor:
        """One train sample's score at one step against one test sample."""
        col = self._column_of(test_hash)
        rows = [r for s, r in self._rows_of(train_hash) if s == step]
        if not rows:
            raise self._missing_step(train_hash, step)
        return self.scores[rows[0], col] if len(rows) == 1 else self.scores[rows, col].sum()

    def query(self, train_hashes: Sequence[str] | None = None, test_hashes: Sequence[str] | None = None,
              trajectory: str = "agnostic") -> torch.Tensor:
        """Scores of the given train and test identities (``"agnostic"``: summed over steps;
        ``"aware"``: one row per ``(sample, step)``)."""
        if trajectory not in ("aware", "agnostic"):
            raise ValueError(f"trajectory is 'aware' or 'agnostic', not {trajectory!r}.")
        samples = self.train_ids if train_hashes is None else list(train_hashes)
        cols = list(range(self.num_test)) if test_hashes is None else [self._column_of(h) for h in test_hashes]
        if trajectory == "aware":
            rows = [r for h in samples for _, r in self._rows_of(h)]
            return self.scores[rows][:, cols]
        rows, keys = [], []
        for i, h in enumerate(samples):
            for _, r in self._rows_of(h):
                rows.append(r)
                keys.append(i)
        _keys, sums = _grouped_sum(self.scores, rows, keys)
        return sums[:, cols]

    def topk(self, k: int, *, largest: bool = True) -> tuple[torch.Tensor, list[list[str]]]:
        """Per test sample, the *k* highest-scoring train samples (trajectory-agnostic):
        ``(values (num_test, k), [[train_id] * k] * num_test)``."""
        ids, per_sample = self.agnostic_matrix()
        vals, idx = torch.topk(per_sample.T, min(k, len(ids)), dim=1, largest=largest)
        return vals, [[ids[j] for j in row] for row in idx.cpu().tolist()]

    # ------------------------------------------------------------------ files
    def save(self, out_dir: str | Path) -> Path:
        """Write ``scores.pt`` and ``metadata.json`` under *out_dir*."""
        out = Path(out_dir)
        out.mkdir(parents=True, exist_ok=True)
        torch.save(self.scores.cpu(), out / SCORES_FILE)
        meta = {"row_train_ids": self.row_train_ids, "row_steps": self.row_steps, "test_ids": self.test_ids,
                "algorithm": self.algorithm, "algorithm_meta": self.algorithm_meta,
                "layer_name": self.layer_name, "row_token_ids": self.row_token_ids,
                "granularity": self.granularity, "num_train": self.num_train, "num_test": self.num_test,
                "num_rows": self.num_rows}
        (out / METADATA_FILE).write_text(json.dumps(meta, indent=2, default=str), encoding="utf-8")
        return out

    @classmethod
    def load(cls, out_dir: str | Path) -> AttributionScore:
        """Read a saved score."""
        root = Path(out_dir)
        meta = json.loads((root / METADATA_FILE).read_text(encoding="utf-8"))
        algorithm_meta = dict(meta.get("algorithm_meta", {}))
        if "normalized_grad" in meta:  # older files keep the flag at the top level
            algorithm_meta.setdefault("normalized_grad", meta["normalized_grad"])
        return cls(scores=torch.load(root / SCORES_FILE, weights_only=True), row_train_ids=meta["row_train_ids"],
                   row_steps=meta["row_steps"], test_ids=meta["test_ids"], algorithm=meta["algorithm"],
                   algorithm_meta=algorithm_meta, layer_name=meta["layer_name"],
                   row_token_ids=meta.get("row_token_ids"))
