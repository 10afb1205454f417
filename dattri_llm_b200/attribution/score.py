"""``AttributionScore``: trajectory-aware attribution scores keyed by sample identity.

Rows are ``(train sample, step)`` pairs (or ``(sample, step, token position)`` for
token granularity), columns are test samples.  Saved as ``scores.pt`` +
``metadata.json`` with the reference's field names
(``dattri_llm/attribution/score.py:50-470``), so a saved score loads in either
framework.  :meth:`topk` (per-test top-k over train samples) runs on whatever
device holds the scores.
"""

from __future__ import annotations

from dattri_llm_b200.options import ScoreTrajectory  # noqa: F401  (re-exported option types)
import json
from collections.abc import Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch


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

    _SCORES_FILE = "scores.pt"
    _META_FILE = "metadata.json"

    def __post_init__(self) -> None:
        n = self.scores.shape[0]
        if not len(self.row_train_ids) == len(self.row_steps) == n:
            raise ValueError(f"row_train_ids ({len(self.row_train_ids)}) and row_steps ({len(self.row_steps)}) "
                             f"must both equal num_rows ({n}).")
        if len(self.test_ids) != self.scores.shape[1]:
            raise ValueError(f"test_ids ({len(self.test_ids)}) must equal num_test ({self.scores.shape[1]}).")
        if self.row_token_ids is not None and len(self.row_token_ids) != n:
            raise ValueError(f"row_token_ids ({len(self.row_token_ids)}) must equal num_rows ({n}).")
        index: dict[str, list[tuple[int, int]]] = {}
        for r, (h, s) in enumerate(zip(self.row_train_ids, self.row_steps, strict=True)):
            index.setdefault(h, []).append((s, r))
        for entries in index.values():
            entries.sort()
        self.train_index = index
        self.test_index = {h: c for c, h in enumerate(self.test_ids)}

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

    def _require_train(self, h: str) -> list[tuple[int, int]]:
        if h not in self.train_index:
            raise KeyError(f"train hash {h[:16]}... not in scores.")
        return self.train_index[h]

    def _require_test(self, h: str) -> int:
        if h not in self.test_index:
            raise KeyError(f"test hash {h[:16]}... not in scores.")
        return self.test_index[h]

    def trajectory_aware(self, train_hash: str) -> tuple[list[int], torch.Tensor]:
        """``(steps, (n_steps, num_test))`` of one train sample (token rows summed per step)."""
        entries = self._require_train(train_hash)
        if self.row_token_ids is None:
            return [s for s, _ in entries], self.scores[[r for _, r in entries]]
        by_step: dict[int, list[int]] = {}
        for s, r in entries:
            by_step.setdefault(s, []).append(r)
        steps = sorted(by_step)
        return steps, torch.stack([self.scores[by_step[s]].sum(0) for s in steps])

    def token_scores(self, train_hash: str, step: int | None = None) -> tuple[list[int], torch.Tensor]:
        """``(positions, (n_pos, num_test))`` per token position of one train sample."""
        if self.row_token_ids is None:
            raise ValueError("token_scores() needs a token-level score; attribute with "
                             "attribution_granularity='token'.")
        entries = self._require_train(train_hash)
        rows = [r for s, r in entries if step is None or s == step]
        if not rows:
            raise KeyError(f"train sample {train_hash[:16]}... has no row at step {step}; known steps: "
                           f"{sorted({s for s, _ in entries})}")
        by_pos: dict[int, list[int]] = {}
        for r in rows:
            by_pos.setdefault(self.row_token_ids[r], []).append(r)
        pos = sorted(by_pos)
        return pos, torch.stack([self.scores[by_pos[p]].sum(0) for p in pos])

    def trajectory_agnostic(self, train_hash: str) -> torch.Tensor:
        """One train sample's scores summed over steps."""
        return self.trajectory_aware(train_hash)[1].sum(0)

    def agnostic_matrix(self) -> tuple[list[str], torch.Tensor]:
        """``(train_ids, (num_train, num_test))`` summed over steps (one scatter-add)."""
        ids = self.train_ids
        where = {h: i for i, h in enumerate(ids)}
        rows = torch.tensor([where[h] for h in self.row_train_ids], dtype=torch.long, device=self.scores.device)
        out = self.scores.new_zeros(len(ids), self.num_test)
        out.index_add_(0, rows, self.scores)
        return ids, out

    def column(self, test_hash: str) -> torch.Tensor:
        """Every row's score against one test sample."""
        return self.scores[:, self._require_test(test_hash)]

    def step_matrix(self, step: int) -> tuple[list[str], torch.Tensor]:
        """``(train_ids, rows)`` of one step (token rows summed per sample)."""
        rows = [i for i, s in enumerate(self.row_steps) if s == step]
        if not rows:
            raise KeyError(f"step {step} not present in scores.")
        if self.row_token_ids is None:
            return [self.row_train_ids[i] for i in rows], self.scores[rows]
        by_hash: dict[str, list[int]] = {}
        for i in rows:
            by_hash.setdefault(self.row_train_ids[i], []).append(i)
        ids = list(by_hash)
        return ids, torch.stack([self.scores[by_hash[h]].sum(0) for h in ids])

    def step_matrices(self) -> dict[int, tuple[list[str], torch.Tensor]]:
        """:meth:`step_matrix` for every step present."""
        return {s: self.step_matrix(s) for s in sorted(set(self.row_steps))}

    def score_at(self, train_hash: str, step: int, test_hash: str) -> torch.Tensor:
        """One train sample's score at one step against one test sample."""
        col = self._require_test(test_hash)
        rows = [r for s, r in self._require_train(train_hash) if s == step]
        if rows:
            return self.scores[rows, col].sum() if len(rows) > 1 else self.scores[rows[0], col]
        raise KeyError(f"train sample {train_hash[:16]}... has no row at step {step}; known steps: "
                       f"{sorted({s for s, _ in self.train_index[train_hash]})}")

    def query(self, train_hashes: Sequence[str] | None = None, test_hashes: Sequence[str] | None = None,
              trajectory: str = "agnostic") -> torch.Tensor:
        """Scores of the given train and test identities (``"agnostic"``: summed over steps;
        ``"aware"``: one row per ``(sample, step)``)."""
        if trajectory not in ("aware", "agnostic"):
            raise ValueError(f"trajectory must be 'aware' or 'agnostic', got {trajectory!r}.")
        train_hashes = list(train_hashes) if train_hashes is not None else self.train_ids
        cols = list(range(self.num_test)) if test_hashes is None else [self._require_test(h) for h in test_hashes]
        if trajectory == "agnostic":
            return torch.stack([self.trajectory_agnostic(h) for h in train_hashes])[:, cols]
        rows = [r for h in train_hashes for _, r in self._require_train(h)]
        return self.scores[rows][:, cols]

    def topk(self, k: int, *, largest: bool = True) -> tuple[torch.Tensor, list[list[str]]]:
        """Per test sample, the *k* highest-scoring train samples (trajectory-agnostic):
        ``(values (num_test, k), [[train_id] * k] * num_test)``."""
        ids, m = self.agnostic_matrix()
        k = min(k, len(ids))
        vals, idx = torch.topk(m.T, k, dim=1, largest=largest)
        idx = idx.cpu().tolist()
        return vals, [[ids[j] for j in row] for row in idx]

    def save(self, out_dir: str | Path) -> Path:
        """Write ``scores.pt`` and ``metadata.json`` under *out_dir*."""
        out = Path(out_dir)
        out.mkdir(parents=True, exist_ok=True)
        torch.save(self.scores.cpu(), out / self._SCORES_FILE)
        meta = {"row_train_ids": self.row_train_ids, "row_steps": self.row_steps, "test_ids": self.test_ids,
                "algorithm": self.algorithm, "algorithm_meta": self.algorithm_meta,
                "layer_name": self.layer_name, "row_token_ids": self.row_token_ids,
                "granularity": self.granularity, "num_train": self.num_train, "num_test": self.num_test,
                "num_rows": self.num_rows}
        (out / self._META_FILE).write_text(json.dumps(meta, indent=2, default=str), encoding="utf-8")
        return out

    @classmethod
    def load(cls, out_dir: str | Path) -> AttributionScore:
        """Read a saved score."""
        out = Path(out_dir)
        scores = torch.load(out / cls._SCORES_FILE, weights_only=True)
        meta = json.loads((out / cls._META_FILE).read_text(encoding="utf-8"))
        am = meta.get("algorithm_meta", {})
        if "normalized_grad" in meta:
            am.setdefault("normalized_grad", meta["normalized_grad"])
        return cls(scores=scores, row_train_ids=meta["row_train_ids"], row_steps=meta["row_steps"],
                   test_ids=meta["test_ids"], algorithm=meta["algorithm"], algorithm_meta=am,
                   layer_name=meta["layer_name"], row_token_ids=meta.get("row_token_ids"))
