"""Column-sharded distributed scoring with the all-gather fused into the score GEMM.

The reference scores each rank's train rows against the whole (replicated) test set
(``attribution/base.py:896-915``).  Here each rank keeps only its shard of the packed
test matrix; every step, each rank's packed train block goes into a symmetric-memory
buffer, the ranks meet at a bounded :class:`PeerBarrier`, and ONE kernel per rank
(``csrc/score_ag.cu``) pulls every peer's block over NVLink tile by tile while it
multiplies it against the local test shard.  Each rank ends with the scores of ALL
ranks' train rows against ITS test columns, so the per-test top-k needs no cross-rank
merge until the end.  Per GPU this holds ``1/world`` of the test matrix and reads
``(world - 1)`` peer blocks over NVLink instead of re-reading the whole test matrix
from HBM every step.  The two buffers alternate between steps, so one barrier per step
covers both "block written" and "peers done reading the buffer I am about to reuse".
"""

from __future__ import annotations

import torch

from dattri_llm_b200.parallel.symm import PeerBarrier, SymmetricBuffer


class AllGatherScorer:
    """``score(block) -> (n_local, world * rows)``: every rank's ``(rows, K)`` train block
    against this rank's ``(n_local, K)`` test shard (bf16 operands, fp32 scores)."""

    def __init__(self, test_shard: torch.Tensor, rows: int, *, group=None, splits: int | None = None) -> None:
        if test_shard.dtype != torch.bfloat16 or test_shard.dim() != 2:
            raise ValueError("test_shard must be a 2-D bf16 tensor")
        if rows % 8:
            raise ValueError("rows per rank must be a multiple of 8")
        dev = test_shard.device
        self.test = test_shard.contiguous()
        self.rows = rows
        k = self.test.shape[1]
        self._bufs = [SymmetricBuffer((rows, k), torch.bfloat16, dev, group) for _ in range(2)]
        self.world = self._bufs[0].world
        self.rank = self._bufs[0].rank
        if self.world * rows > 128:
            raise ValueError(f"world * rows = {self.world * rows} exceeds the fused kernel's 128-row tile")
        self._barrier = PeerBarrier(dev, group)
        m_tiles = (self.test.shape[0] + 127) // 128
        self.splits = splits or max(1, (148 + m_tiles - 1) // m_tiles)
        self._step = 0

    def score(self, block: torch.Tensor) -> torch.Tensor:
        """Scores ``(n_local, world * rows)``; column ``r * rows + b`` is rank r's row b."""
        from dattri_llm_b200.ops import count_launch, error_word, native

        if block.shape != (self.rows, self.test.shape[1]):
            raise ValueError(f"block must be {(self.rows, self.test.shape[1])}, got {tuple(block.shape)}")
        buf = self._bufs[self._step % 2]
        self._step += 1
        buf.local.copy_(block)
        self._barrier.wait()
        out = torch.zeros(self.test.shape[0], self.world * self.rows, dtype=torch.float32, device=block.device)
        count_launch()
        native().ag_score(self.test, buf.peers, out, 1.0, int(self.splits), error_word(block.device))
        return out
