"""Cross-rank reduction of K-FAC covariance accumulators.

The reference all-reduces every layer's ``A``, ``G`` and row count separately
(``dattri_llm/gradient/ops/kronecker.py:516-527``): three collectives per layer,
one of them host-synchronous.  Here every accumulator of a model is packed into
one fp32 buffer reduced with ONE collective (the row counts follow in one small
float64 collective).
On a single-node NCCL group of sm_100 GPUs the reduction is the library's
NVLink all-reduce kernel (:mod:`dattri_llm_b200.parallel.symm`), reading every
peer's buffer directly; elsewhere it is one ``dist.all_reduce``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from dattri_llm_b200.utils.distributed import dist_world_size


def all_reduce_accumulators(accs: list) -> None:
    """Sum ``(A, G, count)`` of every :class:`LayerKroneckerAccumulator` in *accs* over ranks.

    Every rank must pass its accumulators in the same order with the same shapes.
    """
    fused = [a for a in accs if getattr(a, "_symm", None) is not None]
    if fused:
        for a in fused:  # accumulated in symmetric memory: reduced straight out of it
            a.all_reduce()
        accs = [a for a in accs if getattr(a, "_symm", None) is None]
        if not accs:
            return
    if dist_world_size() == 1 or not accs:
        for a in accs:
            if a._A is None:
                raise RuntimeError("No gradient-carrying data has been accumulated")
            a._count = a._n
        return
    for a in accs:
        if a._A is None:
            raise RuntimeError("No gradient-carrying data has been accumulated")
    device = accs[0]._A.device
    if "nccl" in str(dist.get_backend()).lower():
        device = torch.device("cuda", torch.cuda.current_device())
    flat = torch.cat([torch.cat([a._A.reshape(-1), a._G.reshape(-1)]) for a in accs]).to(device)
    counts = torch.tensor([float(a._n) for a in accs], dtype=torch.float64, device=device)
    from dattri_llm_b200.parallel import symm

    if not symm.all_reduce_sum_(flat):
        dist.all_reduce(flat)
    dist.all_reduce(counts)
    off = 0
    for a, n in zip(accs, counts.tolist(), strict=True):
        na, ng = a._A.numel(), a._G.numel()
        a._A.copy_(flat[off : off + na].view_as(a._A))
        off += na
        a._G.copy_(flat[off : off + ng].view_as(a._G))
        off += ng
        a._count = int(round(n))


class SymmetricGram:
    """A ``(w, w)`` fp32 Gram sum ``sum x^T x`` kept in symmetric memory and reduced across
    ranks over NVLink.  Every :meth:`add` is a local tcgen05 GEMM accumulating in its
    epilogue (nothing crosses NVLink per batch: the covariance is needed only once, at the
    end); :meth:`reduced` is a two-shot peer all-reduce straight out of the symmetric
    buffers (reduce-scatter in place, then every rank gathers the owners' slices), with no
    packing copy.  The reference all-reduces each factor with NCCL after the fit
    (``dattri_llm/gradient/ops/kronecker.py:516-527``).  Create collectively (same ``w``,
    same order on every rank)."""

    _barriers: dict = {}

    def __init__(self, w: int, device: torch.device) -> None:
        from dattri_llm_b200.parallel.symm import PeerBarrier, SymmetricBuffer

        self.w = w
        self.n4 = (w * w + 3) // 4
        self.buf = SymmetricBuffer((self.n4 * 4,), torch.float32, device)
        self.buf.local.zero_()
        self.world, self.rank = self.buf.world, self.buf.rank
        if device not in SymmetricGram._barriers:
            SymmetricGram._barriers[device] = PeerBarrier(device)
        self.barrier = SymmetricGram._barriers[device]

    def add(self, x: torch.Tensor) -> None:
        """Add ``x^T x`` of ``x (N, w)`` (bf16, CUDA) into this rank's partial sum."""
        from dattri_llm_b200.gradient.ops.kronecker import gram_accumulate

        gram_accumulate(x, self.buf.local[: self.w * self.w].view(self.w, self.w))

    def reduced(self) -> torch.Tensor:
        """The summed ``(w, w)`` matrix on this rank (collective: every rank calls it)."""
        from dattri_llm_b200.ops import count_launch, native

        n = self.n4 * 4
        self.barrier.wait()  # every rank's partial sum is complete
        count_launch()
        native().allreduce_phase(self.buf.peers, self.buf.local, n, 1, self.rank)  # own slice, in place
        self.barrier.wait()
        out = torch.empty(n, dtype=torch.float32, device=self.buf.local.device)
        count_launch()
        native().allreduce_phase(self.buf.peers, out, n, 2, self.rank)
        self.barrier.wait()  # nobody reads this buffer any more
        return out[: self.w * self.w].view(self.w, self.w)
