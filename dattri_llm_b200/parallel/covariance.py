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
        for a in fused:  # reduced inside their accumulation GEMMs; gather the owners' slices
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
    """A ``(w, w)`` fp32 Gram sum ``sum x^T x`` reduced ACROSS RANKS inside the accumulation
    GEMM: the tcgen05 GEMM's epilogue adds every element with fp32 atomics into its owner
    rank's symmetric buffer over NVLink (``kPeerAtomicF32``), so no separate all-reduce
    follows the fit; :meth:`reduced` only gathers the owners' slices.  Create collectively
    (same ``w``, same order on every rank)."""

    _barriers: dict = {}

    def __init__(self, w: int, device: torch.device) -> None:
        from dattri_llm_b200.parallel.symm import PeerBarrier, SymmetricBuffer

        self.w = w
        self.n4 = (w * w + 3) // 4
        self.buf = SymmetricBuffer((self.n4 * 4,), torch.float32, device)
        self.buf.local.zero_()
        self.world, self.rank = self.buf.world, self.buf.rank
        self.per4 = (self.n4 + self.world - 1) // self.world
        self.ptrs = torch.tensor([int(p.data_ptr()) for p in self.buf.peers], dtype=torch.int64, device=device)
        if device not in SymmetricGram._barriers:
            SymmetricGram._barriers[device] = PeerBarrier(device)
        else:  # the zeroed buffers must be in place on every rank before any rank adds
            torch.cuda.synchronize(device)
            dist.barrier()
        self.barrier = SymmetricGram._barriers[device]

    def add(self, x: torch.Tensor) -> None:
        """Add ``x^T x`` of ``x (N, w)`` (bf16, CUDA) into the cross-rank sum."""
        from dattri_llm_b200 import ops as native_ops

        xt = x.t().contiguous()
        w, n = xt.shape
        splits = native_ops.gemm.auto_splits(w, w, n, 1, 128 if w > 64 else 64)
        native_ops.count_launch()
        native_ops.native().gemm_tn_peer(xt, xt, self.ptrs, self.world, self.per4, w, w, w, 1.0, splits,
                                         native_ops.error_word(x.device), self.rank)

    def reduced(self) -> torch.Tensor:
        """The summed ``(w, w)`` matrix on this rank (collective: every rank calls it)."""
        from dattri_llm_b200.ops import count_launch, native

        self.barrier.wait()  # every rank's atomics have landed
        out = torch.empty(self.n4 * 4, dtype=torch.float32, device=self.buf.local.device)
        count_launch()
        native().allreduce_phase(self.buf.peers, out, self.n4 * 4, 2, self.rank)
        self.barrier.wait()
        return out[: self.w * self.w].view(self.w, self.w)
