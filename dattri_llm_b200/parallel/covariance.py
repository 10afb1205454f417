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

from dattri_llm_b200.utils.distributed import dist_world_size


def all_reduce_accumulators(accs: list) -> None:
    """Sum ``(A, G, count)`` of every :class:`LayerKroneckerAccumulator` in *accs* over ranks.

    Every rank must pass its accumulators in the same order with the same shapes.
    """
    if dist_world_size() == 1 or not accs:
        for a in accs:
            if a._A is None:
                raise RuntimeError("No gradient-carrying data has been accumulated")
            a._count = a._n
        return
    for a in accs:
        if a._A is None:
            raise RuntimeError("No gradient-carrying data has been accumulated")
    import torch.distributed as dist

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
