"""Timings of the fused compute + collective kernels against their rooflines.

    python -m dattri_llm_b200.parallel.bench_fused --emulate 8          # one GPU, 8 emulated peers
    torchrun --nproc-per-node N -m dattri_llm_b200.parallel.bench_fused  # N GPUs over NVLink

With ``--emulate W`` every "peer" buffer is a separate allocation on the local GPU, so the
kernels run their multi-peer code paths with HBM in place of NVLink (the compute side of
the roofline; this is also the form a single-GPU profiler capture can see).  Under
torchrun the peers are the other ranks' symmetric-memory buffers.  Each kernel is timed
with CUDA events after warm-up (max over ranks); the roofline is the slower of the math at
the measured bf16 peak and the bytes that must cross NVLink (each remote byte once) at the
measured per-direction peer bandwidth (770 GB/s) or the HBM bytes at the measured copy
bandwidth (only the latter when emulated).
Prints one JSON object per kernel.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

BF16_PEAK = 1.63e15     # measured cuBLAS bf16 burst on this B200 pool (FLOP/s)
HBM = 6.55e12           # measured copy bandwidth (B/s)
NVLINK = 770e9          # measured peer copy, per direction per GPU (B/s)


def _time(fn, iters: int = 20) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e-3


def _max_over_ranks(x: float) -> float:
    import torch.distributed as dist

    if not dist.is_initialized():
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def _peers(shape, dtype, world, emulate, gen, device):
    """``(local tensor, [peer views])``: symmetric buffers, or W local allocations."""
    if emulate:
        bufs = [torch.randn(shape, device=device, generator=gen).to(dtype) for _ in range(world)]
        return bufs[0], bufs
    from dattri_llm_b200.parallel.symm import SymmetricBuffer

    b = SymmetricBuffer(shape, dtype, device)
    b.local.copy_(torch.randn(shape, device=device, generator=gen).to(dtype))
    torch.cuda.synchronize()
    import torch.distributed as dist

    dist.barrier()
    return b.local, b.peers


def run(world: int, emulate: bool, rank: int) -> list[dict]:
    from dattri_llm_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(rank)
    nat = ops.native()
    err = ops.error_word(dev)
    rows = []

    def report(name, secs, flops, nvlink_bytes, hbm_bytes, extra=None):
        secs = _max_over_ranks(secs)
        link = hbm_bytes / HBM if emulate else max(nvlink_bytes / NVLINK, hbm_bytes / HBM)
        roof = max(flops / BF16_PEAK, link)
        rows.append({"kernel": name, "world": world, "emulated": emulate, "us": secs * 1e6,
                     "roofline_us": roof * 1e6, "fraction_of_roofline": roof / secs,
                     "tflops": flops / secs / 1e12, **(extra or {})})

    # 1) distributed score: all ranks' packed train blocks gathered into the score GEMM
    k, b, n_local = 458752, 8, 1024 // world
    test = torch.randn(n_local, k, device=dev, generator=gen).bfloat16()
    _, blocks = _peers((b, k), torch.bfloat16, world, emulate, gen, dev)
    out = torch.zeros(n_local, world * b, device=dev)
    splits = max(1, 148 // ((n_local + 127) // 128))
    secs = _time(lambda: (out.zero_(), nat.ag_score(test, blocks, out, 1.0, splits, err)))
    report("ag_score (all-gather + score GEMM)", secs, 2.0 * n_local * world * b * k,
           (world - 1) * b * k * 2, n_local * k * 2 + world * b * k * 2)

    # 2) sharded-weight forward: weight tiles all-gathered inside the GEMM (Llama-1B q/o shape)
    m, kk, n = 8192, 2048, 2048
    x = torch.randn(m, kk, device=dev, generator=gen).bfloat16()
    _, shards = _peers((n // world, kk), torch.bfloat16, world, emulate, gen, dev)
    y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    secs = _time(lambda: nat.gemm_tn_peers(x, shards, y, 0, ops.STORE_BF16, 1.0, err))
    report("gemm_tn_peers mode 0 (FSDP all-gather -> forward GEMM)", secs, 2.0 * m * n * kk,
           (world - 1) / world * n * kk * 2, (m * kk + m * n) * 2)
    w_full = torch.cat(list(shards)) if emulate else None
    if w_full is not None:
        secs_ref = _time(lambda: torch.matmul(x, w_full.T))
        rows[-1]["cublas_same_shape_us"] = secs_ref * 1e6

    stage = torch.empty(n, kk, device=dev, dtype=torch.bfloat16)
    flags = torch.zeros(world, dtype=torch.int32, device=dev)
    epoch = [0]

    def staged(a_, peers_, out_, mode):
        epoch[0] += 1
        nat.gemm_tn_staged(a_, peers_, stage, out_, flags, epoch[0], mode, rank, ops.STORE_BF16, 1.0, err)

    secs = _time(lambda: staged(x, shards, y, 0))
    report("gemm_tn_staged mode 0 (FSDP all-gather -> forward GEMM, one launch)", secs, 2.0 * m * n * kk,
           (world - 1) / world * n * kk * 2, (m * kk + m * n + n * kk) * 2)

    # 3) input gradient against the peers' transposed shards
    _, shards_t = _peers((kk, n // world), torch.bfloat16, world, emulate, gen, dev)
    dy = torch.randn(m, n, device=dev, generator=gen).bfloat16()
    dx = torch.empty(m, kk, device=dev, dtype=torch.bfloat16)
    secs = _time(lambda: nat.gemm_tn_peers(dy, shards_t, dx, 1, ops.STORE_BF16, 1.0, err))
    report("gemm_tn_peers mode 1 (all-gather -> input-gradient GEMM)", secs, 2.0 * m * n * kk,
           (world - 1) / world * n * kk * 2, (m * n + m * kk) * 2)
    stage = torch.empty(kk, n, device=dev, dtype=torch.bfloat16)
    flags = torch.zeros(world, dtype=torch.int32, device=dev)
    epoch[0] = 0
    secs = _time(lambda: staged(dy, shards_t, dx, 1))
    report("gemm_tn_staged mode 1 (all-gather -> input-gradient GEMM, one launch)", secs, 2.0 * m * n * kk,
           (world - 1) / world * n * kk * 2, (m * n + m * kk + n * kk) * 2)

    # 4) weight-gradient GEMM reduce-scattered in its epilogue (FSDP wgrad, Llama-1B q/o shape):
    #    16-byte peer stores into the owners' slots, a bounded barrier, the owner's slot sum
    w = 2048
    dyt = torch.randn(w, m, device=dev, generator=gen).bfloat16()
    xt = torch.randn(w, m, device=dev, generator=gen).bfloat16()
    shard = w * w // world
    _, slots = _peers((world * shard,), torch.float32, world, emulate, gen, dev)
    ptrs = torch.tensor([int(p.data_ptr()) for p in slots], dtype=torch.int64, device=dev)
    gshard = torch.zeros(shard, device=dev)
    barrier = None
    if not emulate:
        from dattri_llm_b200.parallel.symm import PeerBarrier

        barrier = PeerBarrier(dev)

    def wgrad_rs():
        nat.gemm_tn_rs(dyt, xt, ptrs, world, shard // 4, w, w, w, 1.0, err, rank)
        if barrier is not None:
            barrier.wait()
        nat.slot_reduce(slots[rank], world, shard, gshard, shard, True)

    secs = _time(wgrad_rs)
    report("gemm_tn_rs (wgrad GEMM -> reduce-scatter in the epilogue + owner slot sum)", secs, 2.0 * w * w * m,
           (world - 1) / world * w * w * 4, 2 * w * m * 2 + 2 * w * w * 4 + shard * 4)
    secs_local = _time(lambda: nat.gemm_tn(dyt, xt, torch.empty(w, w, device=dev), 1.0, ops.STORE_F32, 1, False, err))
    rows[-1]["local_gemm_only_us"] = secs_local * 1e6

    # 4b) Kronecker covariance: the local Gram partial (2048^2 fp32, symmetric memory)
    #     all-reduced by the two-shot NVLink peer kernel (real ranks only)
    if not emulate:
        from dattri_llm_b200.parallel.symm import SymmetricBuffer

        cov = SymmetricBuffer((w * w,), torch.float32, dev)
        cov.local.normal_(generator=gen)
        out_cov = torch.empty(w * w, device=dev)

        def cov_allreduce():
            barrier.wait()
            nat.allreduce_phase(cov.peers, cov.local, w * w, 1, rank)
            barrier.wait()
            nat.allreduce_phase(cov.peers, out_cov, w * w, 2, rank)

        secs = _time(cov_allreduce)
        report("covariance all-reduce (two-shot NVLink peer kernel, 2048^2 fp32)", secs, 0.0,
               2 * (world - 1) / world * w * w * 4, (world + 2) * w * w * 4 / world)
    # 5) expert-parallel MoE
    if emulate:
        # The owner-side kernels with the peers' buffers emulated locally: dispatch of 4096
        # tokens x top-8 rows into W receive buffers, the ragged gate/up GEMM over this owner's
        # 64 / W experts, the split SwiGLU, and the ragged down GEMM scattering its rows home.
        h, inter, n_exp, top_k, t = 2048, 1024, 64, 8, 4096
        e_l = n_exp // world
        rows_in = t * top_k
        x2 = torch.randn(t, h, device=dev, generator=gen).bfloat16()
        dest = torch.randint(0, world, (rows_in,), device=dev, generator=gen)
        order = torch.argsort(dest, stable=True)
        per = torch.bincount(dest, minlength=world)
        start = torch.cumsum(per, 0) - per
        row = torch.empty_like(dest)
        row[order] = torch.arange(rows_in, device=dev) - start[dest[order]]
        recv = [torch.empty(rows_in, h, device=dev, dtype=torch.bfloat16) for _ in range(world)]
        meta = [torch.empty(rows_in, 2, device=dev, dtype=torch.int32) for _ in range(world)]
        d32, r32 = dest.int().contiguous(), row.int().contiguous()
        secs = _time(lambda: nat.moe_dispatch(x2, top_k, d32, r32, recv, meta, rank))
        report("moe_dispatch (rows stored into the owners' receive buffers)", secs, 0.0, 0.0,
               rows_in * h * 2 + t * h * 2)  # every routed row written once; each token read once
        n_i = torch.full((e_l,), rows_in // e_l, dtype=torch.int32, device=dev)
        base = (torch.cumsum(n_i, 0) - n_i).int().contiguous()
        prefix = torch.zeros(e_l + 1, dtype=torch.int32, device=dev)
        prefix[1:] = torch.cumsum((n_i + 255) // 256, 0)  # 256-row blocks
        max_tiles = rows_in // 256 + e_l
        gate_up = (0.02 * torch.randn(e_l, 2 * inter, h, device=dev, generator=gen)).bfloat16()
        down = (0.02 * torch.randn(e_l, h, inter, device=dev, generator=gen)).bfloat16()
        xin = torch.randn(rows_in, h, device=dev, generator=gen).bfloat16()
        hh = torch.empty(rows_in, 2 * inter, device=dev, dtype=torch.bfloat16)
        secs = _time(lambda: nat.gemm_ragged(xin, gate_up, hh, prefix, base, n_i, max_tiles, [], None, err))
        report("gemm_ragged gate/up (persistent, all local experts in one launch)", secs,
               2.0 * rows_in * h * 2 * inter, 0.0, (rows_in * h + rows_in * 2 * inter + e_l * 2 * inter * h) * 2)
        secs_bmm = _time(lambda: torch.bmm(xin.view(e_l, -1, h), gate_up.transpose(1, 2)))
        rows[-1]["cublas_bmm_same_flops_us"] = secs_bmm * 1e6
        act = torch.empty(rows_in, inter, device=dev, dtype=torch.bfloat16)
        nrows = torch.tensor([rows_in], dtype=torch.int32, device=dev)
        secs = _time(lambda: nat.swiglu_split(hh, act, nrows))
        report("swiglu_split", secs, 0.0, 0.0, rows_in * 3 * inter * 2)
        homes = [torch.empty(rows_in // world + 1, h, device=dev, dtype=torch.bfloat16) for _ in range(world)]
        idx = torch.arange(rows_in, device=dev)
        home_meta = torch.stack([idx % world, idx // world], 1).int().contiguous()
        secs = _time(lambda: nat.gemm_ragged(act, down, None, prefix, base, n_i, max_tiles, homes, home_meta, err))
        report("gemm_ragged down + scatter home (combine in the epilogue)", secs, 2.0 * rows_in * inter * h, 0.0,
               (rows_in * inter + rows_in * h + e_l * h * inter) * 2)
    else:
        from dattri_llm_b200.parallel.moe import ExpertParallelMoE

        h, inter, n_exp, top_k, t = 2048, 1024, 64, 8, 4096
        g = torch.Generator(device=dev).manual_seed(11)
        moe = ExpertParallelMoE(h, inter, n_exp, top_k, max_tokens=t)
        moe.load_experts((0.02 * torch.randn(n_exp, 2 * inter, h, device=dev, generator=g)).bfloat16(),
                         (0.02 * torch.randn(n_exp, h, inter, device=dev, generator=g)).bfloat16(),
                         (0.02 * torch.randn(n_exp, h, device=dev, generator=g)).bfloat16())
        xm = torch.randn(t, h, device=dev, generator=gen).bfloat16()
        with torch.no_grad():
            secs = _time(lambda: moe(xm), iters=10)
        rows_moved = t * top_k * (world - 1) / world
        fwd_flops = 2.0 * t * top_k * (h * 2 * inter + inter * h) + 2.0 * t * h * n_exp
        report("expert-parallel MoE forward (dispatch + expert GEMMs + combine in the down-GEMM epilogue)",
               secs, fwd_flops, 2 * rows_moved * h * 2, 4 * t * top_k * h * 2,
               {"tokens_per_rank": t, "experts": n_exp, "top_k": top_k})
        xg = xm.clone().requires_grad_()

        def fwd_bwd():
            y = moe(xg)
            y.backward(torch.ones_like(y))

        secs = _time(fwd_bwd, iters=10)
        report("expert-parallel MoE forward + backward (input and router gradients; experts frozen)",
               secs, 2 * fwd_flops, 4 * rows_moved * h * 2, 8 * t * top_k * h * 2,
               {"tokens_per_rank": t, "experts": n_exp, "top_k": top_k})
    ops.check_device_errors(dev)
    return rows


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--emulate", type=int, default=0, help="emulate this many peers on one GPU")
    a = ap.parse_args()
    if a.emulate:
        torch.cuda.set_device(0)
        rows = run(a.emulate, True, 0)
        rank = 0
    else:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        rank = dist.get_rank()
        rows = run(dist.get_world_size(), False, rank)
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
