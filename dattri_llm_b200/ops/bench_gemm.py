"""Timings of the native tcgen05 GEMMs against cuBLAS on one GPU.

    python -m dattri_llm_b200.ops.bench_gemm            # dense shapes + staged all-gather GEMM
    python -m dattri_llm_b200.ops.bench_gemm --shape 8192x2048x2048

Dense ``C = A B^T`` (bf16 in, bf16 out) through :func:`dattri_llm_b200.ops.gemm_tn`
(multi-wave wide shapes run on the CTA-pair persistent kernel) against ``torch.matmul`` on
the same operands, then the staged all-gather GEMM (``gemm_tn_staged``) with W ranks
emulated by separate allocations on this GPU (the copies run at HBM rather than NVLink
speed).  CUDA events after three warm-up launches; one JSON object per line.
"""

from __future__ import annotations

import argparse
import json

import torch

SHAPES = [(8192, 2048, 2048), (16384, 4096, 2048), (8192, 8192, 2048), (32768, 2048, 2048), (2048, 2048, 8192)]


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


def main() -> None:
    from dattri_llm_b200 import ops

    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default=None, help="MxNxK of one dense problem")
    ap.add_argument("--no-staged", action="store_true")
    a_ = ap.parse_args()
    dev = torch.device("cuda", torch.cuda.current_device())
    err = ops.error_word(dev)
    shapes = [tuple(int(v) for v in a_.shape.split("x"))] if a_.shape else SHAPES
    for m, n, k in shapes:
        a = torch.randn(m, k, device=dev).bfloat16()
        b = torch.randn(n, k, device=dev).bfloat16()
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        ours = _time(lambda: ops.native().gemm_tn(a, b, out, 1.0, ops.STORE_BF16, 1, False, err))
        ref = _time(lambda: torch.matmul(a, b.T))
        flops = 2.0 * m * n * k
        print(json.dumps({"gemm": f"{m}x{n}x{k}", "ours_us": ours * 1e6, "cublas_us": ref * 1e6,
                          "ours_tflops": flops / ours / 1e12, "cublas_tflops": flops / ref / 1e12,
                          "ours_over_cublas": ref / ours}), flush=True)
    if not a_.no_staged:
        m, n, k = 8192, 2048, 2048
        a = torch.randn(m, k, device=dev).bfloat16()
        b = torch.randn(n, k, device=dev).bfloat16()
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        dense = _time(lambda: ops.native().gemm_tn(a, b, out, 1.0, ops.STORE_BF16, 1, False, err))
        for world in (1, 2, 8):
            for mode in (0, 1):
                shards = [s.contiguous() for s in (b.chunk(world, 0) if mode == 0 else b.chunk(world, 1))]
                stage = torch.empty(n, k, device=dev, dtype=torch.bfloat16)
                flags = torch.zeros(world, dtype=torch.int32, device=dev)
                epoch = [0]

                def run(shards=shards, stage=stage, flags=flags, epoch=epoch, mode=mode):
                    epoch[0] += 1
                    ops.native().gemm_tn_staged(a, shards, stage, out, flags, epoch[0], mode, 0, ops.STORE_BF16,
                                                1.0, err)

                t = _time(run)
                print(json.dumps({"staged": f"{m}x{n}x{k}", "emulated_world": world, "mode": mode,
                                  "us": t * 1e6, "dense_gemm_us": dense * 1e6}), flush=True)
    ops.check_device_errors(dev)


if __name__ == "__main__":
    main()
