"""Timings of the native tcgen05 GEMMs against cuBLAS on one GPU.

    python -m dattri_llm_b200.ops.bench_gemm            # dense shapes + staged all-gather GEMM
    python -m dattri_llm_b200.ops.bench_gemm --shape 8192x2048x2048
    python -m dattri_llm_b200.ops.bench_gemm --step   # the Llama-3.2-1B bench step's GEMMs

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
# (name, M, N, K, projection tail rows): the forward and input-gradient GEMMs of one decoder
# layer of the bench step (8 x 1024 tokens) and the LM head; the tail is the fused LoGra
# projection (64 rows; none where a sibling layer already projected the same input).
STEP = [("q_fwd", 8192, 2048, 2048, 64), ("k_fwd", 8192, 512, 2048, 0), ("o_fwd", 8192, 2048, 2048, 64),
        ("gate_fwd", 8192, 8192, 2048, 64), ("up_fwd", 8192, 8192, 2048, 0), ("down_fwd", 8192, 2048, 8192, 64),
        ("q_dgrad", 8192, 2048, 2048, 64), ("k_dgrad", 8192, 2048, 512, 64), ("o_dgrad", 8192, 2048, 2048, 64),
        ("gate_dgrad", 8192, 2048, 8192, 64), ("down_dgrad", 8192, 8192, 2048, 64),
        ("lm_fwd", 8184, 128256, 2048, 0), ("lm_dgrad", 8184, 2048, 128256, 0)]


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
    ap.add_argument("--step", action="store_true", help="time the bench step's GEMM shapes only")
    a_ = ap.parse_args()
    dev = torch.device("cuda", torch.cuda.current_device())
    err = ops.error_word(dev)
    if a_.step:
        from dattri_llm_b200.ops.linear import gemm_with_tail

        for name, m, n, k, tail in STEP:
            a = torch.randn(m, k, device=dev).bfloat16()
            b = torch.randn(n, k, device=dev).bfloat16()
            out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            if tail:
                p_t = torch.randn(tail, k, device=dev).bfloat16()
                ours = _time(lambda: gemm_with_tail(a, b, p_t, 1024, out=out))
                proj = _time(lambda: ops.gemm_tn_seg(a, p_t, 1024))
            else:
                ours = _time(lambda: ops.native().gemm_tn(a, b, out, 1.0, ops.STORE_BF16, 1, False, err))
                proj = 0.0
            ref = _time(lambda: torch.matmul(a, b.T))
            flops = 2.0 * m * n * k
            print(json.dumps({"gemm": name, "mnk": f"{m}x{n}x{k}", "tail": tail, "ours_us": ours * 1e6,
                              "cublas_us": ref * 1e6, "cublas_plus_proj_us": (ref + proj) * 1e6,
                              "ours_tflops": flops / ours / 1e12, "cublas_tflops": flops / ref / 1e12,
                              "ours_over_cublas_plus_proj": (ref + proj) / ours}), flush=True)
        ops.check_device_errors(dev)
        return
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
