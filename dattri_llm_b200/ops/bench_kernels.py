"""A/B timings of the native kernels against the PyTorch ops they replace, on one GPU.

    python -m dattri_llm_b200.ops.bench_kernels            # every kernel, JSON lines
    python -m dattri_llm_b200.ops.bench_kernels --only ghost_gram,norm_grad

Each row times the native entry point and the PyTorch formulation of the same math the
reference uses (its ``gradient/ops`` functions: matmuls, einsums, elementwise chains),
on the same bf16 operands, with CUDA events around every launch and the 126 MB L2
flushed (a 256 MiB write) before each one, after three warm-up runs.  The median of the
timed runs is reported with the algorithmic bytes and FLOPs and their fractions of the
measured copy bandwidth and bf16 GEMM rate (``MEASURED_PEAKS.json`` when present).

Rows (ids of the hot-op inventory):
  ghost_gram      K6  fused (A1 A2^T) . (G1 G2^T) block sum  vs two matmuls + Hadamard + view-sum
  ghost_dot       K8  per-sample <dW_i, dW'_i>                vs the (B, T, T) einsum pair
  ghost_tokens    K10 embedding gram by token equality        vs one-hot scatter per sample
  norm_grad       K11 per-sample RMSNorm dgamma               vs x_hat recompute + einsum over T
  mask_gather     K12 fixed coordinates of g^T a             vs index_select + mul + sum
  gram_acc        K13 A += a^T a (fp32)                       vs (a^T @ a).float() + add
  ekfac_lambda    K17 lam += sum_i (U_G^T dW_i U_A)^2         vs einsum rotate + square + sum
  per_sample_outer K5 (B, T, d)^T (B, T, k) -> (B, d, k)      vs torch.bmm
  adam_dir        K18 m_hat / (sqrt(v_hat) + eps)             vs the elementwise chain
  project_seg     K1  a @ P stored token-major (B, k, T)      vs matmul + transpose copy
  embed_dense     K10 dense (B, vocab * E) embedding grads    vs zero fill + index_add
  gated_norm      Mamba2 gated RMSNorm, forward + backward   vs the module's elementwise chain
  causal_conv     Mamba2 conv1d (4 taps) + SiLU, fwd + bwd    vs cuDNN depthwise conv + SiLU
  ssd_intra       Mamba2 intra-chunk SSD, fwd + bwd          vs materialized decay + einsum
"""

from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

_FLUSH = None


def _peaks() -> tuple[float, float, str]:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]) * 1e9, float(p["bf16_tflops"]) * 1e12, "measured"
    except (OSError, KeyError, ValueError):
        return 6.65e12, 1.59e15, "fallback"


def _flush() -> None:
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def _time(fn, iters: int = 10) -> float:
    """Median device seconds of *fn* over *iters* cold-L2 launches."""
    for _ in range(3):
        fn()
    times = []
    for _ in range(iters):
        _flush()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e) * 1e-3)
    return statistics.median(times)


def _row(name, ours, torch_s, nbytes, flops, peaks, extra=None):
    bw, fl, src = peaks
    out = {"kernel": name, "ours_us": round(ours * 1e6, 2), "torch_us": round(torch_s * 1e6, 2),
           "speedup": round(torch_s / ours, 2), "bytes": int(nbytes), "flops": int(flops),
           "hbm_frac": round(nbytes / ours / bw, 3), "tensor_frac": round(flops / ours / fl, 3),
           "peaks": src}
    if extra:
        out.update(extra)
    print(json.dumps(out), flush=True)


def bench_ghost_gram(peaks):
    from dattri_llm_b200 import ops

    b1, b2, s, k, d = 8, 32, 512, 64, 64
    a1, g1 = torch.randn(b1, s, k, device="cuda").bfloat16(), torch.randn(b1, s, d, device="cuda").bfloat16()
    a2, g2 = torch.randn(b2, s, k, device="cuda").bfloat16(), torch.randn(b2, s, d, device="cuda").bfloat16()

    def ref():
        ka = a1.reshape(-1, k) @ a2.reshape(-1, k).T
        kg = g1.reshape(-1, d) @ g2.reshape(-1, d).T
        return (ka * kg).view(b1, s, b2, s).sum((1, 3), dtype=torch.float32)

    ours = _time(lambda: ops.ghost_gram(a1, g1, a2, g2))
    nbytes = 2 * (a1.numel() + g1.numel() + a2.numel() + g2.numel())
    flops = 2 * (b1 * s) * (b2 * s) * (k + d) + 2 * (b1 * s) * (b2 * s)
    _row("ghost_gram", ours, _time(ref), nbytes, flops, peaks, {"shape": f"B1={b1} B2={b2} S={s} K={k} D={d}"})


def bench_ghost_dot(peaks):
    from dattri_llm_b200 import ops

    b, s, k, d = 16, 1024, 64, 64
    a1, g1 = torch.randn(b, s, k, device="cuda").bfloat16(), torch.randn(b, s, d, device="cuda").bfloat16()

    def ref():
        return (torch.einsum("bsk,btk->bst", a1, a1) * torch.einsum("bsd,btd->bst", g1, g1)).sum((1, 2),
                                                                                               dtype=torch.float32)

    ours = _time(lambda: ops.ghost_dot(a1, g1, a1, g1))
    flops = 2 * b * s * s * (k + d)
    _row("ghost_dot", ours, _time(ref), 2 * (a1.numel() + g1.numel()), flops, peaks,
         {"shape": f"B={b} S={s} K={k} D={d}"})


def bench_ghost_tokens(peaks):
    from dattri_llm_b200 import ops

    b1, b2, s, e, v = 4, 8, 512, 2048, 32000
    tok1 = torch.randint(0, v, (b1, s), device="cuda")
    tok2 = torch.randint(0, v, (b2, s), device="cuda")
    g1 = torch.randn(b1, s, e, device="cuda").bfloat16()
    g2 = torch.randn(b2, s, e, device="cuda").bfloat16()

    def ref():  # the reference's form: per-sample scatter-add into (V, E), then the dense dot
        out = torch.empty(b1, b2, device="cuda")
        w1 = [torch.zeros(v, e, device="cuda").index_add_(0, tok1[i], g1[i].float()) for i in range(b1)]
        for j in range(b2):
            w2 = torch.zeros(v, e, device="cuda").index_add_(0, tok2[j], g2[j].float())
            for i in range(b1):
                out[i, j] = (w1[i] * w2).sum()
        return out

    ours = _time(lambda: ops.ghost_gram_tokens(tok1, g1, tok2, g2))
    flops = 2 * (b1 * s) * (b2 * s) * e
    _row("ghost_tokens", ours, _time(ref, iters=3), 2 * (g1.numel() + g2.numel()), flops, peaks,
         {"shape": f"B1={b1} B2={b2} S={s} E={e} V={v}"})


def bench_norm_grad(peaks):
    from dattri_llm_b200 import ops

    b, t, d, eps = 8, 1024, 2048, 1e-5
    x = torch.randn(b, t, d, device="cuda").bfloat16()
    g = torch.randn(b, t, d, device="cuda").bfloat16()

    def ref():
        xf = x.float()
        xh = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        return torch.einsum("btd,btd->bd", xh, g.float())

    ours = _time(lambda: ops.norm_per_sample_grad(x, g, eps=eps, layer_norm=False, bias=False))
    _row("norm_grad", ours, _time(ref), 2 * (x.numel() + g.numel()) + 4 * b * d, 0, peaks,
         {"shape": f"B={b} T={t} d={d}"})


def bench_mask_gather(peaks):
    from dattri_llm_b200 import ops

    b, t, kr, kc, m = 8, 1024, 2048, 2048, 4096
    r = torch.randn(b, t, kr, device="cuda").bfloat16()
    c = torch.randn(b, t, kc, device="cuda").bfloat16()
    rows = torch.randint(0, kr, (m,), device="cuda")
    cols = torch.randint(0, kc, (m,), device="cuda")

    def ref():
        return (r.index_select(2, rows).float() * c.index_select(2, cols).float()).sum(1)

    ours = _time(lambda: ops.mask_gather(r, c, rows, cols))
    _row("mask_gather", ours, _time(ref), 2 * (r.numel() + c.numel()) + 4 * b * m, 2 * b * t * m, peaks,
         {"shape": f"B={b} T={t} Kr={kr} Kc={kc} M={m}"})


def bench_gram_acc(peaks):
    from dattri_llm_b200.gradient.ops.kronecker import gram_accumulate

    n, w = 16384, 2048
    x = torch.randn(n, w, device="cuda").bfloat16()
    out = torch.zeros(w, w, device="cuda")

    def ref():
        out.add_((x.T @ x).float())

    ours = _time(lambda: gram_accumulate(x, out))
    _row("gram_acc", ours, _time(ref), 2 * x.numel() + 8 * w * w, 2 * n * w * w, peaks, {"shape": f"N={n} w={w}"})


def bench_ekfac_lambda(peaks):
    from dattri_llm_b200.gradient.gradient import Factorized
    from dattri_llm_b200.gradient.ops.kronecker import ekfac_lambda_accumulate

    b, t, k, d = 8, 1024, 64, 64
    a = torch.randn(b, t, k, device="cuda").bfloat16()
    g = torch.randn(b, t, d, device="cuda").bfloat16()
    ua = torch.linalg.qr(torch.randn(k, k, device="cuda"))[0]
    ug = torch.linalg.qr(torch.randn(d, d, device="cuda"))[0]
    f = Factorized(activation=a, pre_activation_grad=g, module_kwargs=None)
    lam = torch.zeros(d * k, device="cuda")

    def ref():
        dw = torch.einsum("btd,btk->bdk", g.float(), a.float())
        m = ug.T @ dw @ ua
        lam.add_((m * m).sum(0).reshape(-1))

    ours = _time(lambda: ekfac_lambda_accumulate(f, "nn.Linear", ua, ug, lam, include_bias=False))
    flops = 2 * b * t * (k * k + d * d) + 2 * b * t * d * k
    _row("ekfac_lambda", ours, _time(ref), 2 * (a.numel() + g.numel()) + 4 * d * k, flops, peaks,
         {"shape": f"B={b} T={t} k={k} d={d}"})


def bench_per_sample_outer(peaks):
    from dattri_llm_b200 import ops

    b, t, dl, dr = 8, 1024, 2048, 512
    left = torch.randn(b, t, dl, device="cuda").bfloat16()
    right = torch.randn(b, t, dr, device="cuda").bfloat16()
    lt, rt = left.transpose(1, 2).contiguous(), right.transpose(1, 2).contiguous()

    def ref():
        return torch.bmm(left.transpose(1, 2), right).float()

    ours = _time(lambda: ops.per_sample_outer(left, right, left_t=lt, right_t=rt))
    _row("per_sample_outer", ours, _time(ref), 2 * (left.numel() + right.numel()) + 4 * b * dl * dr,
         2 * b * t * dl * dr, peaks, {"shape": f"B={b} T={t} L={dl} R={dr}"})


def bench_adam_dir(peaks):
    from dattri_llm_b200 import ops

    b, p = 64, 1 << 16
    g = torch.randn(b, p, device="cuda")
    m0, v0 = torch.randn(p, device="cuda"), torch.rand(p, device="cuda")
    b1, b2, eps, step = 0.9, 0.999, 1e-8, 10

    def ref():
        m = b1 * m0 + (1 - b1) * g
        v = b2 * v0 + (1 - b2) * g * g
        return (m / (1 - b1 ** step)) / ((v / (1 - b2 ** step)).sqrt() + eps)

    ours = _time(lambda: ops.adam_direction(g, m0, v0, step=step, beta1=b1, beta2=b2, eps=eps))
    _row("adam_dir", ours, _time(ref), 4 * (2 * g.numel() + 2 * p), 0, peaks, {"shape": f"B={b} p={p}"})


def bench_project_seg(peaks):
    from dattri_llm_b200 import ops

    b, t, d, k = 8, 1024, 8192, 64
    a = torch.randn(b * t, d, device="cuda").bfloat16()
    p_t = torch.randn(k, d, device="cuda").bfloat16()  # the projection, K-major
    p = p_t.T.contiguous()

    def ref():
        return (a @ p).view(b, t, k).transpose(1, 2).contiguous()

    ours = _time(lambda: ops.gemm_tn_seg(a, p_t, t))
    _row("project_seg", ours, _time(ref), 2 * (a.numel() + p.numel() + b * t * k), 2 * b * t * d * k, peaks,
         {"shape": f"T={b * t} d={d} k={k}"})


def bench_embed_dense(peaks):
    from dattri_llm_b200 import ops

    b, t, e, v = 8, 1024, 1024, 8192
    ids = torch.randint(0, v, (b, t), device="cuda")
    g = torch.randn(b, t, e, device="cuda").bfloat16()

    def ref():  # zero fill + scatter-add of every token row at its (sample, id)
        out = torch.zeros(b * v, e, dtype=g.dtype, device="cuda")
        out.index_add_(0, (ids + torch.arange(b, device="cuda")[:, None] * v).reshape(-1), g.reshape(-1, e))
        return out

    ours = _time(lambda: ops.embedding_dense_grad(ids, g, v))
    _row("embed_dense", ours, _time(ref), 2 * (g.numel() + b * v * e), 0, peaks,
         {"shape": f"B={b} T={t} E={e} V={v}"})


def bench_gated_norm(peaks):
    from dattri_llm_b200.ops import fused

    rows, d, eps = 2048, 5120, 1e-5
    y = torch.randn(rows, d, device="cuda", requires_grad=True)
    g = torch.randn(rows, d, device="cuda").bfloat16().requires_grad_()
    w = torch.ones(d, device="cuda").bfloat16().requires_grad_()
    dout = torch.randn(rows, d, device="cuda").bfloat16()

    def ref():  # the Hugging Face module's chain (fp32), its cast, and the backward
        h = y * torch.nn.functional.silu(g.float())
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
        (w * h).to(torch.bfloat16).backward(dout)

    def ours_fn():
        fused.gated_rms_norm(y, g, w, eps).backward(dout)

    nbytes = (4 + 2 + 2) * rows * d + (2 + 4 + 2 + 2 + 4 + 2) * rows * d  # forward + backward streams
    _row("gated_norm_fwd_bwd", _time(ours_fn), _time(ref), nbytes, 0, peaks, {"shape": f"rows={rows} d={d}"})


def bench_causal_conv(peaks):
    from dattri_llm_b200.ops import fused

    b, length, c = 1, 2048, 5376
    proj = torch.randn(b, length, c + 5200, device="cuda").bfloat16()
    x = proj[..., 5120:5120 + c].detach().requires_grad_()
    conv = torch.nn.Conv1d(c, c, 4, groups=c, padding=3).cuda().bfloat16()
    dout = torch.randn(b, length, c, device="cuda").bfloat16()

    def ref():  # the mixer's module call: transposes, cuDNN depthwise conv, slice, SiLU
        out = torch.nn.functional.silu(conv(x.transpose(1, 2))[..., :length].transpose(1, 2))
        out.backward(dout)

    def ours_fn():
        fused.causal_conv_silu(x, conv.weight, conv.bias).backward(dout)

    _row("causal_conv_silu_fwd_bwd", _time(ours_fn), _time(ref), 2 * b * length * c * 5, 0, peaks,
         {"shape": f"B={b} L={length} C={c}"})


def bench_ssd_intra(peaks):
    from dattri_llm_b200.ops import fused

    b, c, s, h, g, p = 1, 8, 256, 80, 1, 64  # one Mamba2-2.7B layer at 2,048 tokens
    cb = torch.randn(b, g, c, s, s, device="cuda", requires_grad=True)
    cum = (-0.05 * torch.rand(b, h, c, s, device="cuda")).cumsum(-1).requires_grad_()
    x = torch.randn(b, c, s, h, p, device="cuda", requires_grad=True)
    dy = torch.randn(b, c, s, h, p, device="cuda")
    causal = torch.ones(s, s, dtype=torch.bool, device="cuda").tril()

    def ref():  # the materialized form: per-head decayed (chunk x chunk) matrices, einsum
        decay = (cum[..., :, None] - cum[..., None, :]).masked_fill(~causal, float("-inf")).exp()
        mix = cb.repeat_interleave(h // g, dim=1) * decay
        torch.einsum("bhcst,bcthp->bcshp", mix, x).backward(dy)

    def ours_fn():
        fused.ssd_intra(cb, cum, x).backward(dy)

    flops = 3 * 2 * b * h * c * (s * (s + 1) // 2) * p  # y, dx and dM over the causal half
    _row("ssd_intra_fwd_bwd", _time(ours_fn), _time(ref), 4 * (3 * x.numel() + 2 * cb.numel()), flops, peaks,
         {"shape": f"B={b} C={c} S={s} H={h} G={g} P={p}", "note": "fp32 CUDA cores; tensor_frac vs the bf16 peak"})


BENCHES = {
    "ghost_gram": bench_ghost_gram,
    "ghost_dot": bench_ghost_dot,
    "ghost_tokens": bench_ghost_tokens,
    "norm_grad": bench_norm_grad,
    "mask_gather": bench_mask_gather,
    "gram_acc": bench_gram_acc,
    "ekfac_lambda": bench_ekfac_lambda,
    "per_sample_outer": bench_per_sample_outer,
    "adam_dir": bench_adam_dir,
    "project_seg": bench_project_seg,
    "embed_dense": bench_embed_dense,
    "gated_norm": bench_gated_norm,
    "causal_conv": bench_causal_conv,
    "ssd_intra": bench_ssd_intra,
}


def main() -> None:
    from dattri_llm_b200 import ops

    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="", help="comma-separated subset of: " + ",".join(BENCHES))
    args = ap.parse_args()
    names = [n for n in args.only.split(",") if n] or list(BENCHES)
    ops.native()
    peaks = _peaks()
    torch.manual_seed(0)
    for n in names:
        BENCHES[n](peaks)
    ops.check_device_errors()


if __name__ == "__main__":
    main()
