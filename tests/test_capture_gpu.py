"""Native capture path on the GPU vs the CPU fp32 reference path of the same ops."""

import copy

import pytest
import torch

from dattri_llm_b200 import CaptureCallback, HookManager, HookManagerConfig, ops as _ops  # noqa: F401
from dattri_llm_b200 import ops as native_ops
from dattri_llm_b200.gradient import ops

pytestmark = pytest.mark.gpu


class _Tiny(torch.nn.Module):
    def __init__(self, vocab=64, d=64, ff=128):
        super().__init__()
        self.emb = torch.nn.Embedding(vocab, d)
        self.q = torch.nn.Linear(d, d, bias=False)
        self.k = torch.nn.Linear(d, d, bias=False)
        self.up = torch.nn.Linear(d, ff, bias=False)
        self.down = torch.nn.Linear(ff, d, bias=False)
        self.head = torch.nn.Linear(d, vocab, bias=False)

    def forward(self, input_ids):
        h = self.emb(input_ids)
        h = h + self.q(h) * torch.sigmoid(self.k(h))
        h = h + self.down(torch.nn.functional.silu(self.up(h)))
        return self.head(h)


def _capture(model, x, style, proj_dim=16):
    cb = CaptureCallback()
    cfg = HookManagerConfig(linear_io=[r"^(q|k|up|down)$"], capture_style=style,
                            projection_kwargs={"__default__": {"style": "logra", "proj_dim": proj_dim}})
    hm = HookManager(model, cfg, callbacks=[cb])
    with hm.collect():
        out = model(input_ids=x)
        loss = torch.nn.functional.cross_entropy(out.float().reshape(-1, out.shape[-1]), x.reshape(-1))
        loss.backward()
    hm.remove()
    return cb.record.gradient


@pytest.mark.parametrize("style", ["materialized", "factorized"])
def test_projected_capture_native_matches_cpu(style):
    torch.manual_seed(0)
    cpu = _Tiny()
    gpu = copy.deepcopy(cpu).cuda().bfloat16()
    x = torch.randint(0, 64, (4, 32))
    ref = _capture(cpu, x, style).materialize()
    got = _capture(gpu, x.cuda(), style).materialize()
    native_ops.check_device_errors()
    for name in ref.layer_names:
        r, g = ref.data[name].float(), got.data[name].float().cpu()
        err = (r - g).norm() / r.norm()
        assert err < 5e-2, (name, float(err))


def test_ghost_route_matches_materialized_route_on_gpu():
    torch.manual_seed(1)
    a1 = torch.randn(3, 40, 64, device="cuda").bfloat16()
    g1 = torch.randn(3, 40, 32, device="cuda").bfloat16()
    a2 = torch.randn(5, 24, 64, device="cuda").bfloat16()
    g2 = torch.randn(5, 24, 32, device="cuda").bfloat16()
    ghost = ops.cross_gram(a1, g1, a2, g2, "nn.Linear", mode="factorized").float()
    mat = ops.cross_gram(a1, g1, a2, g2, "nn.Linear", mode="materialized").float()
    ref = ops.cross_gram(a1.double().cpu(), g1.double().cpu(), a2.double().cpu(), g2.double().cpu(),
                         "nn.Linear", mode="factorized")
    scale = ref.abs().max().item()
    torch.testing.assert_close(ghost.cpu().double(), ref, rtol=0, atol=1e-2 * scale)
    torch.testing.assert_close(mat.cpu().double(), ref, rtol=0, atol=2e-2 * scale)


def test_host_record_batches_dense_layers_and_keeps_values():
    from dattri_llm_b200.gradient.gradient import Factorized, Gradient, GradientRecord
    from dattri_llm_b200.gradient.storage_manager import _host_record

    gen = torch.Generator(device="cuda").manual_seed(1)
    dense = {f"l{i}": torch.randn(3, 5 + i, device="cuda", generator=gen).to(dt)
             for i, dt in enumerate([torch.bfloat16, torch.float32, torch.bfloat16])}
    fac = Factorized(torch.randn(3, 4, 6, device="cuda", generator=gen), torch.randn(3, 4, 2, device="cuda",
                                                                                     generator=gen))
    data = {**dense, "f": fac}
    g = Gradient({n: "materialized" for n in dense} | {"f": "factorized"}, data,
                 {n: "nn.Linear" for n in data}, {n: "batch" for n in data})
    host = _host_record(GradientRecord(0, ["a", "b", "c"], g)).gradient
    for n, v in dense.items():
        assert host.data[n].device.type == "cpu" and host.data[n].dtype == v.dtype
        assert torch.equal(host.data[n], v.cpu())
    assert host.data["f"].activation.device.type == "cpu"
    assert torch.equal(host.data["f"].activation, fac.activation.cpu())


def test_gradient_to_gpu_moves_host_layers_together():
    from dattri_llm_b200.gradient.gradient import Gradient

    gen = torch.Generator().manual_seed(2)
    data = {f"l{i}": torch.randn(2, 3 + i, generator=gen).to(torch.bfloat16 if i % 3 else torch.float32)
            for i in range(12)}
    g = Gradient({n: "materialized" for n in data}, data, {n: "nn.Linear" for n in data}, {n: "batch" for n in data})
    moved = g.to("cuda")
    torch.cuda.synchronize()
    for n, v in data.items():
        assert moved.data[n].is_cuda and moved.data[n].dtype == v.dtype and moved.data[n].shape == v.shape
        assert torch.equal(moved.data[n].cpu(), v)


def test_grouped_kfac_accumulation_matches_per_layer_updates():
    from dattri_llm_b200.gradient.ops.kronecker import LayerKroneckerAccumulator, kfac_accumulate_grouped

    gen = torch.Generator(device="cuda").manual_seed(4)
    layers = 5
    a_fs = [torch.randn(600, 64, device="cuda", generator=gen).bfloat16() for _ in range(layers)]
    g_fs = [torch.randn(600, 64, device="cuda", generator=gen).bfloat16() for _ in range(layers)]
    for g in g_fs:
        g[::7] = 0  # rows without a gradient are masked out of A and of the count
    one = [LayerKroneckerAccumulator(fused_reduce=False) for _ in range(layers)]
    grouped = [LayerKroneckerAccumulator(fused_reduce=False) for _ in range(layers)]
    for _ in range(2):  # two steps
        for acc, a, g in zip(one, a_fs, g_fs, strict=True):
            acc.update(a, g, "nn.Linear", None, include_bias=False)
        kfac_accumulate_grouped(grouped, a_fs, g_fs)
    for want, got in zip(one, grouped, strict=True):
        (wa, wg), (ga, gg) = want.result(), got.result()
        assert want._n == got._n
        torch.testing.assert_close(ga, wa, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(gg, wg, rtol=1e-4, atol=1e-4)


def test_fused_adamw_step_count_and_preconditioning_match_foreach():
    """The streamer gives GPU parameters torch's fused AdamW, which keeps the update count on
    the GPU; the optimizer snapshot counts it on the host after one read, and its Adam
    preconditioning matches the multi-tensor optimizer's."""
    from dattri_llm_b200.gradient.optimizer_state import OptimizerSnapshot

    snaps, dirs = [], []
    for fused in (True, False):
        torch.manual_seed(0)
        model = torch.nn.Sequential(torch.nn.Linear(16, 32, bias=False), torch.nn.Linear(32, 8, bias=False)).cuda()
        opt = torch.optim.AdamW(model.parameters(), lr=1e-2, fused=fused, foreach=None if fused else True)
        snap = OptimizerSnapshot(model, opt)
        x = torch.randn(4, 16, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
        for i in range(3):
            model(x).pow(2).sum().backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
            if i == 0:
                assert snap.step_count("0") == 1  # first read of the GPU count
        assert snap.step_count("0") == 3 and snap.step_count("1") == 3
        g = torch.randn(5, 32 * 16, device="cuda", generator=torch.Generator(device="cuda").manual_seed(2))
        dirs.append(snap.precondition("0", g))
        snaps.append(snap)
    torch.testing.assert_close(dirs[0], dirs[1], rtol=1e-3, atol=1e-3)
