"""Peer-memory kernels on 2+ GPUs (one process per GPU, NCCL): the bounded cross-GPU
barrier and the fused all-gather + score GEMM against NCCL all-gather + fp32 matmul;
expert parallelism (fused path, and per-sample capture over NCCL all-to-all against the
replicated-expert capture).  Skipped with fewer than two GPUs."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fsdp_worker(rank: int, world: int, port: int, results) -> None:
    import datetime
    import faulthandler

    import torch.distributed as dist

    faulthandler.enable()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from dattri_llm_b200 import ops

        gen = torch.Generator(device=dev).manual_seed(300 + rank)
        worst = 0.0
        # Row-sharded linear: all-gather fused into the forward and input-gradient GEMMs,
        # weight gradient reduce-scattered inside its GEMM.
        from dattri_llm_b200.parallel.fsdp import ShardedLinear, sync_sharded_grads

        torch.manual_seed(7)
        full = torch.nn.Linear(320, 256, bias=False).to(dev)
        w_full = full.weight.detach().bfloat16().float().clone()
        layer = ShardedLinear(full)
        x = torch.randn(3, 40, 320, device=dev, generator=gen).bfloat16().requires_grad_()
        y = layer(x)
        want_y = x.detach().float() @ w_full.T
        worst = max(worst, float((y.float() - want_y).abs().max() / want_y.abs().max()))
        dy = torch.randn_like(y)
        y.backward(dy)
        want_dx = dy.float() @ w_full
        worst = max(worst, float((x.grad.float() - want_dx).abs().max() / want_dx.abs().max()))
        sync_sharded_grads(torch.nn.ModuleList([layer]))
        dw = dy.float().reshape(-1, 256).T @ x.detach().float().reshape(-1, 320)
        dist.all_reduce(dw)
        mine = dw[rank * layer.rows:(rank + 1) * layer.rows]
        worst = max(worst, float((layer.grad_shard() - mine).abs().max() / mine.abs().max()))
        # a second backward accumulates (and takes the other buffer of the slot ring)
        dy2 = torch.randn_like(y)
        layer(x).backward(dy2)
        sync_sharded_grads(torch.nn.ModuleList([layer]))
        dw2 = dy2.float().reshape(-1, 256).T @ x.detach().float().reshape(-1, 320)
        dist.all_reduce(dw2)
        mine = mine + dw2[rank * layer.rows:(rank + 1) * layer.rows]
        worst = max(worst, float((layer.grad_shard() - mine).abs().max() / mine.abs().max()))
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        results[rank] = worst
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _worker(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from dattri_llm_b200 import ops
        from dattri_llm_b200.parallel.score import AllGatherScorer

        rows, k, n_local = 8, 4160, 200
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        test = torch.randn(n_local, k, device=dev, generator=gen).bfloat16()
        scorer = AllGatherScorer(test, rows)
        worst = 0.0
        for step in range(3):
            block = torch.randn(rows, k, device=dev, generator=gen).bfloat16()
            got = scorer.score(block)
            gathered = [torch.empty_like(block) for _ in range(world)]
            dist.all_gather(gathered, block)
            want = test.float() @ torch.cat(gathered).float().T
            err = float((got - want).abs().max() / want.abs().max())
            worst = max(worst, err)
        # NVLink peer all-reduce (one-shot and reduce-scatter + all-gather) against NCCL.
        from dattri_llm_b200.parallel import symm

        for n in (1000, 3 * (1 << 20) + 5):
            x = torch.randn(n, device=dev, generator=gen)
            want = x.clone()
            dist.all_reduce(want)
            assert symm.all_reduce_sum_(x)
            worst = max(worst, float((x - want).abs().max() / want.abs().max()))
        # K-FAC covariances accumulated in symmetric memory, reduced by the peer all-reduce.
        from dattri_llm_b200.gradient.ops.kronecker import LayerKroneckerAccumulator

        acc = LayerKroneckerAccumulator()
        ref_a = torch.zeros(192, 192, device=dev)
        ref_g = torch.zeros(64, 64, device=dev)
        for _ in range(3):
            a = torch.randn(4, 100, 192, device=dev, generator=gen).bfloat16()
            g = torch.randn(4, 100, 64, device=dev, generator=gen).bfloat16()
            acc.update(a, g, "nn.Linear", include_bias=False)
            ref_a += a.float().reshape(-1, 192).T @ a.float().reshape(-1, 192)
            ref_g += g.float().reshape(-1, 64).T @ g.float().reshape(-1, 64)
        assert acc._symm is not None, "the fused cross-rank path was not taken"
        acc.all_reduce()
        dist.all_reduce(ref_a)
        dist.all_reduce(ref_g)
        assert acc._n == 3 * 400 * world
        worst = max(worst, float((acc._A - ref_a).abs().max() / ref_a.abs().max()),
                    float((acc._G - ref_g).abs().max() / ref_g.abs().max()))
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        results[rank] = worst
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_score_allreduce_and_covariance_match_nccl():
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        errs = dict(results)
    assert len(errs) == world
    assert max(errs.values()) < 1e-2, errs


def _moe_worker(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch.distributed as dist
    import torch.nn.functional as F

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from dattri_llm_b200 import ops
        from dattri_llm_b200.parallel.moe import ExpertParallelMoE

        h, inter, n_exp, k = 128, 64, 8, 2
        g = torch.Generator(device=dev).manual_seed(11)  # same weights on every rank
        weights = []
        layers = []
        for _ in range(2):  # two stacked layers of one shape share the receive buffers
            gate_up = (0.1 * torch.randn(n_exp, 2 * inter, h, device=dev, generator=g)).bfloat16()
            down = (0.1 * torch.randn(n_exp, h, inter, device=dev, generator=g)).bfloat16()
            router = (0.1 * torch.randn(n_exp, h, device=dev, generator=g)).bfloat16()
            moe = ExpertParallelMoE(h, inter, n_exp, k, max_tokens=256)
            moe.load_experts(gate_up, down, router)
            weights.append((gate_up, down, router.float().requires_grad_()))
            layers.append(moe)

        def ref_layer(xr, gate_up, down, router):
            # the same bf16 router GEMM as the module, so near-ties pick the same experts
            probs = torch.softmax(F.linear(xr.bfloat16(), router.bfloat16()).float(), -1)
            topv, topi = probs.topk(k, -1)
            out = torch.zeros_like(xr)
            for j in range(k):
                e = topi[:, j]
                hh = torch.einsum("th,tnh->tn", xr, gate_up.float()[e])
                gg, uu = hh.chunk(2, -1)
                a = F.silu(gg) * uu
                out = out + topv[:, j:j + 1] * torch.einsum("ti,thi->th", a, down.float()[e])
            return out

        gx = torch.Generator(device=dev).manual_seed(50 + rank)
        worst = 0.0
        for _ in range(2):
            for m_ in layers:
                m_.gate.weight.grad = None
            for _, _, r_ in weights:
                r_.grad = None
            x = torch.randn(3, 37, h, device=dev, generator=gx).bfloat16().requires_grad_()
            y0 = layers[0](x)
            y = layers[1](y0)
            dy = torch.randn_like(y)
            y.backward(dy)
            # replicated-expert reference in fp32 on this rank's tokens; layer 1 reads the
            # module's own layer-0 output so both route on identical inputs
            xr = x.detach().float().reshape(-1, h).requires_grad_()
            mid = y0.detach().float().reshape(-1, h).requires_grad_()
            out = ref_layer(mid, *weights[1])
            out.backward(dy.float().reshape(-1, h))
            mid_ref = ref_layer(xr, *weights[0])
            mid_ref.backward(mid.grad)
            pairs = [(y0.float().reshape(-1, h), mid_ref.detach()), (y.float().reshape(-1, h), out.detach()),
                     (x.grad.float().reshape(-1, h), xr.grad)]
            pairs += [(m_.gate.weight.grad.float(), w_[2].grad) for m_, w_ in zip(layers, weights)]
            for got, want in pairs:
                worst = max(worst, float((got - want).abs().max() / want.abs().max()))
            x.grad = None
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        results[rank] = worst
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_moe_matches_replicated():
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_moe_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        errs = dict(results)
    assert len(errs) == world
    assert max(errs.values()) < 3e-2, errs


def _ep_capture_worker(rank: int, world: int, port: int, results) -> None:
    import copy
    import datetime

    import torch.distributed as dist
    import torch.nn.functional as F

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import transformers

        import dattri_llm_b200 as bw
        from dattri_llm_b200.parallel.moe import expert_parallelize

        cfg = transformers.OlmoeConfig(vocab_size=64, hidden_size=32, intermediate_size=16, num_hidden_layers=1,
                                       num_attention_heads=4, num_key_value_heads=4, num_experts=4,
                                       num_experts_per_tok=2, max_position_embeddings=64)
        torch.manual_seed(0)
        model = transformers.OlmoeForCausalLM(cfg).eval().to(dev)
        ep_model = copy.deepcopy(model)
        expert_parallelize(ep_model, max_tokens=64)  # fp32: the all-to-all form over NCCL
        ids = torch.randint(0, 64, (3, 8), generator=torch.Generator().manual_seed(7 + rank)).to(dev)

        def capture(m, **kw):
            cap = bw.CaptureCallback()
            hm = bw.HookManager(m, bw.HookManagerConfig(linear_io=[r"mlp"]), callbacks=[cap], **kw)
            with hm.collect():
                logits = m(input_ids=ids).logits
                F.cross_entropy(logits[:, :-1].reshape(-1, 64).float(), ids[:, 1:].reshape(-1),
                                reduction="sum").backward()
            hm.remove()
            return cap.record.gradient.materialize()

        want = capture(model, moe_routed_layers=["model.layers.0.mlp"])
        got = capture(ep_model)
        worst = 0.0 if set(got.data) == set(want.data) else float("inf")
        for n, v in want.data.items():
            if n in got.data:
                a, b = got.data[n].float().reshape(v.shape[0], -1), v.float().reshape(v.shape[0], -1)
                worst = max(worst, float((a - b).abs().max() / b.abs().max().clamp_min(1e-12)))
        torch.cuda.synchronize()
        results[rank] = worst
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_capture_matches_replicated_over_nccl():
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_ep_capture_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        errs = dict(results)
    assert len(errs) == world
    assert max(errs.values()) < 1e-3, errs


def _ep_grouped_worker(rank: int, world: int, port: int, results) -> None:
    """bf16 OLMoE block with LoGra 16 x 16 materialized expert captures: the fused
    expert-parallel path with the grouped capture against the replicated-expert grouped
    capture of the same rank's samples."""
    import copy
    import datetime
    import warnings

    import torch.distributed as dist
    import torch.nn.functional as F

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import transformers

        import dattri_llm_b200 as bw
        from dattri_llm_b200 import ops
        from dattri_llm_b200.parallel.moe import ExpertTap, expert_parallelize

        cfg = transformers.OlmoeConfig(vocab_size=96, hidden_size=128, intermediate_size=64, num_hidden_layers=1,
                                       num_attention_heads=4, num_key_value_heads=4, num_experts=8,
                                       num_experts_per_tok=2, max_position_embeddings=64)
        torch.manual_seed(0)
        model = transformers.OlmoeForCausalLM(cfg).to(dev, torch.bfloat16).eval()
        model.requires_grad_(False)
        model.get_input_embeddings().requires_grad_(True)
        ep_model = copy.deepcopy(model)
        expert_parallelize(ep_model, max_tokens=64)
        ids = torch.randint(0, 96, (3, 16), generator=torch.Generator().manual_seed(11 + rank)).to(dev)
        proj = {"__default__": {"style": "logra", "proj_dim": 16, "proj_type": "rademacher", "proj_seed": 0}}
        taps = {"n": 0}
        for m in ep_model.modules():
            if isinstance(m, ExpertTap):
                m.register_forward_hook(lambda *_: taps.__setitem__("n", taps["n"] + 1))

        def capture(m, **kw):
            cap = bw.CaptureCallback()
            hc = bw.HookManagerConfig(linear_io=[r"\.mlp\.(experts|gate)$", r"dattri_(experts|router)"],
                                      projection_kwargs=proj, capture_style="auto", include_frozen=True)
            hm = bw.HookManager(m, hc, callbacks=[cap], **kw)
            with warnings.catch_warnings():
                warnings.simplefilter("ignore")
                with hm.collect():
                    logits = m(input_ids=ids).logits
                    F.cross_entropy(logits[:, :-1].reshape(-1, 96).float(), ids[:, 1:].reshape(-1),
                                    reduction="sum").backward()
            hm.remove()
            return {n: v.float() for n, v in cap.record.gradient.data.items()}

        want = capture(model, moe_routed_layers=["model.layers.0.mlp"])
        got = capture(ep_model)
        ops.check_device_errors(dev)
        names = [n for n in want if ".dattri_experts." in n]
        worst = 0.0 if (set(got) == set(want) and len(names) == 16 and taps["n"] == 0) else float("inf")
        for n in names:
            a, b = got[n].reshape(got[n].shape[0], -1), want[n].reshape(want[n].shape[0], -1)
            if b.abs().max() == 0:
                worst = max(worst, float(a.abs().max()))
                continue
            worst = max(worst, float((a - b).norm() / b.norm()))
        torch.cuda.synchronize()
        results[rank] = (worst, taps["n"], sorted(set(got) ^ set(want))[:4])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_expert_parallel_grouped_capture_matches_replicated(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_ep_grouped_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        errs = dict(results)
    assert len(errs) == world
    assert max(e[0] for e in errs.values()) < 3e-2, errs


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_linear_fused_collectives_match_dense():
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_fsdp_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        errs = dict(results)
    assert len(errs) == world
    assert max(errs.values()) < 2e-2, errs


def _fused_fsdp_capture_worker(rank: int, world: int, port: int, results) -> None:
    import datetime
    import tempfile

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from dattri_llm_b200 import AttributionArguments, CaptureCallback, HookManager, HookManagerConfig, ops
        from dattri_llm_b200.gradient.streaming import GradientStreamer
        from dattri_llm_b200.models.llama import LlamaConfig, LlamaForCausalLM, token_sum_loss

        cfg = LlamaConfig.tiny(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                               vocab_size=1024)

        def build():
            m = LlamaForCausalLM(cfg, frozen_probe=True)
            m.reset_parameters(seed=0)
            return m.to(dev).bfloat16().requires_grad_(False)

        ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=torch.Generator().manual_seed(rank)).to(dev)
        proj = {"__default__": {"style": "logra", "proj_dim": 64}}
        regex = [r"\.(q_proj|k_proj|v_proj|o_proj|gate_proj|up_proj|down_proj)$"]

        def manager(model):
            cb = CaptureCallback()
            hm = HookManager(model, HookManagerConfig(linear_io=regex, projection_kwargs=proj, include_frozen=True,
                                                      capture_style="auto"), callbacks=[cb])
            return hm, cb

        plain = build()
        hm, cb = manager(plain)
        with hm.collect():
            token_sum_loss(plain, {"input_ids": ids}).backward()
        want = cb.record.gradient
        hm.remove()
        # the streamer's FSDP wrapping of a frozen probe: hooks first, then in-place sharding
        sharded = build()
        hm, cb = manager(sharded)
        args = AttributionArguments(output_dir=tempfile.mkdtemp(), fsdp="full_shard")
        assert GradientStreamer._wrap_model(sharded, args, frozen=True) is sharded
        n_sharded = sum(getattr(m, "_bw_frozen_shard", None) is not None for m in sharded.modules())
        assert n_sharded == 14, n_sharded
        with hm.collect():
            token_sum_loss(sharded, {"input_ids": ids}).backward()
        got = cb.record.gradient
        worst = 0.0
        for name, w in want.data.items():
            g = got.data[name]
            worst = max(worst, float((g.float() - w.float()).abs().max() / w.float().abs().max()))
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        results[rank] = worst
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_fsdp_frozen_probe_capture_matches_unsharded():
    """The streamer's FSDP path for a frozen probe shards the linears in place (weights
    all-gathered inside their GEMMs over NVLink); the per-sample LoGra capture equals the
    unsharded model's on every rank."""
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_fused_fsdp_capture_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        errs = dict(results)
    assert len(errs) == world
    assert max(errs.values()) < 3e-2, errs
