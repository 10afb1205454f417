"""Expert parallelism on CPU (gloo, two ranks, and one process): the all-to-all form of
:class:`ExpertParallelMoE` gives the replicated-expert MoE's output and input / router
gradients, and its expert taps capture every sample's gradient of every expert's gate/up
and down weights (owner-side factors returned to the source), equal to per-sample
autograd on a dense replicated model.  A Hugging Face OLMoE model converted with
``expert_parallelize`` records the same layers, with the same values (raw and LoGra
projected), as the replicated-expert capture of the original model.  TracIn through the
public API on two ranks (the streamer's DDP or FSDP wrapping, which must leave each rank's
expert shard alone) gives the single-process scores."""

from __future__ import annotations

import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F
from torch import nn

H, INTER, E, K, B, T, D_IN = 8, 8, 4, 2, 3, 5, 6


def _weights():
    g = torch.Generator().manual_seed(21)
    return {
        "gate_up": 0.5 * torch.randn(E, 2 * INTER, H, generator=g),
        "down": 0.5 * torch.randn(E, H, INTER, generator=g),
        "router": torch.randn(E, H, generator=g),
        "fc_w": 0.5 * torch.randn(H, D_IN, generator=g),
        "fc_b": 0.1 * torch.randn(H, generator=g),
        "head_w": torch.randn(1, H, generator=g),
    }


def _data(rank: int):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(B, T, D_IN, generator=g), torch.randn(B, generator=g)


def _dense_moe(x, gate_up, down, router):
    x2 = x.reshape(-1, H)
    probs = torch.softmax(x2 @ router.t(), -1)
    topv, topi = probs.topk(K, -1)
    out = torch.zeros_like(x2)
    for j in range(K):
        e = topi[:, j]
        hh = torch.einsum("th,tnh->tn", x2, gate_up[e])
        gg, uu = hh.chunk(2, -1)
        out = out + topv[:, j:j + 1] * torch.einsum("ti,thi->th", F.silu(gg) * uu, down[e])
    return out.view(x.shape)


def _close(got, want, msg=None):
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5 * max(1.0, float(want.abs().max())), msg=msg)


def _oracle(w, x, y):
    """Per-sample gradients of the dense replicated model, one sample at a time."""
    per = []
    for i in range(x.shape[0]):
        p = {n: t.clone().requires_grad_() for n, t in w.items()}
        hid = F.linear(x[i:i + 1], p["fc_w"], p["fc_b"])
        out = F.linear(_dense_moe(hid, p["gate_up"], p["down"], p["router"]), p["head_w"]).sum((1, 2))
        ((out - y[i:i + 1]) ** 2).sum().backward()
        per.append({n: t.grad.clone() for n, t in p.items()})
    return per


class _Net(nn.Module):
    def __init__(self, w):
        from dattri_llm_b200.parallel.moe import ExpertParallelMoE

        super().__init__()
        self.fc_in = nn.Linear(D_IN, H)
        self.moe = ExpertParallelMoE(H, INTER, E, K, max_tokens=64, device=torch.device("cpu"),
                                     dtype=torch.float32)
        self.head = nn.Linear(H, 1, bias=False)
        with torch.no_grad():
            self.fc_in.weight.copy_(w["fc_w"])
            self.fc_in.bias.copy_(w["fc_b"])
            self.head.weight.copy_(w["head_w"])
        self.moe.load_experts(w["gate_up"], w["down"], w["router"])

    def forward(self, x):
        return self.head(self.moe(self.fc_in(x))).sum((1, 2))


def _check(rank: int) -> None:
    import dattri_llm_b200 as bw
    from dattri_llm_b200.gradient.callbacks import CaptureCallback

    w = _weights()
    x, y = _data(rank)
    model = _Net(w)
    # plain forward / backward against the dense model
    xr = x.clone().requires_grad_()
    out = model(xr)
    ((out - y) ** 2).sum().backward()
    p = {n: t.clone().requires_grad_() for n, t in w.items()}
    xd = x.clone().requires_grad_()
    want = F.linear(_dense_moe(F.linear(xd, p["fc_w"], p["fc_b"]), p["gate_up"], p["down"], p["router"]),
                    p["head_w"]).sum((1, 2))
    ((want - y) ** 2).sum().backward()
    torch.testing.assert_close(out, want.detach(), rtol=1e-5, atol=1e-5)
    _close(xr.grad, xd.grad)
    _close(model.moe.gate.weight.grad, p["router"].grad)
    model.zero_grad()

    # per-sample capture through the expert taps
    cap = CaptureCallback()
    hm = bw.HookManager(model, bw.HookManagerConfig(), callbacks=[cap])
    with hm.collect():
        ((model(x) - y) ** 2).sum().backward()
    hm.remove()
    grad = cap.record.gradient.materialize()
    per = _oracle(w, x, y)
    names = set(grad.data)
    for e in range(E):
        for proj, key in (("gate_up", "gate_up"), ("down", "down")):
            name = f"moe.experts.dattri_experts.{e}.{proj}"
            want_e = torch.stack([s[key][e].reshape(-1) for s in per])
            if name not in names:  # no token of this rank's batch was routed to e
                assert float(want_e.abs().max()) == 0.0, name
                continue
            _close(grad.data[name].reshape(B, -1), want_e, msg=name)
    assert any(n.startswith("moe.experts.dattri_experts.") for n in names)
    assert "moe.gate" not in names  # the router weight is captured once, through its tap
    router = torch.stack([s["router"].reshape(-1) for s in per])
    _close(grad.data["moe.gate.dattri_router"].reshape(B, -1), router)
    fc = torch.stack([torch.cat([s["fc_w"], s["fc_b"][:, None]], 1).reshape(-1) for s in per])
    _close(grad.data["fc_in"].reshape(B, -1), fc)


def _olmoe():
    import transformers

    cfg = transformers.OlmoeConfig(vocab_size=64, hidden_size=32, intermediate_size=16, num_hidden_layers=1,
                                   num_attention_heads=4, num_key_value_heads=4, num_experts=4,
                                   num_experts_per_tok=2, max_position_embeddings=64)
    torch.manual_seed(0)
    return transformers.OlmoeForCausalLM(cfg).eval()


def _lm_capture(model, ids, cfg, **kw):
    import dattri_llm_b200 as bw

    cap = bw.CaptureCallback()
    hm = bw.HookManager(model, cfg, callbacks=[cap], **kw)
    with hm.collect():
        logits = model(input_ids=ids).logits
        F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1),
                        reduction="sum").backward()
    hm.remove()
    model.zero_grad(set_to_none=True)
    return cap.record.gradient.materialize()


def _check_olmoe(rank: int) -> None:
    import copy

    import dattri_llm_b200 as bw
    from dattri_llm_b200.parallel.moe import ExpertParallelMoE, expert_parallelize

    model = _olmoe()
    ep_model = copy.deepcopy(model)
    assert expert_parallelize(ep_model, max_tokens=64, device=torch.device("cpu")) == ["model.layers.0.mlp"]
    assert isinstance(ep_model.model.layers[0].mlp, ExpertParallelMoE)
    ids = torch.randint(0, 64, (3, 8), generator=torch.Generator().manual_seed(7 + rank))
    for proj in (None, {"__default__": {"style": "logra", "proj_dim": 4}}):
        cfg = bw.HookManagerConfig(linear_io=[r"mlp"], projection_kwargs=proj)
        want = _lm_capture(model, ids, cfg, moe_routed_layers=["model.layers.0.mlp"])
        got = _lm_capture(ep_model, ids, cfg)
        assert set(got.data) == set(want.data), (sorted(got.data), sorted(want.data))
        assert any(".experts.dattri_experts." in n for n in got.data)
        for n, v in want.data.items():
            _close(got.data[n].reshape(v.shape[0], -1), v.reshape(v.shape[0], -1), msg=n)


class _SeqNet(_Net):
    def forward(self, x, y=None):
        return super().forward(x)


def _ep_scores(fsdp: str = ""):
    """TracIn scores of a model with an expert-parallel layer through the public API
    (the streamer wraps it for data parallelism when a process group is up)."""
    import tempfile

    import dattri_llm_b200 as bw

    g = torch.Generator().manual_seed(5)
    xtr, ytr = torch.randn(8, T, D_IN, generator=g), torch.randn(8, generator=g)
    xte, yte = torch.randn(3, T, D_IN, generator=g), torch.randn(3, generator=g)
    model = _SeqNet(_weights())

    def loss(m, batch):
        return ((m(x=batch["x"], y=batch["y"]) - batch["y"]) ** 2).sum()

    args = bw.AttributionArguments(output_dir=tempfile.mkdtemp(), per_device_train_batch_size=2,
                                   per_device_eval_batch_size=3, fsdp=fsdp)
    att = bw.TracInAttributor(args, task=bw.AttributionTask(loss, model))
    ds = [{"x": xtr[i], "y": ytr[i]} for i in range(8)]
    ts = [{"x": xte[i], "y": yte[i]} for i in range(3)]
    score = att.attribute(ds, ts, hook_config=bw.HookManagerConfig())
    return {h: score.trajectory_agnostic(h) for h in score.train_ids}


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        _check(rank)
        _check_olmoe(rank)
        out[f"scores{rank}"] = _ep_scores()
        out[f"fsdp{rank}"] = _ep_scores("full_shard")
        out[rank] = "ok"
    except Exception as e:  # surfaced in the parent
        import traceback

        out[rank] = traceback.format_exc() + repr(e)
    finally:
        dist.destroy_process_group()


def test_single_process():
    _check(0)


def test_olmoe_converted_matches_replicated_capture():
    _check_olmoe(0)


def test_two_ranks_gloo():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    assert res[0] == "ok" and res[1] == "ok", res
    want = _ep_scores()
    for key in ("scores", "fsdp"):  # DDP, then FSDP full shard
        merged = {**res[f"{key}0"], **res[f"{key}1"]}
        assert set(merged) == set(want)
        for h, row in want.items():
            _close(merged[h], row, msg=key)


def test_taps_are_not_hooked_outside_capture():
    from dattri_llm_b200.parallel.moe import ExpertTap

    model = _Net(_weights())
    assert not model.moe.capturing()
    tap = model.moe.dattri_experts[0]["gate_up"]
    assert isinstance(tap, ExpertTap) and tap.out_features == 2 * INTER
    assert not any(True for _ in tap.parameters())


def _collect_olmoe(model, batches, path, **kw):
    import dattri_llm_b200 as bw

    store = bw.GradientStorageManager(str(path))
    hm = bw.HookManager(model, bw.HookManagerConfig(linear_io=[r"mlp"]),
                        callbacks=[bw.OffloadCallback(offload_interval=1, file_manager=store)], **kw)
    for ids in batches:
        with hm.collect():
            logits = model(input_ids=ids).logits
            F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1),
                            reduction="sum").backward()
        model.zero_grad(set_to_none=True)
    hm.remove()
    store.close()
    return str(path)


def test_kfac_and_tracin_from_expert_parallel_stores(tmp_path):
    """K-FAC (zero rows of tokens not routed to an expert dropped from its covariances) and
    TracIn scored from stores captured under expert parallelism equal the scores from
    replicated-expert stores of the same model and data."""
    import copy

    import dattri_llm_b200 as bw
    from dattri_llm_b200.parallel.moe import expert_parallelize

    model = _olmoe()
    ep_model = copy.deepcopy(model)
    expert_parallelize(ep_model, max_tokens=64, device=torch.device("cpu"))
    g = torch.Generator().manual_seed(9)
    train = [torch.randint(0, 64, (3, 8), generator=g) for _ in range(2)]
    test = [torch.randint(0, 64, (2, 8), generator=g)]
    moe = {"moe_routed_layers": ["model.layers.0.mlp"]}
    rep = (_collect_olmoe(model, train, tmp_path / "rtr", **moe), _collect_olmoe(model, test, tmp_path / "rte", **moe))
    ep = (_collect_olmoe(ep_model, train, tmp_path / "etr"), _collect_olmoe(ep_model, test, tmp_path / "ete"))
    args = bw.AttributionArguments(output_dir=str(tmp_path / "o"), use_cpu=True)
    for cls, kw in ((bw.TracInAttributor, {}), (bw.KFACAttributor, {"damping": 0.1})):
        want = cls(args).attribute_from_cache(*rep, **kw)
        got = cls(args).attribute_from_cache(*ep, **kw)
        assert got.row_train_ids == want.row_train_ids
        _close(got.scores, want.scores, msg=cls.__name__)
