"""Routed-expert capture under DDP (two gloo ranks on CPU): OLMoE's fused experts are
captured per expert and regrouped per sample on each rank, through the DDP wrapper, and
every rank's per-sample router and expert gradients equal the single-sample autograd
oracle on that rank's batch."""

from __future__ import annotations

import datetime
import os
import socket
import warnings

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

transformers = pytest.importorskip("transformers")
E = 4


def _model():
    cfg = transformers.OlmoeConfig(vocab_size=64, hidden_size=32, intermediate_size=16, num_hidden_layers=1,
                                   num_attention_heads=4, num_key_value_heads=4, num_experts=E,
                                   num_experts_per_tok=2, max_position_embeddings=64)
    torch.manual_seed(0)
    return transformers.OlmoeForCausalLM(cfg).eval()


def _loss(model, ids):
    logits = model(input_ids=ids).logits
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1),
                           reduction="sum")


def _ids(rank):
    return torch.randint(0, 64, (3, 8), generator=torch.Generator().manual_seed(20 + rank))


def _oracle(ids):
    model = _model()
    mlp = model.model.layers[0].mlp
    out = {"router": []} | {f"gu{e}": [] for e in range(E)} | {f"dn{e}": [] for e in range(E)}
    for i in range(ids.shape[0]):
        model.zero_grad(set_to_none=True)
        _loss(model, ids[i : i + 1]).backward()
        out["router"].append(mlp.gate.weight.grad.clone())
        for e in range(E):
            out[f"gu{e}"].append(mlp.experts.gate_up_proj.grad[e].clone())
            out[f"dn{e}"].append(mlp.experts.down_proj.grad[e].clone())
    return {k: torch.stack(v).reshape(ids.shape[0], -1) for k, v in out.items()}


def _worker(rank, world, port, out):
    warnings.filterwarnings("ignore")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import dattri_llm_b200 as bw
        from dattri_llm_b200.gradient import ops

        model = _model()
        wrapped = torch.nn.parallel.DistributedDataParallel(model, find_unused_parameters=True)
        cap = bw.CaptureCallback()
        hm = bw.HookManager(wrapped, bw.HookManagerConfig(linear_io=[r"mlp"]), callbacks=[cap],
                            moe_routed_layers=["model.layers.0.mlp"])
        with hm.collect():
            _loss(wrapped, _ids(rank)).backward()
        hm.remove()
        g = cap.record.gradient
        names = {"router": "model.layers.0.mlp.gate.dattri_router"}
        for e in range(E):
            names[f"gu{e}"] = f"model.layers.0.mlp.experts.dattri_experts.{e}.gate_up"
            names[f"dn{e}"] = f"model.layers.0.mlp.experts.dattri_experts.{e}.down"
        out[rank] = {k: ops.materialize(g.data[n], g.layer_types[n]).reshape(3, -1).clone() for k, n in names.items()}
    except Exception as e:  # surfaced in the parent
        out[rank] = repr(e)
    finally:
        dist.destroy_process_group()


def test_routed_expert_capture_under_ddp():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    for rank in range(2):
        got = res[rank]
        assert not isinstance(got, str), got
        want = _oracle(_ids(rank))
        for k, w in want.items():
            scale = float(w.abs().max()) or 1.0
            torch.testing.assert_close(got[k], w, rtol=1e-3, atol=1e-4 * scale, msg=f"rank {rank} {k}")
