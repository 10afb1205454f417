"""Shared fixtures for the CPU tests: a bias-free two-layer MLP on single-token
inputs, so each per-sample weight gradient of a linear layer is exactly the
rank-1 outer product ``g a^T`` -- which makes brute-force oracles transparent."""

from __future__ import annotations

from pathlib import Path

import torch
from torch import nn

from dattri_llm_b200.gradient.callbacks import OffloadCallback
from dattri_llm_b200.gradient.hooks import HookManager, HookManagerConfig
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.utils.hashing import hash_sample

IN, HID, OUT = 5, 7, 3
N_TRAIN, N_TEST = 8, 4
LAYERS = ["mlp.fc1", "mlp.fc2"]
WEIGHTS = ["mlp.fc1.weight", "mlp.fc2.weight"]


class MLP(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.mlp = nn.Sequential()
        self.mlp.add_module("fc1", nn.Linear(IN, HID, bias=False))
        self.mlp.add_module("act", nn.Tanh())
        self.mlp.add_module("fc2", nn.Linear(HID, OUT, bias=False))

    def forward(self, x: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
        return self.mlp(x)


def make_model(seed: int = 0) -> MLP:
    torch.manual_seed(seed)
    return MLP().eval()


def make_data(seed: int = 0, n_train: int = N_TRAIN, n_test: int = N_TEST):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n_train, IN, generator=g), torch.randn(n_train, OUT, generator=g),
            torch.randn(n_test, IN, generator=g), torch.randn(n_test, OUT, generator=g))


def as_dataset(x: torch.Tensor, y: torch.Tensor) -> list[dict]:
    return [{"x": x[i], "y": y[i]} for i in range(x.shape[0])]


def hashes(x: torch.Tensor, y: torch.Tensor) -> list[str]:
    return [hash_sample({"x": x[i], "y": y[i]}) for i in range(x.shape[0])]


def sq_loss(model, batch) -> torch.Tensor:
    """Sum over the batch of the squared error (each sample's loss is independent).  The
    model receives both fields, so the manager's hash of its inputs covers ``{x, y}``."""
    return ((model(x=batch["x"], y=batch["y"]) - batch["y"]) ** 2).sum()


def per_sample_grads(model: nn.Module, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """``(n, p)``: each sample's flattened gradient over :data:`WEIGHTS` (autograd, one by one)."""
    params = [dict(model.named_parameters())[n] for n in WEIGHTS]
    rows = []
    for i in range(x.shape[0]):
        loss = ((model(x=x[i:i + 1]) - y[i:i + 1]) ** 2).sum()
        gs = torch.autograd.grad(loss, params)
        rows.append(torch.cat([g.reshape(-1) for g in gs]))
    return torch.stack(rows)


def factors(model: nn.Module, x: torch.Tensor, y: torch.Tensor) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """``{layer: (a, g)}``: each layer's inputs and output gradients, per sample."""
    acts: dict[str, torch.Tensor] = {}
    outs: dict[str, torch.Tensor] = {}
    mods = {"mlp.fc1": model.mlp.fc1, "mlp.fc2": model.mlp.fc2}
    hs = []

    def keep(name):
        def hook(_m, inputs, out):
            acts[name] = inputs[0].detach()
            out.retain_grad()
            outs[name] = out
        return hook

    for n, m in mods.items():
        hs.append(m.register_forward_hook(keep(n)))
    try:
        loss = ((model(x=x) - y) ** 2).sum()
        loss.backward()
    finally:
        for h in hs:
            h.remove()
        model.zero_grad(set_to_none=True)
    return {n: (acts[n], outs[n].grad.detach()) for n in mods}


def collect_to_disk(model: nn.Module, state_dicts: list[dict], x: torch.Tensor, y: torch.Tensor, out_dir: Path,
                    *, config: HookManagerConfig | None = None, batch_size: int | None = None) -> None:
    """One step per state dict: forward/backward of (x, y) with per-sample records on disk."""
    store = GradientStorageManager(str(out_dir))
    off = OffloadCallback(offload_interval=1, file_manager=store, recording_type="per_sample")
    hm = HookManager(model, config=config or HookManagerConfig(linear_io=[r"mlp\."]), callbacks=[off])
    bs = batch_size or x.shape[0]
    with hm.collect():
        for sd in state_dicts:
            model.load_state_dict(sd)
            for s in range(0, x.shape[0], bs):
                model.zero_grad(set_to_none=True)
                hm.set_sample_ids(hashes(x[s:s + bs], y[s:s + bs]))
                sq_loss(model, {"x": x[s:s + bs], "y": y[s:s + bs]}).backward()
    hm.remove()
    model.zero_grad(set_to_none=True)


def checkpoints(model: nn.Module, n: int = 2, seed: int = 1) -> list[dict]:
    sd0 = {k: v.detach().clone() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(seed)
    out = [sd0]
    for _ in range(n - 1):
        out.append({k: v + 0.1 * torch.randn(v.shape, generator=g) for k, v in sd0.items()})
    return out
