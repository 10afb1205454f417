"""Per-sample update directions (``gradient.ops.optimizer.precondition``) against real
``torch.optim`` steps: after a few warm-up steps build the optimizer state, the direction
predicted from the pre-step state must equal ``-(theta_after - theta_before) / lr`` of the
optimizer's next step on that gradient."""

from __future__ import annotations

import copy

import pytest
import torch

from dattri_llm_b200.gradient.ops.optimizer import OPTIMIZER_STATE_KEYS, precondition

LR = 0.05
K = 24

CASES = [
    ("SGD", lambda p: torch.optim.SGD([p], lr=LR), {}),
    ("SGD", lambda p: torch.optim.SGD([p], lr=LR, momentum=0.9), {"momentum": 0.9}),
    ("SGD", lambda p: torch.optim.SGD([p], lr=LR, momentum=0.8, nesterov=True), {"momentum": 0.8, "nesterov": True}),
    ("SGD", lambda p: torch.optim.SGD([p], lr=LR, momentum=0.7, dampening=0.3),
     {"momentum": 0.7, "dampening": 0.3}),
    ("Adam", lambda p: torch.optim.Adam([p], lr=LR), {}),
    ("Adam", lambda p: torch.optim.Adam([p], lr=LR, betas=(0.8, 0.95), eps=1e-6), {"betas": (0.8, 0.95), "eps": 1e-6}),
    ("Adam", lambda p: torch.optim.Adam([p], lr=LR, amsgrad=True), {"amsgrad": True}),
    ("AdamW", lambda p: torch.optim.AdamW([p], lr=LR, weight_decay=0.0), {}),
    ("Adamax", lambda p: torch.optim.Adamax([p], lr=LR), {}),
    ("NAdam", lambda p: torch.optim.NAdam([p], lr=LR), {}),
    ("RAdam", lambda p: torch.optim.RAdam([p], lr=LR), {}),
    ("RMSprop", lambda p: torch.optim.RMSprop([p], lr=LR), {}),
    ("RMSprop", lambda p: torch.optim.RMSprop([p], lr=LR, centered=True), {"centered": True}),
    ("RMSprop", lambda p: torch.optim.RMSprop([p], lr=LR, momentum=0.5), {"momentum": 0.5}),
    ("Adagrad", lambda p: torch.optim.Adagrad([p], lr=LR), {}),
    ("Adagrad", lambda p: torch.optim.Adagrad([p], lr=LR, lr_decay=0.1), {"lr_decay": 0.1}),
    ("Adadelta", lambda p: torch.optim.Adadelta([p], lr=LR), {}),
]


def _state_view(opt_type: str, state: dict) -> dict:
    out = {}
    for key in OPTIMIZER_STATE_KEYS[opt_type]:
        if key in state:
            v = state[key]
            out[key] = v.clone() if isinstance(v, torch.Tensor) else v
    return out


@pytest.mark.parametrize("warmup", [0, 1, 7])
@pytest.mark.parametrize(("name", "make", "hp"), CASES, ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_direction_matches_a_real_optimizer_step(name, make, hp, warmup):
    torch.manual_seed(11)
    p = torch.nn.Parameter(torch.randn(K, dtype=torch.float64))
    opt = make(p)
    for _ in range(warmup):
        p.grad = torch.randn(K, dtype=torch.float64)
        opt.step()
    before = p.detach().clone()
    state = copy.deepcopy(opt.state[p]) if p in opt.state else {}
    step = int(state["step"]) + 1 if "step" in state else 1
    g = torch.randn(K, dtype=torch.float64)
    p.grad = g.clone()
    opt.step()
    taken = -(p.detach() - before) / LR
    got = precondition(g[None].float(), _state_view(name, state), optimizer_type=name, step=step, **hp)[0]
    torch.testing.assert_close(got.double(), taken, rtol=2e-4, atol=2e-5)


def test_rows_are_independent_samples():
    torch.manual_seed(0)
    state = {"exp_avg": 0.1 * torch.randn(K), "exp_avg_sq": 0.01 * torch.rand(K)}
    g = torch.randn(5, K)
    batch = precondition(g, state, optimizer_type="Adam", step=4)
    rows = torch.stack([precondition(g[i : i + 1], state, optimizer_type="Adam", step=4)[0] for i in range(5)])
    torch.testing.assert_close(batch, rows)


def test_lion_is_a_sign_direction():
    torch.manual_seed(1)
    g = torch.randn(3, K)
    state = {"exp_avg": torch.randn(K)}
    d = precondition(g, state, optimizer_type="Lion", step=2)
    want = torch.sign(0.9 * state["exp_avg"] + 0.1 * g)
    torch.testing.assert_close(d, want)


def test_unknown_optimizer_and_bad_step_raise():
    g = torch.randn(2, K)
    with pytest.raises(NotImplementedError):
        precondition(g, {}, optimizer_type="LBFGS", step=1)
    with pytest.raises(ValueError):
        precondition(g, {}, optimizer_type="Adam", step=0)
