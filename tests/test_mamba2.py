"""The library's SSD forward for Hugging Face Mamba2 equals the model's own (naive) path:
logits and every parameter gradient, fp32 on CPU, with a sequence that is not a multiple
of the chunk length and grouped B/C."""

from __future__ import annotations

import copy
import warnings

import pytest
import torch

transformers = pytest.importorskip("transformers")

from dattri_llm_b200.models.mamba2 import accelerate_mamba2, ssd_chunked  # noqa: E402


def _model():
    cfg = transformers.Mamba2Config(vocab_size=64, hidden_size=64, num_hidden_layers=2, expand=2, state_size=16,
                                    head_dim=16, num_heads=8, n_groups=2, chunk_size=16)
    torch.manual_seed(0)
    return transformers.Mamba2ForCausalLM(cfg).float()


def test_ssd_forward_matches_the_library_model():
    warnings.filterwarnings("ignore")
    theirs = _model()
    ours = copy.deepcopy(theirs)
    assert accelerate_mamba2(ours, linears=False) == 2
    ids = torch.randint(0, 64, (3, 40), generator=torch.Generator().manual_seed(1))
    want, got = theirs(input_ids=ids).logits, ours(input_ids=ids).logits
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)
    want.pow(2).mean().backward()
    got.pow(2).mean().backward()
    for (name, p_ref), p_ours in zip(theirs.named_parameters(), ours.parameters(), strict=True):
        torch.testing.assert_close(p_ours.grad, p_ref.grad, rtol=1e-4, atol=1e-6, msg=name)


def test_ssd_chunked_matches_the_recurrence():
    g = torch.Generator().manual_seed(2)
    b, l, h, p, n = 2, 21, 3, 4, 5
    x, bb, cc = torch.randn(b, l, h, p, generator=g), torch.randn(b, l, h, n, generator=g), torch.randn(b, l, h, n,
                                                                                                          generator=g)
    dt = torch.rand(b, l, h, generator=g) * 0.5
    a = -torch.rand(h, generator=g) - 0.1
    state = torch.zeros(b, h, p, n)
    want = []
    for t in range(l):
        state = torch.exp(dt[:, t, :, None, None] * a[None, :, None, None]) * state \
            + dt[:, t, :, None, None] * x[:, t, :, :, None] * bb[:, t, :, None, :]
        want.append(torch.einsum("bhpn,bhn->bhp", state, cc[:, t]))
    torch.testing.assert_close(ssd_chunked(x, dt, a, bb, cc, chunk=8), torch.stack(want, 1), rtol=1e-4, atol=1e-5)
