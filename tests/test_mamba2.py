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


@pytest.mark.parametrize("recompute", [False, True])
def test_ssd_forward_matches_the_library_model(recompute, monkeypatch):
    from dattri_llm_b200.models import mamba2 as m2

    monkeypatch.setattr(m2, "_RECOMPUTE_TOKENS", 0 if recompute else 1 << 30)
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


def test_capture_overrides_keep_the_installed_forward():
    """A capture manager wraps the mixers while it collects; removing it must put back the
    library's SSD forward, not the model class's naive one, and the forward it wraps while
    collecting must be the SSD one too."""
    import dattri_llm_b200 as bw
    from dattri_llm_b200.models import mamba2 as m2

    warnings.filterwarnings("ignore")
    model = _model()
    accelerate_mamba2(model, linears=False)
    mixers = [m for m in model.modules() if isinstance(m, transformers.models.mamba2.modeling_mamba2.Mamba2Mixer)]
    ids = torch.randint(0, 64, (2, 16), generator=torch.Generator().manual_seed(3))
    calls = {"n": 0}
    real = m2.ssd_chunked

    def counting(*args, **kwargs):
        calls["n"] += 1
        return real(*args, **kwargs)

    m2.ssd_chunked = counting
    try:
        for _ in range(2):  # the second manager wraps what the first one's removal left
            hm = bw.HookManager(model, bw.HookManagerConfig(linear_io=[r"mixer\.(in_proj|out_proj)$"]),
                                callbacks=[bw.CaptureCallback()])
            with hm.collect():
                model(input_ids=ids).logits.float().pow(2).sum().backward()
            hm.remove()
            assert all(m.forward.__func__ is m2._mixer_forward for m in mixers)
    finally:
        m2.ssd_chunked = real
    assert calls["n"] >= 2 * len(mixers)  # every mixer's forward ran the SSD scan, in both passes
