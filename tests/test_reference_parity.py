"""Parity with the reference implementation (skipped when it is not installed under
``baseline/_ref``): the gradient-cache format in both directions, sample hashing, and
TracIn / K-FAC scores on the same captures."""

from __future__ import annotations

import os
import sys
import warnings

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
if not os.path.isdir(os.path.join(REF, "dattri_llm")):
    pytest.skip("reference not installed under baseline/_ref", allow_module_level=True)
if REF not in sys.path:
    sys.path.append(REF)

import dattri_llm as R  # noqa: E402

import dattri_llm_b200 as O  # noqa: E402
from tests import tiny  # noqa: E402

warnings.filterwarnings("ignore", category=UserWarning)


def _records(lib, seed: int):
    g = torch.Generator().manual_seed(seed)
    fac = lib.Factorized(torch.randn(3, 4, 5, generator=g), torch.randn(3, 4, 6, generator=g))
    data = {"a": torch.randn(3, 10, generator=g), "b": fac}
    grad = lib.Gradient({"a": "materialized", "b": "factorized"}, data, {"a": "nn.Linear", "b": "nn.Linear"},
                        {"a": "batch", "b": "batch_token"})
    return [lib.GradientRecord(7, [f"h{seed}_{i}" for i in range(3)], grad)]


def _load(lib, path, step):
    store = lib.GradientStorageManager(str(path))
    out = []
    for f, by in store.iter_steps(step):
        recs = store.load_records(f)
        out.extend(recs[i] for i in by[step])
    return out


@pytest.mark.parametrize(("writer", "reader"), [(R, O), (O, R)])
def test_store_format_is_shared(tmp_path, writer, reader):
    src = _records(writer, 1)
    store = writer.GradientStorageManager(str(tmp_path / "s"))
    store.save_bulk(src)
    store.close()
    (got,) = _load(reader, tmp_path / "s", 7)
    assert got.input_hash == src[0].input_hash
    torch.testing.assert_close(got.gradient.data["a"], src[0].gradient.data["a"])
    fb, sb = got.gradient.data["b"], src[0].gradient.data["b"]
    torch.testing.assert_close(fb.activation, sb.activation)
    torch.testing.assert_close(fb.pre_activation_grad, sb.pre_activation_grad)


def test_hash_sample_matches():
    from dattri_llm.utils.hashing import hash_sample as ref_hash

    from dattri_llm_b200.utils.hashing import hash_sample

    g = torch.Generator().manual_seed(3)
    samples = [{"input_ids": torch.randint(0, 100, (12,), generator=g)},
               {"input_ids": torch.randint(0, 100, (9,), generator=g), "attention_mask": torch.tensor([1] * 6 + [0] * 3)},
               {"x": torch.randn(4, generator=g), "y": torch.randn(2, generator=g)}]
    for s in samples:
        assert hash_sample(s) == ref_hash(s)


@pytest.mark.parametrize("algo", ["TracInAttributor", "KFACAttributor"])
def test_scores_match_reference(tmp_path, algo):
    model = tiny.make_model()
    xtr, ytr, xte, yte = tiny.make_data()
    sd = tiny.checkpoints(model, 1)
    tiny.collect_to_disk(model, sd, xtr, ytr, tmp_path / "tr")
    tiny.collect_to_disk(model, sd, xte, yte, tmp_path / "te")
    out = {}
    for name, lib in (("ref", R), ("ours", O)):
        args = lib.AttributionArguments(output_dir=str(tmp_path / name), use_cpu=True)
        kw = {"damping": 0.1} if algo == "KFACAttributor" else {}
        res = getattr(lib, algo)(args).attribute_from_cache(str(tmp_path / "tr"), str(tmp_path / "te"), **kw)
        out[name] = res.query(tiny.hashes(xtr, ytr), tiny.hashes(xte, yte), trajectory="agnostic")
    torch.testing.assert_close(out["ours"], out["ref"], rtol=1e-4, atol=1e-5)
