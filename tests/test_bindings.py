"""Every native entry point the package calls exists in the built extension (CPU check)."""

import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1] / "dattri_llm_b200"


def _called_names() -> set[str]:
    pat = re.compile(r"(?:native\(\)|\bnat)\.(\w+)\(")
    names = set()
    for path in ROOT.rglob("*.py"):
        names.update(pat.findall(path.read_text()))
    return names


def test_native_entry_points_are_registered():
    try:
        import dattri_llm_b200._C as ext
    except ImportError as e:  # extension not built in this checkout
        pytest.skip(f"extension not built: {e}")
    missing = sorted(n for n in _called_names() if not hasattr(ext, n))
    assert not missing, f"called from Python but not registered in the extension: {missing}"
