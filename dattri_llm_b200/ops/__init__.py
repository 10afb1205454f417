"""Native sm_100a kernels and their Python entry points.

The compiled extension ``dattri_llm_b200._C`` is built in place
(``python setup.py build_ext --inplace``).  Every op here runs only on CUDA
tensors; on a CUDA device a missing extension raises instead of silently falling
back, so a GPU run always exercises the native path.  CPU tensors are handled one
level up, by the PyTorch reference implementations in
:mod:`dattri_llm_b200.gradient.ops`.

Kernels report a bounded-wait timeout through a per-device int32 error word;
:func:`check_device_errors` raises if any launch since the last check set it.
"""

from __future__ import annotations

import importlib
import threading

import torch

from dattri_llm_b200.ops import checks as _checks

_C = None
_IMPORT_ERROR: Exception | None = None
_LAUNCHES = [0]


def count_launch(n: int = 1) -> None:
    """Record *n* native kernel launches (every entry point of this package calls it)."""
    _LAUNCHES[0] += n


def launch_count() -> int:
    """Native kernels launched by this process so far."""
    return _LAUNCHES[0]


_lock = threading.Lock()
_err_words: dict[int, torch.Tensor] = {}
_checked = None


def native():
    """The compiled extension module; raises with the build command if absent.

    With launch checks on (:func:`dattri_llm_b200.ops.checks.set_checks` or
    ``DATTRI_B200_CHECKS=1``) the module comes wrapped so that the index arguments of
    data-dependent launches are validated first.
    """
    global _checked
    mod = _C if _C is not None else _load()
    if not _checks.checks_enabled():
        return mod
    if _checked is None or _checked._module is not mod:
        _checked = _checks.CheckedNative(mod)
    return _checked


def _load():
    global _C, _IMPORT_ERROR
    if _C is not None:
        return _C
    with _lock:
        if _C is None:
            try:
                _C = importlib.import_module("dattri_llm_b200._C")
            except ImportError as exc:  # pragma: no cover - depends on the build
                _IMPORT_ERROR = exc
                raise RuntimeError(
                    "dattri_llm_b200._C is not built; run "
                    "`python setup.py build_ext --inplace` at the repository root "
                    f"({exc})",
                ) from exc
    return _C


def available() -> bool:
    """``True`` when the extension imports (it is built for sm_100a only)."""
    try:
        native()
    except RuntimeError:
        return False
    return True


def use_native(*tensors: torch.Tensor) -> bool:
    """Whether an op on *tensors* runs the native kernels.

    ``True`` for CUDA tensors on an sm_100 device.  A CUDA tensor on a box
    without the extension raises (the native path is mandatory on the GPU).
    """
    if not tensors or not all(t.is_cuda for t in tensors):
        return False
    dev = tensors[0].device
    major, _ = torch.cuda.get_device_capability(dev)
    if major != 10:
        return False
    native()
    return True


def error_word(device: torch.device | int) -> torch.Tensor:
    """The device's int32 kernel error word (zero = no error)."""
    idx = torch.device(device).index if not isinstance(device, int) else device
    if idx is None:
        idx = torch.cuda.current_device()
    w = _err_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _err_words[idx] = w
    return w


_ERR_NAMES = {
    1: "a tensor-core stage never arrived (TMA wait timed out)",
    2: "a pipeline stage never drained (MMA wait timed out)",
    3: "the accumulator never completed",
    4: "a peer GPU flag never arrived",
    5: "a kernel rejected its arguments",
    6: "a peer-staged tile never became ready",
}


def check_device_errors(device: torch.device | int | None = None) -> None:
    """Raise if a native kernel on *device* (default: every used device) timed out."""
    words = (
        _err_words.items()
        if device is None
        else [(torch.device(device).index, error_word(device))]
    )
    for idx, w in list(words):
        code = int(w.item())
        if code:
            w.zero_()
            raise RuntimeError(
                f"native kernel on cuda:{idx} reported error {code}: "
                f"{_ERR_NAMES.get(code, 'unknown')}",
            )


from dattri_llm_b200.ops.gemm import (  # noqa: E402
    STORE_ATOMIC_F32,
    STORE_BF16,
    STORE_BF16_T,
    STORE_F32,
    STORE_SQ_SUM_F32,
    gemm_grouped,
    gemm_tn,
    gemm_tn_seg,
    matmul_f32,
    matmul_tn,
    transpose_last2,
)
from dattri_llm_b200.ops.gram import (  # noqa: E402
    ghost_dot,
    ghost_gram,
    ghost_gram_tokens,
    mask_gather,
    per_sample_outer,
)
from dattri_llm_b200.ops.norm import embedding_dense_grad, norm_per_sample_grad  # noqa: E402
from dattri_llm_b200.ops.optim import adam_direction  # noqa: E402
from dattri_llm_b200.ops.projection import projection_matrix_t  # noqa: E402

__all__ = [
    "STORE_ATOMIC_F32",
    "STORE_BF16",
    "STORE_BF16_T",
    "STORE_SQ_SUM_F32",
    "STORE_F32",
    "adam_direction",
    "available",
    "check_device_errors",
    "count_launch",
    "error_word",
    "gemm_grouped",
    "gemm_tn",
    "gemm_tn_seg",
    "launch_count",
    "ghost_dot",
    "ghost_gram",
    "ghost_gram_tokens",
    "mask_gather",
    "matmul_f32",
    "transpose_last2",
    "matmul_tn",
    "native",
    "embedding_dense_grad",
    "norm_per_sample_grad",
    "per_sample_outer",
    "projection_matrix_t",
    "use_native",
]
