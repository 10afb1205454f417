"""The no-allocation C entry point against the PyTorch entry point of the same GEMM.

Named to be collected last: it must pass alone and after every other test, i.e.
whatever earlier tests left in the device's state.  The entry point is reached
through its exported C symbol (ctypes on the extension's shared object), the way a
caller without PyTorch would reach it.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from dattri_llm_b200 import ops

    lib = ctypes.CDLL(ops.native().__file__)
    fn = lib.dattri_b200_gemm_bf16_splitk_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_float, ctypes.c_int,
                   ctypes.c_void_p]
    lib.dattri_b200_noalloc_status.restype = ctypes.c_int
    lib.dattri_b200_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    lib.dattri_b200_noalloc_max_output.restype = ctypes.c_longlong
    return lib


def _call(lib, a, b, c, splits, alpha=1.0):
    m, k = a.shape
    n = b.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return lib.dattri_b200_gemm_bf16_splitk_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, a.stride(0),
                                                   b.stride(0), c.stride(0), alpha, splits, stream)


def _existing(a, b, alpha=1.0):
    """The PyTorch entry point of the same tcgen05 GEMM, bf16 store."""
    from dattri_llm_b200 import ops

    out = torch.empty(a.shape[0], b.shape[0], dtype=torch.bfloat16, device=a.device)
    ops.gemm_tn(a, b, out, alpha=alpha, mode=ops.STORE_BF16)
    return out


# Shapes reach every kernel the entry point can launch: per-tile split-K (splits >= 2),
# the CTA-pair kernel (splits 1, N > 128), the persistent kernel (splits 1, N <= 128 and
# more tiles than SMs) and a K shorter than one 64-wide block (splits clamped to 1).
@pytest.mark.parametrize(("m", "n", "k", "splits"), [(256, 128, 4096, 8), (200, 72, 1000, 3), (1024, 2048, 512, 2),
                                                     (1024, 1024, 512, 1), (19200, 96, 64, 1), (300, 200, 48, 4)])
def test_two_consecutive_calls_match_existing_entry_point(m, n, k, splits):
    lib = _lib()
    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    for call in range(2):  # the second call checks that the scratch was cleared in between
        a = torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
        b = torch.randn(n, k, device="cuda", generator=gen).to(torch.bfloat16)
        c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
        assert _call(lib, a, b, c, splits, alpha=0.5) == 0
        status = ctypes.c_int(-1)
        stream = torch.cuda.current_stream().cuda_stream
        assert lib.dattri_b200_noalloc_status(ctypes.byref(status), stream) == 0
        assert status.value == 0, f"device error word {status.value} on call {call}"
        want = _existing(a, b, alpha=0.5)
        exact = 0.5 * (a.float() @ b.float().T)
        # Both round an fp32 sum to bf16 once; summation order differs, so allow one bf16 ulp.
        torch.testing.assert_close(c.float(), want.float(), rtol=1.6e-2, atol=1e-2)
        torch.testing.assert_close(c.float(), exact, rtol=1.6e-2, atol=1e-2)


def test_rejects_oversize_and_bad_arguments():
    lib = _lib()
    cap = lib.dattri_b200_noalloc_max_output()
    assert cap == 1 << 21
    a = torch.zeros(4096, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(1024, 64, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(4096, 1024, device="cuda", dtype=torch.bfloat16)  # 4 Mi outputs > cap
    assert _call(lib, a, b, c, 1) != 0
    odd = torch.zeros(8, 60, device="cuda", dtype=torch.bfloat16)  # K not a multiple of 8
    assert _call(lib, odd, odd, torch.zeros(8, 8, device="cuda", dtype=torch.bfloat16), 1) != 0
