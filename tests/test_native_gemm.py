"""tcgen05 GEMM and device projection generator vs fp32 PyTorch references."""

import pytest
import torch

from dattri_llm_b200 import ops
from dattri_llm_b200.utils.rng import counter_projection_matrix

pytestmark = pytest.mark.gpu


def _ref(a, b, alpha=1.0):
    return alpha * (a.float() @ b.float().transpose(-1, -2))


@pytest.mark.parametrize(
    ("m", "n", "k"),
    [(128, 64, 64), (1, 16, 64), (100, 100, 200), (300, 256, 2048), (8192, 64, 2048),
     (77, 1000, 136), (1024, 8, 4096)],
)
def test_gemm_f32_matches_torch(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    b = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    out = torch.empty(m, n, device="cuda")
    ops.gemm_tn(a, b, out, alpha=0.5)
    ops.check_device_errors(a.device)
    torch.testing.assert_close(out, _ref(a, b, 0.5), rtol=1e-3, atol=1e-3 * k ** 0.5)


def test_gemm_batched_bf16_and_transposed():
    z, m, n, k = 5, 64, 64, 1024
    a = torch.randn(z, m, k, device="cuda").bfloat16()
    b = torch.randn(z, n, k, device="cuda").bfloat16()
    out = torch.empty(z, m, n, device="cuda", dtype=torch.bfloat16)
    ops.gemm_tn(a, b, out, mode=ops.STORE_BF16)
    torch.testing.assert_close(out.float(), _ref(a, b), rtol=2e-2, atol=0.3)
    out_t = torch.empty(z, n, m, device="cuda", dtype=torch.bfloat16)
    ops.gemm_tn(a, b, out_t, mode=ops.STORE_BF16_T)
    torch.testing.assert_close(out_t.float(), _ref(a, b).transpose(1, 2), rtol=2e-2, atol=0.3)
    ops.check_device_errors(a.device)


def test_gemm_shared_b_and_split_k():
    z, m, n, k = 3, 200, 48, 8192
    a = torch.randn(z, m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    out = torch.zeros(z, m, n, device="cuda")
    ops.gemm_tn(a, b, out, mode=ops.STORE_ATOMIC_F32, splits=7)
    torch.testing.assert_close(out, _ref(a, b), rtol=1e-3, atol=1e-2 * k ** 0.5)
    got = ops.matmul_tn(a[0], b)
    torch.testing.assert_close(got, _ref(a[0], b), rtol=1e-3, atol=1e-2 * k ** 0.5)
    ops.check_device_errors(a.device)


@pytest.mark.parametrize("kind", ["rademacher", "normal"])
def test_device_projection_matches_host_generator(kind):
    d, k = 1000, 64
    dev = ops.projection_matrix_t(d, k, 3, kind=kind, dtype=torch.float32)
    host = counter_projection_matrix(d, k, 3, kind=kind)
    torch.testing.assert_close(dev.cpu(), host.t(), rtol=1e-6, atol=1e-6)
