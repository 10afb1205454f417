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


@pytest.mark.parametrize(("b1", "s1", "b2", "s2", "k", "d"),
                         [(2, 64, 3, 64, 64, 64), (3, 50, 5, 17, 72, 40), (4, 1, 6, 1, 128, 64),
                          (2, 300, 2, 200, 256, 128), (1, 7, 300, 3, 16, 24), (8, 512, 32, 512, 64, 64),
                          (5, 700, 9, 333, 128, 128)])
def test_ghost_gram_matches_dense_oracle(b1, s1, b2, s2, k, d):
    a1 = torch.randn(b1, s1, k, device="cuda").bfloat16()
    g1 = torch.randn(b1, s1, d, device="cuda").bfloat16()
    a2 = torch.randn(b2, s2, k, device="cuda").bfloat16()
    g2 = torch.randn(b2, s2, d, device="cuda").bfloat16()
    got = ops.ghost_gram(a1, g1, a2, g2)
    ops.check_device_errors(a1.device)
    m1 = torch.einsum("bsk,bsd->bdk", a1.double(), g1.double()).flatten(1)
    m2 = torch.einsum("bsk,bsd->bdk", a2.double(), g2.double()).flatten(1)
    ref = (m1 @ m2.T).float()
    torch.testing.assert_close(got, ref, rtol=2e-3, atol=2e-3 * ref.abs().max().item())


def test_per_sample_outer_matches_bmm():
    left = torch.randn(3, 100, 64, device="cuda").bfloat16()
    right = torch.randn(3, 100, 48, device="cuda").bfloat16()
    got = ops.per_sample_outer(left, right)
    ref = torch.bmm(left.double().transpose(1, 2), right.double()).float()
    torch.testing.assert_close(got, ref, rtol=1e-3, atol=1e-2)


def test_gemm_tn_seg_layout():
    b, t, d, k = 3, 96, 256, 64
    x = torch.randn(b * t, d, device="cuda").bfloat16()
    p = torch.randn(k, d, device="cuda").bfloat16()
    out = ops.gemm_tn_seg(x, p, t)
    assert out.shape == (b, k, t) and out.is_contiguous()
    want = (x.float() @ p.float().T).view(b, t, k).transpose(1, 2)
    torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-1)
    ops.check_device_errors()


@pytest.mark.parametrize("shared_b", [False, True])
@pytest.mark.parametrize("mode", ["bf16", "f32"])
def test_gemm_grouped_matches_per_job(shared_b, mode):
    jobs, z, m, n, kk = 5, 4, 64, 48, 320
    a = [torch.randn(z, m, kk, device="cuda").bfloat16() for _ in range(jobs)]
    b = [torch.randn(n, kk, device="cuda").bfloat16() if shared_b else torch.randn(z, n, kk, device="cuda").bfloat16()
         for _ in range(jobs)]
    dt = torch.bfloat16 if mode == "bf16" else torch.float32
    out = torch.full((jobs, z, m, n), float("nan"), device="cuda", dtype=dt)
    store = ops.STORE_BF16 if mode == "bf16" else ops.STORE_F32
    for _ in range(2):  # the second call reuses the uploaded job table
        ops.gemm_grouped(a, b, list(out.unbind(0)), mode=store)
        for i in range(jobs):
            bi = b[i].float() if b[i].dim() == 3 else b[i].float().expand(z, n, kk)
            want = a[i].float() @ bi.transpose(1, 2)
            torch.testing.assert_close(out[i].float(), want, rtol=2e-2, atol=2e-1)
    ops.check_device_errors()


@pytest.mark.parametrize("mode", ["f32", "f32acc", "bf16", "bf16t", "seg"])
@pytest.mark.parametrize(("m", "n", "k"), [(8192, 64, 2048), (1000, 32, 1032), (4096, 128, 640)])
def test_skinny_cluster_split_k(mode, m, n, k):
    """Few output tiles and a long K take the 2-CTA cluster split-K path (DSMEM reduction)."""
    a = torch.randn(m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    want = a.float() @ b.float().T
    if mode == "seg":
        t = 8 if m % 8 == 0 else 1
        out = ops.gemm_tn_seg(a, b, t).float()
        got = out.transpose(1, 2).reshape(m, n)
    elif mode in ("f32", "f32acc"):
        out = torch.ones(m, n, device="cuda") if mode == "f32acc" else torch.empty(m, n, device="cuda")
        ops.gemm_tn(a, b, out, mode=ops.STORE_F32, accumulate=mode == "f32acc")
        got = out - 1 if mode == "f32acc" else out
    elif mode == "bf16":
        out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        got = ops.gemm_tn(a, b, out, mode=ops.STORE_BF16).float()
    else:
        out = torch.empty(n, m, device="cuda", dtype=torch.bfloat16)
        got = ops.gemm_tn(a, b, out, mode=ops.STORE_BF16_T).float().T
    tol = 2e-2 if mode in ("bf16", "bf16t", "seg") else 1e-3
    torch.testing.assert_close(got, want, rtol=tol, atol=tol * float(want.abs().max()))
    ops.check_device_errors()


@pytest.mark.parametrize("checked", [False, True])
@pytest.mark.parametrize("scatter", [False, True])
def test_gemm_ragged_expert_segments(scatter, checked, monkeypatch):
    """Ragged grouped GEMM over expert row segments (empty and partial-tile segments
    included), stored in place or scattered to rows of several destination buffers; with
    launch checks on, the validator accepts these tables and metadata."""
    from dattri_llm_b200.ops import checks

    monkeypatch.setattr(checks, "_enabled", checked)
    lens = [0, 130, 7, 256, 0, 61]
    n, kk = 192, 320
    rows = sum(lens)
    a = torch.randn(rows, kk, device="cuda").bfloat16()
    b3 = torch.randn(len(lens), n, kk, device="cuda").bfloat16()
    n_i = torch.tensor(lens, dtype=torch.int32, device="cuda")
    base = (torch.cumsum(n_i, 0) - n_i).int()
    prefix = torch.zeros(len(lens) + 1, dtype=torch.int32, device="cuda")
    prefix[1:] = torch.cumsum((n_i + 255) // 256, 0)  # 256-row blocks
    max_tiles = rows // 256 + len(lens) + 2  # an upper bound: the kernel reads the real count
    want = torch.empty(rows, n, device="cuda")
    start = 0
    for j, ln in enumerate(lens):
        want[start:start + ln] = a[start:start + ln].float() @ b3[j].float().T
        start += ln
    err = ops.error_word(torch.device("cuda", torch.cuda.current_device()))
    if not scatter:
        out = torch.full((rows, n), float("nan"), device="cuda", dtype=torch.bfloat16)
        ops.native().gemm_ragged(a, b3, out, prefix, base.contiguous(), n_i, max_tiles, [], None, err)
        got = out.float()
    else:
        dests = [torch.full((rows, n), float("nan"), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
        g = torch.Generator(device="cuda").manual_seed(3)
        owner = torch.randint(0, 3, (rows,), device="cuda", generator=g)
        slot = torch.randperm(rows, device="cuda", generator=g)
        meta = torch.stack([owner, slot], 1).int().contiguous()
        ops.native().gemm_ragged(a, b3, None, prefix, base.contiguous(), n_i, max_tiles, dests, meta, err)
        got = torch.stack([dests[int(o)][int(s)] for o, s in meta.tolist()]).float()
    torch.testing.assert_close(got, want, rtol=2e-2, atol=2e-1)
    ops.check_device_errors()


def test_gemm_reduce_scatter_slots_emulated():
    """GEMM -> reduce-scatter with three ranks emulated on one GPU: every "rank" stores its
    product into the owners' slots, then every owner sums its slots into its shard."""
    world, m, n, k = 3, 200, 136, 384
    elems = m * n
    per4 = -(-elems // 4 // world)
    slot = 4 * per4
    bufs = [torch.full((world * slot,), float("nan"), device="cuda") for _ in range(world)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    a = [torch.randn(m, k, device="cuda").bfloat16() for _ in range(world)]
    b = [torch.randn(n, k, device="cuda").bfloat16() for _ in range(world)]
    err = ops.error_word(torch.device("cuda", torch.cuda.current_device()))
    for s in range(world):
        ops.native().gemm_tn_rs(a[s], b[s], ptrs, world, per4, m, n, n, 0.5, err, s)
    want = sum(a[s].float() @ b[s].float().T for s in range(world)).reshape(-1) * 0.5
    got = torch.empty(world * slot, device="cuda")
    for r in range(world):
        got[r * slot:(r + 1) * slot] = 1.0
        ops.native().slot_reduce(bufs[r], world, slot, got[r * slot:], min(slot, elems - r * slot) // 4 * 4, True)
    torch.testing.assert_close(got[:elems] - 1.0, want, rtol=1e-3, atol=1e-2)
    ops.check_device_errors()


@pytest.mark.parametrize("mode", ["f32", "f32acc", "bf16", "bf16t", "atomic"])
@pytest.mark.parametrize(("z", "m", "n", "k"), [(1, 8192, 2048, 512), (1, 8000, 1000, 328), (3, 4096, 640, 256),
                                                 (1, 1000, 33000, 1024)])
def test_persistent_gemm_many_tiles(mode, z, m, n, k):
    """More than one wave of output tiles takes the persistent kernel (two TMEM accumulators,
    epilogue overlapped with the next tile's MMAs); partial row / column tiles included.  The
    last shape's B (66 MB) outgrows half the L2 while A does not: row-block-fastest order."""
    a = torch.randn(z, m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    want = a.float() @ b.float().T
    if mode in ("f32", "f32acc", "atomic"):
        out = torch.ones(z, m, n, device="cuda") if mode != "f32" else torch.empty(z, m, n, device="cuda")
        store = ops.STORE_ATOMIC_F32 if mode == "atomic" else ops.STORE_F32
        ops.gemm_tn(a, b, out, mode=store, accumulate=mode == "f32acc")
        got = out - 1 if mode != "f32" else out
    elif mode == "bf16":
        out = torch.empty(z, m, n, device="cuda", dtype=torch.bfloat16)
        got = ops.gemm_tn(a, b, out, mode=ops.STORE_BF16).float()
    else:
        out = torch.empty(z, n, m, device="cuda", dtype=torch.bfloat16)
        got = ops.gemm_tn(a, b, out, mode=ops.STORE_BF16_T).float().transpose(1, 2)
    tol = 2e-2 if mode in ("bf16", "bf16t") else 1e-3
    torch.testing.assert_close(got, want, rtol=tol, atol=tol * float(want.abs().max()))
    ops.check_device_errors()


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize(("world", "self_rank", "m", "n", "k"), [(4, 1, 1000, 1024, 512), (2, 0, 640, 384, 384),
                                                                 (3, 2, 512, 384, 192)])
def test_staged_allgather_gemm_emulated(mode, world, self_rank, m, n, k):
    """All-gather fused into the GEMM, ranks emulated by separate allocations on one GPU:
    mode 0 shards B's rows, mode 1 its K columns; the launch copies the other ranks'
    shards into the staging matrix while its own-shard tiles start."""
    a = torch.randn(m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    if mode == 0:
        shards = [s.contiguous() for s in b.chunk(world, 0)]
    else:
        shards = [s.contiguous() for s in b.chunk(world, 1)]
    if any(s.shape != shards[0].shape for s in shards):
        pytest.skip("uneven shards")
    stage = torch.empty(n, k, device="cuda", dtype=torch.bfloat16)
    flags = torch.zeros(world, dtype=torch.int32, device="cuda")
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    err = ops.error_word(torch.device("cuda", torch.cuda.current_device()))
    want = a.float() @ b.float().T
    for epoch in (1, 2):  # the flags keep counting across launches
        out.fill_(float("nan"))
        ops.native().gemm_tn_staged(a, shards, stage, out, flags, epoch, mode, self_rank, ops.STORE_BF16, 1.0, err)
        torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-2 * float(want.abs().max()))
    ops.check_device_errors()


@pytest.mark.parametrize(("b1", "s1", "b2", "s2", "e", "vocab"), [(3, 100, 5, 37, 64, 50), (8, 256, 4, 256, 200, 1000)])
def test_embedding_token_gram_matches_dense(b1, s1, b2, s2, e, vocab):
    """Embedding cross-gram: gradient Gram masked by token equality, per sample pair and per
    side-1 token, against the fp32 one-hot formula."""
    from dattri_llm_b200.gradient.ops.dot import _embedding_gram

    tok1 = torch.randint(0, vocab, (b1, s1), device="cuda")
    tok2 = torch.randint(0, vocab, (b2, s2), device="cuda")
    g1 = torch.randn(b1, s1, e, device="cuda").bfloat16()
    g2 = torch.randn(b2, s2, e, device="cuda").bfloat16()
    match = (tok1.reshape(-1, 1) == tok2.reshape(1, -1)).float()
    prod = (g1.float().reshape(-1, e) @ g2.float().reshape(-1, e).T) * match
    want_tok = prod.view(b1, s1, b2, s2).sum(3)
    got = ops.ghost_gram_tokens(tok1, g1, tok2, g2)
    torch.testing.assert_close(got, want_tok.sum(1), rtol=1e-3, atol=1e-2)
    got_tok = _embedding_gram(tok1, g1, tok2, g2, per_token=True).float()
    torch.testing.assert_close(got_tok, want_tok, rtol=2e-2, atol=2e-1)
    ops.check_device_errors()


@pytest.mark.parametrize(("b", "s", "k", "d"), [(6, 100, 64, 96), (4, 300, 128, 64)])
def test_fused_per_sample_dot_and_norm(b, s, k, d):
    """Per-sample <dW1_i, dW2_i> and ||dW_i||^2 from factors: the diagonal sample blocks of
    the fused ghost gram only (linear and embedding layers) against fp32 materialized grads."""
    from dattri_llm_b200.gradient.ops.dot import dot_factors, grad_norm_sq_factors

    a1, g1 = torch.randn(b, s, k, device="cuda").bfloat16(), torch.randn(b, s, d, device="cuda").bfloat16()
    a2, g2 = torch.randn(b, s, k, device="cuda").bfloat16(), torch.randn(b, s, d, device="cuda").bfloat16()
    w1 = torch.einsum("btd,btk->bdk", g1.float(), a1.float())
    w2 = torch.einsum("btd,btk->bdk", g2.float(), a2.float())
    want_dot = (w1 * w2).sum((1, 2))
    want_norm = (w1 * w1).sum((1, 2))
    got_dot = ops.ghost_dot(a1, g1, a2, g2)
    torch.testing.assert_close(got_dot, want_dot, rtol=1e-2, atol=1e-2 * float(want_norm.max()))
    got_norm = grad_norm_sq_factors(a1, g1, "nn.Linear", include_bias=False, mode="factorized").float()
    torch.testing.assert_close(got_norm, want_norm, rtol=2e-2, atol=0)
    tok = torch.randint(0, 40, (b, s), device="cuda")
    onehot = torch.nn.functional.one_hot(tok, 40).float()
    we = torch.einsum("btd,btv->bvd", g1.float(), onehot)
    got_emb = grad_norm_sq_factors(tok, g1, "nn.Embedding", include_bias=False).float()
    torch.testing.assert_close(got_emb, (we * we).sum((1, 2)), rtol=2e-2, atol=0)
    got_emb_dot = dot_factors(tok, g1, tok, g2, "nn.Embedding", include_bias=False).float()
    we2 = torch.einsum("btd,btv->bvd", g2.float(), onehot)
    torch.testing.assert_close(got_emb_dot, (we * we2).sum((1, 2)), rtol=2e-2,
                               atol=2e-2 * float((we * we).sum((1, 2)).max()))
    ops.check_device_errors()


def test_ekfac_lambda_fused_rotate_square_reduce():
    """EK-FAC eigenvalue accumulation: rotate the factors into the eigenbasis, form every
    sample's rotated gradient and square-sum it into lambda inside one batched GEMM's
    epilogue; against fp32 materialized U_G^T dW U_A."""
    from dattri_llm_b200.gradient.gradient import Factorized
    from dattri_llm_b200.gradient.ops.kronecker import ekfac_lambda_accumulate

    b, t, k, d = 6, 200, 96, 64
    a = torch.randn(b, t, k, device="cuda").bfloat16()
    g = torch.randn(b, t, d, device="cuda").bfloat16()
    u_a = torch.linalg.qr(torch.randn(k, k, device="cuda"))[0]
    u_g = torch.linalg.qr(torch.randn(d, d, device="cuda"))[0]
    f = Factorized(activation=a, pre_activation_grad=g, module_kwargs=None)
    lam, n = ekfac_lambda_accumulate(f, "nn.Linear", u_a, u_g, None)
    lam, n2 = ekfac_lambda_accumulate(f, "nn.Linear", u_a, u_g, lam)  # accumulates
    dw = torch.einsum("btd,btk->bdk", g.float(), a.float())
    m = u_g.T @ dw @ u_a
    want = 2 * (m * m).sum(0).reshape(-1)
    assert n == n2 == b
    torch.testing.assert_close(lam, want, rtol=3e-2, atol=3e-2 * float(want.mean()))
    ops.check_device_errors()


@pytest.mark.parametrize(("b", "t", "kr", "kc", "m"), [(3, 300, 64, 96, 1000), (2, 1024, 2048, 512, 4096)])
def test_mask_gather_matches_materialized(b, t, kr, kc, m):
    """Mask projection: fixed coordinates of every per-sample gradient R_b^T C_b gathered
    from shared-memory token tiles, against the fp32 materialized gradient."""
    r = torch.randn(b, t, kr, device="cuda").bfloat16()
    c = torch.randn(b, t, kc, device="cuda").bfloat16()
    rows = torch.randint(0, kr, (m,), device="cuda")
    cols = torch.randint(0, kc, (m,), device="cuda")
    dense = torch.einsum("btr,btc->brc", r.float(), c.float())
    want = dense[:, rows, cols]
    got = ops.mask_gather(r, c, rows, cols)
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-2)
    ops.check_device_errors()


@pytest.mark.parametrize(("b1", "t", "b2", "t2", "k", "d"), [(3, 50, 5, 37, 64, 64), (2, 200, 7, 64, 40, 24)])
def test_per_token_cross_gram_on_tensor_cores(b1, t, b2, t2, k, d):
    """Per-token cross-gram (factorized and dense side 2) against an fp32 einsum."""
    from dattri_llm_b200.gradient.ops.dot import cross_gram_per_token, cross_gram_per_token_dense

    g = torch.Generator(device="cuda").manual_seed(5)
    a1, g1 = (torch.randn(b1, t, n, device="cuda", generator=g).bfloat16() for n in (k, d))
    a2, g2 = (torch.randn(b2, t2, n, device="cuda", generator=g).bfloat16() for n in (k, d))
    m2 = torch.einsum("csd,csk->cdk", g2.float(), a2.float())
    want = torch.einsum("btk,btd,cdk->btc", a1.float(), g1.float(), m2)
    scale = float(want.abs().max())
    got = cross_gram_per_token(a1, g1, a2, g2, "nn.Linear").float()
    torch.testing.assert_close(got, want, rtol=3e-2, atol=2e-2 * scale)
    got_dense = cross_gram_per_token_dense(a1, g1, m2.bfloat16().reshape(b2, -1), "nn.Linear").float()
    torch.testing.assert_close(got_dense, want, rtol=3e-2, atol=2e-2 * scale)
    ops.check_device_errors()
