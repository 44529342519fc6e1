"""llattn_pool_proj_fwd / _bwd (the pooling fused with rkv_proj / rq_proj by
linearity) against the oracle's pooling of x followed by the projections
(models.py:159-230, :333-347), and its gradient against autograd through the
oracle's pooling of z. Ragged chunks, ragged query blocks, token-wise
queries, a latent width that is not a multiple of the vector width.

Tolerances: max|a-b|/max|b| <= 1e-5 in float32 (float64 oracle), 1e-2 in
bfloat16 (the rounding of z's rows and of the outputs)."""

import pytest
import torch

import llattn_oracle as O

pytestmark = pytest.mark.gpu

CASES = [  # B, T, latent_tokens, query_block, latent_heads, latent_head_dim
    (2, 2048, 64, 0, 2, 32),
    (2, 1000, 64, 0, 2, 32),     # ragged last chunk
    (1, 777, 48, 128, 2, 32),    # ragged chunk and query block
    (2, 512, 64, 64, 4, 16),
    (1, 300, 7, 0, 1, 64),
    (2, 96, 5, 3, 2, 3),         # Ld = 6: scalar path
    (1, 40, 64, 100, 1, 8),      # query block > T, more latents than tokens
]


def _reference(x, w_rkv, b_rkv, w_rq, b_rq, T, latent_tokens, query_block):
    cs, nc = O.chunk_layout(T, latent_tokens)
    gkv = O.pool_chunks(x, cs) @ w_rkv.t() + b_rkv
    if query_block > 1:
        bs, _ = O.query_block_layout(T, query_block)
        qsrc = O.pool_query_blocks(x, bs, O.chunk_ids(T, cs, nc))[0]
    else:
        qsrc = x
    return gkv, qsrc @ w_rq.t() + b_rq


def _rel(a, b):
    return ((a.double().cpu() - b.double().cpu()).abs().max() / b.double().abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
def test_pool_proj_fwd(case, dtype):
    from llattn_b200 import ops

    B, T, Nl, QB, Lh, ldh = case
    Ld, d = Lh * ldh, 64
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(B, T, d, generator=gen, dtype=torch.float64)
    w_rkv = torch.randn(2 * Ld, d, generator=gen, dtype=torch.float64) / d ** 0.5
    w_rq = torch.randn(Ld, d, generator=gen, dtype=torch.float64) / d ** 0.5
    b_rkv = torch.randn(2 * Ld, generator=gen, dtype=torch.float64)
    b_rq = torch.randn(Ld, generator=gen, dtype=torch.float64)
    rnd = lambda t: t.to(dtype).double()  # noqa: E731
    x, w_rkv, w_rq, b_rkv, b_rq = map(rnd, (x, w_rkv, w_rq, b_rkv, b_rq))
    gkv_ref, rq_ref = _reference(x, w_rkv, b_rkv, w_rq, b_rq, T, Nl, QB)
    dev = lambda t: t.to("cuda", dtype).contiguous()  # noqa: E731
    z = dev(x).view(B * T, d) @ dev(torch.cat([w_rkv, w_rq])).t()
    gkv, rq = ops.pool_proj_fwd(z, dev(b_rkv), dev(b_rq), B, Lh, Nl, QB)
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert gkv.shape == gkv_ref.shape and rq.shape == rq_ref.shape
    assert _rel(gkv, gkv_ref) <= tol
    assert _rel(rq, rq_ref) <= tol
    # no biases
    gkv0, rq0 = ops.pool_proj_fwd(z, None, None, B, Lh, Nl, QB)
    assert _rel(gkv0, gkv_ref - b_rkv) <= 2 * tol
    assert _rel(rq0, rq_ref - b_rq) <= 2 * tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
def test_pool_proj_bwd(case, dtype):
    from llattn_b200 import ops

    B, T, Nl, QB, Lh, ldh = case
    Ld = Lh * ldh
    cs, nc = O.chunk_layout(T, Nl)
    gen = torch.Generator().manual_seed(11)
    z = torch.randn(B, T, 3 * Ld, generator=gen, dtype=torch.float64, requires_grad=True)
    gkv = O.pool_chunks(z[..., :2 * Ld], cs)
    if QB > 1:
        bs, _ = O.query_block_layout(T, QB)
        rq = O.pool_query_blocks(z[..., 2 * Ld:], bs, O.chunk_ids(T, cs, nc))[0]
    else:
        rq = z[..., 2 * Ld:]
    dgkv = torch.randn(gkv.shape, generator=gen, dtype=torch.float64).to(dtype).double()
    drq = torch.randn(rq.shape, generator=gen, dtype=torch.float64).to(dtype).double()
    torch.autograd.backward([gkv, rq], [dgkv, drq])
    dz = ops.pool_proj_bwd(dgkv.to("cuda", dtype), drq.to("cuda", dtype), T, Lh, Nl, QB)
    torch.cuda.synchronize()
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert dz.shape == (B * T, 3 * Ld)
    assert _rel(dz, z.grad.view(B * T, 3 * Ld)) <= tol


def test_pool_proj_rejects_bad_args():
    import ctypes

    from llattn_b200 import _lib

    L = _lib.lib()
    dims = _lib.make_dims(1, 64, latent_heads=2, latent_head_dim=32, latent_tokens=8, dtype=_lib.F32)
    buf = torch.empty(64 * 192, device="cuda")
    p = ctypes.c_void_p(buf.data_ptr())
    assert L.llattn_pool_proj_fwd(ctypes.byref(dims), p, 100, None, None, p, p, None) == 1  # ldz < 3 Ld
    assert L.llattn_pool_proj_fwd(ctypes.byref(dims), None, 192, None, None, p, p, None) == 1
    assert L.llattn_pool_proj_bwd(ctypes.byref(dims), p, p, p, 191, None) == 1
    wide = _lib.make_dims(1, 64, latent_heads=4, latent_head_dim=64, latent_tokens=8, dtype=_lib.F32)
    assert L.llattn_pool_proj_fwd(ctypes.byref(wide), p, 768, None, None, p, p, None) == 1  # Ld 256 > 128
