"""The block as one autograd node (``ops.BlockFunction``) and its two native
helpers: ``llattn_colsum`` (bias gradients) and ``llattn_pool_bwd`` with
LLATTN_POOL_ACCUMULATE.

The fused node must give what autograd over the separate layers gives (the
module's per-layer path, taken when profiling is on): same output, same
gradients up to the rounding of the fused accumulation, and both within the
parity tolerance of the CPU oracle.
"""

from __future__ import annotations

import pytest
import torch

import llattn_b200
import llattn_oracle as O
from parity import TOL, make_cfg, model_config, oracle_block, rel_err

pytestmark = pytest.mark.gpu

CASES = {
    "tokenwise": dict(B=2, T=300, d_model=256, n_heads=2, local_window=64, local_block_size=128,
                      latent_tokens=16, latent_d_model=64, latent_heads=2, latent_query_block_size=0),
    "qblocks": dict(B=2, T=257, d_model=256, n_heads=4, local_window=32, local_block_size=64,
                    latent_tokens=12, latent_d_model=64, latent_heads=4, latent_query_block_size=16),
}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("shape", [(1, 1), (7, 3), (1000, 64), (4096, 4608), (333, 1537)])
def test_colsum_matches_torch_sum(shape, dtype):
    from llattn_b200 import ops

    g = torch.randn(*shape, generator=torch.Generator().manual_seed(3)).to(device="cuda", dtype=dtype)
    got = ops.colsum(g)
    want = g.double().sum(0)
    assert got.dtype == dtype and got.shape == (shape[1],)
    assert rel_err(got, want) < (1e-6 if dtype == torch.float32 else 8e-3)
    assert torch.equal(ops.colsum(g), got)  # fixed summation order


@pytest.mark.parametrize("mode", ["chunks", "qblocks"])
def test_pool_bwd_accumulate(mode):
    from llattn_b200 import _lib, ops

    B, T, d, Nl, qb = 2, 37, 64, 5, 8
    m = _lib.POOL_CHUNKS if mode == "chunks" else _lib.POOL_QBLOCKS
    rows = ops.geometry(T, Nl, qb if mode == "qblocks" else 0)["n_chunks" if mode == "chunks" else "n_qrows"]
    gen = torch.Generator().manual_seed(5)
    dp = torch.randn(B, rows, d, generator=gen, device="cpu").cuda()
    dx0 = torch.randn(B, T, d, generator=gen, device="cpu").cuda()
    want = dx0 + ops.pool_bwd(dp, T, Nl, qb if mode == "qblocks" else 0, m)
    got = dx0.clone()
    ops.pool_bwd_accumulate_(got, dp, Nl, qb if mode == "qblocks" else 0, m)
    assert torch.allclose(got, want, rtol=0, atol=1e-6)


def _run(m, x, gy):
    x = x.clone().requires_grad_(True)
    m.zero_grad(set_to_none=True)
    y = m(x)
    y.backward(gy)
    return y.detach(), x.grad, {k: p.grad.detach().clone() for k, p in m.named_parameters()}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", sorted(CASES))
def test_block_function_matches_per_layer_autograd(case, dtype):
    import llattn_b200

    B, T, cfg = make_cfg(CASES[case])
    params = O.init_params(cfg, 0)
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg))
    m.load_state_dict(params)
    m = m.to(device="cuda", dtype=dtype)
    gen = torch.Generator().manual_seed(2)
    x = torch.randn(B, T, cfg.d_model, generator=gen).to(device="cuda", dtype=dtype)
    gy = torch.randn(B, T, cfg.d_model, generator=gen).to(device="cuda", dtype=dtype)
    fused = _run(m, x, gy)
    m.set_profile(True)  # per-layer path
    layered = _run(m, x, gy)
    m.set_profile(False)
    # the fused node pools the projected rows (llattn_pool_proj), the layers
    # project the pooled rows: equal up to rounding
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel_err(fused[0], layered[0]) < tol, "y"
    assert rel_err(fused[1], layered[1]) < tol, "dx"
    for k in fused[2]:
        assert rel_err(fused[2][k], layered[2][k]) < tol, k
    # and the fused gradients against the oracle
    y_ref, dx_ref, g_ref = oracle_block(params, x.float().cpu(), gy.float().cpu(), cfg)
    assert rel_err(fused[0], y_ref) < TOL[dtype]
    assert rel_err(fused[1], dx_ref) < TOL[dtype]
    for k in fused[2]:
        assert rel_err(fused[2][k], g_ref[k]) < TOL[dtype], k


def test_block_function_under_autocast_matches_per_layer():
    """fp32 parameters under bf16 autocast (the LM's training setup): the
    fused node on cast inputs/weights against autocast over the layers."""
    import llattn_b200

    B, T, cfg = make_cfg(CASES["tokenwise"])
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg))
    m.load_state_dict(O.init_params(cfg, 0))
    m = m.cuda()
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(B, T, cfg.d_model, generator=gen).cuda()
    gy = torch.randn(B, T, cfg.d_model, generator=gen).cuda()

    def run():
        xx = x.clone().requires_grad_(True)
        m.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(xx)
        y.float().backward(gy)
        return y.detach(), xx.grad, {k: p.grad.detach().clone() for k, p in m.named_parameters()}

    fused = run()
    m.set_profile(True)
    layered = run()
    m.set_profile(False)
    assert fused[0].dtype == layered[0].dtype == torch.bfloat16
    assert rel_err(fused[0], layered[0]) < 1e-2
    assert fused[1].dtype == torch.float32 and rel_err(fused[1], layered[1]) < 1e-2
    for k in fused[2]:
        assert fused[2][k].dtype == torch.float32
        assert rel_err(fused[2][k], layered[2][k]) < 1e-2, k


def test_block_under_torch_compile_matches_eager():
    """torch.compile over the drop-in block (aot_eager: FakeTensor tracing of
    the custom ops, their register_fake / register_autograd entries and the
    autograd graph, with the library kernels as the executed ops) gives the
    eager outputs and gradients."""
    B, T, cfg = make_cfg(CASES["tokenwise"])
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg))
    m.load_state_dict(O.init_params(cfg, 0))
    m = m.cuda().to(torch.bfloat16)
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(B, T, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()
    gy = torch.randn(B, T, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()

    def run(fn):
        xx = x.clone().requires_grad_(True)
        m.zero_grad(set_to_none=True)
        y = fn(xx)
        y.backward(gy)
        return y.detach(), xx.grad, {k: p.grad.detach().clone() for k, p in m.named_parameters()}

    eager = run(m)
    compiled = run(torch.compile(m, backend="aot_eager", fullgraph=True))
    assert torch.equal(eager[0], compiled[0])
    assert torch.equal(eager[1], compiled[1])
    for k in eager[2]:
        assert torch.equal(eager[2][k], compiled[2][k]), k


@pytest.mark.parametrize("bias", [0.0, 8.0, -8.0])
def test_profile_stats_gate_mean(bias):
    """Profile mode fills the reference's keys; gate_mean is the mean local
    gate weight (models.py:450), near 1 / 0 when the gate bias saturates it."""
    B, T, cfg = make_cfg(CASES["tokenwise"])
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg)).cuda().to(torch.bfloat16)
    m.gate_bias = bias
    m.set_profile(True)
    x = torch.randn(B, T, cfg.d_model, device="cuda", dtype=torch.bfloat16)
    m(x)
    st = m.get_profile_stats()
    m.set_profile(False)
    assert st["profile_local_latent_total_ms"] > 0 and 0.0 < st["profile_gate_mean"] < 1.0
    if bias > 0:
        assert st["profile_gate_mean"] > 0.99
    elif bias < 0:
        assert st["profile_gate_mean"] < 0.01
