"""The tensor-core latent kernels for more than 64 chunks (up to 512) against
the SIMT kernels of the same math and against the oracle, bf16, through the
C ABI (torch op -> llattn_fwd / llattn_bwd). Latent attention is
models.py:361-375: row r sees chunks j < qid(r); rows that see none give 0.
After every tensor-core launch the device fault word must be 0."""

import math
import os

import pytest
import torch

import llattn_oracle as O
from parity import TOL, frob_err, rel_err

pytestmark = pytest.mark.gpu

# B, T, latent_tokens, ldh, Lh, query block (0 = token-wise)
CASES = [
    (1, 1000, 100, 32, 2, 0),      # 100 chunks of 10
    (2, 2048, 128, 64, 1, 0),      # two full key tiles
    (1, 4100, 256, 32, 2, 0),      # ragged last chunk
    (1, 700, 512, 48, 2, 0),       # 350 chunks of 2, ldh 48 as a 64-wide tile
    (1, 8192, 512, 32, 2, 0),      # the cfg5 latent size
    (1, 8192, 512, 64, 2, 64),     # block-pooled queries
    (2, 16384, 256, 32, 2, 64),    # cfg3's latent branch
    (1, 1300, 65, 32, 3, 7),       # one chunk past a tile, odd query blocks
]


def _fault():
    from llattn_b200 import _lib
    return _lib.lib().llattn_fault_status(1)


def _inputs(B, T, Nl, ldh, Lh, QB, H=1, hd=64, seed=0):
    gen = torch.Generator().manual_seed(seed)
    d, Ld = H * hd, Lh * ldh
    cs, nc = O.chunk_layout(T, Nl)
    tq = math.ceil(T / min(T, QB)) if QB > 1 else T
    f = lambda *s: torch.randn(*s, generator=gen)
    return dict(qkv=f(B, T, 3 * d), rq=f(B, tq, Ld), gkv=f(B, nc, 2 * Ld), w=f(d, Ld) / math.sqrt(Ld),
                b=f(d) * 0.1, gl=f(hd) / math.sqrt(hd), gr=f(hd) / math.sqrt(hd))


def _run(inp, Lh, Nl, QB, force_simt, H=1, W=64, LBS=256, backward=False, seed=5):
    import llattn_b200  # noqa: F401  (registers the ops)

    os.environ["LLATTN_FORCE_SIMT"] = "1" if force_simt else "0"
    try:
        dev = {k: v.cuda().to(torch.bfloat16 if k in ("qkv", "rq", "gkv", "w") else torch.float32)
               for k, v in inp.items()}
        outs = torch.ops.llattn_b200.attn_fwd(dev["qkv"], dev["rq"], dev["gkv"], dev["w"], dev["b"],
                                              dev["gl"], dev["gr"], H, Lh, W, LBS, Nl, QB, 0.0)
        grads = None
        if backward:
            gen = torch.Generator().manual_seed(seed)
            dm = torch.randn(outs[0].shape, generator=gen).to(torch.bfloat16).cuda()
            grads = torch.ops.llattn_b200.attn_bwd(dm, dev["qkv"], dev["rq"], dev["gkv"], dev["w"], dev["b"],
                                                   dev["gl"], dev["gr"], outs[1], outs[2], outs[3], outs[4],
                                                   H, Lh, W, LBS, Nl, QB, 0.0)
            grads = [g_.cpu() for g_ in grads]
        torch.cuda.synchronize()
    finally:
        os.environ["LLATTN_FORCE_SIMT"] = "0"
    return [o.cpu() for o in outs], grads


def _oracle_lat(inp, T, Nl, ldh, Lh, QB):
    """lat [B, Tq, Ld] of the oracle on the bf16-rounded rows, float64."""
    B = inp["rq"].shape[0]
    cs, nc = O.chunk_layout(T, Nl)
    tok = O.chunk_ids(T, cs, nc)
    qchunk = tok if QB <= 1 else tok[torch.arange(math.ceil(T / min(T, QB))) * min(T, QB)]
    rq = inp["rq"].to(torch.bfloat16).double().view(B, -1, Lh, ldh).transpose(1, 2)
    gkv = inp["gkv"].to(torch.bfloat16).double().view(B, nc, 2, Lh, ldh)
    gk, gv = gkv[:, :, 0].transpose(1, 2), gkv[:, :, 1].transpose(1, 2)
    out = O.latent_attention(rq, gk, gv, qchunk)
    return out.transpose(1, 2).reshape(B, -1, Lh * ldh)


@pytest.mark.parametrize("case", CASES)
def test_latent_fwd_tc_long(case):
    B, T, Nl, ldh, Lh, QB = case
    inp = _inputs(B, T, Nl, ldh, Lh, QB)
    tc, _ = _run(inp, Lh, Nl, QB, False)
    assert _fault() == 0
    simt, _ = _run(inp, Lh, Nl, QB, True)
    lat, lse = tc[3].float(), tc[4]
    ref = _oracle_lat(inp, T, Nl, ldh, Lh, QB)
    for got, want in ((lat, ref), (lat, simt[3].float())):
        assert rel_err(got, want) < TOL[torch.bfloat16], rel_err(got, want)
        assert frob_err(got, want) < TOL[torch.bfloat16], frob_err(got, want)
    fin = torch.isfinite(simt[4])
    assert torch.equal(fin, torch.isfinite(lse))
    if fin.any():
        assert (lse[fin] - simt[4][fin]).abs().max().item() < 1e-3


@pytest.mark.parametrize("case", CASES)
def test_latent_bwd_tc_long(case):
    """Every gradient of the block op, tensor-core latent kernels against the
    SIMT ones (which the parity suite holds to the oracle)."""
    B, T, Nl, ldh, Lh, QB = case
    inp = _inputs(B, T, Nl, ldh, Lh, QB)
    _, gt = _run(inp, Lh, Nl, QB, False, backward=True)
    assert _fault() == 0
    _, gr = _run(inp, Lh, Nl, QB, True, backward=True)
    names = ["dqkv", "drq", "dgkv", "dw_rout", "db_rout", "dg_local", "dg_remote", "db_qkv"]
    for name, a, b_ in zip(names, gt, gr):
        a, b_ = a.float(), b_.float()
        assert rel_err(a, b_) < TOL[torch.bfloat16], (name, rel_err(a, b_))
        assert frob_err(a, b_) < TOL[torch.bfloat16], (name, frob_err(a, b_))


def test_latent_bwd_tc_long_deterministic():
    inp = _inputs(1, 8192, 512, 32, 2, 0)
    _, g1 = _run(inp, 2, 512, 0, False, backward=True)
    _, g2 = _run(inp, 2, 512, 0, False, backward=True)
    assert _fault() == 0
    for a, b_ in zip(g1, g2):
        assert torch.equal(a, b_)
