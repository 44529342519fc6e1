"""The tcgen05 (sm_100a tensor-core) local-branch kernels against the exact
SIMT kernels of the same math and against the oracle, on bf16 inputs.

Both implementations run through the C ABI (torch op -> llattn_fwd/bwd); the
SIMT one is selected with LLATTN_FORCE_SIMT=1. After every launch the
device fault word (bounded waits that ran out) must be 0."""

import math
import os

import pytest
import torch

import llattn_oracle as O
from parity import rel_err

pytestmark = pytest.mark.gpu


def _fault():
    from llattn_b200 import _lib
    return _lib.lib().llattn_fault_status(1)


def _inputs(B, T, H, hd, Lh=2, ldh=32, Nl=32, QB=0, seed=0):
    gen = torch.Generator().manual_seed(seed)
    d, Ld = H * hd, Lh * ldh
    cs, nc = O.chunk_layout(T, Nl)
    tq = math.ceil(T / min(T, QB)) if QB > 1 else T
    f = lambda *s: torch.randn(*s, generator=gen)
    return dict(qkv=f(B, T, 3 * d), rq=f(B, tq, Ld), gkv=f(B, nc, 2 * Ld), w=f(d, Ld) / math.sqrt(Ld),
                b=f(d) * 0.1, gl=f(hd) / math.sqrt(hd), gr=f(hd) / math.sqrt(hd))


def _run_fwd(inp, H, Lh, W, LBS, Nl, QB, force_simt):
    import llattn_b200

    os.environ["LLATTN_FORCE_SIMT"] = "1" if force_simt else "0"
    try:
        dev = {k: v.cuda().to(torch.bfloat16 if k in ("qkv", "rq", "gkv", "w") else torch.float32)
               for k, v in inp.items()}
        outs = torch.ops.llattn_b200.attn_fwd(dev["qkv"], dev["rq"], dev["gkv"], dev["w"], dev["b"],
                                              dev["gl"], dev["gr"], H, Lh, W, LBS, Nl, QB, 0.0)
        torch.cuda.synchronize()
    finally:
        os.environ["LLATTN_FORCE_SIMT"] = "0"
    return [o.cpu() for o in outs]


FWD_CASES = [
    # B, T, H, hd, W, LBS
    (1, 256, 1, 128, 256, 256),
    (1, 300, 2, 64, 128, 256),
    (2, 1000, 2, 128, 256, 256),
    (1, 777, 3, 64, 300, 200),
    (1, 2100, 1, 128, 1024, 256),
    (2, 129, 2, 128, 16, 32),
    (1, 1, 1, 128, 4, 256),
    (1, 4096, 2, 128, 512, 256),
    (1, 700, 2, 88, 256, 256),
    (2, 333, 3, 96, 64, 128),
]


@pytest.mark.parametrize("case", FWD_CASES)
def test_local_fwd_tc_matches_simt(case):
    B, T, H, hd, W, LBS = case
    inp = _inputs(B, T, H, hd)
    tc = _run_fwd(inp, H, 2, W, LBS, 32, 0, False)
    assert _fault() == 0
    ref = _run_fwd(inp, H, 2, W, LBS, 32, 0, True)
    # local_out (bf16) and lse
    assert rel_err(tc[1].float(), ref[1].float()) < 1e-2, rel_err(tc[1].float(), ref[1].float())
    fin = torch.isfinite(ref[2])
    assert torch.equal(fin, torch.isfinite(tc[2]))
    if fin.any():
        assert (tc[2][fin] - ref[2][fin]).abs().max().item() < 1e-3
    assert rel_err(tc[0].float(), ref[0].float()) < 1e-2


def test_local_fwd_tc_against_oracle():
    B, T, H, hd, W, LBS = 1, 700, 2, 128, 256, 256
    inp = _inputs(B, T, H, hd)
    tc = _run_fwd(inp, H, 2, W, LBS, 32, 0, False)
    assert _fault() == 0
    qkv = inp["qkv"].to(torch.bfloat16).double()
    q, k, v = qkv.view(B, T, 3, H, hd).unbind(2)
    ref = O.local_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), W, LBS)
    got = tc[1].view(B, T, H, hd).transpose(1, 2)
    assert rel_err(got, ref) < 2e-2


def _run_fwd_bwd(inp, H, Lh, W, LBS, Nl, QB, force_simt, seed=5):
    os.environ["LLATTN_FORCE_SIMT"] = "1" if force_simt else "0"
    try:
        dev = {k: v.cuda().to(torch.bfloat16 if k in ("qkv", "rq", "gkv", "w") else torch.float32)
               for k, v in inp.items()}
        outs = torch.ops.llattn_b200.attn_fwd(dev["qkv"], dev["rq"], dev["gkv"], dev["w"], dev["b"],
                                              dev["gl"], dev["gr"], H, Lh, W, LBS, Nl, QB, 0.0)
        gen = torch.Generator().manual_seed(seed)
        dm = torch.randn(outs[0].shape, generator=gen).to(torch.bfloat16).cuda()
        grads = torch.ops.llattn_b200.attn_bwd(dm, dev["qkv"], dev["rq"], dev["gkv"], dev["w"], dev["b"],
                                               dev["gl"], dev["gr"], outs[1], outs[2], outs[3], outs[4],
                                               H, Lh, W, LBS, Nl, QB, 0.0)
        torch.cuda.synchronize()
    finally:
        os.environ["LLATTN_FORCE_SIMT"] = "0"
    return [o.cpu() for o in outs], [g_.cpu() for g_ in grads]


BWD_CASES = [
    # B, T, H, hd, W, LBS
    (1, 256, 1, 128, 256, 256),
    (1, 300, 2, 64, 128, 256),
    (2, 1000, 2, 128, 256, 256),
    (1, 777, 3, 64, 300, 200),
    (1, 2100, 1, 128, 1024, 256),
    (2, 129, 2, 128, 16, 32),
    (1, 1, 1, 128, 4, 256),
    (1, 4096, 2, 128, 512, 256),
    (1, 700, 2, 88, 256, 256),
    (2, 333, 3, 96, 64, 128),
]


@pytest.mark.parametrize("case", BWD_CASES)
def test_local_bwd_tc_matches_simt(case):
    B, T, H, hd, W, LBS = case
    inp = _inputs(B, T, H, hd)
    _, gt = _run_fwd_bwd(inp, H, 2, W, LBS, 32, 0, False)
    assert _fault() == 0
    _, gr = _run_fwd_bwd(inp, H, 2, W, LBS, 32, 0, True)
    names = ["dqkv", "drq", "dgkv", "dw_rout", "db_rout", "dg_local", "dg_remote", "db_qkv"]
    assert len(gt) == len(names)
    d = H * hd
    for name, a, b_ in zip(names, gt, gr):
        if name == "dqkv":
            for slot, sname in enumerate(("dq", "dk", "dv")):
                x = a.view(B, T, 3, d)[:, :, slot].float()
                y = b_.view(B, T, 3, d)[:, :, slot].float()
                assert rel_err(x, y) < 2e-2, (sname, rel_err(x, y))
        else:
            assert rel_err(a.float(), b_.float()) < 2e-2, (name, rel_err(a.float(), b_.float()))


def test_recorded_fault_fails_later_launches_until_cleared():
    """A fault recorded in the host-mapped fault word (injected on the host:
    no GPU wait is made to run out) makes the launching entry points fail
    with LLATTN_ERR_DEVICE, so the op raises instead of returning outputs of
    abandoned kernels; clearing the word restores normal launches."""
    from llattn_b200 import _lib

    L = _lib.lib()
    inp = _inputs(1, 300, 2, 64)
    ref = _run_fwd(inp, 2, 2, 128, 256, 32, 0, False)
    assert _fault() == 0
    assert L.llattn_fault_inject_host(4) == 0
    try:
        with pytest.raises(RuntimeError, match="status 5"):
            _run_fwd(inp, 2, 2, 128, 256, 32, 0, False)
    finally:
        assert _fault() == 4  # reads and clears both words
    again = _run_fwd(inp, 2, 2, 128, 256, 32, 0, False)
    for a, b in zip(again, ref):
        assert torch.equal(a, b)
    assert _fault() == 0


STRIDE_CASES = [
    # B, T, H, hd, Lh, ldh, force_simt, dtype
    (2, 300, 2, 128, 2, 32, False, torch.bfloat16),
    (2, 257, 3, 64, 2, 32, False, torch.bfloat16),
    (1, 300, 2, 88, 2, 32, False, torch.bfloat16),   # padded head_dim
    (1, 200, 2, 64, 4, 64, False, torch.bfloat16),   # latent_d_model 256: the general path
    (2, 150, 2, 32, 2, 16, True, torch.bfloat16),    # SIMT kernels
    (2, 150, 2, 32, 2, 16, False, torch.float32),
]


@pytest.mark.parametrize("case", STRIDE_CASES)
def test_wide_qkv_and_dqkv_rows_match_contiguous(case):
    """qkv read from, and dqkv written into, the first 3d columns of a wider
    row-major buffer (llattn_dims.qkv_row_stride / dqkv_row_stride): the
    same bits as with contiguous rows, and the extra columns untouched."""
    B, T, H, hd, Lh, ldh, simt, dt = case
    d, Ld, extra = H * hd, Lh * ldh, 24
    W, LBS, Nl = 64, 128, 16
    inp = _inputs(B, T, H, hd, Lh, ldh, Nl)
    dev = {k: v.cuda().to(dt if k in ("qkv", "rq", "gkv", "w") else torch.float32) for k, v in inp.items()}
    wide = torch.full((B, T, 3 * d + extra), 7.0, dtype=dt, device="cuda")
    wide[..., :3 * d] = dev["qkv"]
    qkv_view = wide[..., :3 * d]
    cfg = (H, Lh, W, LBS, Nl, 0, 0.0)
    os.environ["LLATTN_FORCE_SIMT"] = "1" if simt else "0"
    try:
        ref = torch.ops.llattn_b200.attn_fwd(dev["qkv"], dev["rq"], dev["gkv"], dev["w"], dev["b"], dev["gl"],
                                             dev["gr"], *cfg)
        got = torch.ops.llattn_b200.attn_fwd(qkv_view, dev["rq"], dev["gkv"], dev["w"], dev["b"], dev["gl"],
                                             dev["gr"], *cfg)
        dm = torch.randn(B, T, d, generator=torch.Generator().manual_seed(3)).to("cuda", dt)
        saved = lambda q, o: (q, dev["rq"], dev["gkv"], dev["w"], dev["b"], dev["gl"], dev["gr"], o[1], o[2],  # noqa: E731
                              o[3], o[4])
        bref = torch.ops.llattn_b200.attn_bwd(dm, *saved(dev["qkv"], ref), *cfg)
        bgot = torch.ops.llattn_b200.attn_bwd(dm, *saved(qkv_view, got), *cfg, 0, 0, 3 * d + extra)
        torch.cuda.synchronize()
    finally:
        os.environ["LLATTN_FORCE_SIMT"] = "0"
    assert _fault() == 0
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    assert bgot[0].shape == (B, T, 3 * d + extra)
    assert torch.equal(bgot[0][..., :3 * d], bref[0])
    for a, b in zip(bref[1:], bgot[1:]):
        assert torch.equal(a, b)
    assert torch.equal(wide[..., 3 * d:], torch.full_like(wide[..., 3 * d:], 7.0))
