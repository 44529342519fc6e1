"""llattn_bwd_noalloc against llattn_bwd, through the C ABI.

llattn_bwd_noalloc serves callers that cannot allocate device memory (hosts
that only lend the library tensors from their own preallocated pool, or code
that must not trigger an allocation): it runs the same backward with a fixed
scratch array built into the library instead of a caller workspace. This file
is collected last so that a stop-at-first-failure run has run everything else
before it; it passes alone in a fresh process and after the other tests.
"""

import ctypes
import math

import pytest
import torch

from parity import TOL, rel_err

pytestmark = pytest.mark.gpu


def _case(dtype, B=2, T=777, H=2, hd=128, Lh=2, ldh=32, Nl=32, W=256, LBS=256, QB=0, seed=0):
    gen = torch.Generator().manual_seed(seed)
    d, Ld = H * hd, Lh * ldh
    cs = math.ceil(T / min(Nl, T))
    nc = math.ceil(T / cs)
    tq = math.ceil(T / min(T, QB)) if QB > 1 else T
    f = lambda *s: torch.randn(*s, generator=gen)
    act = lambda t: t.to(dtype).cuda()
    f32 = lambda t: t.float().cuda()
    inp = dict(qkv=act(f(B, T, 3 * d)), rq=act(f(B, tq, Ld)), gkv=act(f(B, nc, 2 * Ld)),
               w=act(f(d, Ld) / math.sqrt(Ld)), b=f32(f(d) * 0.1), gl=f32(f(hd) / math.sqrt(hd)),
               gr=f32(f(hd) / math.sqrt(hd)))
    fwd = torch.ops.llattn_b200.attn_fwd(inp["qkv"], inp["rq"], inp["gkv"], inp["w"], inp["b"], inp["gl"],
                                         inp["gr"], H, Lh, W, LBS, Nl, QB, 0.0)
    dm = act(f(B, T, d))
    cfg = (H, Lh, hd, ldh, W, LBS, Nl, QB)
    return inp, fwd, dm, cfg


def _run(entry, inp, fwd, dm, cfg, with_workspace):
    from llattn_b200 import _lib

    H, Lh, hd, ldh, W, LBS, Nl, QB = cfg
    qkv = inp["qkv"]
    B, T = qkv.shape[:2]
    code = _lib.BF16 if qkv.dtype == torch.bfloat16 else _lib.F32
    dims = _lib.make_dims(B, T, H, hd, Lh, ldh, W, LBS, Nl, QB, code, 0.0)
    outs = [torch.empty_like(qkv), torch.empty_like(inp["rq"]), torch.empty_like(inp["gkv"]),
            torch.empty(inp["w"].shape, device="cuda"), torch.empty(H * hd, device="cuda"),
            torch.empty(hd, device="cuda"), torch.empty(hd, device="cuda"), torch.empty(3 * H * hd, device="cuda")]
    ws = None
    if with_workspace:
        n = _lib.lib().llattn_bwd_workspace_bytes(ctypes.byref(dims))
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    p = lambda t: t.data_ptr()
    args = _lib.BwdArgs(dims, p(qkv), p(inp["rq"]), p(inp["gkv"]), p(inp["w"]), p(inp["b"]), p(inp["gl"]),
                        p(inp["gr"]), p(fwd[1]), p(fwd[2]), p(fwd[3]), p(fwd[4]), p(dm), *[p(o) for o in outs[:7]],
                        p(ws) if ws is not None else None, ws.numel() if ws is not None else 0, p(outs[7]))
    rc = entry(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, _lib.lib().llattn_last_error().decode()
    return outs


def _near_full_T(dtype, **kw):
    """Largest T whose backward workspace still fits the fixed scratch: the
    case that puts the last workspace region at the end of the array."""
    from llattn_b200 import _lib

    H, Lh, hd, ldh, W, LBS, Nl, QB = (kw[k] for k in ("H", "Lh", "hd", "ldh", "W", "LBS", "Nl", "QB"))
    code = _lib.BF16 if dtype == torch.bfloat16 else _lib.F32
    need = lambda T: _lib.lib().llattn_bwd_workspace_bytes(
        ctypes.byref(_lib.make_dims(kw["B"], T, H, hd, Lh, ldh, W, LBS, Nl, QB, code, 0.0)))
    lo, hi = 1, 65535
    while lo < hi:  # the workspace grows with T
        mid = (lo + hi + 1) // 2
        lo, hi = (mid, hi) if need(mid) <= _lib.BWD_NOALLOC_SCRATCH_BYTES else (lo, mid - 1)
    assert _lib.BWD_NOALLOC_SCRATCH_BYTES - need(lo) < 64 * 1024, "workspace not within 64 KiB of the scratch"
    return lo


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_bwd_matches_workspace_bwd_twice(dtype):
    """Two calls in a row on different dims. The first fills the scratch almost
    to its end, with block-pooled queries and more than 64 latent chunks (the
    paths with the most workspace regions); the second, smaller call then
    runs over what the first left behind. Each must give exactly the bytes of
    llattn_bwd with a fresh caller workspace (the backward is deterministic)."""
    from llattn_b200 import _lib

    L = _lib.lib()
    big = dict(B=1, H=2, hd=128, Lh=2, ldh=32, Nl=128, W=256, LBS=256, QB=64)
    T_big = _near_full_T(dtype, **big)
    for kw in (dict(big, T=T_big), dict(T=777, seed=1)):
        inp, fwd, dm, cfg = _case(dtype, **kw)
        ref = _run(L.llattn_bwd, inp, fwd, dm, cfg, True)
        got = _run(L.llattn_bwd_noalloc, inp, fwd, dm, cfg, False)
        for a, b in zip(got, ref):
            assert torch.equal(a, b), f"T={kw['T']}: max diff {(a.float() - b.float()).abs().max().item()}"
            assert rel_err(a.float(), b.float()) <= TOL[dtype]


def test_noalloc_rejects_dims_beyond_its_scratch():
    from llattn_b200 import _lib

    dims = _lib.make_dims(16, 2048, 12, 128, 2, 32, 256, 256, 64, 0, _lib.BF16, 0.0)
    L = _lib.lib()
    assert L.llattn_bwd_workspace_bytes(ctypes.byref(dims)) > _lib.BWD_NOALLOC_SCRATCH_BYTES
    args = _lib.BwdArgs()
    args.dims = dims
    for name, _ in _lib.BwdArgs._fields_:
        if name not in ("dims", "workspace", "workspace_bytes"):
            setattr(args, name, 256)  # never dereferenced: the size check comes first
    assert L.llattn_bwd_noalloc(ctypes.byref(args), None) == 4
    assert "scratch" in L.llattn_last_error().decode()
