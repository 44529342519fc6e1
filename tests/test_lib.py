"""The C-ABI library: it loads, exports every symbol include/llattn.h
declares, and its host-side logic (geometry, workspace sizing, argument
validation) behaves — no kernel launches, so no GPU needed."""

import ctypes
import os
import re

import pytest

import llattn_b200
from llattn_b200 import _lib, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    with open(os.path.join(ROOT, "include", "llattn.h")) as fh:
        text = fh.read()
    return re.findall(r"LLATTN_API\s+[\w\s\*]+?\b(llattn_\w+)\s*\(", text)


def test_header_declares_the_binding_symbols():
    assert sorted(declared_symbols()) == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert L.llattn_version() == 3


@pytest.mark.parametrize("T,Nl,QB,W,LBS", [
    (512, 16, 0, 128, 256), (2048, 64, 0, 256, 256), (16384, 256, 64, 512, 256),
    (37, 5, 8, 6, 10), (1, 4, 0, 4, 256), (20, 64, 0, 5, 8), (5, 3, 8, 3, 4),
    (32805, 512, 0, 1024, 256), (8191, 32, 0, 64, 256), (130, 128, 0, 64, 256),
])
def test_geometry_matches_reference_formulas(T, Nl, QB, W, LBS):
    g = _lib.geometry(_lib.make_dims(2, T, window=W, local_block=LBS, latent_tokens=Nl,
                                     query_block=QB))
    py = ops.geometry(T, Nl, QB, W, LBS)
    assert (g.chunk, g.n_chunks, g.local_span, g.qblock, g.n_qrows) == (
        py["chunk"], py["n_chunks"], py["local_span"], py["qblock"], py["n_qrows"])
    import llattn_oracle as O
    assert (g.chunk, g.n_chunks) == O.chunk_layout(T, Nl)


@pytest.mark.parametrize("bad,msg", [
    (dict(seq_len=0), "seq_len"), (dict(head_dim=256), "head_dim"), (dict(window=0), "local_window"),
    (dict(latent_tokens=0), "latent_tokens"), (dict(dtype=7), "dtype"),
    (dict(latent_head_dim=128), "latent_head_dim"),
    (dict(qkv_row_stride=95), "row strides"), (dict(dqkv_row_stride=64), "row strides"),
    (dict(qkv_row_stride=100, dtype=1), "multiples of 8"), (dict(dqkv_row_stride=97, dtype=1), "multiples of 8"),
])
def test_bad_dims_are_rejected_on_the_host(bad, msg):
    kw = dict(batch=2, seq_len=64, n_heads=2, head_dim=16, latent_heads=2, latent_head_dim=4,
              window=8, local_block=16, latent_tokens=8)
    kw.update(bad)
    dims = _lib.make_dims(**kw)
    g = _lib.Geom()
    rc = _lib.lib().llattn_geometry(ctypes.byref(dims), ctypes.byref(g))
    assert rc == 1
    assert msg in _lib.lib().llattn_last_error().decode()
    assert _lib.lib().llattn_bwd_workspace_bytes(ctypes.byref(dims)) == 0


def test_wide_row_strides_are_accepted():
    """qkv / dqkv rows inside a wider buffer (3d = 96 here): any stride >= 3d
    in fp32, a multiple of 8 in bf16."""
    L = _lib.lib()
    g = _lib.Geom()
    for ld, dt in ((96, _lib.F32), (97, _lib.F32), (104, _lib.BF16), (96 + 192, _lib.BF16)):
        dims = _lib.make_dims(2, 64, 2, 16, 2, 4, 8, 16, 8, dtype=dt, qkv_row_stride=ld, dqkv_row_stride=ld)
        assert L.llattn_geometry(ctypes.byref(dims), ctypes.byref(g)) == 0, (ld, dt)


def test_entry_points_reject_null_args_without_launching():
    L = _lib.lib()
    assert L.llattn_fwd(None, None) == 1
    assert L.llattn_bwd(None, None) == 1
    args = _lib.FwdArgs()
    args.dims = _lib.make_dims(1, 8, 1, 8, 1, 4, 4, 256, 2)
    assert L.llattn_fwd(ctypes.byref(args), None) == 1
    assert "NULL" in L.llattn_last_error().decode()


def test_workspace_grows_with_problem():
    small = _lib.make_dims(1, 64, 2, 16, 2, 4, 8, 16, 8, dtype=_lib.BF16)
    big = _lib.make_dims(16, 2048, 12, 128, 2, 32, 256, 256, 64, dtype=_lib.BF16)
    L = _lib.lib()
    a = L.llattn_bwd_workspace_bytes(ctypes.byref(small))
    b = L.llattn_bwd_workspace_bytes(ctypes.byref(big))
    assert 0 < a < b and b % 256 == 0


def test_bwd_rejects_small_workspace():
    import torch  # noqa: F401
    dims = _lib.make_dims(1, 8, 1, 8, 1, 4, 4, 256, 2)
    args = _lib.BwdArgs()
    args.dims = dims
    fake = 256  # never dereferenced: validation fails first
    for name, _ in _lib.BwdArgs._fields_:
        if name not in ("dims", "workspace", "workspace_bytes"):
            setattr(args, name, fake)
    args.workspace = fake
    args.workspace_bytes = 16
    assert _lib.lib().llattn_bwd(ctypes.byref(args), None) == 4
    assert "workspace" in _lib.lib().llattn_last_error().decode()


def test_shard_offset_validation():
    """Sequence shards: geometry follows total_len, bad offsets are rejected on the host."""
    from llattn_b200 import _lib

    g = _lib.Geom()
    L = _lib.lib()
    # offset + length beyond the total, and an offset off the query-block grid, are rejected
    bad = _lib.make_dims(1, 100, 1, 64, 1, 32, 16, 256, 8, 0, _lib.BF16, 0.0, 950, 1000)
    assert L.llattn_geometry(ctypes.byref(bad), ctypes.byref(g)) == 1
    bad = _lib.make_dims(1, 100, 1, 64, 1, 32, 16, 256, 8, 64, _lib.BF16, 0.0, 100, 1000)
    assert L.llattn_geometry(ctypes.byref(bad), ctypes.byref(g)) == 1
    ok = _lib.make_dims(1, 128, 1, 64, 1, 32, 16, 256, 8, 64, _lib.BF16, 0.0, 128, 1000)
    assert L.llattn_geometry(ctypes.byref(ok), ctypes.byref(g)) == 0
    assert (g.chunk, g.n_chunks, g.qblock, g.n_qrows) == (125, 8, 64, 2)


def test_pool_proj_rejects_bad_args_on_the_host():
    """llattn_pool_proj_fwd / _bwd validate before launching (no GPU needed):
    NULL pointers, ldz below 3 * latent_d_model, latent_d_model above 128,
    sequence shards."""
    L = _lib.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: every case fails validation first
    ok = _lib.make_dims(1, 64, latent_heads=2, latent_head_dim=32, latent_tokens=8, dtype=_lib.BF16)
    cases = [
        (ok, None, 192, "NULL"),
        (ok, p, 100, "ldz"),
        (_lib.make_dims(1, 64, latent_heads=4, latent_head_dim=64, latent_tokens=8, dtype=_lib.BF16), p, 768, "> 128"),
        (_lib.make_dims(1, 64, latent_heads=2, latent_head_dim=32, latent_tokens=8, dtype=_lib.BF16,
                        seq_offset=0, total_len=128), p, 192, "whole sequences"),
    ]
    for dims, z, ldz, msg in cases:
        assert L.llattn_pool_proj_fwd(ctypes.byref(dims), z, ldz, None, None, p, p, None) == 1
        assert msg in L.llattn_last_error().decode(), (msg, L.llattn_last_error())
        assert L.llattn_pool_proj_bwd(ctypes.byref(dims), z, p, p, ldz, None) == 1
        assert msg in L.llattn_last_error().decode(), (msg, L.llattn_last_error())


@pytest.mark.parametrize("T,Nl,QB", [(8192, 512, 0), (16384, 256, 64), (1000, 100, 0)])
def test_workspace_holds_the_long_latent_regions(T, Nl, QB):
    """Past 64 chunks the tensor-core latent backward needs delta [B, Lh, Tq]
    fp32 and one dgk/dgv partial [B, Nc, 2, Ld] per row split of its keys
    kernel (splits: about two waves of (128-key tile, split, head, b) CTAs
    on 148 SMs); the workspace must hold both beside everything else."""
    B, Lh, ldh = 4, 2, 32
    dims = _lib.make_dims(B, T, 8, 128, Lh, ldh, 1024, 256, Nl, QB, _lib.BF16)
    g = _lib.geometry(dims)
    nc, tq, Ld = g.n_chunks, g.n_qrows, Lh * ldh
    assert nc > 64
    splits = max(1, min(-(-tq // 64), (2 * 148) // (B * Lh * -(-nc // 128))))
    need = 4 * B * Lh * tq + 4 * splits * B * nc * 2 * Ld
    assert _lib.lib().llattn_bwd_workspace_bytes(ctypes.byref(dims)) >= need
