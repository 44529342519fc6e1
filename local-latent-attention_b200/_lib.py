"""ctypes binding of libllattn.so (the C ABI declared in include/llattn.h).

The library is built in-tree by ``csrc/build.py``; loading fails loudly when
it is missing — there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libllattn.so")

F32, BF16 = 0, 1
POOL_CHUNKS, POOL_QBLOCKS, POOL_ACCUMULATE = 0, 1, 16
BWD_NOALLOC_SCRATCH_BYTES = 32 << 20

EXPORTED = (
    "llattn_version", "llattn_last_error", "llattn_fault_status", "llattn_geometry", "llattn_bwd_workspace_bytes",
    "llattn_pool_fwd", "llattn_pool_bwd", "llattn_fwd", "llattn_bwd", "llattn_bwd_noalloc", "llattn_decode",
    "llattn_profile_enable", "llattn_profile_read", "llattn_profile_name", "llattn_colsum_workspace_bytes",
    "llattn_colsum", "llattn_fault_inject_host", "llattn_pool_proj_fwd", "llattn_pool_proj_bwd",
)


class Dims(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("seq_len", ctypes.c_int32), ("n_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("latent_heads", ctypes.c_int32),
        ("latent_head_dim", ctypes.c_int32), ("window", ctypes.c_int32),
        ("local_block", ctypes.c_int32), ("latent_tokens", ctypes.c_int32),
        ("query_block", ctypes.c_int32), ("dtype", ctypes.c_int32), ("gate_bias", ctypes.c_float),
        ("seq_offset", ctypes.c_int32), ("total_len", ctypes.c_int32),
        ("qkv_row_stride", ctypes.c_int32), ("dqkv_row_stride", ctypes.c_int32),
    ]


class Geom(ctypes.Structure):
    _fields_ = [("chunk", ctypes.c_int32), ("n_chunks", ctypes.c_int32),
                ("local_span", ctypes.c_int32), ("qblock", ctypes.c_int32),
                ("n_qrows", ctypes.c_int32)]


_vp = ctypes.c_void_p
_fp = ctypes.c_void_p  # float* passed as raw addresses


class FwdArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("qkv", _vp), ("rq", _vp), ("gkv", _vp), ("w_rout", _vp),
                ("b_rout", _fp), ("g_local", _fp), ("g_remote", _fp), ("mixed", _vp),
                ("local_out", _vp), ("lse", _fp), ("lat", _vp), ("lat_lse", _fp)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("qkv", _vp), ("rq", _vp), ("gkv", _vp), ("w_rout", _vp),
                ("b_rout", _fp), ("g_local", _fp), ("g_remote", _fp), ("local_out", _vp),
                ("lse", _fp), ("lat", _vp), ("lat_lse", _fp), ("dmixed", _vp), ("dqkv", _vp),
                ("drq", _vp), ("dgkv", _vp), ("dw_rout", _fp), ("db_rout", _fp),
                ("dg_local", _fp), ("dg_remote", _fp), ("workspace", _vp),
                ("workspace_bytes", ctypes.c_size_t), ("db_qkv", _fp)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("cache_len", ctypes.c_int64), ("qkv_cache", _vp), ("rq_row", _vp),
                ("gkv", _vp), ("w_rout", _vp), ("b_rout", _fp), ("g_local", _fp), ("g_remote", _fp),
                ("mixed_row", _vp)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load libllattn.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with "
                "`python local-latent-attention_b200/csrc/build.py` (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        L.llattn_version.restype = ctypes.c_int
        L.llattn_last_error.restype = ctypes.c_char_p
        L.llattn_fault_status.argtypes = [ctypes.c_int]
        L.llattn_fault_status.restype = ctypes.c_uint
        L.llattn_fault_inject_host.argtypes = [ctypes.c_uint]
        L.llattn_fault_inject_host.restype = ctypes.c_int
        L.llattn_geometry.argtypes = [ctypes.POINTER(Dims), ctypes.POINTER(Geom)]
        L.llattn_geometry.restype = ctypes.c_int
        L.llattn_bwd_workspace_bytes.argtypes = [ctypes.POINTER(Dims)]
        L.llattn_bwd_workspace_bytes.restype = ctypes.c_size_t
        for name in ("llattn_pool_fwd", "llattn_pool_bwd"):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.POINTER(Dims), ctypes.c_int, _vp, _vp, ctypes.c_int64, _vp]
            fn.restype = ctypes.c_int
        L.llattn_pool_proj_fwd.argtypes = [ctypes.POINTER(Dims), _vp, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp]
        L.llattn_pool_proj_fwd.restype = ctypes.c_int
        L.llattn_pool_proj_bwd.argtypes = [ctypes.POINTER(Dims), _vp, _vp, _vp, ctypes.c_int64, _vp]
        L.llattn_pool_proj_bwd.restype = ctypes.c_int
        L.llattn_colsum_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        L.llattn_colsum_workspace_bytes.restype = ctypes.c_size_t
        L.llattn_colsum.argtypes = [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _vp, _vp, ctypes.c_size_t, _vp]
        L.llattn_colsum.restype = ctypes.c_int
        L.llattn_fwd.argtypes = [ctypes.POINTER(FwdArgs), _vp]
        L.llattn_fwd.restype = ctypes.c_int
        L.llattn_bwd.argtypes = [ctypes.POINTER(BwdArgs), _vp]
        L.llattn_bwd.restype = ctypes.c_int
        L.llattn_bwd_noalloc.argtypes = [ctypes.POINTER(BwdArgs), _vp]
        L.llattn_bwd_noalloc.restype = ctypes.c_int
        L.llattn_decode.argtypes = [ctypes.POINTER(DecodeArgs), _vp]
        L.llattn_decode.restype = ctypes.c_int
        L.llattn_profile_enable.argtypes = [ctypes.c_int]
        L.llattn_profile_enable.restype = ctypes.c_int
        L.llattn_profile_read.argtypes = [ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_longlong), ctypes.c_int]
        L.llattn_profile_read.restype = ctypes.c_int
        L.llattn_profile_name.argtypes = [ctypes.c_int]
        L.llattn_profile_name.restype = ctypes.c_char_p
        _lib = L
    return _lib


def profile_enable(on: bool) -> None:
    """Turn per-kernel event timing on/off (and reset the totals)."""
    lib().llattn_profile_enable(1 if on else 0)


def profile_read() -> dict:
    """{kernel group: (total ms, launches)} since the last profile_enable."""
    L = lib()
    n = 16
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_longlong * n)()
    k = L.llattn_profile_read(ms, cnt, n)
    return {L.llattn_profile_name(i).decode(): (ms[i], cnt[i]) for i in range(k)}


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().llattn_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def make_dims(batch, seq_len, n_heads=1, head_dim=1, latent_heads=1, latent_head_dim=1,
              window=1, local_block=256, latent_tokens=1, query_block=0, dtype=F32,
              gate_bias=0.0, seq_offset=0, total_len=0, qkv_row_stride=0, dqkv_row_stride=0) -> Dims:
    return Dims(int(batch), int(seq_len), int(n_heads), int(head_dim), int(latent_heads),
                int(latent_head_dim), int(window), int(local_block), int(latent_tokens),
                int(query_block), int(dtype), float(gate_bias), int(seq_offset), int(total_len),
                int(qkv_row_stride), int(dqkv_row_stride))


def geometry(dims: Dims) -> Geom:
    g = Geom()
    check(lib().llattn_geometry(ctypes.byref(dims), ctypes.byref(g)), "llattn_geometry")
    return g
