"""torch custom ops over libllattn.so: pooling and the fused attention core.

``llattn_b200::pool_fwd/pool_bwd`` and ``llattn_b200::attn_fwd/attn_bwd`` are
registered with ``torch.library.custom_op`` for CUDA only, with fake (meta)
implementations for tracing and ``register_autograd`` for the backward. They
launch on torch's current stream, allocate every output and the backward
workspace through torch, and raise ``RuntimeError`` with the library's
message on any argument error. There is no CPU implementation: calling them
on CPU tensors is an error.

Reference API mirrored: ``LLAttnFunction.apply`` of
``kernels/llattn_op.py:184-238`` — the forward saves the local-branch
logsumexp and the branch outputs, the backward returns one gradient per
tensor input. The math is that of the PyTorch module (models.py:307-462).
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch
from torch import Tensor

from . import _lib

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def geometry(seq_len: int, latent_tokens: int, query_block: int, window: int = 1,
             local_block: int = 256, total_len: int = 0) -> dict:
    """Derived sizes, as models.py derives them (cs/Nc :175-183, bsL :249,
    bs/Tq :216-219). Pure Python so fake tensors need no library call. For a
    shard of a total_len-token sequence the chunking, block span and query
    block follow total_len and n_qrows counts the shard's query rows."""
    TT = total_len if total_len > 0 else seq_len
    target = min(latent_tokens, TT)
    cs = math.ceil(TT / target)
    qbs = min(TT, query_block) if query_block > 1 else 1
    return {"chunk": cs, "n_chunks": math.ceil(TT / cs),
            "local_span": min(TT, max(window, local_block)),
            "qblock": qbs, "n_qrows": math.ceil(seq_len / qbs)}


def visible_pairs(seq_len: int, window: int, local_block: int = 256) -> int:
    """Visible (query, key) pairs of one (batch, head) sequence under the
    local mask (models.py:245-292: key j visible from t iff 0 < t-j <= W and
    j >= qs(t) - W + 1): the local branch's work is 4*hd FLOPs per pair
    forward and 8*hd backward."""
    bsl = min(seq_len, max(window, local_block))
    t = torch.arange(seq_len, dtype=torch.int64)
    qs = (t // bsl) * bsl
    lo = torch.clamp(torch.maximum(t - window, qs - window + 1), min=0)
    return int((t - lo).clamp(min=0).sum())


def _ptr(t: Tensor) -> int:
    return t.data_ptr()


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _dtype_code(t: Tensor) -> int:
    if t.dtype not in _DT:
        raise RuntimeError(f"llattn: unsupported dtype {t.dtype} (float32 or bfloat16)")
    return _DT[t.dtype]


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError("llattn: " + msg)


# --------------------------------------------------------------------------
# pooling (K1): models.py:159-214 (chunks) and :216-230 (query blocks)

@torch.library.custom_op("llattn_b200::pool_fwd", mutates_args=(), device_types="cuda")
def pool_fwd(x: Tensor, latent_tokens: int, query_block: int, mode: int) -> Tensor:
    _require(x.dim() == 3 and x.is_contiguous(), "pool_fwd expects a contiguous [B, T, d] tensor")
    B, T, d = x.shape
    geo = geometry(T, latent_tokens, query_block)
    rows = geo["n_chunks"] if mode == _lib.POOL_CHUNKS else geo["n_qrows"]
    out = torch.empty(B, rows, d, dtype=x.dtype, device=x.device)
    dims = _lib.make_dims(B, T, latent_tokens=latent_tokens, query_block=query_block,
                          dtype=_dtype_code(x))
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().llattn_pool_fwd(ctypes.byref(dims), mode, _ptr(x), _ptr(out), d,
                                              _stream(x)), "llattn_pool_fwd")
    return out


@pool_fwd.register_fake
def _pool_fwd_fake(x, latent_tokens, query_block, mode):
    B, T, d = x.shape
    geo = geometry(T, latent_tokens, query_block)
    rows = geo["n_chunks"] if mode == _lib.POOL_CHUNKS else geo["n_qrows"]
    return x.new_empty(B, rows, d)


@torch.library.custom_op("llattn_b200::pool_bwd", mutates_args=(), device_types="cuda")
def pool_bwd(dpooled: Tensor, seq_len: int, latent_tokens: int, query_block: int, mode: int) -> Tensor:
    _require(dpooled.dim() == 3 and dpooled.is_contiguous(), "pool_bwd expects a contiguous gradient")
    B, _, d = dpooled.shape
    dx = torch.empty(B, seq_len, d, dtype=dpooled.dtype, device=dpooled.device)
    dims = _lib.make_dims(B, seq_len, latent_tokens=latent_tokens, query_block=query_block,
                          dtype=_dtype_code(dpooled))
    with torch.cuda.device(dpooled.device):
        _lib.check(_lib.lib().llattn_pool_bwd(ctypes.byref(dims), mode, _ptr(dpooled), _ptr(dx), d,
                                              _stream(dpooled)), "llattn_pool_bwd")
    return dx


@pool_bwd.register_fake
def _pool_bwd_fake(dpooled, seq_len, latent_tokens, query_block, mode):
    B, _, d = dpooled.shape
    return dpooled.new_empty(B, seq_len, d)


def _pool_setup(ctx, inputs, output):
    x, latent_tokens, query_block, mode = inputs
    ctx.cfg = (x.shape[1], latent_tokens, query_block, mode)


def _pool_backward(ctx, grad):
    return pool_bwd(grad.contiguous(), *ctx.cfg), None, None, None


pool_fwd.register_autograd(_pool_backward, setup_context=_pool_setup)


# Pooling fused with the latent projections (llattn_pool_proj_fwd/bwd): z =
# x [W_rkv; W_rq]^T per token, then the chunk / query-block means of z's rows.

def _pp_dims(B, T, latent_heads, latent_d_model, latent_tokens, query_block, t):
    return _lib.make_dims(B, T, latent_heads=latent_heads, latent_head_dim=latent_d_model // latent_heads,
                          latent_tokens=latent_tokens, query_block=query_block, dtype=_dtype_code(t))


@torch.library.custom_op("llattn_b200::pool_proj_fwd", mutates_args=(), device_types="cuda")
def pool_proj_fwd(z: Tensor, b_rkv: Optional[Tensor], b_rq: Optional[Tensor], batch: int, latent_heads: int,
                  latent_tokens: int, query_block: int) -> tuple[Tensor, Tensor]:
    """z [B*T, 3Ld] (x W_rkv^T | x W_rq^T, no bias) -> gkv [B, Nc, 2Ld] (chunk
    means + b_rkv), rq [B, Tq, Ld] (query-block means or the rows, + b_rq)."""
    _require(z.dim() == 2 and z.stride(1) == 1 and z.is_cuda, "pool_proj_fwd expects a row-major 2-D CUDA tensor")
    _require(z.shape[1] % 3 == 0 and z.shape[0] % batch == 0, "pool_proj_fwd: z must be [B*T, 3*latent_d_model]")
    Ld, T = z.shape[1] // 3, z.shape[0] // batch
    geo = geometry(T, latent_tokens, query_block)
    gkv = torch.empty(batch, geo["n_chunks"], 2 * Ld, dtype=z.dtype, device=z.device)
    rq = torch.empty(batch, geo["n_qrows"], Ld, dtype=z.dtype, device=z.device)
    for b in (b_rkv, b_rq):
        _require(b is None or (b.is_contiguous() and b.dtype == z.dtype), "pool_proj_fwd: biases must match z")
    dims = _pp_dims(batch, T, latent_heads, Ld, latent_tokens, query_block, z)
    with torch.cuda.device(z.device):
        _lib.check(_lib.lib().llattn_pool_proj_fwd(ctypes.byref(dims), _ptr(z), z.stride(0),
                                                   _ptr(b_rkv) if b_rkv is not None else None,
                                                   _ptr(b_rq) if b_rq is not None else None, _ptr(gkv), _ptr(rq),
                                                   _stream(z)), "llattn_pool_proj_fwd")
    return gkv, rq


@pool_proj_fwd.register_fake
def _pool_proj_fwd_fake(z, b_rkv, b_rq, batch, latent_heads, latent_tokens, query_block):
    Ld, T = z.shape[1] // 3, z.shape[0] // batch
    geo = geometry(T, latent_tokens, query_block)
    return z.new_empty(batch, geo["n_chunks"], 2 * Ld), z.new_empty(batch, geo["n_qrows"], Ld)


@torch.library.custom_op("llattn_b200::pool_proj_bwd", mutates_args=(), device_types="cuda")
def pool_proj_bwd(dgkv: Tensor, drq: Tensor, seq_len: int, latent_heads: int, latent_tokens: int,
                  query_block: int) -> Tensor:
    """dgkv [B, Nc, 2Ld], drq [B, Tq, Ld] -> dz [B*T, 3Ld], the gradient of
    pool_proj_fwd with respect to z."""
    _require(dgkv.is_contiguous() and drq.is_contiguous() and dgkv.dtype == drq.dtype,
             "pool_proj_bwd expects contiguous gradients of one dtype")
    B, Ld = dgkv.shape[0], drq.shape[-1]
    dz = torch.empty(B * seq_len, 3 * Ld, dtype=dgkv.dtype, device=dgkv.device)
    dims = _pp_dims(B, seq_len, latent_heads, Ld, latent_tokens, query_block, dgkv)
    with torch.cuda.device(dgkv.device):
        _lib.check(_lib.lib().llattn_pool_proj_bwd(ctypes.byref(dims), _ptr(dgkv), _ptr(drq), _ptr(dz), dz.stride(0),
                                                   _stream(dgkv)), "llattn_pool_proj_bwd")
    return dz


@torch.library.custom_op("llattn_b200::pool_proj_bwd_into_", mutates_args=("buf",), device_types="cuda")
def pool_proj_bwd_into_(buf: Tensor, dgkv: Tensor, drq: Tensor, col0: int, latent_heads: int, latent_tokens: int,
                        query_block: int) -> None:
    """pool_proj_bwd written into columns [col0, col0 + 3Ld) of a row-major
    [B*T, W] buffer (beside the other per-token gradients held there)."""
    _require(buf.dim() == 2 and buf.is_contiguous() and buf.dtype == dgkv.dtype, "buf must be a contiguous [B*T, W]")
    _require(dgkv.is_contiguous() and drq.is_contiguous() and dgkv.dtype == drq.dtype,
             "pool_proj_bwd expects contiguous gradients of one dtype")
    B, Ld = dgkv.shape[0], drq.shape[-1]
    _require(col0 >= 0 and col0 + 3 * Ld <= buf.shape[1] and buf.shape[0] % B == 0, "pool_proj_bwd_into_: bad columns")
    dims = _pp_dims(B, buf.shape[0] // B, latent_heads, Ld, latent_tokens, query_block, dgkv)
    with torch.cuda.device(buf.device):
        _lib.check(_lib.lib().llattn_pool_proj_bwd(ctypes.byref(dims), _ptr(dgkv), _ptr(drq),
                                                   buf.data_ptr() + col0 * buf.element_size(), buf.stride(0),
                                                   _stream(buf)), "llattn_pool_proj_bwd")


@pool_proj_bwd_into_.register_fake
def _pool_proj_bwd_into_fake(buf, dgkv, drq, col0, latent_heads, latent_tokens, query_block):
    return None


@pool_proj_bwd.register_fake
def _pool_proj_bwd_fake(dgkv, drq, seq_len, latent_heads, latent_tokens, query_block):
    return dgkv.new_empty(dgkv.shape[0] * seq_len, 3 * drq.shape[-1])


# the per-token latent projections cost 3 * 2 M d 3Ld FLOPs over the step
# against the pooled ones' 2 M d Ld plus the x reads of the pooling: they pay
# for small latent widths only
POOL_PROJ_MAX_LATENT = 128


def _fused_projections(x: Tensor, d: int, Ld: int) -> bool:
    """Whether BlockFunction runs qkv_proj and the latent projections as one
    GEMM: small latent widths, and (bf16) 16-byte row strides for the tensor
    maps of the wide rows."""
    return Ld <= POOL_PROJ_MAX_LATENT and (x.dtype != torch.bfloat16 or (3 * d + 3 * Ld) % 8 == 0)


def pool_chunks(x: Tensor, latent_tokens: int) -> Tensor:
    """Chunk means of x [B,T,d] -> [B,Nc,d] (models.py:159-214)."""
    return pool_fwd(x.contiguous(), latent_tokens, 0, _lib.POOL_CHUNKS)


def pool_query_blocks(x: Tensor, latent_tokens: int, query_block: int) -> Tensor:
    """Zero-padded query-block means of x [B,T,d] -> [B,Tq,d] (models.py:216-230)."""
    return pool_fwd(x.contiguous(), latent_tokens, query_block, _lib.POOL_QBLOCKS)


# --------------------------------------------------------------------------
# fused attention core: local + latent + r_out + gate + mix

def _row_stride(t: Tensor) -> int:
    """Row stride of a [B, T, C] tensor whose rows may sit in a wider
    row-major buffer (t = buf[..., :C]); 0 when t is contiguous."""
    if t.is_contiguous():
        return 0
    B, T, C = t.shape
    ok = t.stride(2) == 1 and t.stride(1) >= C and (B == 1 or t.stride(0) == T * t.stride(1))
    _require(ok, "qkv must be contiguous or a column slice [..., :3d] of a row-major [B, T, W] buffer")
    return t.stride(1)


def _core_dims(qkv: Tensor, w_rout: Tensor, n_heads: int, latent_heads: int, window: int,
               local_block: int, latent_tokens: int, query_block: int, gate_bias: float,
               seq_offset: int = 0, total_len: int = 0, dqkv_row_stride: int = 0):
    B, T, three_d = qkv.shape
    d = three_d // 3
    _require(three_d == 3 * d and d % n_heads == 0, "qkv last dim must be 3 * n_heads * head_dim")
    Ld = w_rout.shape[1]
    _require(Ld % latent_heads == 0, "latent_d_model must be divisible by latent_heads")
    return _lib.make_dims(B, T, n_heads, d // n_heads, latent_heads, Ld // latent_heads, window,
                          local_block, latent_tokens, query_block, _dtype_code(qkv), gate_bias,
                          seq_offset, total_len, _row_stride(qkv), dqkv_row_stride)


def _check_core_inputs(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, dims, geo):
    dt = qkv.dtype
    B, T = dims.batch, dims.seq_len
    d, Ld = dims.n_heads * dims.head_dim, dims.latent_heads * dims.latent_head_dim
    for name, t, shape, want in (
        ("qkv", qkv, (B, T, 3 * d), dt), ("rq", rq, (B, geo["n_qrows"], Ld), dt),
        ("gkv", gkv, (B, geo["n_chunks"], 2 * Ld), dt), ("w_rout", w_rout, (d, Ld), dt),
        ("b_rout", b_rout, (d,), torch.float32), ("g_local", g_local, (dims.head_dim,), torch.float32),
        ("g_remote", g_remote, (dims.head_dim,), torch.float32),
    ):
        _require(tuple(t.shape) == shape, f"{name} has shape {tuple(t.shape)}, expected {shape}")
        _require(t.dtype == want, f"{name} has dtype {t.dtype}, expected {want}")
        _require(t is qkv or t.is_contiguous(), f"{name} must be contiguous")
        _require(t.device == qkv.device, f"{name} is on {t.device}, expected {qkv.device}")


@torch.library.custom_op("llattn_b200::attn_fwd", mutates_args=(), device_types="cuda")
def attn_fwd(qkv: Tensor, rq: Tensor, gkv: Tensor, w_rout: Tensor, b_rout: Tensor,
             g_local: Tensor, g_remote: Tensor, n_heads: int, latent_heads: int, window: int,
             local_block: int, latent_tokens: int, query_block: int,
             gate_bias: float, seq_offset: int = 0,
             total_len: int = 0) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    dims = _core_dims(qkv, w_rout, n_heads, latent_heads, window, local_block, latent_tokens,
                      query_block, gate_bias, seq_offset, total_len)
    geo = geometry(dims.seq_len, latent_tokens, query_block, window, local_block, total_len)
    _check_core_inputs(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, dims, geo)
    B, T, H = dims.batch, dims.seq_len, dims.n_heads
    d, Ld, Tq = H * dims.head_dim, w_rout.shape[1], geo["n_qrows"]
    kw = dict(device=qkv.device)
    mixed = torch.empty(B, T, d, dtype=qkv.dtype, **kw)
    local_out = torch.empty(B, T, d, dtype=qkv.dtype, **kw)
    lse = torch.empty(B, H, T, dtype=torch.float32, **kw)
    lat = torch.empty(B, Tq, Ld, dtype=qkv.dtype, **kw)
    lat_lse = torch.empty(B, latent_heads, Tq, dtype=torch.float32, **kw)
    args = _lib.FwdArgs(dims, _ptr(qkv), _ptr(rq), _ptr(gkv), _ptr(w_rout), _ptr(b_rout),
                        _ptr(g_local), _ptr(g_remote), _ptr(mixed), _ptr(local_out), _ptr(lse),
                        _ptr(lat), _ptr(lat_lse))
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.lib().llattn_fwd(ctypes.byref(args), _stream(qkv)), "llattn_fwd")
    return mixed, local_out, lse, lat, lat_lse


@attn_fwd.register_fake
def _attn_fwd_fake(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, n_heads, latent_heads, window,
                   local_block, latent_tokens, query_block, gate_bias, seq_offset=0, total_len=0):
    B, T, three_d = qkv.shape
    d = three_d // 3
    Tq = geometry(T, latent_tokens, query_block, total_len=total_len)["n_qrows"]
    f32 = torch.float32
    return (qkv.new_empty(B, T, d), qkv.new_empty(B, T, d), qkv.new_empty(B, n_heads, T, dtype=f32),
            qkv.new_empty(B, Tq, w_rout.shape[1]), qkv.new_empty(B, latent_heads, Tq, dtype=f32))


@torch.library.custom_op("llattn_b200::attn_bwd", mutates_args=(), device_types="cuda")
def attn_bwd(dmixed: Tensor, qkv: Tensor, rq: Tensor, gkv: Tensor, w_rout: Tensor, b_rout: Tensor,
             g_local: Tensor, g_remote: Tensor, local_out: Tensor, lse: Tensor, lat: Tensor,
             lat_lse: Tensor, n_heads: int, latent_heads: int, window: int, local_block: int,
             latent_tokens: int, query_block: int, gate_bias: float, seq_offset: int = 0,
             total_len: int = 0, dqkv_cols: int = 0,
             want_db_qkv: bool = True) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """The backward of attn_fwd. dqkv_cols > 3d returns dqkv as the first 3d
    columns of a [B, T, dqkv_cols] buffer (the rest unwritten), for a caller
    that puts other per-token gradients beside it; want_db_qkv=False skips
    the qkv bias gradient (the last output is then left unwritten)."""
    B, T, three_d = qkv.shape
    wide = dqkv_cols > three_d
    dims = _core_dims(qkv, w_rout, n_heads, latent_heads, window, local_block, latent_tokens,
                      query_block, gate_bias, seq_offset, total_len, dqkv_cols if wide else 0)
    _require(dmixed.shape == local_out.shape and dmixed.dtype == qkv.dtype and dmixed.is_contiguous(),
             "dmixed must be a contiguous [B, T, d] tensor of the activation dtype")
    d, hd = dims.n_heads * dims.head_dim, dims.head_dim
    kw = dict(device=qkv.device)
    dqkv = torch.empty(B, T, dqkv_cols if wide else three_d, dtype=qkv.dtype, **kw)
    drq = torch.empty_like(rq)
    dgkv = torch.empty_like(gkv)
    dw = torch.empty(w_rout.shape, dtype=torch.float32, **kw)
    db = torch.empty(d, dtype=torch.float32, **kw)
    dgl = torch.empty(hd, dtype=torch.float32, **kw)
    dgr = torch.empty(hd, dtype=torch.float32, **kw)
    dbqkv = torch.empty(3 * d, dtype=torch.float32, **kw)
    ws_bytes = _lib.lib().llattn_bwd_workspace_bytes(ctypes.byref(dims))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, **kw)
    args = _lib.BwdArgs(dims, _ptr(qkv), _ptr(rq), _ptr(gkv), _ptr(w_rout), _ptr(b_rout),
                        _ptr(g_local), _ptr(g_remote), _ptr(local_out), _ptr(lse), _ptr(lat),
                        _ptr(lat_lse), _ptr(dmixed), _ptr(dqkv), _ptr(drq), _ptr(dgkv), _ptr(dw),
                        _ptr(db), _ptr(dgl), _ptr(dgr), _ptr(ws), ws.numel(), _ptr(dbqkv) if want_db_qkv else 0)
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.lib().llattn_bwd(ctypes.byref(args), _stream(qkv)), "llattn_bwd")
    return dqkv, drq, dgkv, dw, db, dgl, dgr, dbqkv


@attn_bwd.register_fake
def _attn_bwd_fake(dmixed, qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, local_out, lse, lat,
                   lat_lse, n_heads, latent_heads, window, local_block, latent_tokens, query_block, gate_bias,
                   seq_offset=0, total_len=0, dqkv_cols=0, want_db_qkv=True):
    f32 = torch.float32
    B, T, three_d = qkv.shape
    return (qkv.new_empty(B, T, max(dqkv_cols, three_d)), torch.empty_like(rq), torch.empty_like(gkv),
            w_rout.new_empty(w_rout.shape, dtype=f32), b_rout.new_empty(b_rout.shape, dtype=f32),
            g_local.new_empty(g_local.shape, dtype=f32), g_remote.new_empty(g_remote.shape, dtype=f32),
            qkv.new_empty(qkv.shape[-1], dtype=f32))


def _attn_setup(ctx, inputs, output):
    qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, *cfg = inputs
    _, local_out, lse, lat, lat_lse = output
    ctx.save_for_backward(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, local_out, lse, lat,
                          lat_lse)
    ctx.cfg = cfg


def _attn_backward(ctx, dmixed, _d_local, _d_lse, _d_lat, _d_lat_lse):
    saved = ctx.saved_tensors
    qkv = saved[0]
    if dmixed is None:
        dmixed = torch.zeros_like(saved[7])
    # (the qkv bias gradient belongs to the caller's qkv projection: not asked for)
    dqkv, drq, dgkv, dw, db, dgl, dgr, _ = attn_bwd(dmixed.to(qkv.dtype).contiguous(), *saved, *ctx.cfg,
                                                    want_db_qkv=False)
    return (dqkv, drq, dgkv, dw.to(saved[3].dtype), db, dgl, dgr) + (None,) * 9


attn_fwd.register_autograd(_attn_backward, setup_context=_attn_setup)


def llattn_attention(qkv: Tensor, rq: Tensor, gkv: Tensor, w_rout: Tensor, b_rout: Tensor,
                     g_local: Tensor, g_remote: Tensor, *, n_heads: int, latent_heads: int,
                     window: int, local_block_size: int, latent_tokens: int,
                     latent_query_block_size: int = 0, gate_bias: float = 0.0) -> Tensor:
    """Differentiable attention core between the projections -> mixed [B,T,d].

    qkv [B,T,3d] (qkv_proj output), rq [B,Tq,Ld] (rq_proj output),
    gkv [B,Nc,2Ld] (rkv_proj output of the chunk means), r_out weight/bias,
    gate vectors [hd]. The activation dtype is qkv's (float32 -> exact SIMT
    kernels, bfloat16 -> tcgen05 kernels); the other tensors are cast to it,
    bias and gates to float32, under autograd."""
    dt = qkv.dtype
    outs = attn_fwd(qkv.contiguous(), rq.to(dt).contiguous(), gkv.to(dt).contiguous(),
                    w_rout.to(dt).contiguous(), b_rout.float().contiguous(),
                    g_local.float().reshape(-1).contiguous(), g_remote.float().reshape(-1).contiguous(),
                    n_heads, latent_heads, window, local_block_size, latent_tokens,
                    latent_query_block_size, float(gate_bias))
    return outs[0]


# --------------------------------------------------------------------------
# whole block: projections, pooling, attention core, output projection

@torch.library.custom_op("llattn_b200::colsum", mutates_args=(), device_types="cuda")
def colsum(g: Tensor) -> Tensor:
    """Column sums of a contiguous [rows, cols] CUDA tensor, in its dtype with
    fp32 accumulation in a fixed order: the bias gradient of a linear layer
    whose output gradient is g (llattn_colsum)."""
    _require(g.dim() == 2 and g.is_contiguous() and g.is_cuda, "colsum expects a contiguous 2-D CUDA tensor")
    rows, cols = g.shape
    code = _dtype_code(g)
    L = _lib.lib()
    ws = torch.empty(max(int(L.llattn_colsum_workspace_bytes(rows, cols, code)), 16), dtype=torch.uint8,
                     device=g.device)
    out = torch.empty(cols, dtype=g.dtype, device=g.device)
    with torch.cuda.device(g.device):
        _lib.check(L.llattn_colsum(_ptr(g), rows, cols, code, _ptr(out), _ptr(ws), ws.numel(), _stream(g)),
                   "llattn_colsum")
    return out


@colsum.register_fake
def _colsum_fake(g):
    return g.new_empty(g.shape[1])


@torch.library.custom_op("llattn_b200::pool_bwd_accumulate", mutates_args=("dx",), device_types="cuda")
def pool_bwd_accumulate_(dx: Tensor, dpooled: Tensor, latent_tokens: int, query_block: int, pool_mode: int) -> None:
    """dx [B,T,d] += the pooling gradient of dpooled [B,rows,d] (in place)."""
    _require(dx.is_contiguous() and dpooled.is_contiguous() and dx.dtype == dpooled.dtype,
             "pool_bwd_accumulate_ expects contiguous tensors of one dtype")
    B, T, d = dx.shape
    dims = _lib.make_dims(B, T, latent_tokens=latent_tokens, query_block=query_block, dtype=_dtype_code(dx))
    with torch.cuda.device(dx.device):
        _lib.check(_lib.lib().llattn_pool_bwd(ctypes.byref(dims), pool_mode | _lib.POOL_ACCUMULATE, _ptr(dpooled),
                                              _ptr(dx), d, _stream(dx)), "llattn_pool_bwd")


@pool_bwd_accumulate_.register_fake
def _pool_bwd_accumulate_fake(dx, dpooled, latent_tokens, query_block, pool_mode):
    return None


class BlockFunction(torch.autograd.Function):
    """The whole attention block (models.py:307-462 with the projections of
    models.py:80-84) as one autograd node, so its backward can fuse what
    autograd would run as separate kernels: x's three gradient contributions
    accumulate in place (the rq_proj input gradient as a beta=1 GEMM into the
    qkv_proj one, the pooling gradients through llattn_pool_bwd's accumulate
    mode) instead of two elementwise adds, and the four bias gradients are
    llattn_colsum reductions. Same math and the same GEMMs as autograd over
    the separate layers; activations, weights and biases share one dtype.

    Inputs: x [B,T,d], then weight/bias of qkv_proj, rq_proj, rkv_proj,
    r_out, the gate_local / gate_remote weights [1, hd], weight/bias of out,
    and cfg = (n_heads, latent_heads, window, local_block_size, latent_tokens,
    latent_query_block_size, gate_bias)."""

    @staticmethod
    def forward(ctx, x, w_qkv, b_qkv, w_rq, b_rq, w_rkv, b_rkv, w_rout, b_rout, g_local, g_remote, w_out,
                b_out, cfg):
        n_heads, latent_heads, window, local_block, latent_tokens, query_block, gate_bias = cfg
        B, T, d = x.shape
        x = x.contiguous()
        F = torch.nn.functional
        Ld = w_rq.shape[0]
        w_cat = None
        if _fused_projections(x, d, Ld):
            # one GEMM for qkv_proj and the per-token latent projections:
            # [qkv | x W_rkv^T | x W_rq^T], whose last 3 Ld columns are pooled
            w_cat = torch.cat([w_qkv, w_rkv, w_rq])
            b_cat = torch.cat([b_qkv, b_qkv.new_zeros(3 * Ld)])
            full = F.linear(x, w_cat, b_cat)
            qkv = full[..., :3 * d]
            gkv, rq = pool_proj_fwd(full.view(B * T, -1)[:, 3 * d:], b_rkv, b_rq, B, latent_heads, latent_tokens,
                                    query_block)
            pooled = qsrc = None
        else:
            qkv = F.linear(x, w_qkv, b_qkv)
            pooled = pool_fwd(x, latent_tokens, 0, _lib.POOL_CHUNKS)
            gkv = F.linear(pooled, w_rkv, b_rkv)
            qsrc = pool_fwd(x, latent_tokens, query_block, _lib.POOL_QBLOCKS) if query_block > 1 else None
            rq = F.linear(x if qsrc is None else qsrc, w_rq, b_rq)
        b_rout_f = b_rout.float().contiguous()
        gl = g_local.float().reshape(-1).contiguous()
        gr = g_remote.float().reshape(-1).contiguous()
        mixed, local_out, lse, lat, lat_lse = attn_fwd(
            qkv, rq, gkv, w_rout.contiguous(), b_rout_f, gl, gr, n_heads, latent_heads, window, local_block,
            latent_tokens, query_block, float(gate_bias))
        y = F.linear(mixed, w_out, b_out)
        ctx.save_for_backward(x, qkv, pooled, qsrc, rq, gkv, mixed, local_out, lse, lat, lat_lse, w_qkv, w_rq,
                              w_rkv, w_rout, b_rout_f, gl, gr, w_out, w_cat)
        ctx.cfg = cfg
        ctx.dtypes = (b_rout.dtype, g_local.dtype, g_local.shape, g_remote.dtype, g_remote.shape)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x, qkv, pooled, qsrc, rq, gkv, mixed, local_out, lse, lat, lat_lse, w_qkv, w_rq, w_rkv, w_rout,
         b_rout_f, gl, gr, w_out, w_cat) = ctx.saved_tensors
        n_heads, latent_heads, window, local_block, latent_tokens, query_block, gate_bias = ctx.cfg
        b_rout_dt, gl_dt, gl_shape, gr_dt, gr_shape = ctx.dtypes
        need = ctx.needs_input_grad
        B, T, d = x.shape
        M, Ld = B * T, w_rq.shape[0]
        dy2 = dy.to(x.dtype).contiguous().view(M, d)
        x2 = x.view(M, d)
        g = [None] * 14
        dmixed = torch.mm(dy2, w_out)
        if need[11]:
            g[11] = torch.mm(dy2.t(), mixed.view(M, d))
        if need[12]:
            g[12] = colsum(dy2)
        fused = w_cat is not None
        dqkv, drq, dgkv, dw_rout, db_rout, dgl, dgr, db_qkv = attn_bwd(
            dmixed.view(B, T, d), qkv, rq, gkv, w_rout, b_rout_f, gl, gr, local_out, lse, lat, lat_lse,
            n_heads, latent_heads, window, local_block, latent_tokens, query_block, float(gate_bias), 0, 0,
            w_cat.shape[0] if fused else 0, not fused)
        drq2 = drq.view(-1, drq.shape[-1])
        dgkv2 = dgkv.view(-1, dgkv.shape[-1])
        if fused:
            # [dqkv | dz] in one buffer: x's gradient is one GEMM against
            # [W_qkv; W_rkv; W_rq] and the three weight gradients one GEMM
            dfull = dqkv.view(M, -1)
            pool_proj_bwd_into_(dfull, dgkv, drq, 3 * d, latent_heads, latent_tokens, query_block)
            if need[0]:
                g[0] = torch.mm(dfull, w_cat).view(B, T, d)
            if need[2] or need[4] or need[6]:
                # the bias gradients as one column sum over the buffer (for
                # rkv: sum_t dgkv[c(t)] / cnt(c), the chunk gradients summed).
                # Block-pooled queries count zero padding, so a ragged last
                # block's bias gradient is its whole drq row, not the
                # n_valid / bs share its tokens carry in dz: rq's own sum then
                db_cat = colsum(dfull)
                g[2] = db_cat[:3 * d] if need[2] else None
                g[6] = db_cat[3 * d:3 * d + 2 * Ld] if need[6] else None
                if need[4]:
                    g[4] = db_cat[3 * d + 2 * Ld:] if query_block <= 1 else colsum(drq2)
            if need[1] or need[3] or need[5]:
                dw_cat = torch.mm(dfull.t(), x2)
                g[1] = dw_cat[:3 * d] if need[1] else None
                g[5] = dw_cat[3 * d:3 * d + 2 * Ld] if need[5] else None
                g[3] = dw_cat[3 * d + 2 * Ld:] if need[3] else None
        else:
            dqkv2 = dqkv.view(M, 3 * d)
            if need[0]:
                dx = torch.mm(dqkv2, w_qkv)
                if qsrc is None:
                    dx.addmm_(drq2, w_rq)
                dx = dx.view(B, T, d)
                if qsrc is not None:
                    pool_bwd_accumulate_(dx, torch.mm(drq2, w_rq).view(B, -1, d), latent_tokens, query_block,
                                         _lib.POOL_QBLOCKS)
                pool_bwd_accumulate_(dx, torch.mm(dgkv2, w_rkv).view(B, -1, d), latent_tokens, 0,
                                     _lib.POOL_CHUNKS)
                g[0] = dx
            if need[1]:
                g[1] = torch.mm(dqkv2.t(), x2)
            if need[3]:
                g[3] = torch.mm(drq2.t(), x2 if qsrc is None else qsrc.view(-1, d))
            if need[5]:
                g[5] = torch.mm(dgkv2.t(), pooled.view(-1, d))
            if need[2]:  # column sums of dqkv, taken by the library's backward
                g[2] = db_qkv.to(dqkv.dtype)
            if need[4]:
                g[4] = colsum(drq2)
            if need[6]:
                g[6] = colsum(dgkv2)
        g[7] = dw_rout.to(w_rout.dtype) if need[7] else None
        g[8] = db_rout.to(b_rout_dt) if need[8] else None
        g[9] = dgl.to(gl_dt).view(gl_shape) if need[9] else None
        g[10] = dgr.to(gr_dt).view(gr_shape) if need[10] else None
        return tuple(g)


def decode_core(qkv_cache: Tensor, seq_len: int, rq_row: Tensor, gkv: Tensor, w_rout: Tensor,
                b_rout: Tensor, g_local: Tensor, g_remote: Tensor, *, n_heads: int, latent_heads: int,
                window: int, local_block_size: int, latent_tokens: int,
                latent_query_block_size: int = 0, gate_bias: float = 0.0) -> Tensor:
    """One decode step of the attention core (no autograd) -> mixed row [B, d].

    The last row (t = seq_len - 1) of ``llattn_attention`` over the
    seq_len-token prefix whose qkv_proj rows fill qkv_cache[:, :seq_len]
    ([B, cache_len, 3d]); rq_row [B, Ld] is the rq_proj row of t's latent
    query and gkv [B, Nc, 2Ld] the rkv_proj output of the prefix's chunk means
    (Nc of seq_len). Launches ``llattn_decode``; CUDA only."""
    dt = qkv_cache.dtype
    _require(qkv_cache.is_cuda, "decode_core needs CUDA tensors")
    _require(qkv_cache.is_contiguous() and qkv_cache.dim() == 3, "qkv_cache must be a contiguous [B, cache_len, 3d]")
    B, cache_len, three_d = qkv_cache.shape
    _require(1 <= seq_len <= cache_len, f"seq_len {seq_len} outside [1, cache_len={cache_len}]")
    d = three_d // 3
    Ld = w_rout.shape[1]
    dims = _lib.make_dims(B, seq_len, n_heads, d // n_heads, latent_heads, Ld // latent_heads, window,
                          local_block_size, latent_tokens, latent_query_block_size, _dtype_code(qkv_cache),
                          float(gate_bias))
    geo = geometry(seq_len, latent_tokens, latent_query_block_size, window, local_block_size)
    rq_row = rq_row.to(dt).reshape(B, Ld).contiguous()
    gkv = gkv.to(dt).contiguous()
    _require(tuple(gkv.shape) == (B, geo["n_chunks"], 2 * Ld),
             f"gkv has shape {tuple(gkv.shape)}, expected {(B, geo['n_chunks'], 2 * Ld)}")
    w = w_rout.to(dt).contiguous()
    b = b_rout.float().contiguous()
    gl = g_local.float().reshape(-1).contiguous()
    gr = g_remote.float().reshape(-1).contiguous()
    out = torch.empty(B, d, dtype=dt, device=qkv_cache.device)
    args = _lib.DecodeArgs(dims, cache_len, _ptr(qkv_cache), _ptr(rq_row), _ptr(gkv), _ptr(w), _ptr(b),
                           _ptr(gl), _ptr(gr), _ptr(out))
    with torch.cuda.device(qkv_cache.device):
        _lib.check(_lib.lib().llattn_decode(ctypes.byref(args), _stream(qkv_cache)), "llattn_decode")
    return out


class LLAttnFunction:
    """Name-compatible entry of the reference's autograd op
    (kernels/llattn_op.py:184-238). ``apply`` takes the PyTorch module's
    tensors (see ``llattn_attention``), not the Triton path's per-head
    Q/K/V/GQ/GK/GV layout, because the PyTorch module is the semantic target."""

    @staticmethod
    def apply(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, n_heads, latent_heads, window,
              local_block_size, latent_tokens, latent_query_block_size=0, gate_bias=0.0):
        return llattn_attention(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, n_heads=n_heads,
                                latent_heads=latent_heads, window=window,
                                local_block_size=local_block_size, latent_tokens=latent_tokens,
                                latent_query_block_size=latent_query_block_size,
                                gate_bias=gate_bias)
