"""CPU restatement of the reference LocalLatentAttention block — TEST INFRASTRUCTURE.

This module is the parity checker for the CUDA kernels of this repository.
Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` legs may import it; the product path never calls it.

It restates, in plain PyTorch on the CPU (any float dtype, float64 for tight
checks), the math of the reference's PyTorch module
``LocalLatentAttention`` (Fenix46/local-latent-attention ``models.py:61-462``).
Each function cites the reference lines it follows. It is pinned against
golden vectors produced by the reference module itself
(``tests/golden/make_golden.py``; checked by ``tests/test_oracle.py``).

Parameters are passed as a dict keyed by the reference's state_dict names
(``qkv_proj.weight``, ``rq_proj.bias``, ... ``gate_local.weight``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class BlockCfg:
    """The ModelConfig fields the block reads (models.py:21-37)."""

    d_model: int
    n_heads: int
    local_window: int
    local_block_size: int = 256
    latent_tokens: int = 16
    latent_d_model: int = 64
    latent_heads: int = 2
    latent_query_block_size: int = 0

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def latent_head_dim(self) -> int:
        return self.latent_d_model // self.latent_heads


def chunk_layout(seq_len: int, latent_tokens: int) -> tuple[int, int]:
    """(chunk size cs, chunk count Nc) — models.py:175-183, 201-212."""
    target = min(latent_tokens, seq_len)
    cs = math.ceil(seq_len / target)
    return cs, math.ceil(seq_len / cs)


def query_block_layout(seq_len: int, qb: int) -> tuple[int, int]:
    """(block size bs, block count) for block-pooled latent queries, models.py:218-219."""
    bs = min(seq_len, qb)
    return bs, math.ceil(seq_len / bs)


def pool_chunks(x: torch.Tensor, cs: int) -> torch.Tensor:
    """Chunk means of x [B,T,d] -> [B,Nc,d]; the last partial chunk is averaged
    over its true token count (models.py:185-199)."""
    B, T, d = x.shape
    nc = math.ceil(T / cs)
    sums = F.pad(x, (0, 0, 0, nc * cs - T)).view(B, nc, cs, d).sum(2)
    counts = (T - torch.arange(nc) * cs).clamp(max=cs).to(x.dtype)
    return sums / counts.view(1, nc, 1)


def chunk_ids(T: int, cs: int, nc: int) -> torch.Tensor:
    """Latent chunk index of each token, models.py:208-212."""
    return (torch.arange(T) // cs).clamp(max=nc - 1)


def pool_query_blocks(x: torch.Tensor, bs: int, token_chunk: torch.Tensor):
    """Zero-padded block means (divisor bs, padding counted) and each block's
    smallest chunk id (models.py:216-230)."""
    B, T, d = x.shape
    nb = math.ceil(T / bs)
    pooled = F.pad(x, (0, 0, 0, nb * bs - T)).view(B, nb, bs, d).sum(2) / bs
    # chunk ids are non-decreasing in t, so a block's min is at its first token
    return pooled, token_chunk[torch.arange(nb) * bs]


def local_allowed(T: int, window: int, local_block_size: int) -> torch.Tensor:
    """Boolean [T,T] mask of the reference's blockwise local attention
    (models.py:245-292): key j is visible from query t iff 0 < t-j <= W and
    j >= max(0, qs(t) - W + 1), qs(t) the start of t's query block of size
    bsL = min(T, max(W, local_block_size))."""
    bsl = min(T, max(window, local_block_size))
    t = torch.arange(T).view(T, 1)
    j = torch.arange(T).view(1, T)
    qs = (t // bsl) * bsl
    dist = t - j
    return (dist > 0) & (dist <= window) & (j >= (qs - window + 1).clamp(min=0))


def local_attention(q, k, v, window: int, local_block_size: int) -> torch.Tensor:
    """Blockwise windowed causal attention, q/k/v [B,H,T,hd] (models.py:232-276).

    Same blocking as the reference: one SDPA per query block of bsL rows over
    keys [max(0, qs-W+1), qe), additive mask allowing 0 < t-j <= W. A query
    with no visible key (t = 0) yields 0 (torch >= 2.5 SDPA semantics)."""
    if window <= 0:
        raise ValueError("local_window must be positive")
    B, H, T, hd = q.shape
    bsl = min(T, max(window, local_block_size))
    out = q.new_empty(B, H, T, hd)
    for qs in range(0, T, bsl):
        qe = min(qs + bsl, T)
        ks = max(0, qs - window + 1)
        tq = torch.arange(qs, qe).view(-1, 1)
        tk = torch.arange(ks, qe).view(1, -1)
        dist = tq - tk
        ok = (dist > 0) & (dist <= window)
        mask = torch.zeros(ok.shape, dtype=q.dtype).masked_fill(~ok, float("-inf"))
        out[:, :, qs:qe] = F.scaled_dot_product_attention(
            q[:, :, qs:qe], k[:, :, ks:qe], v[:, :, ks:qe], attn_mask=mask
        )
    return out


def latent_attention(rq, gk, gv, query_chunk: torch.Tensor) -> torch.Tensor:
    """Causal-chunk latent attention (models.py:361-375).

    rq [B,Lh,Tq,ldh], gk/gv [B,Lh,Nc,ldh]; query row r sees chunks j < qid(r);
    rows with qid = 0 see nothing and output 0."""
    ldh = rq.shape[-1]
    nc = gk.shape[2]
    scores = torch.matmul(rq, gk.transpose(-2, -1)) / math.sqrt(ldh)
    blocked = torch.arange(nc).view(1, -1) >= query_chunk.view(-1, 1)
    valid = (~blocked).any(-1).view(1, 1, -1, 1)
    scores = scores.masked_fill(blocked, float("-inf"))
    scores = torch.where(valid, scores, torch.zeros_like(scores))
    attn = torch.softmax(scores, -1) * valid
    return torch.matmul(attn, gv)


def attention_core(qkv, rq, gkv, w_rout, b_rout, g_local, g_remote, cfg: BlockCfg,
                   seq_len: int, gate_bias: float = 0.0) -> torch.Tensor:
    """Everything between the projections (the part the CUDA op computes).

    qkv [B,T,3d] (qkv_proj output), rq [B,Tq,Ld] (rq_proj output),
    gkv [B,Nc,2Ld] (rkv_proj output) -> mixed [B,T,d].
    Follows models.py:315-319 (split), 333-342 (gk/gv), 348-353 (rq),
    355 (local), 361-375 (latent), 392-414 (r_out + block broadcast),
    417-438 (gate + mix). ``gate_bias`` is added to the local gate logit,
    which equals a forward hook adding it to ``gate_local``'s output."""
    B, T = qkv.shape[0], seq_len
    H, hd, d = cfg.n_heads, cfg.head_dim, cfg.d_model
    Lh, ldh = cfg.latent_heads, cfg.latent_head_dim
    q, k, v = qkv.view(B, T, 3, H, hd).unbind(2)
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    cs, nc = chunk_layout(T, cfg.latent_tokens)
    tok_chunk = chunk_ids(T, cs, nc)
    gk, gv = gkv.view(B, nc, 2, Lh, ldh).unbind(2)
    gk, gv = gk.transpose(1, 2), gv.transpose(1, 2)
    if cfg.latent_query_block_size > 1:
        bs, nb = query_block_layout(T, cfg.latent_query_block_size)
        qid = tok_chunk[torch.arange(nb) * bs]
    else:
        bs, nb, qid = 1, T, tok_chunk
    rqh = rq.view(B, nb, Lh, ldh).transpose(1, 2)
    local = local_attention(q, k, v, cfg.local_window, cfg.local_block_size)
    lat = latent_attention(rqh, gk, gv, qid)
    remote = F.linear(lat.transpose(1, 2).reshape(B, nb, Lh * ldh), w_rout, b_rout)
    if bs > 1:
        reps = torch.full((nb,), bs, dtype=torch.long)
        if T % bs:
            reps[-1] = T % bs
        remote = torch.repeat_interleave(remote, reps, dim=1)
    remote_h = remote.view(B, T, H, hd).transpose(1, 2)
    s_l = torch.matmul(local, g_local.view(hd, 1)) + gate_bias
    s_r = torch.matmul(remote_h, g_remote.view(hd, 1))
    w_l = torch.sigmoid(s_l - s_r)
    mixed = w_l * local + (1.0 - w_l) * remote_h
    return mixed.transpose(1, 2).reshape(B, T, d)


def block_forward(params: dict, x: torch.Tensor, cfg: BlockCfg, gate_bias: float = 0.0):
    """Full LocalLatentAttention.forward (models.py:307-462): projections,
    pooling, the attention core and the output projection."""
    B, T, d = x.shape
    qkv = F.linear(x, params["qkv_proj.weight"], params["qkv_proj.bias"])
    cs, nc = chunk_layout(T, cfg.latent_tokens)
    pooled = pool_chunks(x, cs)
    gkv = F.linear(pooled, params["rkv_proj.weight"], params["rkv_proj.bias"])
    if cfg.latent_query_block_size > 1:
        bs, _ = query_block_layout(T, cfg.latent_query_block_size)
        qsrc, _ = pool_query_blocks(x, bs, chunk_ids(T, cs, nc))
    else:
        qsrc = x
    rq = F.linear(qsrc, params["rq_proj.weight"], params["rq_proj.bias"])
    mixed = attention_core(qkv, rq, gkv, params["r_out.weight"], params["r_out.bias"],
                           params["gate_local.weight"].view(-1),
                           params["gate_remote.weight"].view(-1), cfg, T, gate_bias)
    return F.linear(mixed, params["out.weight"], params["out.bias"])


def init_params(cfg: BlockCfg, seed: int = 0, dtype=torch.float32) -> dict:
    """Parameters drawn like the reference constructor's default nn.Linear init
    (models.py:80-90: kaiming-uniform weights, uniform biases), in the same
    construction order, so seed 0 reproduces the reference module's weights."""
    g = torch.manual_seed(seed)
    d, Ld, hd = cfg.d_model, cfg.latent_d_model, cfg.head_dim
    shapes = [("qkv_proj", 3 * d, d, True), ("rq_proj", Ld, d, True),
              ("rkv_proj", 2 * Ld, d, True), ("r_out", d, Ld, True),
              ("out", d, d, True), ("gate_local", 1, hd, False),
              ("gate_remote", 1, hd, False)]
    p = {}
    for name, fo, fi, bias in shapes:
        w = torch.empty(fo, fi)
        torch.nn.init.kaiming_uniform_(w, a=math.sqrt(5), generator=g)
        p[name + ".weight"] = w
        if bias:
            bound = 1.0 / math.sqrt(fi)
            p[name + ".bias"] = torch.empty(fo).uniform_(-bound, bound, generator=g)
    return {k: v.to(dtype) for k, v in p.items()}


def local_pairs(T: int, window: int, local_block_size: int) -> int:
    """Number of visible (query, key) pairs of one (batch, head) sequence; the
    local branch costs 4*hd FLOPs per pair forward and 8*hd backward."""
    bsl = min(T, max(window, local_block_size))
    total = 0
    for t in range(T):
        qs = (t // bsl) * bsl
        lo = max(0, t - window, qs - window + 1)
        total += max(0, t - lo)
    return total
