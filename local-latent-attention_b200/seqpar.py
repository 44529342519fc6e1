"""Sequence (context) parallelism for the attention block: one long sequence
split over the ranks of a process group, each rank holding a contiguous
shard of tokens.

The reference runs a whole sequence on one device (models.py:307-462); this
is the long-context extension of its blockwise local attention: every
shard's queries need the W keys before the shard, and every query sees
the latent chunks of the whole prefix. Per rank r (shard of Tl tokens at
global position p0 = r * Tl of a T = R * Tl token sequence):

  * local branch: the previous rank sends its last h rows of qkv (the halo,
    h = W rounded up to the query block), and the library runs the shard
    with that halo in front, told its global offset (llattn_dims.seq_offset
    / total_len), so masks and block spans follow global positions. The
    halo rows' outputs are dropped; in the backward their dK / dV go back to
    the previous rank (and their dQ is zero).
  * latent branch: each rank sums its tokens per global chunk; one
    all-reduce gives every rank the chunk sums of the whole sequence, hence
    the same pooled rows and gk / gv; the backward all-reduces their
    gradient (torch.distributed.nn's differentiable all_reduce).
  * projections and everything else are per-token and stay local.

After the backward the parameter gradients of the ranks are partial sums
over their shards: their sum over the group (all_reduce SUM) is the gradient
of the whole sequence. Collectives: one P2P halo exchange and one
all-reduce of [B, Nc, d] chunk sums per forward, the same per backward.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor

from . import ops


def halo_rows(window: int, query_block: int, total_len: int) -> int:
    """Rows of qkv a shard needs from before its first token: the W keys a
    query can reach back (0 < t - j <= W, models.py:286-292), rounded up to
    whole query blocks (a shard's offset must be a multiple of the query
    block)."""
    need = max(window, 0)
    qbs = min(total_len, query_block) if query_block > 1 else 1
    return -(-need // qbs) * qbs


class HaloExchange(torch.autograd.Function):
    """[halo | local] rows: rank r receives the last h rows of rank r - 1's
    tensor (h = 0 on rank 0) and sends its own last h rows to rank r + 1. The
    backward returns the halo rows' gradient to their owner, which adds it to
    its last h rows."""

    @staticmethod
    def forward(ctx, t: Tensor, h: int, group) -> Tensor:
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        ctx.h, ctx.group = h, group
        B, _, C = t.shape
        recv = t.new_empty(B, h, C) if rank > 0 else t.new_empty(B, 0, C)
        p2p = []
        if rank + 1 < world and h:
            p2p.append(dist.P2POp(dist.isend, t[:, -h:].contiguous(), dist.get_global_rank(group, rank + 1), group))
        if rank > 0 and h:
            p2p.append(dist.P2POp(dist.irecv, recv, dist.get_global_rank(group, rank - 1), group))
        for req in dist.batch_isend_irecv(p2p) if p2p else []:
            req.wait()
        return torch.cat([recv, t], dim=1)

    @staticmethod
    def backward(ctx, g: Tensor):
        h, group = ctx.h, ctx.group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        mine = h if rank > 0 else 0
        g_local = g[:, mine:].contiguous()
        back = g.new_empty(g.shape[0], h, g.shape[2])
        p2p = []
        if rank > 0 and h:
            p2p.append(dist.P2POp(dist.isend, g[:, :h].contiguous(), dist.get_global_rank(group, rank - 1), group))
        if rank + 1 < world and h:
            p2p.append(dist.P2POp(dist.irecv, back, dist.get_global_rank(group, rank + 1), group))
        for req in dist.batch_isend_irecv(p2p) if p2p else []:
            req.wait()
        if rank + 1 < world and h:
            g_local[:, -h:] += back
        return g_local, None, None


def chunk_sums(x: Tensor, p0: int, total_len: int, latent_tokens: int) -> tuple[Tensor, Tensor]:
    """Per-chunk sums of this shard's tokens [B, Nc, d] with the chunking of
    the whole sequence (models.py:159-214: cs = ceil(T / min(Nl, T)), the
    last chunk holding the remainder), and the chunks' token counts [Nc]."""
    geo = ops.geometry(total_len, latent_tokens, 0)
    cs, nc = geo["chunk"], geo["n_chunks"]
    pos = torch.arange(p0, p0 + x.shape[1], device=x.device)
    cid = torch.clamp(pos // cs, max=nc - 1)
    sums = x.new_zeros(x.shape[0], nc, x.shape[2]).index_add(1, cid, x)
    allpos = torch.arange(total_len, device=x.device)
    counts = torch.bincount(torch.clamp(allpos // cs, max=nc - 1), minlength=nc).to(x.dtype)
    return sums, counts


def sequence_parallel_forward(module, x: Tensor, group=None) -> Tensor:
    """This rank's rows of module(x_full), for x = the rank's contiguous
    shard [B, Tl, d] of a sequence split evenly over the group (rank order =
    sequence order). `module` is a LocalLatentAttentionB200 (the same weights
    on every rank). Differentiable; parameter gradients are per-shard partial
    sums (sum them over the group). Under autocast the block runs in the
    autocast dtype, as the single-device module does."""
    import torch.distributed.nn.functional as dnnf

    group = group or dist.group.WORLD
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, Tl, d = x.shape
    T, p0 = world * Tl, rank * Tl
    W, LBS, Nl, QB = module.window, module.local_block_size, module.latent_tokens, module.latent_query_block_size
    h = halo_rows(W, QB, T)
    if rank > 0 and h > Tl:
        raise ValueError(f"sequence parallel: the halo ({h} rows) exceeds a shard ({Tl} tokens)")
    qbs = min(T, QB) if QB > 1 else 1
    if Tl % qbs:
        raise ValueError(f"sequence parallel: shard length {Tl} is not a multiple of the query block {qbs}")
    dt = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype
    with torch.autocast("cuda", enabled=False):
        cast = lambda p: p.to(dt)  # noqa: E731
        xx = x.to(dt)
        qkv = F.linear(xx, cast(module.qkv_proj.weight), cast(module.qkv_proj.bias))
        qkv_v = HaloExchange.apply(qkv, h, group)
        hv = h if rank > 0 else 0
        # latent memory: chunk sums of the whole sequence on every rank
        sums, counts = chunk_sums(xx.float(), p0, T, Nl)
        sums = dnnf.all_reduce(sums, group=group)
        pooled = (sums / counts.view(1, -1, 1)).to(dt)
        gkv = F.linear(pooled, cast(module.rkv_proj.weight), cast(module.rkv_proj.bias))
        qsrc = ops.pool_query_blocks(xx, Nl, QB) if qbs > 1 else xx
        rq = F.linear(qsrc, cast(module.rq_proj.weight), cast(module.rq_proj.bias))
        rq_v = torch.cat([rq.new_zeros(B, hv // qbs, rq.shape[2]), rq], dim=1)
        mixed_v = ops.attn_fwd(qkv_v.contiguous(), rq_v.contiguous(), gkv.contiguous(),
                               cast(module.r_out.weight).contiguous(), module.r_out.bias.float().contiguous(),
                               module.gate_local.weight.float().reshape(-1).contiguous(),
                               module.gate_remote.weight.float().reshape(-1).contiguous(), module.n_heads,
                               module.latent_heads, W, LBS, Nl, QB, float(module.gate_bias), p0 - hv, T)[0]
        mixed = mixed_v[:, hv:]
        return F.linear(mixed, cast(module.out.weight), cast(module.out.bias))
