"""Host-side plumbing of sequence parallelism (llattn_b200.seqpar) on
world_size-2 gloo process groups on the CPU: the halo exchange and the
chunk sums of the latent memory, forward and backward, against the same
operations on the whole sequence in one process."""

import os
import socket
import sys

import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import torch.distributed.nn.functional as dnnf

    from llattn_b200 import seqpar

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        B, T, C, h, Nl = 2, 40, 6, 7, 6
        Tl = T // world
        gen = torch.Generator().manual_seed(0)
        full = torch.randn(B, T, C, generator=gen)
        gfull = torch.randn(B, T + h * (world - 1), C, generator=gen)  # upstream grads of every rank's [halo|local]
        mine = full[:, rank * Tl:(rank + 1) * Tl].clone().requires_grad_(True)
        v = seqpar.HaloExchange.apply(mine, h, dist.group.WORLD)
        start = max(0, rank * Tl - h)
        fwd_ok = torch.equal(v, full[:, start:(rank + 1) * Tl])
        # rank r's [halo | local] block of upstream gradients, laid out per rank
        off = sum(Tl + (h if r > 0 else 0) for r in range(rank))
        gv = gfull[:, off:off + v.shape[1]]
        v.backward(gv)
        # chunk sums of the whole sequence through the differentiable all-reduce
        x = full[:, rank * Tl:(rank + 1) * Tl].clone().requires_grad_(True)
        sums, counts = seqpar.chunk_sums(x, rank * Tl, T, Nl)
        sums = dnnf.all_reduce(sums)
        w = torch.randn(sums.shape, generator=torch.Generator().manual_seed(1))
        (sums * w).sum().backward()
        # by value (numpy): a tensor would travel as a shared-memory handle
        # that is gone once this process exits
        q.put((rank, fwd_ok, *(t.detach().numpy().copy() for t in (mine.grad, sums, counts, x.grad))))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_halo_exchange_and_chunk_sums_two_ranks():
    import llattn_b200.seqpar as sp

    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        item = q.get(timeout=120)
        assert len(item) > 2, item
        res[item[0]] = (item[1], *(torch.from_numpy(a) for a in item[2:]))
    for p in ps:
        p.join(timeout=60)
    B, T, C, h, Nl = 2, 40, 6, 7, 6
    Tl = T // world
    gen = torch.Generator().manual_seed(0)
    full = torch.randn(B, T, C, generator=gen)
    gfull = torch.randn(B, T + h * (world - 1), C, generator=gen)
    # expected gradient of each token: its own row of its rank's block plus, for
    # the last h rows of rank 0, the halo rows of rank 1's block
    g0 = gfull[:, :Tl].clone()
    g1 = gfull[:, Tl:Tl + h + Tl]
    g0[:, -h:] += g1[:, :h]
    want = [g0, g1[:, h:]]
    sums_ref = torch.zeros(B, 0)
    geo = __import__("llattn_b200").ops.geometry(T, Nl, 0)
    cs, nc = geo["chunk"], geo["n_chunks"]
    cid = torch.clamp(torch.arange(T) // cs, max=nc - 1)
    sums_ref = torch.zeros(B, nc, C).index_add(1, cid, full)
    w = torch.randn(B, nc, C, generator=torch.Generator().manual_seed(1))
    for r in range(world):
        fwd_ok, grad, sums, counts, xgrad = res[r]
        assert fwd_ok
        assert torch.allclose(grad, want[r])
        assert torch.allclose(sums, sums_ref, atol=1e-5)
        assert torch.equal(counts, torch.bincount(cid, minlength=nc).float())
        # d(sum(all_reduce(S) * w))/dx: every rank's w, all-reduced = world * w gathered at the token's chunk
        assert torch.allclose(xgrad, (world * w)[:, cid[r * Tl:(r + 1) * Tl]], atol=1e-5)
    assert sp.halo_rows(256, 0, 4096) == 256 and sp.halo_rows(300, 64, 4096) == 320
