"""Sequence shards through the C ABI on one GPU: a sequence split into three
shards, each run with the halo of W rows before it and its global
offset (llattn_dims.seq_offset / total_len), gives the rows of the whole
sequence's forward, and the shards' backward outputs (halo rows' dK / dV
returned to their owner, gk / gv gradients summed) give its gradients. This
is the kernel-level half of llattn_b200.seqpar, without the collectives
(which test_seqpar_cpu.py checks on gloo ranks)."""

import math

import pytest
import torch

from parity import TOL, frob_err, rel_err

pytestmark = pytest.mark.gpu

CASES = [
    # dtype, T, H, hd, W, LBS, Nl, Lh, ldh, QB
    (torch.bfloat16, 1536, 2, 128, 256, 256, 32, 2, 32, 0),   # fused gate epilogue
    (torch.bfloat16, 1536, 2, 88, 300, 200, 40, 8, 64, 64),   # padded head dim, general path, query blocks
    (torch.float32, 1200, 2, 64, 128, 256, 16, 2, 16, 0),     # exact SIMT path
    (torch.bfloat16, 1536, 2, 128, 256, 256, 200, 2, 32, 0),  # 192 chunks: the tensor-core long-latent kernels
    (torch.bfloat16, 1536, 2, 64, 128, 256, 300, 1, 64, 64),  # 256 chunks with query blocks
]


@pytest.mark.parametrize("case", CASES, ids=["bf16-fused", "bf16-general-qb", "fp32", "bf16-long-latent",
                                             "bf16-long-latent-qb"])
def test_shards_with_halo_equal_the_whole_sequence(case):
    from llattn_b200.seqpar import halo_rows

    dt, T, H, hd, W, LBS, Nl, Lh, ldh, QB = case
    B, R = 2, 3
    Tl = T // R
    d, Ld = H * hd, Lh * ldh
    cs = math.ceil(T / min(Nl, T))
    nc = math.ceil(T / cs)
    qbs = min(T, QB) if QB > 1 else 1
    tq = math.ceil(T / qbs)
    gen = torch.Generator().manual_seed(0)
    f = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    act = lambda t: t.to(dt).cuda()  # noqa: E731
    qkv, rq, gkv = act(f(B, T, 3 * d)), act(f(B, tq, Ld)), act(f(B, nc, 2 * Ld))
    w, b = act(f(d, Ld) / math.sqrt(Ld)), (f(d) * 0.1).cuda()
    gl, gr = (f(hd) / math.sqrt(hd)).cuda(), (f(hd) / math.sqrt(hd)).cuda()
    dm = act(f(B, T, d))
    cfg = (H, Lh, W, LBS, Nl, QB, 0.0)
    full = torch.ops.llattn_b200.attn_fwd(qkv, rq, gkv, w, b, gl, gr, *cfg)
    gfull = torch.ops.llattn_b200.attn_bwd(dm, qkv, rq, gkv, w, b, gl, gr, *full[1:], *cfg)
    acc = [torch.zeros(t.shape, dtype=torch.float32, device="cuda") for t in gfull]
    h = halo_rows(W, QB, T)
    tol = TOL[dt]
    for r in range(R):
        p0 = r * Tl
        hv = min(p0, h)
        s0 = p0 - hv
        qkv_v, rq_v = qkv[:, s0:p0 + Tl].contiguous(), rq[:, s0 // qbs:(p0 + Tl) // qbs].contiguous()
        out = torch.ops.llattn_b200.attn_fwd(qkv_v, rq_v, gkv, w, b, gl, gr, *cfg, s0, T)
        assert rel_err(out[0][:, hv:], full[0][:, p0:p0 + Tl]) <= tol
        assert rel_err(out[1][:, hv:], full[1][:, p0:p0 + Tl]) <= tol
        lse, lse_full = out[2][:, :, hv:], full[2][:, :, p0:p0 + Tl]
        fin = torch.isfinite(lse_full)
        assert torch.equal(fin, torch.isfinite(lse)) and (lse[fin] - lse_full[fin]).abs().max() < 1e-2
        dm_v = dm[:, s0:p0 + Tl].clone()
        dm_v[:, :hv] = 0  # the halo rows' outputs are not this shard's
        g = torch.ops.llattn_b200.attn_bwd(dm_v, qkv_v, rq_v, gkv, w, b, gl, gr, *out[1:], *cfg, s0, T)
        acc[0][:, s0:p0 + Tl] += g[0].float()
        acc[1][:, s0 // qbs:(p0 + Tl) // qbs] += g[1].float()
        for i in range(2, 8):
            acc[i] += g[i].float()
    names = ["dqkv", "drq", "dgkv", "dw_rout", "db_rout", "dg_local", "dg_remote", "db_qkv"]
    for name, a, b_ in zip(names, acc, gfull):
        assert rel_err(a, b_.float()) <= tol, (name, rel_err(a, b_.float()))
        assert frob_err(a, b_.float()) <= tol, (name, frob_err(a, b_.float()))


def _sp_worker(rank, world, port, q):
    import os
    import sys

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests"))
    import datetime

    import torch.distributed as dist

    import llattn_b200
    from llattn_b200.seqpar import sequence_parallel_forward
    from parity import model_config

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=120))
        import llattn_oracle as O
        from parity import make_cfg

        B, T, cfg = make_cfg(dict(B=2, T=2048, d_model=512, n_heads=4, local_window=256, latent_tokens=64,
                                  latent_d_model=64, latent_heads=2))
        torch.manual_seed(0)
        m = llattn_b200.LocalLatentAttentionB200(model_config(cfg)).cuda().to(torch.bfloat16)
        gen = torch.Generator().manual_seed(1)
        x = torch.randn(B, T, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()
        g = torch.randn(B, T, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()
        Tl = T // world
        xs = x[:, rank * Tl:(rank + 1) * Tl].clone().requires_grad_(True)
        y = sequence_parallel_forward(m, xs)
        y.backward(g[:, rank * Tl:(rank + 1) * Tl])
        grads = torch.cat([p.grad.float().reshape(-1) for p in m.parameters()])
        dist.all_reduce(grads)
        out = (y.detach().cpu(), xs.grad.cpu(), grads.cpu())
        if rank == 0:  # the whole sequence on one device
            m.zero_grad()
            xf = x.clone().requires_grad_(True)
            yf = m(xf)
            yf.backward(g)
            gf = torch.cat([p.grad.float().reshape(-1) for p in m.parameters()])
            out = out + (yf.detach().cpu(), xf.grad.cpu(), gf.cpu())
        # by value (numpy): a tensor would travel as a shared-memory handle
        # that is gone once this process exits
        q.put((rank,) + tuple(t.float().numpy().copy() for t in out))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, traceback.format_exc()))


def test_sequence_parallel_two_gpus_equals_one_device():
    """llattn_b200.seqpar on 2 GPUs (NCCL: halo exchange and chunk-sum
    all-reduce) against the module on the whole sequence on one device: each
    rank's rows, dx and the group-summed parameter gradients within 2e-2."""
    import socket

    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_sp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        item = q.get(timeout=300)
        assert len(item) > 2, item[1]
        res[item[0]] = tuple(torch.from_numpy(a) for a in item[1:])
    for p in ps:
        p.join(timeout=60)
    yf, dxf, gf = res[0][3:]
    Tl = yf.shape[1] // world
    tol = TOL[torch.bfloat16]
    for r in range(world):
        y, dx, grads = res[r][:3]
        assert rel_err(y.float(), yf[:, r * Tl:(r + 1) * Tl].float()) <= tol
        assert rel_err(dx.float(), dxf[:, r * Tl:(r + 1) * Tl].float()) <= tol
        assert rel_err(grads, gf) <= tol and frob_err(grads, gf) <= tol
