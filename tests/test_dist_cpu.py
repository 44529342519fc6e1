"""Data-parallel plumbing (llattn_b200.dist, the reference's dist_utils
API) on world_size-2 gloo process groups on the CPU, including failure
detection: a rank that dies makes the survivor's next collective fail
within the process-group timeout instead of hanging."""

import os
import socket
import sys
import time

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)


def _worker_collectives(rank, world, port, q):
    _env(rank, world, port)
    import llattn_b200.dist as D

    try:
        D.setup_distributed("gloo", timeout_s=30)
        t = torch.full((4,), float(rank + 1))
        D.all_reduce_mean(t)
        ok_mean = torch.allclose(t, torch.full((4,), 1.5))
        s = torch.tensor([float(rank)])
        D.all_reduce_sum(s)
        # DDP: no_sync skips the all-reduce, the final micro-step syncs
        model = torch.nn.Linear(3, 1, bias=False)
        with torch.no_grad():
            model.weight.fill_(1.0)
        ddp = torch.nn.parallel.DistributedDataParallel(model)
        x = torch.full((1, 3), float(rank + 1))
        with D.maybe_no_sync(ddp, sync=False):
            ddp(x).sum().backward()
        local = model.weight.grad.clone()
        model.weight.grad = None
        with D.maybe_no_sync(ddp, sync=True):
            ddp(x).sum().backward()
        synced = model.weight.grad.clone()
        q.put((rank, ok_mean, s.item(), local.tolist(), synced.tolist(), D.unwrap(ddp) is model,
               D.get_world_size(), D.is_main_process()))
        D.cleanup_distributed()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_gloo_collectives_and_no_sync():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_collectives, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert len(res[r]) == 8, res[r]
        _, ok_mean, ssum, local, synced, unwrapped, world, main = res[r]
        assert ok_mean and ssum == 1.0 and unwrapped and world == 2 and main == (r == 0)
        assert local == [[float(r + 1)] * 3]       # no sync: own gradient
        assert synced == [[1.5, 1.5, 1.5]]         # synced: mean over ranks


def _worker_failure(rank, world, port, q):
    _env(rank, world, port)
    import llattn_b200.dist as D

    D.setup_distributed("gloo", timeout_s=5)
    if rank == 1:
        os._exit(3)  # the rank dies between steps, with nothing in flight
    t0 = time.time()
    try:
        D.all_reduce_mean(torch.ones(2))
        q.put(("no error", time.time() - t0))
    except Exception as e:
        q.put((type(e).__name__, time.time() - t0))


def test_dead_rank_fails_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_failure, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert kind != "no error"
    assert waited < 60


def test_helpers_outside_torchrun():
    sys.path.insert(0, ROOT)
    import llattn_b200.dist as D

    for k in ("RANK", "WORLD_SIZE"):
        os.environ.pop(k, None)
    assert not D.launched_under_torchrun()
    assert D.get_rank() == 0 and D.get_world_size() == 1
    t = torch.ones(3)
    assert D.all_reduce_mean(t) is t
    D.barrier()
    dev = D.setup_distributed("gloo")
    assert dev.type in ("cpu", "cuda")


def test_numa_mask_decoding_and_fake_nvml_binding(monkeypatch):
    """bind_to_gpu_numa: decodes NVML's CPU mask, binds the process to those
    CPUs (restored after the test), and is a no-op when NVML fails."""
    import os
    import types

    from llattn_b200 import dist as D

    assert D.mask_to_cpus([0b1011]) == [0, 1, 3]
    assert D.mask_to_cpus([0, 1]) == [64]
    allowed = sorted(os.sched_getaffinity(0))
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1b, pci_device_id=0)
    monkeypatch.setattr("torch.cuda.get_device_properties", lambda i: props)
    seen = {}

    class FakeNvml:
        def nvmlInit(self):
            pass

        def nvmlShutdown(self):
            pass

        def nvmlDeviceGetHandleByPciBusId(self, bus):
            seen["bus"] = bus
            return "h"

        def nvmlDeviceGetCpuAffinity(self, handle, n):
            return [1 << allowed[0]] + [0] * (n - 1)

    try:
        assert D.bind_to_gpu_numa(0, nvml=FakeNvml()) == [allowed[0]]
        assert seen["bus"] == "00000000:1b:00.0"
        assert os.sched_getaffinity(0) == {allowed[0]}
    finally:
        os.sched_setaffinity(0, allowed)

    class Broken(FakeNvml):
        def nvmlDeviceGetHandleByPciBusId(self, bus):
            raise RuntimeError("no such device")

    assert D.bind_to_gpu_numa(0, nvml=Broken()) is None
    assert sorted(os.sched_getaffinity(0)) == allowed
