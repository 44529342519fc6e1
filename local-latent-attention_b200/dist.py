"""Distributed plumbing of the data-parallel harness (the reference's
dist_utils.py:28-165, same function names and behaviour).

One process per GPU, launched by torchrun; NCCL over NVLink on GPUs, gloo
on CPU (used by the tests). Outside torchrun every function is a no-op.
"""

from __future__ import annotations

import contextlib
import datetime
import os
from typing import Iterator

import torch
import torch.distributed as dist


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank() -> int:
    return dist.get_rank() if is_distributed() else 0


def get_world_size() -> int:
    return dist.get_world_size() if is_distributed() else 1


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def is_main_process() -> bool:
    return get_rank() == 0


def launched_under_torchrun() -> bool:
    return "RANK" in os.environ and "WORLD_SIZE" in os.environ


def setup_distributed(backend: str = "nccl", timeout_s: float | None = None) -> torch.device:
    """Initialise the process group from torchrun's environment (dist_utils.py:61-88).

    Unlike the reference, a `timeout_s` can bound every collective, so a rank
    that dies or stops participating surfaces as an error on the others
    instead of a hang; and backend "gloo" runs on CPU."""
    if not launched_under_torchrun():
        return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    kw = {}
    if timeout_s is not None:
        kw["timeout"] = datetime.timedelta(seconds=timeout_s)
    if backend == "nccl":
        if not torch.cuda.is_available():
            raise RuntimeError("torchrun launched with backend nccl but CUDA is unavailable")
        local = get_local_rank()
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        dist.init_process_group(backend="nccl", init_method="env://", device_id=device, **kw)
        dist.barrier(device_ids=[local])
        return device
    dist.init_process_group(backend=backend, init_method="env://", **kw)
    dist.barrier()
    return torch.device("cpu")


def cleanup_distributed() -> None:
    if is_distributed():
        dist.destroy_process_group()


def all_reduce_mean(tensor: torch.Tensor) -> torch.Tensor:
    """In-place SUM all-reduce divided by the world size (dist_utils.py:99-109)."""
    if not is_distributed():
        return tensor
    dist.all_reduce(tensor, op=dist.ReduceOp.SUM)
    tensor.div_(get_world_size())
    return tensor


def all_reduce_sum(tensor: torch.Tensor) -> torch.Tensor:
    if not is_distributed():
        return tensor
    dist.all_reduce(tensor, op=dist.ReduceOp.SUM)
    return tensor


def barrier() -> None:
    if is_distributed():
        dist.barrier()


@contextlib.contextmanager
def maybe_no_sync(model: torch.nn.Module, sync: bool) -> Iterator[None]:
    """DDP gradient sync off for non-final micro-steps (dist_utils.py:127-144)."""
    no_sync = getattr(model, "no_sync", None)
    if not sync and no_sync is not None and is_distributed():
        with no_sync():
            yield
    else:
        yield


def unwrap(model: torch.nn.Module) -> torch.nn.Module:
    """Strip torch.compile and DDP wrappers (dist_utils.py:147-165)."""
    inner = model
    while True:
        if hasattr(inner, "_orig_mod"):
            inner = inner._orig_mod
            continue
        if isinstance(inner, torch.nn.parallel.DistributedDataParallel):
            inner = inner.module
            continue
        return inner


def mask_to_cpus(words, bits_per_word: int = 64) -> list[int]:
    """CPU ids set in an NVML affinity mask (a list of words, CPU 0 = bit 0
    of word 0)."""
    return [w * bits_per_word + b for w, word in enumerate(words) for b in range(bits_per_word) if (int(word) >> b) & 1]


def bind_to_gpu_numa(device_index: int, nvml=None) -> list[int] | None:
    """Pin this process to the CPUs that NVML reports as local to the GPU
    (nvmlDeviceGetCpuAffinity), so that host memory it allocates afterwards
    (pinned staging buffers) lands on the GPU's NUMA node and its host-device
    copies do not cross the socket link. Changes only this process's CPU
    affinity, never a GPU setting. Returns the CPUs bound to, or None (NVML
    or the affinity call unavailable: nothing changed)."""
    try:
        if nvml is None:
            import pynvml as nvml
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        nvml.nvmlInit()
        try:
            handle = nvml.nvmlDeviceGetHandleByPciBusId(bus)
            n_cpu = os.cpu_count() or 1
            words = nvml.nvmlDeviceGetCpuAffinity(handle, (n_cpu + 63) // 64)
        finally:
            nvml.nvmlShutdown()
        cpus = [c for c in mask_to_cpus(words) if c < n_cpu]
        allowed = os.sched_getaffinity(0)
        cpus = [c for c in cpus if c in allowed]
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return cpus
    except Exception:  # noqa: BLE001 - best effort: no NVML, no PCI ids, no permission
        return None
