"""Benchmark of the LocalLatentAttention block on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg2|cfg3|cfg1|cfg5_nl512|p055|p060] [--no-cpu-baseline]
                    [--no-lm] [--no-presets] [--lm-steps S]

A step is one forward + backward of the drop-in block (LocalLatentAttentionB200:
cuBLAS projections + the libllattn kernels) over one batch of the configured
shape, bf16, with a seeded synthetic input and upstream gradient. Default
workload: cfg2 (B16 T2048 d1536 H12 W256 Nl64 Ld64 Lh2, token-wise latent
queries). Under torchrun each rank runs its own batch (weak scaling) and
all-reduces the block's parameter gradients with NCCL (all_reduce_mean), the
data-parallel exchange of the reference's DDP training. `value` is the whole
job's tokens/s (all ranks); `value_per_gpu` divides it by the GPU count.

Keys beyond the base contract:
  e2e           same metric through the public module API with the step's
                inputs (x, upstream grad) copied from pinned host memory and
                dx copied back, inside the timed region; copy_ms_per_step is
                the same copies alone on the same streams (all ranks at
                once), the host-link bound of the e2e figure
  sustained     the same step repeated for >= 2 s of device time, with its
                own clock samples (the K-step figure is a burst)
  roofline      dominant kernel: its algorithmic FLOPs (local branch: 4*hd*P
                per launch, P = visible query/key pairs) and bytes per launch;
                the bound is the roof whose ideal time is longer; achieved =
                that amount over the kernel's CUDA-event time, against
                MEASURED_PEAKS.json; traffic = DRAM bytes per launch from the
                committed ncu capture (profiles/traffic.json)
  local_branch  local fwd + bwd kernels against the dense-bf16 peak
  cpu_baseline  the CPU oracle (a restatement of the reference PyTorch block)
                on the host cores, bounded sample
  kernels       per-kernel-group event times (ms per step) and launch counts
  graphed       the same step captured once as a CUDA graph and replayed
                (1 GPU): the launch-overhead-free time, for small shapes
  configs       cfg3 (B2 T16384, 256 chunks, query blocks of 64) and cfg5_nl512
                (B4 T8192 W1024, 512 chunks) measured the same way, with their
                kernel groups (rank 0, 1 GPU each)
  presets       the block at the reference's training presets (train.py:71-92:
                0.55b d1408 H16 hd88 latent 512/8 heads, 0.60b d1536 H16 hd96
                latent 384/8 heads) at B16 x T2048, with their kernel groups
  lm            cfg4: the LocalLatentLM training step (24 layers, d1536, B16 x
                T2048 per GPU, AdamW, DDP) at the same N, its own e2e; each
                decoder layer under torch.compile (inductor fuses the norms,
                MLP activation, residual adds and casts; the attention is the
                library's kernels, opaque custom ops in the graph), as the
                reference's published LM numbers use torch.compile;
                --lm-compile 0 for the eager harness
  lm_0.55b      the same step for the reference's 0.55b preset (22 layers,
                d1408, H16, latent 512 over 8 heads), with vs_published = per-GPU
                tok/s over the reference's published 108k tok/s/GPU (H200)
  clocks        nvidia-smi samples taken during the timed region

--impl reference times the reference's CPU implementation of the path on a
bounded sample: its own LocalLatentAttention (models.py) when the reference
is installed in baseline/_ref, else the oracle port; under torchrun only rank
0 runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "cfg1": dict(B=2, T=512, d_model=256, n_heads=4, local_window=128, local_block_size=256,
                 latent_tokens=16, latent_d_model=32, latent_heads=2, latent_query_block_size=0),
    "cfg2": dict(B=16, T=2048, d_model=1536, n_heads=12, local_window=256, local_block_size=256,
                 latent_tokens=64, latent_d_model=64, latent_heads=2, latent_query_block_size=0),
    "cfg3": dict(B=2, T=16384, d_model=1024, n_heads=8, local_window=512, local_block_size=256,
                 latent_tokens=256, latent_d_model=64, latent_heads=2, latent_query_block_size=64),
    # the shape sweep's 512-latent corner (B*T = 32k, 8 heads of 128, the wide
    # window): the point where the latent branch is largest
    "cfg5_nl512": dict(B=4, T=8192, d_model=1024, n_heads=8, local_window=1024, local_block_size=256,
                       latent_tokens=512, latent_d_model=64, latent_heads=2, latent_query_block_size=0),
    # the block of the reference's training presets (train.py:71-92) at the cfg2 batch
    "p055": dict(B=16, T=2048, d_model=1408, n_heads=16, local_window=256, local_block_size=256,
                 latent_tokens=64, latent_d_model=512, latent_heads=8, latent_query_block_size=0),
    "p060": dict(B=16, T=2048, d_model=1536, n_heads=16, local_window=256, local_block_size=256,
                 latent_tokens=64, latent_d_model=384, latent_heads=8, latent_query_block_size=0),
}
METRIC = "llattn fwd+bwd tokens/s, whole job over n_gpus (bf16, T=2048)"
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--batch", type=int, default=0, help="override the config's batch (small profiling runs)")
    p.add_argument("--workload", default="block", choices=["block", "lm", "decode"],
                   help="block: the attention block fwd+bwd (default); lm: cfg4 LM training step")
    p.add_argument("--layers", type=int, default=24, help="lm: decoder layers (cfg4: 24)")
    p.add_argument("--lm-steps", type=int, default=10, help="timed steps of the LM object in the block run")
    p.add_argument("--no-lm", action="store_true", help="leave the cfg4 LM measurement out of the block run")
    p.add_argument("--no-presets", action="store_true", help="leave the preset-shape block points out")
    p.add_argument("--sustain-seconds", type=float, default=2.0)
    p.add_argument("--lm-compile", type=int, default=1,
                   help="lm: 1 (default) = torch.compile each decoder layer (norms, MLP, residuals fused by inductor; the "
                        "attention stays the library's kernels, opaque custom ops in the graph)")
    return p.parse_args()


def block_cfg(name):
    """(B, T, block ModelConfig) of a config; head_dim = d_model / n_heads."""
    from llattn_b200.lm import ModelConfig

    d = dict(CONFIGS[name])
    B, T = d.pop("B"), d.pop("T")
    return B, T, ModelConfig(max_seq_len=T, n_layers=1, dropout=0.0, **d)


def seeded_module(cfg, device):
    """The block with the reference constructor's default init drawn from
    seed 0 (its layers are created in the reference's order, so the weights
    equal the reference module's under the same seed), bf16 on `device`."""
    import torch

    import llattn_b200

    torch.manual_seed(0)
    m = llattn_b200.LocalLatentAttentionB200(cfg)
    return m.to(device=device, dtype=torch.bfloat16)


def config_json(name, n_gpus):
    c = CONFIGS[name]
    return {"workload": f"LocalLatentAttention block fwd+bwd ({name})", "global_batch": c["B"] * n_gpus,
            "seq_len": c["T"], "d_model": c["d_model"], "n_heads": c["n_heads"],
            "local_window": c["local_window"], "latent_tokens": c["latent_tokens"],
            "latent_d_model": c["latent_d_model"], "latent_heads": c["latent_heads"],
            "latent_query_block_size": c["latent_query_block_size"],
            "parallelism": f"dp{n_gpus}", "l2": "inputs larger than L2 (qkv alone > 126 MB)"}


# ---------------------------------------------------------------------------
# CPU legs (oracle = restatement of the reference PyTorch block)

def reference_models():
    """The reference's own models module if it is installed in baseline/_ref
    (the reference tree has no setup.py / pyproject, so `pip install --target`
    cannot install it; __graft_entry__.build() places its unmodified models.py
    there instead), else None."""
    path = os.path.join(REF_DIR, "models.py")
    if not os.path.exists(path):
        return None
    import importlib.util

    spec = importlib.util.spec_from_file_location("llattn_reference_models", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cpu_time_block(name, seconds, steps=None, warmup=1):
    """Median time of one fwd+bwd of one sequence of the config on the host
    cores (autocast bf16, all threads): the reference's own module when
    installed, else the oracle restatement of it."""
    import torch

    fields = {k: v for k, v in CONFIGS[name].items() if k not in ("B", "T")}
    T = CONFIGS[name]["T"]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    Bs = 1  # bounded sample: one sequence of the workload per iteration
    ref = reference_models()
    torch.manual_seed(0)
    if ref is not None:
        kind = "reference"
        m = ref.LocalLatentAttention(ref.ModelConfig(**fields))
        fwd = m
        what = "the reference's own models.py LocalLatentAttention"
    else:
        kind = "port"
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import llattn_oracle as O

        cfg = O.BlockCfg(**fields)
        params = {k: v.requires_grad_(True) for k, v in O.init_params(cfg, 0).items()}
        fwd = lambda xx: O.block_forward(params, xx, cfg)  # noqa: E731
        what = "oracle restatement of models.py LocalLatentAttention"
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(Bs, T, fields["d_model"], generator=gen).requires_grad_(True)
    g = torch.randn(Bs, T, fields["d_model"], generator=gen)

    def one():
        with torch.autocast("cpu", dtype=torch.bfloat16):
            y = fwd(x)
        y.float().backward(g)

    for _ in range(warmup):
        one()
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - t_start > seconds and len(times) >= 2:
            break
    per = statistics.median(times)
    sample = (f"{len(times)} iterations of 1 x {T}-token sequence of {name} ({what}, autocast bf16, "
              f"fwd+bwd), median")
    return Bs * T / per, threads, sample, per, kind


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    tok_s, threads, sample, per, kind = cpu_time_block(args.config, 0, steps=args.steps, warmup=args.warmup)
    import platform

    cpu = platform.processor() or "cpu"
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    cpu = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    out = {"impl": "reference", "metric": METRIC, "value": round(tok_s, 1), "unit": "tokens/s",
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded randn)",
           "config": config_json(args.config, 1),
           "cpu_baseline": {"value": round(tok_s, 1), "unit": "tokens/s", "cores": threads,
                            "kind": kind, "sample": sample, "cpu": cpu},
           "e2e": {"value": round(tok_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# GPU leg

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as fh:
            return json.load(fh)
    except (OSError, ValueError):
        return {}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import llattn_b200
    from llattn_b200 import _lib
    from llattn_b200 import dist as D
    from llattn_b200.ops import visible_pairs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    # each rank's pinned buffers on its GPU's NUMA node (host copies from the
    # far socket's memory cross the socket link, and the N ranks' copies
    # otherwise meet on one socket); the CPU baseline gets the whole host back
    all_cpus = os.sched_getaffinity(0)
    numa_cpus = D.bind_to_gpu_numa(local)

    B, T, cfg = block_cfg(args.config)
    if args.batch:
        B = args.batch
        CONFIGS[args.config] = dict(CONFIGS[args.config], B=B)
    m = seeded_module(cfg, dev)
    params = [p for p in m.parameters()]
    gen = torch.Generator().manual_seed(1 + rank)
    x_h = torch.randn(B, T, cfg.d_model, generator=gen).to(torch.bfloat16).pin_memory()
    g_h = torch.randn(B, T, cfg.d_model, generator=gen).to(torch.bfloat16).pin_memory()
    dx_h = torch.empty_like(x_h).pin_memory()
    x = x_h.to(dev).requires_grad_(True)
    g = g_h.to(dev)
    flat = torch.empty(sum(p.numel() for p in params), dtype=torch.bfloat16, device=dev)

    def step(xx=x, gg=g):
        for p in params:
            p.grad = None
        xx.grad = None
        y = m(xx)
        y.backward(gg)
        if world > 1:
            # data-parallel exchange: one flat bucket, all_reduce_mean. The
            # block is one autograd node, so its gradients all appear at the
            # end of its backward: there is nothing left to overlap the
            # exchange with inside the step (DDP over the block measured
            # slower: 2.50 vs 2.42 ms at N=2); the LM below overlaps DDP
            # buckets with the earlier layers' backward
            torch.cat([p.grad.reshape(-1) for p in params], out=flat)
            D.all_reduce_mean(flat)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t_host = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - t_host) * 1e3 / args.steps  # CPU time to issue a step
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    # per-kernel times from a separate pass of the same steps with the
    # library's event profiler on (its events cost time: not in `ms`)
    _lib.profile_enable(True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    barrier()
    kern = _lib.profile_read()
    _lib.profile_enable(False)

    # the same step captured once as a CUDA graph and replayed (the library
    # is capture-safe after its first call: no allocation, no host sync, cached
    # tensor maps and attributes): what a launch-bound shape gains from graphs
    graphed = None
    if world == 1:
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    step()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(args.steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ms_g = e0.elapsed_time(e1) / args.steps
            graphed = {"ms_per_step": round(ms_g, 4), "value": round(B * T / (ms_g / 1e3), 1)}
            del graph
        except Exception as ex:  # reported, not fatal: the eager figure above is the measurement
            graphed = {"error": repr(ex)[:200]}

    # end to end through the public module: each step's x and upstream grad
    # copied in from pinned host memory and its dx copied back, pipelined
    # over two input/output buffers so that the copies of steps i+1 / i-1
    # overlap the compute of step i (H2D and D2H on their own streams)
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    xs = [torch.empty_like(x).requires_grad_(True) for _ in range(2)]
    gs = [torch.empty_like(g) for _ in range(2)]
    dxh = [torch.empty_like(x_h).pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(comp)
        h2d.wait_event(start)
        with torch.cuda.stream(h2d):
            xs[0].data.copy_(x_h, non_blocking=True)
            gs[0].copy_(g_h, non_blocking=True)
            ev_in[0].record(h2d)
        for i in range(n):
            k = i % 2
            if i + 1 < n:  # inputs of step i+1 into the other buffer once step i-1 is done with it
                if i >= 1:
                    h2d.wait_event(ev_comp[1 - k])
                with torch.cuda.stream(h2d):
                    xs[1 - k].data.copy_(x_h, non_blocking=True)
                    gs[1 - k].copy_(g_h, non_blocking=True)
                    ev_in[1 - k].record(h2d)
            comp.wait_event(ev_in[k])
            if i >= 2:
                comp.wait_event(ev_out[k])  # dx of step i-2 has left this buffer
            step(xs[k], gs[k])
            ev_comp[k].record(comp)
            d2h.wait_event(ev_comp[k])
            with torch.cuda.stream(d2h):
                dxh[k].copy_(xs[k].grad, non_blocking=True)
                xs[k].grad.record_stream(d2h)
                ev_out[k].record(d2h)
        comp.wait_event(ev_out[(n - 1) % 2])
        if n >= 2:
            comp.wait_event(ev_out[(n - 2) % 2])
        end.record(comp)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / n

    e2e_run(3)
    barrier()
    ms_e2e = e2e_run(args.steps)
    barrier()

    # the e2e step's copies alone (H2D of x and the upstream grad, D2H of a
    # dx-sized buffer, on the same two streams, every rank at once): the
    # host-link bound of the e2e figure
    def copy_run(n):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(comp)
        h2d.wait_event(start)
        d2h.wait_event(start)
        for i in range(n):
            k = i % 2
            with torch.cuda.stream(h2d):
                xs[k].data.copy_(x_h, non_blocking=True)
                gs[k].copy_(g_h, non_blocking=True)
            with torch.cuda.stream(d2h):
                dxh[k].copy_(gs[1 - k], non_blocking=True)
        ev_in[0].record(h2d)
        ev_out[0].record(d2h)
        comp.wait_event(ev_in[0])
        comp.wait_event(ev_out[0])
        end.record(comp)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / n

    copy_run(2)
    barrier()
    ms_copy = copy_run(args.steps)
    barrier()

    # sustained: the same step repeated for >= sustain_seconds of device time.
    # The step count comes from the slowest rank's ms so that every rank runs
    # the same number of steps (each step holds a gradient all-reduce)
    ms_all = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_all, op=dist.ReduceOp.MAX)
    n_sus = max(args.steps, min(20000, math.ceil(args.sustain_seconds * 1e3 / max(ms_all.item(), 1e-3))))
    clocks_sus = ClockSampler(local)
    clocks_sus.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n_sus):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk_sus = clocks_sus.stop()
    ms_sus = e0.elapsed_time(e1) / n_sus

    t = torch.tensor([ms, ms_e2e, ms_copy, ms_sus], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_copy, ms_sus = t.tolist()
    tokens = B * T * world
    value = tokens / (ms / 1e3)
    e2e_value = tokens / (ms_e2e / 1e3)

    presets = sweep = None
    if rank == 0 and not args.no_presets and args.config in ("cfg2",):
        presets = {name: measure_block_point(name, dev, args.steps) for name in ("p055", "p060")}
        # the long-context and 512-latent configs beside the headline one
        sweep = {name: measure_block_point(name, dev, args.steps) for name in ("cfg3", "cfg5_nl512")}
    barrier()
    del m, params, x, g, xs, gs, flat
    torch.cuda.empty_cache()
    lm = lm055 = None
    if not args.no_lm and args.config == "cfg2":
        lm = measure_lm(args, world, rank, dev)
        torch.cuda.empty_cache()
        lm055 = measure_lm(args, world, rank, dev, shape="0.55b")

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    # roofline of the dominant kernel group
    hbm, tflops, peak_kind = load_peaks()
    P = visible_pairs(T, cfg.local_window, cfg.local_block_size) * B * cfg.n_heads
    hd = cfg.d_model // cfg.n_heads
    d = cfg.d_model
    BTd2 = B * T * d * 2.0  # one [B,T,d] bf16 tensor
    # per launch-group call: (FLOPs, bytes that must cross HBM)
    alg = {
        "local_fwd": (4.0 * hd * P, 3 * BTd2 + 2 * BTd2),    # qkv in; local_out, mixed out
        "local_bwd": (8.0 * hd * P, 4 * BTd2 + 3 * BTd2),
        "local_dq": (4.0 * hd * P, 4 * BTd2 + BTd2),        # q,k,v,dlocal in; dq out
        "local_dkv": (4.0 * hd * P, 4 * BTd2 + 2 * BTd2),   # q,k,v,dlocal in; dk,dv out
        "gate_fwd": (0.0, (2 * B * T * d + B * T * d + 2 * d * cfg.latent_d_model) * 2.0),
        "gate_bwd": (0.0, 4 * BTd2),                        # local_out, dmixed in; dlocal, dR out
        "pool_fwd": (0.0, BTd2),
        "pool_bwd": (0.0, BTd2),
    }
    per_step = {k: (v[0] / args.steps, v[1] / args.steps) for k, v in kern.items() if v[1] > 0}
    top = max(per_step, key=lambda k: per_step[k][0])
    calls = max(1, round(kern[top][1] / args.steps / {"local_bwd": 2, "rout_bwd": 2, "reduce": 3,
                                                      "latent_bwd": 2}.get(top, 1)))
    avg_ms = kern[top][0] / args.steps / calls
    roof = None
    if top in alg:
        # the binding roof is the one whose ideal time (amount / peak) is longer
        flops, nbytes = alg[top]
        t_tensor = flops / (tflops * 1e12)
        t_hbm = nbytes / (hbm * 1e9)
        f_ach = flops / (avg_ms / 1e3) / 1e12
        b_ach = nbytes / (avg_ms / 1e3) / 1e9
        if t_tensor > t_hbm:
            roof = {"kernel": top, "bound": "tensor", "achieved": round(f_ach, 2), "peak": tflops,
                    "unit": "TFLOP/s", "frac": round(f_ach / tflops, 4), "peak_kind": peak_kind,
                    "hbm_frac": round(b_ach / hbm, 4)}
        else:
            roof = {"kernel": top, "bound": "hbm", "achieved": round(b_ach, 1), "peak": hbm,
                    "unit": "GB/s", "frac": round(b_ach / hbm, 4), "peak_kind": peak_kind,
                    "algorithmic_bytes": nbytes}
            if flops:
                roof["tensor_frac"] = round(f_ach / tflops, 4)
        # measured at the config's default batch; other batches get null
        tr = None if args.batch else load_traffic().get(f"{top}:{args.config}")
        roof["traffic"] = tr
        roof["avg_launch_ms"] = round(avg_ms, 4)
    # also the local branch as a whole (fwd + bwd), the BASELINE target
    local_ms = sum(per_step.get(k, (0, 0))[0] for k in ("local_fwd", "local_bwd", "local_dq", "local_dkv"))
    local_branch = None
    if local_ms > 0:
        ach = 12.0 * hd * P / (local_ms / 1e3) / 1e12
        local_branch = {"ms": round(local_ms, 4), "achieved": round(ach, 2), "unit": "TFLOP/s",
                        "frac": round(ach / tflops, 4), "flops": 12.0 * hd * P}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        os.sched_setaffinity(0, all_cpus)
        tok_s, threads, sample, _, kind = cpu_time_block(args.config, args.cpu_seconds)
        if numa_cpus:
            os.sched_setaffinity(0, numa_cpus)
        cpu = {"value": round(tok_s, 1), "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": sample}

    launches = int(sum(v[1] for v in kern.values()))
    out = {
        "metric": METRIC, "value": round(value, 1), "value_per_gpu": round(value / world, 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "host_issue_ms_per_step": round(host_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded randn inputs and upstream grad; reference default init)",
        "config": config_json(args.config, world),
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * x_h.numel() * 2, "d2h_bytes_per_step": dx_h.numel() * 2,
                "ms_per_step": round(ms_e2e, 4), "copy_ms_per_step": round(ms_copy, 4),
                "copy_bound_frac": round(ms_copy / ms_e2e, 4),
                "rank0_cpus": None if numa_cpus is None else f"{len(numa_cpus)} cpus bound to GPU {local}'s NUMA node"},
        "sustained": {"steps": n_sus, "seconds": round(ms_sus * n_sus / 1e3, 3), "ms_per_step": round(ms_sus, 4),
                      "value": round(tokens / (ms_sus / 1e3), 1), "clocks": clk_sus},
        "roofline": roof,
        "local_branch": local_branch,
        "cpu_baseline": cpu,
        "gpu_launches": launches,
        "kernels": {k: {"ms_per_step": round(v[0], 4), "launches_per_step": v[1]} for k, v in per_step.items()},
        "clocks": clk,
        "graphed": graphed,
        "presets": presets,
        "configs": sweep,
        "lm": lm,
        "lm_0.55b": lm055,
    }
    print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_block_point(name, dev, steps, warmup=3):
    """One GPU's block fwd+bwd at a config (no gradient exchange): K steps
    timed with CUDA events, then a profiled pass for the kernel groups.
    local_backward names the local-branch backward that ran: tcgen05 (the
    dq / dk,dv tensor-core kernels) or simt."""
    import torch

    from llattn_b200 import _lib

    B, T, cfg = block_cfg(name)
    m = seeded_module(cfg, dev)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(B, T, cfg.d_model, generator=gen).to(device=dev, dtype=torch.bfloat16).requires_grad_(True)
    g = torch.randn(B, T, cfg.d_model, generator=gen).to(device=dev, dtype=torch.bfloat16)

    def step():
        x.grad = None
        for p in m.parameters():
            p.grad = None
        m(x).backward(g)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    _lib.profile_enable(True)
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    kern = _lib.profile_read()
    _lib.profile_enable(False)
    c = CONFIGS[name]
    return {"config": {k: c[k] for k in ("B", "T", "d_model", "n_heads", "latent_d_model", "latent_heads")},
            "head_dim": c["d_model"] // c["n_heads"], "ms_per_step": round(ms, 4),
            "value": round(B * T / (ms / 1e3), 1), "unit": "tokens/s",
            "local_backward": "tcgen05" if kern.get("local_dq", (0, 0))[1] > 0 and kern.get("local_bwd", (0, 0))[1] == 0
            else "simt",
            "kernels": {k: {"ms_per_step": round(v[0] / steps, 4), "launches_per_step": v[1] / steps}
                        for k, v in kern.items() if v[1] > 0}}


LM_METRIC = "LM train tok/s (bf16, T=2048, cfg4 0.55B-class, AdamW, DDP)"


def run_lm(args):
    """--workload lm: the cfg4 LM training step alone, as its own JSON line."""
    import torch

    from llattn_b200 import dist as D

    world = int(os.environ.get("WORLD_SIZE", "1"))
    device = D.setup_distributed("nccl") if world > 1 else torch.device("cuda", 0)
    torch.cuda.set_device(device)
    out = measure_lm(args, world, D.get_rank(), device, steps=args.steps)
    if out is not None:
        print(json.dumps(out), flush=True)
    D.cleanup_distributed()


# LM shapes: cfg4 (the benchmark's LM config) and the reference's 0.55b
# training preset (train.py:71-80), whose LM throughput the reference
# publishes (README.md:254-257: 108k tok/s/GPU, 1 H200, torch.compile, batch
# 16 x 2048, PyTorch attention)
LM_SHAPES = {
    "cfg4": dict(d_model=1536, n_heads=12, n_layers=24, d_ff=4096, latent_d_model=64, latent_heads=2),
    "0.55b": dict(d_model=1408, n_heads=16, n_layers=22, d_ff=4096, latent_d_model=512, latent_heads=8),
}
LM_PUBLISHED = {"0.55b": 108000.0}


def measure_lm(args, world, rank, device, steps=None, shape="cfg4"):
    """cfg4: LocalLatentLM (24 x d1536 H12 W256 Nl64 Ld64, d_ff 4096, V32000,
    tied embeddings), B16 x T2048 per GPU, bf16 autocast, fused AdamW, DDP
    gradient all-reduce over NCCL (bucketed, overlapping the backward; the
    process group must exist when world > 1). Returns the measurement on
    rank 0, None elsewhere."""
    import torch
    import torch.distributed as dist

    import llattn_b200  # noqa: F401
    from llattn_b200 import _lib
    from llattn_b200 import dist as D
    from llattn_b200.lm import LocalLatentLM, ModelConfig, build_optimizer, train_step

    steps = steps or args.lm_steps
    warmup = max(3, min(args.warmup, 5))
    B = (args.batch if args.workload == "lm" else 0) or 16
    T = 2048
    sh = dict(LM_SHAPES[shape])
    if shape == "cfg4":
        sh["n_layers"] = args.layers
    cfg = ModelConfig(vocab_size=32000, max_seq_len=T, local_window=256, latent_tokens=64, **sh)
    torch.manual_seed(0)  # identical init on every rank (DDP also broadcasts rank 0's)
    model = LocalLatentLM(cfg).to(device)
    n_params = sum(p.numel() for p in model.parameters())
    t_compile = None
    if args.lm_compile:
        t0 = time.perf_counter()
        for i, layer in enumerate(model.blocks):
            model.blocks[i] = torch.compile(layer, fullgraph=True)
        model.loss_head = torch.compile(model.loss_head, fullgraph=True)  # norm, tied head, fp32 CE
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[device.index], bucket_cap_mb=100,
                                                          gradient_as_bucket_view=True)
    opt = build_optimizer(model)
    gen = torch.Generator().manual_seed(1000 + rank)
    data_h = torch.randint(0, cfg.vocab_size, (B, T + 1), generator=gen, dtype=torch.int64).pin_memory()
    data = data_h.to(device)
    ids, tgt = data[:, :-1].contiguous(), data[:, 1:].contiguous()
    for _ in range(warmup):
        train_step(model, opt, ids, tgt)
    torch.cuda.synchronize()
    if args.lm_compile:
        t_compile = time.perf_counter() - t0
    D.barrier()
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        loss = train_step(model, opt, ids, tgt)
    e1.record()
    torch.cuda.synchronize()
    D.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    # per-kernel times from a separate profiled pass (the profiler's events cost time)
    _lib.profile_enable(True)
    for _ in range(steps):
        train_step(model, opt, ids, tgt)
    torch.cuda.synchronize()
    D.barrier()
    kern = _lib.profile_read()
    _lib.profile_enable(False)
    # end to end: the step's tokens copied from pinned host memory, loss read back
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def e2e_step():
        data.copy_(data_h, non_blocking=True)
        # inputs and targets into the contiguous buffers the compiled step was
        # traced with (a strided slice would be a new guard, i.e. a recompile)
        ids.copy_(data[:, :-1])
        tgt.copy_(data[:, 1:])
        loss_h.copy_(train_step(model, opt, ids, tgt), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e2.record()
    for _ in range(steps):
        e2e_step()
    e3.record()
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3) / steps
    t = torch.tensor([ms, ms_e2e], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = t.tolist()
    if rank == 0:
        hbm, tflops, peak_kind = load_peaks()
        sustained = tflops
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
                sustained = json.load(fh).get("bf16_tflops_sustained", tflops)
        except (OSError, ValueError):
            pass
        tokens = B * T * world
        n_nonemb = n_params - cfg.vocab_size * cfg.d_model - T * cfg.d_model
        flops_tok = 6 * n_nonemb + 6 * cfg.vocab_size * cfg.d_model
        ach = flops_tok * tokens / (ms / 1e3) / 1e12
        per_step = {k: (v[0] / steps, v[1] / steps) for k, v in kern.items() if v[1] > 0}
        out = {
            "metric": LM_METRIC, "value": round(tokens / (ms / 1e3), 1),
            "value_per_gpu": round(tokens / world / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded uniform tokens in [0, 32000))",
            "vs_published": (round(tokens / world / (ms / 1e3) / LM_PUBLISHED[shape], 3)
                             if shape in LM_PUBLISHED else None),
            "config": {"workload": f"LocalLatentLM training step ({shape})", "model": f"LocalLatentLM {shape}",
                       "d_model": cfg.d_model, "n_heads": cfg.n_heads, "latent_d_model": cfg.latent_d_model,
                       "n_layers": cfg.n_layers, "params": n_params, "global_batch": B * world, "seq_len": T,
                       "parallelism": f"dp{world}", "l2": "inputs and activations larger than L2"},
            "e2e": {"value": round(tokens / (ms_e2e / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": data_h.numel() * 8, "d2h_bytes_per_step": 4},
            "roofline": {"kernel": "whole step (6N FLOPs/token model)", "bound": "tensor",
                         "achieved": round(ach / world, 1), "peak": sustained, "unit": "TFLOP/s",
                         "frac": round(ach / world / sustained, 4), "peak_kind": peak_kind + " sustained",
                         "traffic": None},
            "gpu_launches": int(sum(v[1] for v in kern.values())),
            "kernels": {k: {"ms_per_step": round(v[0], 4), "launches_per_step": v[1]} for k, v in per_step.items()},
            "final_loss": float(loss.item()),
            "compiled_layers": bool(args.lm_compile),
            "compile_and_warmup_s": round(t_compile, 1) if t_compile is not None else None,
            "clocks": clk,
        }
        return out
    return None


def run_decode(args):
    """Incremental decode of the cfg2 block: B=16 sequences with a 2047-token
    prefix in the decode caches, then one token per step through
    LocalLatentAttentionB200.decode (qkv row, chunk means re-pooled over the
    prefix, llattn_decode, out row). Metric: generated tokens/s; 1 GPU
    (replicas only: each rank would decode its own sequences)."""
    import torch

    from llattn_b200 import _lib

    if int(os.environ.get("RANK", "0")) != 0:
        return
    B, T, cfg = block_cfg(args.config)
    if args.batch:
        B = args.batch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    m = seeded_module(cfg, dev).eval()
    gen = torch.Generator().manual_seed(0)
    T0 = T - 1
    steps = args.steps + args.warmup
    # room for the timed steps and then a profiled pass of as many steps
    x = torch.randn(B, T0 + steps + args.steps, cfg.d_model, generator=gen).to(device=dev, dtype=torch.bfloat16)
    cache = m.new_decode_cache(T0 + steps + args.steps)
    m.prefill(x[:, :T0], cache)
    for i in range(args.warmup):
        m.decode(x[:, T0 + i:T0 + i + 1], cache)
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.warmup, steps):
        y = m.decode(x[:, T0 + i:T0 + i + 1], cache)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    # per-kernel times from the next steps with the profiler on (its events cost time)
    _lib.profile_enable(True)
    for i in range(steps, steps + args.steps):
        m.decode(x[:, T0 + i:T0 + i + 1], cache)
    torch.cuda.synchronize()
    kern = _lib.profile_read()
    _lib.profile_enable(False)
    # end to end: the new token's input from pinned host memory, its output row back
    xh = x[:, -1:].cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    cache2 = m.new_decode_cache(T0 + steps)
    m.prefill(x[:, :T0], cache2)
    xd = torch.empty_like(x[:, :1])
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(args.steps):
        xd.copy_(xh, non_blocking=True)
        yd = m.decode(xd, cache2)
        yh.copy_(yd, non_blocking=True)
    e3.record()
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3) / args.steps
    per_step = {k: (v[0] / args.steps, v[1] / args.steps) for k, v in kern.items() if v[1] > 0}
    hbm, tflops, peak_kind = load_peaks()
    # the decode kernel reads, per (b, h), the key/value rows of the window and
    # the query row, plus per sequence the rq row, gk/gv and W_rout
    Tn = T0 + steps
    nk = min(cfg.local_window, Tn - 1)
    Ld = cfg.latent_d_model
    hd = cfg.d_model // cfg.n_heads
    dec_bytes = 2.0 * B * (cfg.n_heads * (2 * nk + 1) * hd + cfg.d_model * (1 + Ld) + 2 * 64 * Ld)
    dec_ms = per_step.get("decode", (0.0, 0))[0]
    roof = None
    if dec_ms > 0:
        ach = dec_bytes / (dec_ms / 1e3) / 1e9
        roof = {"kernel": "decode", "bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(ach / hbm, 4), "peak_kind": peak_kind, "algorithmic_bytes": dec_bytes, "traffic": None,
                "avg_launch_ms": round(dec_ms, 4)}
    out = {
        "metric": "llattn decode tokens/s (bf16, cfg2 block, 2047-token prefix)", "value": round(B / (ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded randn token inputs)",
        "config": {"workload": "LocalLatentAttention block decode (cfg2 shapes)", "batch": B, "prefix": T0,
                   "parallelism": "replicas only"},
        "e2e": {"value": round(B / (ms_e2e / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": xh.numel() * 2,
                "d2h_bytes_per_step": yh.numel() * 2},
        "roofline": roof,
        "gpu_launches": int(sum(v[1] for v in kern.values())),
        "kernels": {k: {"ms_per_step": round(v[0], 4), "launches_per_step": v[1]} for k, v in per_step.items()},
        "clocks": clk,
    }
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    # stdout carries exactly one JSON line: keep NCCL's version banner off it
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "lm":
        run_lm(args)
    elif args.workload == "decode":
        run_decode(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
