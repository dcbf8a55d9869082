"""Benchmark of the causal_conv1d hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (benchmark config 2): bf16 x (4, 4096, 2048) channel-last, fp32 weight (4096, 4)
~U(-0.5, 0.5) and bias ~N(0, 0.1), SiLU, initial_states (4, 4096, 3), final states
returned; one step = forward + backward (dx, dweight, dbias, dinitial_states, dfinal fed
back).  Metric: algorithmic HBM GB/s (every tensor element read or written once).  Each
rank runs its own batch (weak scaling); for N > 1 the backward is batch-sharded and
dweight|dbias are summed with one NCCL all-reduce per step.

Inputs rotate over 4 buffer sets (1 GiB in total, > 8x the 126 MB L2); the forward of
step i reads set i % 4 and the backward reads set (i + 2) % 4, so no kernel reads data
another kernel touched within the previous ~300 MB of traffic.  The timed loop replays
one CUDA graph per 16 steps; per-kernel times come from a graph of 16 back-to-back
launches of each pass.

`--impl reference` times the reference algorithm's CPU implementation (the C
restatement in oracle/, OpenMP on all host cores) on a bounded sample of the same
workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "cute-causal-conv1d_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "fwd/bwd/update achieved HBM GB/s and % of 8 TB/s roofline at 1/2/4/8 B200"
CFG2 = dict(batch=4, dim=4096, seqlen=2048, width=4)
NSETS = 4
GRAPH_STEPS = 4 * NSETS  # steps per replay of the timed step graph


def workload_bytes(batch, dim, seqlen, width, es=2, init=True, final=True, bias=True):
    """Algorithmic bytes of one forward and one backward."""
    n = batch * dim * seqlen
    states = batch * dim * (width - 1) * es
    params = dim * width * 4 + (dim * 4 if bias else 0)
    fwd = 2 * n * es + params + (states if init else 0) + (states if final else 0)
    bwd = 3 * n * es + 2 * params + (2 * states if init else 0) + (states if final else 0)
    return fwd, bwd


# ------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period: float = 0.005):
        self.samples, self.reasons = [], 0
        self.period = period
        self._stop = threading.Event()
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nvml = pynvml
            props = torch.cuda.get_device_properties(device_index)
            try:
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                self.reasons |= int(self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self.thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.handle is not None:
            self.thread.join()
        return False

    def result(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(key):
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(key)
    except Exception:
        return None


# ---------------------------------------------------------------- CPU baseline
def cpu_sample_rate(target_s: float, max_channels: int = CFG2["dim"]):
    """Time the C oracle (OpenMP) on a channel slice of the config-2 workload.

    Returns (GB/s, cores, sample description, seconds per sample run)."""
    import numpy as np

    from oracle import c_oracle
    from oracle import numpy_oracle as O

    c_oracle.build()
    cores = c_oracle.use_all_cores()
    b, L, W = CFG2["batch"], CFG2["seqlen"], CFG2["width"]
    rng = np.random.default_rng(0)

    def make(ch):
        x = O.f32_to_bf16_bits(rng.standard_normal((b, L, ch), dtype=np.float32)).transpose(0, 2, 1)
        dout = O.f32_to_bf16_bits(rng.standard_normal((b, L, ch), dtype=np.float32)).transpose(0, 2, 1)
        w = rng.uniform(-0.5, 0.5, (ch, W)).astype(np.float32)
        bias = (0.1 * rng.standard_normal(ch)).astype(np.float32)
        init = O.f32_to_bf16_bits(rng.standard_normal((b, ch, W - 1), dtype=np.float32))
        dfin = np.zeros((b, ch, W - 1), np.uint16)
        return x, dout, w, bias, init, dfin

    def run(ch, data):
        x, dout, w, bias, init, dfin = data
        c_oracle.fwd(x, "bfloat16", w, bias, initial_states=init, silu=True, return_final_states=True)
        c_oracle.bwd(x, "bfloat16", w, dout, bias, initial_states=init, dfinal_states=dfin, silu=True)

    ch = 64
    data = make(ch)
    run(ch, data)
    t0 = time.perf_counter()
    run(ch, data)
    dt = time.perf_counter() - t0
    ch = int(min(max_channels, max(64, 64 * (target_s / max(dt, 1e-6)))))
    ch = max(64, ch // 64 * 64)
    data = make(ch)
    run(ch, data)  # warm
    t0 = time.perf_counter()
    run(ch, data)
    dt = time.perf_counter() - t0
    fb, bb = workload_bytes(b, ch, L, W)
    sample = f"config-2 fwd+bwd on a {ch}-channel slice: x ({b}, {ch}, {L}) bf16 channel-last"
    return (fb + bb) / dt / 1e9, cores, sample, dt, ch


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    # each step is one sample run; size it so that all steps finish in ~2 minutes
    budget = 120.0 / max(1, args.steps + args.warmup)
    budget = min(max(budget, 0.01), 5.0)
    rate, cores, sample, _, ch = cpu_sample_rate(budget)
    import numpy as np  # noqa: F401

    from oracle import c_oracle
    from oracle import numpy_oracle as O

    b, L, W = CFG2["batch"], CFG2["seqlen"], CFG2["width"]
    rng = np.random.default_rng(1)
    x = O.f32_to_bf16_bits(rng.standard_normal((b, L, ch), dtype=np.float32)).transpose(0, 2, 1)
    dout = O.f32_to_bf16_bits(rng.standard_normal((b, L, ch), dtype=np.float32)).transpose(0, 2, 1)
    w = rng.uniform(-0.5, 0.5, (ch, W)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(ch)).astype(np.float32)
    init = O.f32_to_bf16_bits(rng.standard_normal((b, ch, W - 1), dtype=np.float32))
    dfin = np.zeros((b, ch, W - 1), np.uint16)

    def step():
        c_oracle.fwd(x, "bfloat16", w, bias, initial_states=init, silu=True, return_final_states=True)
        c_oracle.bwd(x, "bfloat16", w, dout, bias, initial_states=init, dfinal_states=dfin, silu=True)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    total = time.perf_counter() - t0
    fb, bb = workload_bytes(b, ch, L, W)
    value = (fb + bb) * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample + " per step (oracle/cc1d_oracle.c, OpenMP)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(n):
    return {"workload": "config2: causal_conv1d fwd+bwd, bf16 x (4,4096,2048) channel-last, W=4, silu, "
                        "initial_states + final_states, fp32 weight/bias",
            "global_batch": CFG2["batch"] * n, "seq_len": CFG2["seqlen"], "dim": CFG2["dim"], "width": CFG2["width"],
            "parallelism": f"dp{n}" if n > 1 else "single",
            "l2": "inputs rotate over 4 sets (1 GiB) > L2; fwd reads set i%4, bwd set (i+2)%4"}


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    from causal_conv1d import _abi
    from causal_conv1d.cpp_functions import causal_conv1d_fwd_function
    from causal_conv1d.distributed import GradBucket, allreduce_param_grads, causal_conv1d_bwd_batch_sharded

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        # the per-step all-reduce moves 80 KB: NVLink SHARP brings nothing at that size,
        # so it stays off (no multicast memory objects are created)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _abi.load_library()

    B, D, L, W = CFG2["batch"], CFG2["dim"], CFG2["seqlen"], CFG2["width"]
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    weight = (torch.rand(D, W, generator=gen, device=dev) - 0.5)
    bias = torch.randn(D, generator=gen, device=dev) * 0.1
    sets = []
    for _ in range(NSETS):
        x = torch.randn(B, L, D, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
        dout = torch.randn(B, L, D, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
        init = torch.randn(B, D, W - 1, generator=gen, device=dev).to(torch.bfloat16)
        final = torch.empty(B, W - 1, D, device=dev, dtype=torch.bfloat16).transpose(1, 2)
        dfinal = torch.zeros(B, D, W - 1, device=dev, dtype=torch.bfloat16)
        sets.append(dict(x=x, dout=dout, init=init, final=final, dfinal=dfinal,
                         bucket=GradBucket(D, W, True, dev)))

    def fwd(k):
        s = sets[k]
        s["out"] = causal_conv1d_fwd_function(s["x"], weight, bias, None, s["init"], s["final"], True)

    def bwd(k):
        s = sets[k]
        s["grads"] = causal_conv1d_bwd_batch_sharded(
            s["x"], weight, bias, s["dout"], None, s["init"], s["dfinal"], True, True,
            bucket=s["bucket"], allreduce=False)

    for k in range(NSETS):  # eager warm-up: occupancy queries, allocator pools
        fwd(k)
        bwd(k)
    torch.cuda.synchronize()
    g_fwd, g_bwd = [], []
    for k in range(NSETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fwd(k)
        g_fwd.append(g)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            bwd(k)
        g_bwd.append(g)
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    fb, bb = workload_bytes(B, D, L, W)

    def step(i):
        g_fwd[i % NSETS].replay()
        kb = (i + NSETS // 2) % NSETS
        g_bwd[kb].replay()
        if world > 1:
            allreduce_param_grads(sets[kb]["bucket"])

    # One graph holds GRAPH_STEPS consecutive steps, so that no graph-launch gap sits
    # between the kernels of the timed steps.  With N ranks each step's dweight|dbias
    # all-reduce is captured on a side stream, overlapping the next steps; the backward
    # that rewrites a bucket waits for the all-reduce that read it, and the graph joins
    # the side stream before it ends.
    side = torch.cuda.Stream(dev) if world > 1 else None
    if side is not None:
        allreduce_param_grads(sets[0]["bucket"])  # communicator set up before capture
        torch.cuda.synchronize()
    g_round = torch.cuda.CUDAGraph()
    reduced = [torch.cuda.Event() for _ in range(NSETS)]  # all-reduce of set k's bucket done
    with torch.cuda.graph(g_round):
        cap = torch.cuda.current_stream()
        for i in range(GRAPH_STEPS):
            fwd(i % NSETS)
            kb = (i + NSETS // 2) % NSETS
            if side is not None and i >= NSETS:
                cap.wait_event(reduced[kb])  # the all-reduce that read this bucket, NSETS steps ago
            bwd(kb)
            if side is not None:
                side.wait_stream(cap)
                with torch.cuda.stream(side):
                    allreduce_param_grads(sets[kb]["bucket"])
                    reduced[kb].record(side)
        if side is not None:
            cap.wait_stream(side)
    torch.cuda.synchronize()

    def run_steps(n):
        i = 0
        if g_round is not None:
            while i + GRAPH_STEPS <= n:
                g_round.replay()
                i += GRAPH_STEPS
        while i < n:
            step(i)
            i += 1

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler:
        t_start.record(stream)
        run_steps(args.steps)
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    # per-kernel device times (the roofline's "achieved"): 16 back-to-back launches of
    # each pass in one graph, inputs rotating over the NSETS sets
    fwd_ms = graph_time([lambda k=k: fwd(k) for k in range(NSETS)] * 4) / 1e3
    bwd_ms = graph_time([lambda k=k: bwd(k) for k in range(NSETS)] * 4) / 1e3
    t = torch.tensor([total_ms, fwd_ms, bwd_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, fwd_ms, bwd_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    value = (fb + bb) * world * args.steps / (total_ms / 1e3) / 1e9

    e2e = run_e2e(args, dev, world, weight, bias)
    kernels = {}
    cpu = None
    if world == 1 and not args.no_extras:
        kernels = run_extras(dev)
    peak, peak_kind = measured_peak()
    achieved = bb / (bwd_ms / 1e3) / 1e9
    kernels.update({
        "config2_fwd": {"GB/s": round(fb / (fwd_ms / 1e3) / 1e9, 1), "us": round(fwd_ms * 1e3, 2),
                        "bytes": fb, "frac_of_peak": round(fb / (fwd_ms / 1e3) / 1e9 / peak, 4)},
        "config2_bwd": {"GB/s": round(achieved, 1), "us": round(bwd_ms * 1e3, 2), "bytes": bb,
                        "frac_of_peak": round(achieved / peak, 4)},
    })
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, cores, sample, _, _ = cpu_sample_rate(8.0)
        cpu = {"value": round(rate, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": sample + " (oracle/cc1d_oracle.c, OpenMP), after one warm run"}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config_dict(world),
        "roofline": {"bound": "hbm", "kernel": "bwd_stream_kernel + reduce_unit_partials (config 2 backward)", "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": f"{peak_kind} hbm_gbs", "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": ncu_traffic("config2_bwd"),
                     "algorithmic_bytes": bb},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 3 * args.steps,  # forward kernel + backward kernel + partial-sum kernel
        "clocks": sampler.result(),
        "kernels": kernels,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        del g_fwd, g_bwd, g_round
        dist.destroy_process_group()
    return 0


def run_e2e(args, dev, world, weight, bias):
    """Same metric through the public API (causal_conv1d_fn + autograd) with pinned host
    buffers: H2D of x/dout/initial states and D2H of every result inside the timed region."""
    import torch
    import torch.distributed as dist

    from causal_conv1d import causal_conv1d_fn

    B, D, L, W = CFG2["batch"], CFG2["dim"], CFG2["seqlen"], CFG2["width"]
    gen = torch.Generator().manual_seed(77)
    hx = torch.randn(B, L, D, generator=gen).to(torch.bfloat16).pin_memory()
    hg = torch.randn(B, L, D, generator=gen).to(torch.bfloat16).pin_memory()
    hi = torch.randn(B, D, W - 1, generator=gen).to(torch.bfloat16).pin_memory()
    hw = weight.cpu().pin_memory()
    hb = bias.cpu().pin_memory()
    outs = dict(out=torch.empty(B, L, D, dtype=torch.bfloat16).pin_memory(),
                final=torch.empty(B, W - 1, D, dtype=torch.bfloat16).pin_memory(),
                dx=torch.empty(B, L, D, dtype=torch.bfloat16).pin_memory(),
                dw=torch.empty(D, W).pin_memory(), db=torch.empty(D).pin_memory(),
                di=torch.empty(B, D, W - 1, dtype=torch.bfloat16).pin_memory())
    h2d = sum(t.numel() * t.element_size() for t in (hx, hg, hi, hw, hb))
    d2h = sum(t.numel() * t.element_size() for t in outs.values())

    # Three streams, two device input buffers: the H2D copy of step i+1 and the D2H copy
    # of step i-1 run on the copy engines while step i computes.  Every step still copies
    # its own inputs in and its own results out inside the timed region.
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [dict(x=torch.empty(B, L, D, dtype=torch.bfloat16, device=dev),
                 g=torch.empty(B, L, D, dtype=torch.bfloat16, device=dev),
                 i0=torch.empty(B, D, W - 1, dtype=torch.bfloat16, device=dev),
                 w=torch.empty(D, W, device=dev), b=torch.empty(D, device=dev)) for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    for e in in_free:
        e.record(comp)

    def step(i):
        k = i % 2
        buf = bufs[k]
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[k])
            for name, host in (("x", hx), ("g", hg), ("i0", hi), ("w", hw), ("b", hb)):
                buf[name].copy_(host, non_blocking=True)
            in_ready[k].record(s_in)
        comp.wait_event(in_ready[k])
        x = buf["x"].transpose(1, 2).detach().requires_grad_()
        g = buf["g"].transpose(1, 2)
        i0 = buf["i0"].detach().requires_grad_()
        w = buf["w"].detach().requires_grad_()
        b = buf["b"].detach().requires_grad_()
        out, fin = causal_conv1d_fn(x, w, b, initial_states=i0, return_final_states=True, activation="silu")
        torch.autograd.backward([out], [g])
        if world > 1:
            dist.all_reduce(w.grad)
            dist.all_reduce(b.grad)
        res = dict(out=out.transpose(1, 2), final=fin.transpose(1, 2), dx=x.grad.transpose(1, 2),
                   dw=w.grad, db=b.grad, di=i0.grad)
        in_free[k].record(comp)
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for name, t in res.items():
                t.record_stream(s_out)
                outs[name].copy_(t, non_blocking=True)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    n = args.e2e_steps
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s0.record(comp)
    s_in.wait_stream(comp)
    for i in range(n):
        step(i)
    comp.wait_stream(s_out)
    s1.record(comp)
    torch.cuda.synchronize()
    ms = s0.elapsed_time(s1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    fb, bb = workload_bytes(B, D, L, W)
    return {"value": round((fb + bb) * world * n / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / n, 4),
            "path": "causal_conv1d_fn + autograd backward, pinned host buffers, copies overlapped with compute on two copy streams"}


def graph_time(fns, reps=5):
    """Average device time per call of a list of launch closures, captured in one CUDA
    graph (so launch latency does not hide the kernel time)."""
    import torch

    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(reps):
        g.replay()
    s1.record()
    torch.cuda.synchronize()
    return s0.elapsed_time(s1) / (reps * len(fns)) * 1e3  # us per call


def run_extras(dev):
    """Kernel-level numbers for the other benchmark configs (outside the timed step)."""
    import torch

    from causal_conv1d import causal_conv1d_update
    from causal_conv1d.causal_conv1d_varlen import causal_conv1d_fn_varlen_states, causal_conv1d_varlen_states
    from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function

    peak, _ = measured_peak()
    res = {}
    gen = torch.Generator(device=dev).manual_seed(3)

    def entry(nbytes, us):
        gbs = nbytes / (us * 1e-6) / 1e9
        return {"GB/s": round(gbs, 1), "us": round(us, 3), "bytes": int(nbytes), "frac_of_peak": round(gbs / peak, 4)}

    # config 3: decode update, B=128, D=8192, bf16, silu
    Bu, Du, W = 128, 8192, 4
    w = torch.rand(Du, W, generator=gen, device=dev) - 0.5
    b = torch.randn(Du, generator=gen, device=dev) * 0.1
    for name, S, circular in (("config3a_update_linear", 3, False), ("config3b_update_circular", 16, True)):
        for layout in ("channel_last", "contiguous"):
            nsets = 32 if S == 3 else 16
            fns = []
            for _ in range(nsets):
                x = torch.randn(Bu, Du, generator=gen, device=dev).to(torch.bfloat16)
                if layout == "channel_last":
                    st = torch.randn(Bu, S, Du, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
                else:
                    st = torch.randn(Bu, Du, S, generator=gen, device=dev).to(torch.bfloat16)
                cache = torch.randint(0, 1000, (Bu,), generator=gen, device=dev, dtype=torch.int32) if circular else None
                idx = torch.randperm(Bu, generator=gen, device=dev).to(torch.int32) if circular else None
                fns.append(lambda x=x, st=st, cache=cache, idx=idx: causal_conv1d_update(
                    x, st, w, b, activation="silu", cache_seqlens=cache, conv_state_indices=idx))
            us = graph_time(fns)
            es = 2
            if circular:
                nbytes = Bu * Du * es * (1 + (W - 1) + 1 + 1) + Bu * 8
            else:
                nbytes = Bu * Du * es * (1 + 2 * S + 1)
            res[f"{name}_{layout}"] = entry(nbytes, us)

    # config 4: varlen states on (65536, 5120) fp16, 32 sequences, state_len 3
    T, Dv, S = 65536, 5120, 3
    xv = torch.randn(T, Dv, generator=gen, device=dev).to(torch.float16)
    fns = []
    cpu_gen = torch.Generator().manual_seed(0)
    for _ in range(32):
        lens = 1 + torch.bincount(torch.multinomial(torch.full((32,), 1 / 32), T - 32, replacement=True,
                                                    generator=cpu_gen), minlength=32)
        cu = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).to(dev)
        fns.append(lambda cu=cu: causal_conv1d_varlen_states(xv, cu, S))
    res["config4_varlen_states"] = entry(2 * 32 * S * Dv * 2 + 33 * 4, graph_time(fns))
    del xv

    # config 4: packed varlen fwd+bwd, fp16 (1, 5120, 65536) channel-last, seq_idx from the split
    lens = 1 + torch.bincount(torch.multinomial(torch.full((32,), 1 / 32), T - 32, replacement=True,
                                                generator=torch.Generator().manual_seed(0)), minlength=32)
    seq = torch.repeat_interleave(torch.arange(32, dtype=torch.int32), lens).view(1, T).to(dev)
    x = torch.randn(1, T, Dv, generator=gen, device=dev).to(torch.float16).transpose(1, 2)
    g = torch.randn(1, T, Dv, generator=gen, device=dev).to(torch.float16).transpose(1, 2)
    w4 = torch.rand(Dv, 4, generator=gen, device=dev) - 0.5
    b4 = torch.randn(Dv, generator=gen, device=dev) * 0.1
    n = T * Dv
    us = graph_time([lambda: causal_conv1d_fwd_function(x, w4, b4, seq, None, None, True)] * 4, reps=3)
    res["config4_fwd_seq_idx"] = entry(2 * n * 2 + T * 4 + Dv * 20, us)
    # the same forward also writing the 32 sequences' decode states (state_len 3) in one pass
    cu4 = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).to(dev)
    us = graph_time([lambda: causal_conv1d_fn_varlen_states(x, w4, cu4, S, b4, seq, "silu")] * 4, reps=3)
    res["config4_fwd_seq_idx_with_states"] = entry(2 * n * 2 + T * 4 + Dv * 20 + 33 * 4 + 32 * S * Dv * 2, us)
    us = graph_time([lambda: causal_conv1d_bwd_function(x, w4, b4, g, seq, None, None, None, False, True)] * 4,
                    reps=3)
    res["config4_bwd_seq_idx"] = entry(3 * n * 2 + T * 4 + Dv * 40, us)
    del x, g

    # config 5: (8, 16384, 8192) fp16/bf16 sweep point, W=4, silu, both layouts
    B5, D5, L5 = 8, 16384, 8192
    n5 = B5 * D5 * L5
    w5 = torch.rand(D5, 4, generator=gen, device=dev) - 0.5
    b5 = torch.randn(D5, generator=gen, device=dev) * 0.1
    for layout in ("channel_last", "contiguous"):
        if layout == "channel_last":
            x = torch.randn(B5, L5, D5, generator=gen, device=dev, dtype=torch.bfloat16).transpose(1, 2)
        else:
            x = torch.randn(B5, D5, L5, generator=gen, device=dev, dtype=torch.bfloat16)
        g = torch.randn_like(x)
        us = graph_time([lambda: causal_conv1d_fwd_function(x, w5, b5, None, None, None, True)] * 2, reps=2)
        res[f"config5_fwd_bf16_w4_{layout}"] = entry(2 * n5 * 2 + D5 * 20, us)
        us = graph_time([lambda: causal_conv1d_bwd_function(x, w5, b5, g, None, None, None, None, False, True)] * 2,
                        reps=2)
        res[f"config5_bwd_bf16_w4_{layout}"] = entry(3 * n5 * 2 + D5 * 40, us)
        del x, g
        torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-extras", action="store_true", help="skip the per-config kernel table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
