"""Benchmark of the causal_conv1d hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --case NAME [--repeat R]      # one kernel case, for ncu captures

Headline workload (benchmark config 5, the largest single-GPU config): bf16 x
(8, 16384, 8192) channel-last, fp32 weight (16384, 4) ~U(-0.5, 0.5) and bias ~N(0, 0.1),
SiLU; one step = forward + backward (dx, dweight, dbias).  With N ranks the channels are
sharded: rank r owns 16384/N channels of every batch row, allocates its own shard and
runs the same step on it; there is no collective on this path (strong scaling: the
total problem is fixed).  Metric: algorithmic HBM GB/s (every tensor element read or
written once), summed over ranks, over the max-over-ranks device time.  Every tensor is
larger than L2 (2 GiB / N >= 256 MiB each), so nothing is re-read from L2 across steps.

Timing: each of the K timed steps replays a CUDA graph of the forward and one of the
backward, with a CUDA event after each pass, after W warm-up steps; the step total and each
pass's average duration (the roofline's "achieved") come from those events.

Per-N figures printed beside the headline: the batch-sharded backward (each rank B/N
batch rows of all channels) with its NCCL all-reduce of dweight|dbias, as kernel time,
all-reduce time and overlapped step time; the decode update (config 3) sharded over
batch with no collective.  At N=1 the `kernels` table adds the other configs, the config-5
sweep (fp16/bf16 x width 2/3/4 x activation x both layouts), the strided-slice
(producer/consumer) case and, when the reference is installed under baseline/_ref, its
own CuTe DSL kernels timed on the same inputs (alternating order, median of 5).

`--impl reference` times the reference's own CPU path, `causal_conv1d_ref` with an
autograd backward (PyTorch on all host cores), on a channel slice of the headline
workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_PARENT = os.path.join(ROOT, "cute-causal-conv1d_b200")
REF_INSTALL = os.path.join(ROOT, "baseline", "_ref")

METRIC = "fwd/bwd/update achieved HBM GB/s and % of 8 TB/s roofline at 1/2/4/8 B200"
CFG5 = dict(batch=8, dim=16384, seqlen=8192, width=4)
CFG2 = dict(batch=4, dim=4096, seqlen=2048, width=4)
CFG3 = dict(batch=128, dim=8192, width=4)
CFG4 = dict(tokens=65536, dim=5120, nseq=32, width=4, state_len=3)


def _package_path():
    for p in (ROOT, PKG_PARENT):
        if p not in sys.path:
            sys.path.insert(0, p)


def conv_bytes(batch, dim, seqlen, width, es=2, *, bias=True, init=False, final=False, seq=False, pes=4):
    """Algorithmic bytes of one forward and one backward (each element read or written once)."""
    n = batch * dim * seqlen
    states = batch * dim * (width - 1) * es
    params = dim * width * pes + (dim * pes if bias else 0)
    seqb = batch * seqlen * 4 if seq else 0
    fwd = 2 * n * es + params + (states if init else 0) + (states if final else 0) + seqb
    bwd = 3 * n * es + 2 * params + (2 * states if init else 0) + (states if final else 0) + seqb
    return fwd, bwd


def update_bytes(batch, dim, width, state_len, circular, es=2):
    """Algorithmic bytes of one single-token update: x, the state entries read and written,
    out, the parameters, and cache_seqlens / conv_state_indices when present."""
    params = dim * width * 4 + dim * 4
    if circular:  # W-1 history reads, one state write
        return batch * dim * es * (1 + (width - 1) + 1 + 1) + params + batch * 8
    return batch * dim * es * (1 + 2 * state_len + 1) + params  # the whole state shifts


# ------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples the SM clock and clock-event reasons through NVML every millisecond while
    the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period: float = 0.001):
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

    def _sample(self):
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
            self.reasons |= int(self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
        except Exception:
            pass

    def _run(self):
        while not self._stop.wait(self.period):
            self._sample()

    def __enter__(self):
        if self.handle is not None:
            self._sample()  # one sample as the region starts, then one per period
            self.thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.handle is not None:
            self.thread.join()
            self._sample()  # and one as it ends (before the host synchronises)
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
def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _host_cores():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def _reference_cpu_fn():
    """(causal_conv1d_ref, kind): the reference's own function from its installed copy
    (this process must not have imported the B200 package, which has the same module
    name), else the stand-in restatement in oracle/torch_ref.py."""
    if os.path.isdir(os.path.join(REF_INSTALL, "causal_conv1d")):
        sys.path.insert(0, REF_INSTALL)
        try:
            from causal_conv1d.causal_conv1d_interface import causal_conv1d_ref

            return causal_conv1d_ref, "reference"
        except Exception:
            sys.path.remove(REF_INSTALL)
            for m in [m for m in sys.modules if m == "causal_conv1d" or m.startswith("causal_conv1d.")]:
                del sys.modules[m]
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle.torch_ref import causal_conv1d_ref

    return causal_conv1d_ref, "port"


def cpu_measure(run_target_s: float, runs: int, warmup: int, want_c_port: bool = True):
    """Time the reference's CPU path (causal_conv1d_ref forward + autograd backward, PyTorch
    on every host core) on a channel slice of the headline workload, sized so one run takes
    about ``run_target_s``; ``runs`` timed runs after ``warmup``.  The C restatement
    (oracle/cc1d_oracle.c, OpenMP) is timed on the same slice as a second figure."""
    import torch

    cores = _host_cores()
    torch.set_num_threads(cores)
    fn, kind = _reference_cpu_fn()
    B, D, L, W = CFG5["batch"], CFG5["dim"], CFG5["seqlen"], CFG5["width"]
    gen = torch.Generator().manual_seed(11)

    def make(ch):
        x = torch.randn(B, L, ch, generator=gen).to(torch.bfloat16).transpose(1, 2).requires_grad_()
        w = (torch.rand(ch, W, generator=gen) - 0.5).requires_grad_()
        b = (torch.randn(ch, generator=gen) * 0.1).requires_grad_()
        g = torch.randn(B, L, ch, generator=gen).to(torch.bfloat16).transpose(1, 2)
        return x, w, b, g

    def run(data):
        x, w, b, g = data
        x.grad = w.grad = b.grad = None
        out = fn(x, w, b, activation="silu")
        out.backward(g)

    ch = 64
    data = make(ch)
    run(data)
    t0 = time.perf_counter()
    run(data)
    dt = time.perf_counter() - t0
    ch = int(min(D, max(64, ch * run_target_s / max(dt, 1e-4))))
    ch = max(64, ch // 64 * 64)
    data = make(ch)
    for _ in range(warmup):
        run(data)
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        run(data)
        times.append(time.perf_counter() - t0)
    fb, bb = conv_bytes(B, ch, L, W)
    res = {
        "kind": kind, "cores": cores, "cpu_model": _cpu_model(), "channels": ch,
        "bytes_per_run": fb + bb, "times_s": [round(t, 4) for t in times],
        "median_GBps": (fb + bb) / statistics.median(times) / 1e9,
        "total_GBps": (fb + bb) * runs / sum(times) / 1e9,
        "sample": (f"config-5 fwd+bwd on a {ch}-channel slice: x ({B}, {ch}, {L}) bf16 channel-last, "
                   f"W={W}, silu, bias; causal_conv1d_ref + autograd backward, torch CPU, {cores} threads"),
    }
    if want_c_port:
        res["c_port"] = c_port_measure(ch, runs)
    return res


def c_port_measure(ch, runs):
    """oracle/cc1d_oracle.c (OpenMP, all host cores) on the same config-5 slice."""
    import numpy as np

    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import c_oracle
    from oracle import numpy_oracle as O

    c_oracle.build()
    cores = c_oracle.use_all_cores()
    B, L, W = CFG5["batch"], CFG5["seqlen"], CFG5["width"]
    rng = np.random.default_rng(0)
    x = O.f32_to_bf16_bits(rng.standard_normal((B, L, ch), dtype=np.float32)).transpose(0, 2, 1)
    dout = O.f32_to_bf16_bits(rng.standard_normal((B, L, ch), dtype=np.float32)).transpose(0, 2, 1)
    w = rng.uniform(-0.5, 0.5, (ch, W)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(ch)).astype(np.float32)

    def run():
        c_oracle.fwd(x, "bfloat16", w, bias, silu=True)
        c_oracle.bwd(x, "bfloat16", w, dout, bias, silu=True)

    run()
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    fb, bb = conv_bytes(B, ch, L, W)
    return {"GB/s": round((fb + bb) / statistics.median(times) / 1e9, 3), "cores": cores,
            "kind": "port", "sample": f"oracle/cc1d_oracle.c fwd+bwd on the same {ch}-channel slice, median of {runs}"}


def cpu_child(args):
    """Entry of ``bench.py --cpu-child``: prints one JSON object (run in a fresh process so
    that the reference's package can be imported under its own name)."""
    res = cpu_measure(args.cpu_run_s, args.cpu_runs, 1)
    print("CPUJSON " + json.dumps(res), flush=True)
    return 0


def cpu_baseline_subprocess(run_s=3.0, runs=5):
    cmd = [sys.executable, os.path.abspath(__file__), "--cpu-child", "--cpu-run-s", str(run_s),
           "--cpu-runs", str(runs)]
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    except subprocess.TimeoutExpired:
        return None
    for line in out.stdout.splitlines():
        if line.startswith("CPUJSON "):
            return json.loads(line[len("CPUJSON "):])
    sys.stderr.write(out.stdout[-2000:] + out.stderr[-2000:])
    return None


def config_dict(n):
    d = CFG5["dim"] // n
    return {"workload": "config5: causal_conv1d fwd+bwd, bf16 x (8,16384,8192) channel-last, W=4, silu, bias, "
                        "fp32 weight/bias; channels sharded over ranks (no collective)",
            "global_batch": CFG5["batch"], "seq_len": CFG5["seqlen"], "dim": CFG5["dim"], "width": CFG5["width"],
            "dim_per_rank": d, "parallelism": f"dim-shard{n}" if n > 1 else "single",
            "l2": "no rotation needed: x, dout, out and dx are each 2 GiB/N >= 256 MiB, larger than the 126 MB L2"}


def run_reference(args):
    """The reference arm: the reference's own CPU path on this box's host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n = args.steps + args.warmup
    run_s = min(5.0, max(0.2, 75.0 / max(1, n)))
    res = cpu_measure(run_s, args.steps, args.warmup)
    value = res["total_GBps"]
    total_s = sum(res["times_s"])
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_s / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": res["cores"], "kind": res["kind"],
                         "cpu_model": res["cpu_model"], "sample": res["sample"] + " per step",
                         "median_GBps": round(res["median_GBps"], 3), "c_port": res.get("c_port")},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU helpers
def capture(fns):
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    return g


def replay_ms(g, reps=1):
    import torch

    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(reps):
        g.replay()
    s1.record()
    torch.cuda.synchronize()
    return s0.elapsed_time(s1) / reps


def graph_us(fns, reps=5):
    """Average device time per call of a list of launch closures captured in one CUDA graph
    (launch latency does not hide the kernel time)."""
    import torch

    for f in fns:
        f()
    torch.cuda.synchronize()
    g = capture(fns)
    g.replay()
    torch.cuda.synchronize()
    return replay_ms(g, reps) / len(fns) * 1e3


def rank_max(values, world, dev):
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def entry(nbytes, us, peak):
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"GB/s": round(gbs, 1), "us": round(us, 3), "bytes": int(nbytes), "frac_of_peak": round(gbs / peak, 4)}


def cl_randn(shape_bdl, dtype, gen, dev):
    """(batch, dim, seqlen) tensor stored channel-last."""
    import torch

    B, D, L = shape_bdl
    return torch.randn(B, L, D, generator=gen, device=dev, dtype=dtype).transpose(1, 2)


# ------------------------------------------------------------------ our arm
def headline(args, dev, world, rank, sampler_index):
    """Config-5 forward+backward on this rank's channel shard: K steps, each a replay of a
    one-launch forward graph and of a backward graph."""
    import torch
    import torch.distributed as dist

    from causal_conv1d import _abi
    from causal_conv1d.distributed import shard_range

    B, D, L, W = CFG5["batch"], CFG5["dim"], CFG5["seqlen"], CFG5["width"]
    d0, d1 = shard_range(D, world, rank, 8)
    Dr = d1 - d0
    gen = torch.Generator(device=dev).manual_seed(5000 + rank)
    x = cl_randn((B, Dr, L), torch.bfloat16, gen, dev)
    dout = cl_randn((B, Dr, L), torch.bfloat16, gen, dev)
    out = torch.empty_like(x)
    dx = torch.empty_like(x)
    w = torch.rand(Dr, W, generator=gen, device=dev) - 0.5
    b = torch.randn(Dr, generator=gen, device=dev) * 0.1
    dw = torch.empty(Dr, W, device=dev)
    db = torch.empty(Dr, device=dev)
    need = _abi.bwd_workspace_bytes(x, w, b, dout, None, None, None, dx, None, dw, db, True)
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)

    def fwd():
        _abi.fwd(x, w, b, None, None, None, out, True)

    def bwd():
        _abi.bwd(x, w, b, dout, None, None, None, dx, None, dw, db, True, workspace=ws)

    fwd()
    bwd()
    torch.cuda.synchronize()
    n0 = _abi.launch_count()
    g_fwd = capture([fwd])
    g_bwd = capture([bwd])
    launches = (_abi.launch_count() - n0) * args.steps  # kernels of the K timed steps
    for _ in range(args.warmup):
        g_fwd.replay()
        g_bwd.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # The K timed steps replay the forward and backward graphs in turn, with an event
    # after each pass: the events give the step total and each pass's own duration inside
    # the timed region (the roofline's "achieved").
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    sampler = ClockSampler(sampler_index)
    with sampler:
        ev[0].record()
        for i in range(args.steps):
            g_fwd.replay()
            ev[2 * i + 1].record()
            g_bwd.replay()
            ev[2 * i + 2].record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = ev[0].elapsed_time(ev[-1])
    fwd_us = statistics.mean(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) * 1e3
    bwd_us = statistics.mean(ev[2 * i + 1].elapsed_time(ev[2 * i + 2]) for i in range(args.steps)) * 1e3
    total_ms, fwd_us, bwd_us = rank_max([total_ms, fwd_us, bwd_us], world, dev)
    fb, bb = conv_bytes(B, Dr, L, W)
    res = dict(total_ms=total_ms, fwd_us=fwd_us, bwd_us=bwd_us, fwd_bytes=fb, bwd_bytes=bb,
               launches=launches, clocks=sampler.result(), dim_per_rank=Dr)
    del g_fwd, g_bwd
    return res


def batch_sharded_bwd(args, dev, world, rank):
    """Config-5 backward sharded over batch: each rank runs its B/N rows of all channels,
    then one NCCL all-reduce of the flat fp32 dweight|dbias bucket.  Kernel time,
    all-reduce time and the overlapped step (the all-reduce of step i on a side stream
    under the backward of step i+1, two buckets) are timed separately."""
    import torch
    import torch.distributed as dist

    from causal_conv1d import _abi
    from causal_conv1d.distributed import GradBucket, allreduce_param_grads, shard_range

    B, D, L, W = CFG5["batch"], CFG5["dim"], CFG5["seqlen"], CFG5["width"]
    b0, b1 = shard_range(B, world, rank)
    Br = b1 - b0
    gen = torch.Generator(device=dev).manual_seed(6000 + rank)
    x = cl_randn((Br, D, L), torch.bfloat16, gen, dev)
    dout = cl_randn((Br, D, L), torch.bfloat16, gen, dev)
    dx = torch.empty_like(x)
    pg = torch.Generator(device=dev).manual_seed(6000)  # the same parameters on every rank
    w = torch.rand(D, W, generator=pg, device=dev) - 0.5
    b = torch.randn(D, generator=pg, device=dev) * 0.1
    buckets = [GradBucket(D, W, True, dev) for _ in range(2)]
    need = _abi.bwd_workspace_bytes(x, w, b, dout, None, None, None, dx, None,
                                    buckets[0].dweight, buckets[0].dbias, True)
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)

    def bwd(k):
        _abi.bwd(x, w, b, dout, None, None, None, dx, None, buckets[k].dweight, buckets[k].dbias, True,
                 workspace=ws)

    K = max(4, args.steps)
    bwd(0)
    side = torch.cuda.Stream(dev)
    if world > 1:
        allreduce_param_grads(buckets[0])
        with torch.cuda.stream(side):
            allreduce_param_grads(buckets[1])
    torch.cuda.synchronize()

    def settle():  # every rank starts each timed replay together
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    g_kern = capture([lambda k=i % 2: bwd(k) for i in range(K)])
    settle()
    kern_us = replay_ms(g_kern, 2) / K * 1e3
    del g_kern
    ar_us = 0.0
    step_us = kern_us
    if world > 1:
        g_ar = capture([lambda k=i % 2: allreduce_param_grads(buckets[k]) for i in range(K)])
        g_ar.replay()
        settle()
        ar_us = replay_ms(g_ar, 2) / K * 1e3
        del g_ar
        done = [torch.cuda.Event() for _ in range(2)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            cap = torch.cuda.current_stream()
            for i in range(K):
                k = i % 2
                if i >= 2:
                    cap.wait_event(done[k])  # the all-reduce that last read this bucket
                bwd(k)
                side.wait_stream(cap)
                with torch.cuda.stream(side):
                    allreduce_param_grads(buckets[k])
                    done[k].record(side)
            cap.wait_stream(side)
        g.replay()
        settle()
        step_us = replay_ms(g, 2) / K * 1e3
        del g
    kern_us, ar_us, step_us = rank_max([kern_us, ar_us, step_us], world, dev)
    _, bb = conv_bytes(Br, D, L, W)
    return {"batch_per_rank": Br, "kernel_us": round(kern_us, 2), "allreduce_us": round(ar_us, 2),
            "step_us": round(step_us, 2), "allreduce_bytes": (D * W + D) * 4,
            "GB/s": round(bb * world / (step_us * 1e-6) / 1e9, 1),
            "kernel_GB/s_per_rank": round(bb / (kern_us * 1e-6) / 1e9, 1)}


def update_sharded(dev, world, rank, peak):
    """Config-3 decode update sharded over batch rows (no collective); aggregate GB/s =
    all ranks' bytes over the max-over-ranks device time of one launch."""
    import torch

    from causal_conv1d import causal_conv1d_update
    from causal_conv1d.distributed import shard_range

    Bu, Du, W = CFG3["batch"], CFG3["dim"], CFG3["width"]
    b0, b1 = shard_range(Bu, world, rank)
    Br = b1 - b0
    gen = torch.Generator(device=dev).manual_seed(7000 + rank)
    pg = torch.Generator(device=dev).manual_seed(7000)
    w = torch.rand(Du, W, generator=pg, device=dev) - 0.5
    b = torch.randn(Du, generator=pg, device=dev) * 0.1
    res = {}
    for name, S, circular in (("config3a_update_linear", 3, False), ("config3b_update_circular", 16, True)):
        for layout in ("channel_last", "contiguous"):
            fns = []
            for _ in range(16):
                x = torch.randn(Br, Du, 1, generator=gen, device=dev).to(torch.bfloat16)
                if layout == "channel_last":
                    st = torch.randn(Br, S, Du, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
                else:
                    st = torch.randn(Br, Du, S, generator=gen, device=dev).to(torch.bfloat16)
                cache = torch.randint(0, 1000, (Br,), generator=gen, device=dev, dtype=torch.int32) if circular else None
                idx = torch.randperm(Br, generator=gen, device=dev).to(torch.int32) if circular else None
                fns.append(lambda x=x, st=st, cache=cache, idx=idx: causal_conv1d_update(
                    x, st, w, b, activation="silu", cache_seqlens=cache, conv_state_indices=idx))
            us = rank_max([graph_us(fns)], world, dev)[0]
            nbytes = update_bytes(Br, Du, W, S, circular) * world
            res[f"{name}_{layout}"] = entry(nbytes, us, peak * world)
            res[f"{name}_{layout}"]["batch_per_rank"] = Br
    return res


def run_e2e(args, dev, world, rank):
    """The headline metric through the public API (causal_conv1d_fn + autograd) with
    pinned host buffers: every step copies its inputs (x, dout, weight, bias) in and its
    results (out, dx, dweight, dbias) out inside the timed region."""
    import torch
    import torch.distributed as dist

    from causal_conv1d import causal_conv1d_fn
    from causal_conv1d.distributed import shard_range

    B, D, L, W = CFG5["batch"], CFG5["dim"], CFG5["seqlen"], CFG5["width"]
    d0, d1 = shard_range(D, world, rank, 8)
    Dr = d1 - d0
    gen = torch.Generator(device=dev).manual_seed(8000 + rank)

    def pinned_from_device(t):
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h

    hx = pinned_from_device(torch.randn(B, L, Dr, generator=gen, device=dev, dtype=torch.bfloat16))
    hg = pinned_from_device(torch.randn(B, L, Dr, generator=gen, device=dev, dtype=torch.bfloat16))
    hw = pinned_from_device(torch.rand(Dr, W, generator=gen, device=dev) - 0.5)
    hb = pinned_from_device(torch.randn(Dr, generator=gen, device=dev) * 0.1)
    outs = dict(out=torch.empty(B, L, Dr, dtype=torch.bfloat16, pin_memory=True),
                dx=torch.empty(B, L, Dr, dtype=torch.bfloat16, pin_memory=True),
                dw=torch.empty(Dr, W, pin_memory=True), db=torch.empty(Dr, pin_memory=True))
    h2d = sum(t.numel() * t.element_size() for t in (hx, hg, hw, hb))
    d2h = sum(t.numel() * t.element_size() for t in outs.values())
    torch.cuda.empty_cache()

    # Three streams and two device input buffers: the copy-in of step i+1 and the copy-out
    # of step i-1 run on the copy engines while step i computes.
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [dict(x=torch.empty(B, L, Dr, dtype=torch.bfloat16, device=dev),
                 g=torch.empty(B, L, Dr, dtype=torch.bfloat16, device=dev),
                 w=torch.empty(Dr, W, device=dev), b=torch.empty(Dr, device=dev)) for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    for e in in_free:
        e.record(comp)

    def step(i):
        k = i % 2
        buf = bufs[k]
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[k])
            for name, host in (("x", hx), ("g", hg), ("w", hw), ("b", hb)):
                buf[name].copy_(host, non_blocking=True)
            in_ready[k].record(s_in)
        comp.wait_event(in_ready[k])
        x = buf["x"].transpose(1, 2).detach().requires_grad_()
        w = buf["w"].detach().requires_grad_()
        b = buf["b"].detach().requires_grad_()
        out = causal_conv1d_fn(x, w, b, activation="silu")
        torch.autograd.backward([out], [buf["g"].transpose(1, 2)])
        res = dict(out=out.transpose(1, 2), dx=x.grad.transpose(1, 2), dw=w.grad, db=b.grad)
        in_free[k].record(comp)
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for name, t in res.items():
                t.record_stream(s_out)
                outs[name].copy_(t, non_blocking=True)

    step(0)
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
    ms = rank_max([s0.elapsed_time(s1)], world, dev)[0]
    fb, bb = conv_bytes(B, Dr, L, W)
    del bufs
    torch.cuda.empty_cache()
    return {"value": round((fb + bb) * world * n / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / n, 3),
            "steps": n,
            "path": "causal_conv1d_fn + autograd backward, pinned host buffers, copies overlapped with "
                    "compute on two copy streams"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        # the only collective moves 320 KB: NVLink SHARP brings nothing at that size, so it
        # stays off (no multicast memory objects are created)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from causal_conv1d import _abi

    _abi.load_library()
    peak, peak_kind = measured_peak()

    h = headline(args, dev, world, rank, local)
    torch.cuda.empty_cache()
    ms_per_step = h["total_ms"] / args.steps
    value = (h["fwd_bytes"] + h["bwd_bytes"]) * world * args.steps / (h["total_ms"] / 1e3) / 1e9
    achieved = h["bwd_bytes"] / (h["bwd_us"] * 1e-6) / 1e9  # the dominant kernel: the backward
    per_n = {
        "headline_fwd_us": round(h["fwd_us"], 2), "headline_bwd_us": round(h["bwd_us"], 2),
        "headline_kernel_sum_us": round(h["fwd_us"] + h["bwd_us"], 2),
        "headline_step_us": round(ms_per_step * 1e3, 2),
        "step_over_kernel_sum": round(ms_per_step * 1e3 / (h["fwd_us"] + h["bwd_us"]), 4),
        "dim_per_rank": h["dim_per_rank"],
    }
    if not args.no_extras:
        per_n["bwd_batch_sharded"] = batch_sharded_bwd(args, dev, world, rank)
        torch.cuda.empty_cache()
        per_n["update_batch_sharded"] = update_sharded(dev, world, rank, peak)
        torch.cuda.empty_cache()
    e2e = run_e2e(args, dev, world, rank) if not args.no_e2e else None
    kernels = {}
    if world == 1 and not args.no_extras and not args.no_kernel_table:
        kernels = kernel_table(dev, peak, args)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        res = cpu_baseline_subprocess()
        if res is not None:
            cpu = {"value": round(res["median_GBps"], 3), "unit": "GB/s", "cores": res["cores"], "kind": res["kind"],
                   "cpu_model": res["cpu_model"], "sample": res["sample"] + ", median of 5 after 1 warm run",
                   "c_port": res.get("c_port")}
    fb, bb = h["fwd_bytes"], h["bwd_bytes"]
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config_dict(world),
        "roofline": {"bound": "hbm", "kernel": "bwd_stream_kernel + reduce_unit_partials (config-5 backward, per rank)",
                     "achieved": round(achieved, 1), "peak": peak, "peak_source": f"{peak_kind} hbm_gbs", "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": ncu_traffic(f"config5_bwd_n{world}"),
                     "algorithmic_bytes": bb, "launch_us": round(h["bwd_us"], 2),
                     "fwd_frac": round(fb / (h["fwd_us"] * 1e-6) / 1e9 / peak, 4)},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": h["launches"],
        "clocks": h["clocks"],
        "per_n": per_n,
        "kernels": kernels,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------- kernel table (N=1)
def kernel_table(dev, peak, args):
    """Kernel-level numbers for the other benchmark configs (outside the timed step)."""
    import torch

    from causal_conv1d import causal_conv1d_update
    from causal_conv1d.causal_conv1d_varlen import causal_conv1d_fn_varlen_states, causal_conv1d_varlen_states
    from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function

    res = {}
    gen = torch.Generator(device=dev).manual_seed(3)

    # config 2: bf16 (4, 4096, 2048) channel-last, W=4, silu, initial + final states; 4 input
    # sets (1 GiB) rotate so that no launch reads what the previous ones left in L2
    B, D, L, W = CFG2["batch"], CFG2["dim"], CFG2["seqlen"], CFG2["width"]
    w2 = torch.rand(D, W, generator=gen, device=dev) - 0.5
    b2 = torch.randn(D, generator=gen, device=dev) * 0.1
    sets = []
    for _ in range(4):
        sets.append(dict(x=cl_randn((B, D, L), torch.bfloat16, gen, dev), g=cl_randn((B, D, L), torch.bfloat16, gen, dev),
                         init=torch.randn(B, D, W - 1, generator=gen, device=dev).to(torch.bfloat16),
                         final=torch.empty(B, W - 1, D, device=dev, dtype=torch.bfloat16).transpose(1, 2),
                         dfinal=torch.zeros(B, D, W - 1, device=dev, dtype=torch.bfloat16)))
    fb, bb = conv_bytes(B, D, L, W, init=True, final=True)
    us = graph_us([lambda s=s: causal_conv1d_fwd_function(s["x"], w2, b2, None, s["init"], s["final"], True)
                   for s in sets] * 4)
    res["config2_fwd"] = entry(fb, us, peak)
    us = graph_us([lambda s=s: causal_conv1d_bwd_function(s["x"], w2, b2, s["g"], None, s["init"], s["dfinal"], None,
                                                          True, True) for s in sets] * 4)
    res["config2_bwd"] = entry(bb, us, peak)
    fb0, bb0 = conv_bytes(B, D, L, W)
    us = graph_us([lambda s=s: causal_conv1d_fwd_function(s["x"], w2, b2, None, None, None, True) for s in sets] * 4)
    res["config2_fwd_stateless"] = entry(fb0, us, peak)
    us = graph_us([lambda s=s: causal_conv1d_bwd_function(s["x"], w2, b2, s["g"], None, None, None, None, False, True)
                   for s in sets] * 4)
    res["config2_bwd_stateless"] = entry(bb0, us, peak)
    del sets

    # the reference README's two forward shapes (channel-last, silu), 32 rotating sets
    for name, shape, W_, dt in (("readme_fwd_fp16_w3_1x2048x2048", (1, 2048, 2048), 3, torch.float16),
                                ("readme_fwd_bf16_w4_1x4096x2048", (1, 4096, 2048), 4, torch.bfloat16)):
        xs = [cl_randn(shape, dt, gen, dev) for _ in range(32)]
        wr = torch.rand(shape[1], W_, generator=gen, device=dev) - 0.5
        br = torch.randn(shape[1], generator=gen, device=dev) * 0.1
        us = graph_us([lambda x=x: causal_conv1d_fwd_function(x, wr, br, None, None, None, True) for x in xs])
        res[name] = entry(conv_bytes(*shape, W_)[0], us, peak)
        del xs

    # config 3: decode update, B=128, D=8192, bf16, silu
    res.update(update_sharded(dev, 1, 0, peak))

    # What a plain device copy (torch copy_) of the same number of bytes reaches in the same
    # graph harness: the floor that launch, first-load latency and drain put under a
    # kernel moving 2-34 MB (the update and small forward rows above).
    for mb in (2, 8, 17, 34):
        n = mb * (1 << 20) // 2  # bytes read = bytes written
        pairs = [(torch.empty(n, dtype=torch.uint8, device=dev), torch.empty(n, dtype=torch.uint8, device=dev))
                 for _ in range(max(4, 512 // mb))]
        res[f"calibration_copy_{mb}MB"] = entry(2 * n, graph_us([lambda a=a, c=c: c.copy_(a) for a, c in pairs]), peak)
        del pairs

    # config 4: varlen states on (65536, 5120) fp16, 32 sequences, state_len 3
    T, Dv, S, nseq = CFG4["tokens"], CFG4["dim"], CFG4["state_len"], CFG4["nseq"]
    xv = torch.randn(T, Dv, generator=gen, device=dev).to(torch.float16)
    fns = []
    cpu_gen = torch.Generator().manual_seed(0)
    for _ in range(32):
        lens = 1 + torch.bincount(torch.multinomial(torch.full((nseq,), 1 / nseq), T - nseq, replacement=True,
                                                    generator=cpu_gen), minlength=nseq)
        cu = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).to(dev)
        fns.append(lambda cu=cu: causal_conv1d_varlen_states(xv, cu, S))
    res["config4_varlen_states"] = entry(2 * nseq * S * Dv * 2 + (nseq + 1) * 4, graph_us(fns), peak)
    del xv

    # config 4: packed varlen fwd+bwd, fp16 (1, 5120, 65536) channel-last, seq_idx from the split
    lens = 1 + torch.bincount(torch.multinomial(torch.full((nseq,), 1 / nseq), T - nseq, replacement=True,
                                                generator=torch.Generator().manual_seed(0)), minlength=nseq)
    seq = torch.repeat_interleave(torch.arange(nseq, dtype=torch.int32), lens).view(1, T).to(dev)
    x = cl_randn((1, Dv, T), torch.float16, gen, dev)
    g = cl_randn((1, Dv, T), torch.float16, gen, dev)
    w4 = torch.rand(Dv, 4, generator=gen, device=dev) - 0.5
    b4 = torch.randn(Dv, generator=gen, device=dev) * 0.1
    fb, bb = conv_bytes(1, Dv, T, 4, seq=True)
    us = graph_us([lambda: causal_conv1d_fwd_function(x, w4, b4, seq, None, None, True)] * 4, reps=3)
    res["config4_fwd_seq_idx"] = entry(fb, us, peak)
    cu4 = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).to(dev)
    us = graph_us([lambda: causal_conv1d_fn_varlen_states(x, w4, cu4, S, b4, seq, "silu")] * 4, reps=3)
    res["config4_fwd_seq_idx_with_states"] = entry(fb + (nseq + 1) * 4 + nseq * S * Dv * 2, us, peak)
    us = graph_us([lambda: causal_conv1d_bwd_function(x, w4, b4, g, seq, None, None, None, False, True)] * 4, reps=3)
    res["config4_bwd_seq_idx"] = entry(bb, us, peak)
    del x, g
    torch.cuda.empty_cache()

    # config 5 sweep: fp16/bf16 x width 2/3/4 x activation none/silu x both layouts
    B5, D5, L5 = CFG5["batch"], CFG5["dim"], CFG5["seqlen"]
    for dt, dname in ((torch.bfloat16, "bf16"), (torch.float16, "fp16")):
        for layout in ("channel_last", "contiguous"):
            if layout == "channel_last":
                x = cl_randn((B5, D5, L5), dt, gen, dev)
                g = cl_randn((B5, D5, L5), dt, gen, dev)
            else:
                x = torch.randn(B5, D5, L5, generator=gen, device=dev, dtype=dt)
                g = torch.randn(B5, D5, L5, generator=gen, device=dev, dtype=dt)
            out = torch.empty_like(x)
            dx = torch.empty_like(x)
            for W_ in (2, 3, 4):
                w5 = torch.rand(D5, W_, generator=gen, device=dev) - 0.5
                b5 = torch.randn(D5, generator=gen, device=dev) * 0.1
                fb, bb = conv_bytes(B5, D5, L5, W_)
                for act in ("none", "silu"):
                    silu = act == "silu"
                    tag = f"{dname}_w{W_}_{act}_{layout}"
                    us = graph_us([lambda: causal_conv1d_fwd_function(x, w5, b5, None, None, None, silu)] * 2, reps=2)
                    res[f"config5_fwd_{tag}"] = entry(fb, us, peak)
                    us = graph_us([lambda: causal_conv1d_bwd_function(x, w5, b5, g, None, None, None, dx, False, silu)] * 2,
                                  reps=2)
                    res[f"config5_bwd_{tag}"] = entry(bb, us, peak)
                    torch.cuda.empty_cache()
            del x, g, out, dx
            torch.cuda.empty_cache()

    # producer/consumer fusion: x is the [..., D:2D] channel slice of a (B, L, 3D) projection,
    # dx is written into the same slice of a (B, L, 3D) gradient buffer
    proj = torch.randn(B5, L5, 3 * D5, generator=gen, device=dev, dtype=torch.bfloat16)
    gproj = torch.empty_like(proj)
    x = proj[..., D5:2 * D5].transpose(1, 2)
    dx = gproj[..., D5:2 * D5].transpose(1, 2)
    g = cl_randn((B5, D5, L5), torch.bfloat16, gen, dev)
    w5 = torch.rand(D5, 4, generator=gen, device=dev) - 0.5
    b5 = torch.randn(D5, generator=gen, device=dev) * 0.1
    fb, bb = conv_bytes(B5, D5, L5, 4)
    us = graph_us([lambda: causal_conv1d_fwd_function(x, w5, b5, None, None, None, True)] * 2, reps=2)
    res["config5_fwd_bf16_w4_silu_slice_of_3D"] = entry(fb, us, peak)
    us = graph_us([lambda: causal_conv1d_bwd_function(x, w5, b5, g, None, None, None, dx, False, True)] * 2, reps=2)
    res["config5_bwd_bf16_w4_silu_slice_of_3D_dx_into_slice"] = entry(bb, us, peak)
    del proj, gproj, x, dx, g
    torch.cuda.empty_cache()

    if not args.no_ref_gpu:
        res["reference_gpu_kernels"] = reference_gpu_table(dev, peak)
    return res


# ------------------------------------------- the reference's own GPU kernels (N=1)
def _load_reference_kernels():
    """The reference's CuTe DSL kernel module from its installed copy, loaded under its own
    name (it imports only torch and the CuTe DSL), or None."""
    import importlib.util

    path = os.path.join(REF_INSTALL, "causal_conv1d", "cutedsl_kernels.py")
    if not os.path.exists(path):
        return None, "reference not installed under baseline/_ref"
    try:
        spec = importlib.util.spec_from_file_location("cc1d_reference_cutedsl_kernels", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as e:  # noqa: BLE001
        return None, f"import failed: {type(e).__name__}: {e}"[:300]


def reference_gpu_table(dev, peak):
    """The reference's CuTe DSL kernels (K1 forward, K6/K7 backward, K2 update, K3 varlen
    states) against ours on the same inputs: both captured in CUDA graphs, replayed in
    alternating order 5 times, medians compared (speedup = ref_us / ours_us)."""
    import torch

    from causal_conv1d import _abi
    from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states
    from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function

    K, why = _load_reference_kernels()
    if K is None:
        return {"unavailable": why}
    gen = torch.Generator(device=dev).manual_seed(21)
    table = {}

    def compare(name, ours, ref, nbytes):
        t_start = time.time()
        try:
            for f in ours + ref:
                f()
            torch.cuda.synchronize()
            go, gr = capture(ours), capture(ref)
            go.replay()
            gr.replay()
            torch.cuda.synchronize()
            to, tr = [], []
            for i in range(5):
                for which in ((0, 1) if i % 2 == 0 else (1, 0)):
                    if which == 0:
                        to.append(replay_ms(go) / len(ours) * 1e3)
                    else:
                        tr.append(replay_ms(gr) / len(ref) * 1e3)
            uo, ur = statistics.median(to), statistics.median(tr)
            table[name] = {"ours_us": round(uo, 3), "ref_us": round(ur, 3), "speedup": round(ur / uo, 3),
                           "ours_frac_of_peak": round(nbytes / (uo * 1e-6) / 1e9 / peak, 4),
                           "ref_frac_of_peak": round(nbytes / (ur * 1e-6) / 1e9 / peak, 4),
                           "wall_s": round(time.time() - t_start, 1)}
        except Exception as e:  # noqa: BLE001
            table[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    def fwd_pair(shape, W, dt, nsets):
        xs = [cl_randn(shape, dt, gen, dev) for _ in range(nsets)]
        w = torch.rand(shape[1], W, generator=gen, device=dev) - 0.5
        b = torch.randn(shape[1], generator=gen, device=dev) * 0.1
        return ([lambda x=x: causal_conv1d_fwd_function(x, w, b, None, None, None, True) for x in xs],
                [lambda x=x: K.causal_conv1d_fwd_cutedsl(x, w, b, "silu") for x in xs], conv_bytes(*shape, W)[0])

    def bwd_pair(shape, W, dt, nsets):
        xs = [(cl_randn(shape, dt, gen, dev), cl_randn(shape, dt, gen, dev)) for _ in range(nsets)]
        w = torch.rand(shape[1], W, generator=gen, device=dev) - 0.5
        b = torch.randn(shape[1], generator=gen, device=dev) * 0.1
        return ([lambda x=x, g=g: causal_conv1d_bwd_function(x, w, b, g, None, None, None, None, False, True)
                 for x, g in xs],
                [lambda x=x, g=g: K.causal_conv1d_bwd_cutedsl(x, w, b, g, True) for x, g in xs], conv_bytes(*shape, W)[1])

    compare("fwd_config2_stateless_bf16_w4", *fwd_pair((4, 4096, 2048), 4, torch.bfloat16, 8))
    compare("fwd_readme_fp16_w3_1x2048x2048", *fwd_pair((1, 2048, 2048), 3, torch.float16, 32))
    compare("fwd_readme_bf16_w4_1x4096x2048", *fwd_pair((1, 4096, 2048), 4, torch.bfloat16, 16))
    compare("bwd_config2_stateless_bf16_w4", *bwd_pair((4, 4096, 2048), 4, torch.bfloat16, 4))
    compare("fwd_config5_bf16_w4_channel_last", *fwd_pair((8, 16384, 8192), 4, torch.bfloat16, 1))
    compare("bwd_config5_bf16_w4_channel_last", *bwd_pair((8, 16384, 8192), 4, torch.bfloat16, 1))

    # update (channel-last state: the only layout the reference kernel takes)
    from causal_conv1d import causal_conv1d_update

    Bu, Du, W = CFG3["batch"], CFG3["dim"], CFG3["width"]
    w = torch.rand(Du, W, generator=gen, device=dev) - 0.5
    b = torch.randn(Du, generator=gen, device=dev) * 0.1
    for name, S, circular in (("update_config3a_channel_last", 3, False), ("update_config3b_channel_last", 16, True)):
        ours, ref = [], []
        for _ in range(16):
            x = torch.randn(Bu, Du, 1, generator=gen, device=dev).to(torch.bfloat16)
            st_o = torch.randn(Bu, S, Du, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
            st_r = st_o.clone().transpose(1, 2).contiguous().transpose(1, 2)
            cache = torch.randint(0, 1000, (Bu,), generator=gen, device=dev, dtype=torch.int32) if circular else None
            idx = torch.randperm(Bu, generator=gen, device=dev).to(torch.int32) if circular else None
            ours.append(lambda x=x, st=st_o, c=cache, i=idx: causal_conv1d_update(x, st, w, b, "silu", c, i))
            ref.append(lambda x=x, st=st_r, c=cache, i=idx: K.causal_conv1d_update_cutedsl(x, st, w, b, "silu", c, i))
        compare(name, ours, ref, update_bytes(Bu, Du, W, S, circular))

    T, Dv, S, nseq = CFG4["tokens"], CFG4["dim"], CFG4["state_len"], CFG4["nseq"]
    xv = torch.randn(T, Dv, generator=gen, device=dev).to(torch.float16)
    ours, ref = [], []
    cpu_gen = torch.Generator().manual_seed(0)
    for _ in range(32):
        lens = 1 + torch.bincount(torch.multinomial(torch.full((nseq,), 1 / nseq), T - nseq, replacement=True,
                                                    generator=cpu_gen), minlength=nseq)
        cu = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).to(dev)
        ours.append(lambda cu=cu: causal_conv1d_varlen_states(xv, cu, S))
        ref.append(lambda cu=cu: K.causal_conv1d_varlen_states_cutedsl(xv, cu, S))
    compare("varlen_states_config4", ours, ref, 2 * nseq * S * Dv * 2 + (nseq + 1) * 4)
    _abi.load_library()
    return table


# ------------------------------------------------------------- single kernel cases
def run_case(args):
    """Build one benchmark case and launch it ``--repeat`` times (no graph), for ncu."""
    import torch

    from causal_conv1d import causal_conv1d_update
    from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states
    from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(9)
    name = args.case
    if name.startswith("config5_") or name.startswith("config2_"):
        cfg = CFG5 if name.startswith("config5_") else CFG2
        B = args.case_batch or cfg["batch"]
        D, L, W = cfg["dim"], cfg["seqlen"], cfg["width"]
        contiguous = name.endswith("_contiguous")
        x = (torch.randn(B, D, L, generator=gen, device=dev, dtype=torch.bfloat16) if contiguous
             else cl_randn((B, D, L), torch.bfloat16, gen, dev))
        w = torch.rand(D, W, generator=gen, device=dev) - 0.5
        b = torch.randn(D, generator=gen, device=dev) * 0.1
        states = name.startswith("config2_")
        init = torch.randn(B, D, W - 1, generator=gen, device=dev).to(torch.bfloat16) if states else None
        final = torch.empty(B, W - 1, D, device=dev, dtype=torch.bfloat16).transpose(1, 2) if states else None
        dfinal = torch.zeros(B, D, W - 1, device=dev, dtype=torch.bfloat16) if states else None
        if "_fwd" in name:
            fn = lambda: causal_conv1d_fwd_function(x, w, b, None, init, final, True)  # noqa: E731
        else:
            g = torch.randn_like(x)
            fn = lambda: causal_conv1d_bwd_function(x, w, b, g, None, init, dfinal, None, states, True)  # noqa: E731
    elif name.startswith("config3"):
        Bu, Du, W = CFG3["batch"], CFG3["dim"], CFG3["width"]
        circular = name.startswith("config3b")
        S = 16 if circular else 3
        w = torch.rand(Du, W, generator=gen, device=dev) - 0.5
        b = torch.randn(Du, generator=gen, device=dev) * 0.1
        x = torch.randn(Bu, Du, 1, generator=gen, device=dev).to(torch.bfloat16)
        if name.endswith("channel_last"):
            st = torch.randn(Bu, S, Du, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
        else:
            st = torch.randn(Bu, Du, S, generator=gen, device=dev).to(torch.bfloat16)
        cache = torch.randint(0, 1000, (Bu,), generator=gen, device=dev, dtype=torch.int32) if circular else None
        idx = torch.randperm(Bu, generator=gen, device=dev).to(torch.int32) if circular else None
        fn = lambda: causal_conv1d_update(x, st, w, b, "silu", cache, idx)  # noqa: E731
    elif name.startswith("readme_") or name.startswith("ref_readme_"):
        # the reference README's forward shapes; ref_* runs the reference's own CuTe DSL kernel
        shape, W_, dt = ((1, 2048, 2048), 3, torch.float16) if "fp16" in name else ((1, 4096, 2048), 4, torch.bfloat16)
        x = cl_randn(shape, dt, gen, dev)
        w = torch.rand(shape[1], W_, generator=gen, device=dev) - 0.5
        b = torch.randn(shape[1], generator=gen, device=dev) * 0.1
        if name.startswith("ref_"):
            K, why = _load_reference_kernels()
            if K is None:
                raise SystemExit(why)
            fn = lambda: K.causal_conv1d_fwd_cutedsl(x, w, b, "silu")  # noqa: E731
        else:
            fn = lambda: causal_conv1d_fwd_function(x, w, b, None, None, None, True)  # noqa: E731
    elif name.startswith("calibration_copy_"):  # e.g. calibration_copy_17MB: read + write that many bytes
        n = int(name[len("calibration_copy_"):-2]) * (1 << 20) // 2
        src = torch.empty(n, dtype=torch.uint8, device=dev)
        dst = torch.empty(n, dtype=torch.uint8, device=dev)
        fn = lambda: dst.copy_(src)  # noqa: E731
    elif name == "config4_varlen_states":
        T, Dv, S, nseq = CFG4["tokens"], CFG4["dim"], CFG4["state_len"], CFG4["nseq"]
        xv = torch.randn(T, Dv, generator=gen, device=dev).to(torch.float16)
        lens = 1 + torch.bincount(torch.multinomial(torch.full((nseq,), 1 / nseq), T - nseq, replacement=True,
                                                    generator=torch.Generator().manual_seed(0)), minlength=nseq)
        cu = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).to(dev)
        fn = lambda: causal_conv1d_varlen_states(xv, cu, S)  # noqa: E731
    else:
        raise SystemExit(f"unknown case {name}")
    for _ in range(args.repeat):
        fn()
    torch.cuda.synchronize()
    print(f"case {name}: {args.repeat} launches done", flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-extras", action="store_true", help="skip the per-N side figures and the kernel table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) figure")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip timing the reference's own GPU kernels")
    ap.add_argument("--no-kernel-table", action="store_true", help="skip the N=1 per-config kernel table")
    ap.add_argument("--case", default=None, help="run one kernel case (see run_case) and exit")
    ap.add_argument("--case-batch", type=int, default=0, help="batch of a config-2/5 case (0: the config's)")
    ap.add_argument("--repeat", type=int, default=3)
    ap.add_argument("--cpu-child", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--cpu-run-s", type=float, default=3.0, help=argparse.SUPPRESS)
    ap.add_argument("--cpu-runs", type=int, default=5, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.cpu_child:
        return cpu_child(args)
    if args.impl == "reference":
        return run_reference(args)
    _package_path()
    if args.case:
        return run_case(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
