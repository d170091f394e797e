"""Benchmark: sqrt-block attention forward+backward at B=1, H=16, T=16384, D=128, bf16,
and GPT-2 small training tokens/s with that attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload attn-t16k|attn-t4k|attn-t8k|attn-t32k|attn-t64k|attn-cfg2|
                                attn-cfg5|gpt2-small|gpt2-medium-8k|refsem-cfg2]

Default workload (attn-t16k), one JSON line:
  * top level: one step = one forward (sqb_fwd) and one backward (sqb_bwd) of
    the attention over B=1, H=16 heads per rank, T=16384, D=128 (b=128).
    ``value`` is whole-job algorithmic HBM throughput in GB/s (compulsory
    bytes 12*B*H*T*D*2 + 8*B*H*T per step, summed over ranks, divided by the
    max-over-ranks device time).  Inputs (Q, K, V, dO: 4 x 67 MB, plus O and
    the gradients) exceed the 126 MB L2, so no flush is needed between steps.
    ``e2e`` is the same metric through the public autograd op with every
    step's inputs copied in from pinned host memory and its outputs back.
  * ``h64_split``: the fixed 64-head job at T=16384 split 64/N heads per rank
    (strong scaling), max-over-ranks device time.
  * ``train``: GPT-2 small (12L/12H/768, bias-free, vocab 50257), 16 x 1024
    tokens per rank, fwd + bwd + clip + fused AdamW under bf16 autocast,
    data-parallel over NCCL (DDP's bucketed fp32 gradient all-reduce) when
    N > 1; with the same steps run without the all-reduce, and a flat
    all-reduce of the gradients' size timed alone, to show how much of the
    collective the backward hides.
  * ``train_gpt2_medium_8k``: the same for GPT-2 medium (24L/16H/1024) at
    T=8192 (b=96), 8 sequences per rank.
Multi-GPU: one process per GPU under torchrun; every rank runs its own 16
heads for the top-level metric (weak scaling; the (batch, head) units are
independent, so there is no data-path collective).

``--impl reference`` times the CPU restatement of the operator (the reference
repository has no implementation of it) on the host cores, on a bounded sample
of the same workload (a subset of heads), and prints the same metric.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "sqrt-block attn fwd+bwd ms & HBM GB/s at T=16K; GPT-2 small train tokens/sec"
ELT = 2  # bf16
# attention workloads: (B, H per rank, T, D, block or None = default b)
ATTN = {
    "attn-t4k": (1, 16, 4096, 128, None),
    "attn-t8k": (1, 16, 8192, 128, None),
    "attn-t16k": (1, 16, 16384, 128, None),   # the headline point and the default
    "attn-t32k": (1, 16, 32768, 128, None),
    "attn-t64k": (1, 16, 65536, 128, None),
    "attn-cfg2": (8, 12, 1024, 64, 32),       # the GPT-2 small attention shape
    "attn-cfg5": (8, 16, 8192, 64, 96),       # the GPT-2 medium T=8K attention shape
}
L2_BYTES = 126 * 2**20


def algorithmic_bytes(B_, H_, T_, D_, elt=ELT, fwd=True, bwd=True):
    n = B_ * H_ * T_
    return (4 * n * D_ * elt + 4 * n if fwd else 0) + (8 * n * D_ * elt + 4 * n if bwd else 0)


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def host_info():
    """Host CPU model (from /proc/cpuinfo, as lscpu reports it) and torch version."""
    model = platform.processor() or "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "logical_cpus": os.cpu_count(), "torch": torch.__version__}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64,
                     device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def make_inputs(seed, rank, B_, H_, T_, D_, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    return [torch.randn(B_, T_, H_, D_, generator=g).to(dtype) for _ in range(4)]


# ---- CPU baseline / reference arm ------------------------------------------------------


def cpu_samples(shape, heads=1, reps=1, seconds=0.0):
    """Time the oracle port (fp32 torch, all host threads) on `heads` heads of
    the workload's shape, forward+backward, `reps` times and then until the
    timed work adds up to `seconds`; returns (list of seconds per sample, threads)."""
    from oracle.torch_port import sqrt_block_attention_ref

    B_, _, T_, D_, blk = shape
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v, do = [torch.randn(1, heads, T_, D_, generator=g) for _ in range(4)]
    times = []
    while len(times) < reps or (sum(times) < seconds and len(times) < 5000):
        qs, ks, vs = [x.clone().requires_grad_(True) for x in (q, k, v)]
        t0 = time.perf_counter()
        o, _ = sqrt_block_attention_ref(qs, ks, vs, blk)
        (o * do).sum().backward()
        times.append(time.perf_counter() - t0)
    return times, threads


def attn_config(args, shape, world, block):
    B_, H_, T_, D_, _ = shape
    return {"workload": f"sqrt-block attention fwd+bwd ({args.workload}: B={B_} H={H_} "
                        f"T={T_} D={D_} b={block}, bf16)",
            "B": B_, "H_per_rank": H_, "T": T_, "D": D_, "block": block,
            "parallelism": f"heads x {world} ranks"}


def run_reference(args, world, rank):
    """CPU restatement of the operator, timed on the host cores (rank 0 alone)."""
    if rank != 0:
        return
    from oracle.sqrtblock_oracle import geometry

    shape = ATTN[args.workload]
    B_, H_, T_, D_, blk = shape
    block = geometry(T_, blk)[0]
    # one (batch, head) unit per sample: the whole-job time is the sample's
    # time scaled to every unit the job has at this N (the host's cores are
    # one resource shared by all ranks' work)
    units = B_ * H_ * world
    sample_bytes = algorithmic_bytes(1, 1, T_, D_)
    cpu_samples(shape, 1, 1)  # warm-up allocations and thread pool
    for _ in range(max(args.warmup, 0)):
        cpu_samples(shape, 1, 1)
    times, threads = [], 1
    for _ in range(args.steps):
        t, threads = cpu_samples(shape, 1, 1)
        times.append(t[0])
    per = statistics.median(times)
    gbs = sample_bytes / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * units * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1), seeded", "config": attn_config(args, shape, world, block),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"1 of the job's {units} (batch, head) units per step "
                                   "(fp32 torch fwd+bwd on all host threads); ms_per_step "
                                   "scales it to the whole job at this N. The host's cores are "
                                   "one resource for every N, so value does not grow with N",
                         **host_info()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- attention on the GPU ------------------------------------------------------------


def time_attention(dev, shape, host, steps, warmup, warmup_seconds, kernels, world,
                   clocks=None):
    """Device time of `steps` fwd+bwd steps of the attention over `host` inputs
    (moved to `dev`).  Returns a dict of times (max over ranks), the kernel
    family and the L2 policy."""
    from llm_training_b200 import _lib
    from llm_training_b200.ops import sqrt_block_backward, sqrt_block_forward

    B_, H_, T_, D_, blk = shape
    q, k, v, do = [x.to(dev) for x in host]
    block = _lib.geometry(T_, blk)[0]
    fwd_impl = bwd_impl = kernels
    if kernels == "auto":
        # the tcgen05 family where it has a kernel for this shape, else SIMT
        n0 = min(T_, 256)
        qs, ks, vs, dos = q[:, :n0], k[:, :n0], v[:, :n0], do[:, :n0]
        try:
            o_, l_, kb_, vb_ = sqrt_block_forward(qs, ks, vs, block, None, "tcgen05")
            fwd_impl = "tcgen05"
        except _lib.SqrtBlockError:
            o_, l_, kb_, vb_ = sqrt_block_forward(qs, ks, vs, block, None, "simt")
            fwd_impl = "simt"
        try:
            sqrt_block_backward(qs, ks, vs, o_, l_, kb_, vb_, dos, block, None, "tcgen05")
            bwd_impl = "tcgen05"
        except _lib.SqrtBlockError:
            bwd_impl = "simt"
    # kernels each call launches: tcgen05 fwd 1, bwd 1; SIMT fwd 2 (pool,
    # attention), bwd 4 (delta, summary gradients, dQ, dK/dV)
    launches = {"tcgen05": 1, "simt": 2}[fwd_impl] + {"tcgen05": 1, "simt": 4}[bwd_impl]
    stream = torch.cuda.current_stream(dev)
    # Q, K, V, dO and O resident: above 2x the 126 MB L2 nothing survives from
    # one step to the next; below it L2 is flushed between timed steps (a
    # 512 MB write) and a step is timed from the forward's start to the
    # backward's end, so the flush is not counted.
    resident = 5 * B_ * H_ * T_ * D_ * ELT
    flush = resident < 2 * L2_BYTES
    flush_buf = torch.empty(512 * 2**20, dtype=torch.uint8, device=dev) if flush else None
    f_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]
    b_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]

    def step(i=None):
        if i is not None:
            f_ev[2 * i].record(stream)
        o, lse, kbar, vbar = sqrt_block_forward(q, k, v, block, None, fwd_impl)
        if i is not None:
            f_ev[2 * i + 1].record(stream)
            b_ev[2 * i].record(stream)
        sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do, block, None, bwd_impl)
        if i is not None:
            b_ev[2 * i + 1].record(stream)

    with (clocks if clocks is not None else contextlib.nullcontext()):
        # warm up for at least W steps and `warmup_seconds`, so a clock sampler
        # (100 ms period) has samples under load when the timed region starts
        t_end = time.perf_counter() + warmup_seconds
        i = 0
        while i < max(warmup, 3) or time.perf_counter() < t_end:
            step()
            i += 1
            if i % 16 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(steps):
            if flush:
                flush_buf.zero_()
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = max_over_ranks(start.elapsed_time(end), world)
    fwd_ms = statistics.mean(f_ev[2 * i].elapsed_time(f_ev[2 * i + 1]) for i in range(steps))
    bwd_ms = statistics.mean(b_ev[2 * i].elapsed_time(b_ev[2 * i + 1]) for i in range(steps))
    if flush:
        step_ms = statistics.mean(f_ev[2 * i].elapsed_time(b_ev[2 * i + 1]) for i in range(steps))
        ms_per_step = max_over_ranks(step_ms, world)
    else:
        ms_per_step = total_ms / steps
    return {"fwd_ms": max_over_ranks(fwd_ms, world), "bwd_ms": max_over_ranks(bwd_ms, world),
            "ms_per_step": ms_per_step, "block": block, "flush": flush, "resident": resident,
            "impl": f"fwd:{fwd_impl},bwd:{bwd_impl}", "launches_per_step": launches}


def e2e_attention(dev, shape, host, block, kernels, world, e_steps=30):
    """End to end through the public autograd op: every step copies its inputs
    (Q, K, V, dO) in from pinned host memory and its results (O, dQ, dK, dV)
    back out to pinned host memory.  Steps are pipelined on three streams, as a
    host application streaming batches would run them: the H2D copy of step
    i+1 and the D2H copy of step i-1 overlap step i.  Every step's copies lie
    inside the timed region (first H2D start to last D2H end)."""
    from llm_training_b200.ops import sqrt_block_attention

    B_, H_, T_, D_, _ = shape
    stream = torch.cuda.current_stream(dev)
    pinned = [x.pin_memory() for x in host]
    outs = [[torch.empty(B_, T_, H_, D_, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
            for _ in range(2)]
    dev_in = [[torch.empty_like(x, device=dev) for x in host] for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def run(nsteps, timed):
        ev = lambda: torch.cuda.Event(enable_timing=timed)  # noqa: E731
        in_ready = [ev() for _ in range(nsteps)]
        done = [ev() for _ in range(nsteps)]
        e0, e1 = ev(), ev()
        e0.record(s_in)
        for i in range(nsteps):
            buf = dev_in[i % 2]
            if i >= 2:
                s_in.wait_event(done[i - 2])  # step i-2 has finished with this buffer set
            with torch.cuda.stream(s_in):
                for d_, h_ in zip(buf, pinned):
                    d_.copy_(h_, non_blocking=True)
            in_ready[i].record(s_in)
            stream.wait_event(in_ready[i])
            qd, kd, vd = (x.detach().requires_grad_(True) for x in buf[:3])
            o = sqrt_block_attention(qd, kd, vd, block, None, kernels)
            o.backward(buf[3])
            res = (o.detach(), qd.grad, kd.grad, vd.grad)
            done[i].record(stream)
            s_out.wait_event(done[i])
            with torch.cuda.stream(s_out):
                for dst, src in zip(outs[i % 2], res):
                    src.record_stream(s_out)
                    dst.copy_(src, non_blocking=True)
        e1.record(s_out)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) if timed else 0.0

    run(2, False)
    barrier(world)
    # 30 streamed steps: the pipeline's fill and drain (the first step's H2D
    # and the last step's D2H, which overlap nothing) are ~3 % of the timed
    # region at T=16K, as in a long-running stream of batches
    e2e_ms = max_over_ranks(run(e_steps, True), world) / e_steps
    h2d = sum(x.numel() * x.element_size() for x in pinned)
    d2h = sum(x.numel() * x.element_size() for x in outs[0])
    return e2e_ms, h2d, d2h, e_steps


def run_h64_split(args, dev, world, rank):
    """Config-3's fixed-work job: B=1, H=64, T=16384, D=128 split 64/N heads per rank."""
    if 64 % world:
        return {"skipped": f"64 heads do not split over {world} ranks"}
    shape = (1, 64 // world, 16384, 128, None)
    host = make_inputs(args.seed + 1, rank, 1, 64 // world, 16384, 128)
    t = time_attention(dev, shape, host, args.h64_steps, 3, 0.0, args.kernels, world)
    job_bytes = algorithmic_bytes(1, 64, 16384, 128)
    return {"H_total": 64, "H_per_rank": 64 // world, "T": 16384, "D": 128, "block": t["block"],
            "scaling": "strong", "steps": args.h64_steps,
            "ms_per_step": round(t["ms_per_step"], 4), "fwd_ms": round(t["fwd_ms"], 4),
            "bwd_ms": round(t["bwd_ms"], 4),
            "GBps": round(job_bytes / (t["ms_per_step"] * 1e-3) / 1e9, 1),
            "timing": "max over ranks, CUDA events",
            "l2": "flushed between steps" if t["flush"] else "inputs > 2 x L2, no flush"}


def run_ours(args, world, rank, local):
    from llm_training_b200.ops import read_status

    dev = torch.device("cuda", local)
    shape = ATTN[args.workload]
    B_, H_, T_, D_, _ = shape
    host = make_inputs(args.seed, rank, B_, H_, T_, D_)
    clocks = ClockSampler(torch.cuda.current_device())
    t = time_attention(dev, shape, host, args.steps, args.warmup, args.warmup_seconds,
                       args.kernels, world, clocks)
    status = read_status(dev)
    block, ms_per_step, fwd_ms, bwd_ms = t["block"], t["ms_per_step"], t["fwd_ms"], t["bwd_ms"]
    step_bytes = algorithmic_bytes(B_, H_, T_, D_)
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9
    e2e_ms, h2d, d2h, e_steps = e2e_attention(dev, shape, host, block, args.kernels, world)

    peak, peak_kind = load_peaks()
    bwd_bytes = algorithmic_bytes(B_, H_, T_, D_, fwd=False)
    fwd_bytes = algorithmic_bytes(B_, H_, T_, D_, bwd=False)
    dom = ("backward", bwd_bytes, bwd_ms) if bwd_ms >= fwd_ms else ("forward", fwd_bytes, fwd_ms)
    achieved = dom[1] / (dom[2] * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": None, "kernel": dom[0],
                "peak_source": peak_kind,
                "fwd": {"ms": round(fwd_ms, 4),
                        "GBps": round(fwd_bytes / (fwd_ms * 1e-3) / 1e9, 1)},
                "bwd": {"ms": round(bwd_ms, 4),
                        "GBps": round(bwd_bytes / (bwd_ms * 1e-3) / 1e9, 1)},
                "step_frac": round(value / world / peak, 4)}
    traffic_path = os.path.join(REPO, "profiles", "dram_traffic.json")
    if args.workload == "attn-t16k" and os.path.exists(traffic_path):  # captured at T=16384
        try:
            roofline["traffic"] = json.load(open(traffic_path)).get(dom[0])
        except Exception:
            pass

    extra = {}
    if args.workload == "attn-t16k" and not args.no_h64:
        extra["h64_split"] = run_h64_split(args, dev, world, rank)
    if args.workload == "attn-t16k" and not args.no_train:
        torch.cuda.empty_cache()
        extra["train"] = train_record(args, "gpt2-small", world, rank, local,
                                      args.train_steps, args.train_warmup)
        if not args.no_train_medium:
            torch.cuda.empty_cache()
            extra["train_gpt2_medium_8k"] = train_record(
                args, "gpt2-medium-8k", world, rank, local, max(args.train_steps // 3, 5), 3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        # one head of the workload per sample, repeated until the timed CPU work
        # adds up to 10 s (median sample; a first, untimed call warms the pool)
        cpu_samples(shape, 1, 1)
        samples, threads = cpu_samples(shape, 1, 1, seconds=10.0)
        dt = statistics.median(samples)
        cpu = {"value": round(algorithmic_bytes(1, 1, T_, D_) / dt / 1e9, 3), "unit": "GB/s",
               "cores": threads, "kind": "port",
               "sample": f"1 of {B_ * H_} (batch, head) units, fp32 torch fwd+bwd, median of "
                         f"{len(samples)} samples ({sum(samples):.1f} s; {dt * 1e3:.0f} ms each)",
               **host_info()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded per rank",
            "config": {**attn_config(args, shape, world, block), "kernels": t["impl"],
                       "l2": (f"L2 flushed between steps (512 MB write, not timed); resident "
                              f"Q/K/V/dO/O {t['resident'] / 2**20:.0f} MB" if t["flush"] else
                              f"resident Q/K/V/dO/O {t['resident'] / 2**20:.0f} MB > 2 x 126 MB "
                              "L2; no flush")},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(step_bytes * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e_steps,
                    "pipelined": "H2D of step i+1 and D2H of step i-1 overlap step i "
                                 "(three streams); all copies inside the timed region"},
            "gpu_launches": t["launches_per_step"] * args.steps,
            "clocks": clocks.summary(),
            "device_status": status,
            **extra,
        }
        print(json.dumps(line), flush=True)


# ---- reference-semantics mode ------------------------------------------------------
# (B, H, T, D) of the cfg-2 shape (T a perfect square)
REFSEM = {"refsem-cfg2": (8, 12, 1024, 64)}


def run_refsem(args, world, rank, local):
    """Reference-semantics mode (the reference's own attention core), fwd+bwd."""
    from llm_training_b200.ops import read_status, reference_backward, reference_forward

    Bq, Hq, Tq, Dq = REFSEM[args.workload]
    dev = torch.device("cuda", local)
    g = torch.Generator().manual_seed(args.seed * 1000 + rank)
    host = [torch.randn(Bq, Tq, Hq, Dq, generator=g).to(torch.bfloat16) for _ in range(4)]
    q, k, v, do = [x.to(dev) for x in host]

    def step():
        o, glob, summary = reference_forward(q, k, v)
        reference_backward(q, k, v, glob, summary, do)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    # fwd reads Q, K, V and writes O; bwd reads Q, K, V, dO and writes dQ, dK, dV
    step_bytes = 11 * Bq * Tq * Hq * Dq * 2
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        per, threads = refsem_cpu_sample(Tq, Dq, 3)
        cpu = {"value": round(11 * Tq * Dq * 2 / per / 1e9, 4), "unit": "GB/s",
               "cores": threads, "kind": "port",
               "sample": f"1 of {Bq * Hq} (batch, head) units, fp32 torch restatement of the "
                         f"reference core fwd+bwd, median {per * 1e3:.1f} ms", **host_info()}
    if rank == 0:
        print(json.dumps({
            "metric": "reference-semantics sqrt_block attn fwd+bwd GB/s (B=8 H=12 T=1024 D=64)",
            "value": round(step_bytes * world / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded per rank",
            "config": {"workload": args.workload, "B": Bq, "H": Hq, "T": Tq, "D": Dq,
                       "mode": "reference semantics",
                       "parallelism": f"replicas x {world} ranks"},
            "cpu_baseline": cpu, "gpu_launches": 7 * args.steps, "clocks": clocks.summary(),
            "device_status": read_status(dev),
        }), flush=True)


def refsem_cpu_sample(Tq, Dq, reps, units=1):
    """Median seconds of `reps` fwd+bwd samples of the reference core's torch
    restatement on `units` (batch, head) units, fp32, all host threads."""
    from oracle.refsem_torch_port import reference_core

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v, do = [torch.randn(1, units, Tq, Dq, generator=g) for _ in range(4)]
    times = []
    for _ in range(reps + 1):
        qs, ks, vs = [x.clone().requires_grad_(True) for x in (q, k, v)]
        t0 = time.perf_counter()
        (reference_core(qs, ks, vs) * do).sum().backward()
        times.append(time.perf_counter() - t0)
    return statistics.median(times[1:]), threads


def run_refsem_reference(args, world, rank):
    """Reference arm of the refsem workload: the reference's core restated in
    torch (the reference module is torch ops itself) on the host cores."""
    if rank != 0:
        return
    Bq, Hq, Tq, Dq = REFSEM[args.workload]
    units = Bq * Hq
    for _ in range(max(args.warmup, 0)):
        refsem_cpu_sample(Tq, Dq, 1, units)
    per, threads = refsem_cpu_sample(Tq, Dq, max(args.steps, 1), units)
    gbs = 11 * units * Tq * Dq * 2 / per / 1e9
    print(json.dumps({
        "impl": "reference",
        "metric": "reference-semantics sqrt_block attn fwd+bwd GB/s (B=8 H=12 T=1024 D=64)",
        "value": round(gbs, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per * world * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": args.workload, "B": Bq, "H": Hq, "T": Tq, "D": Dq,
                   "mode": "reference semantics", "parallelism": f"replicas x {world} ranks"},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": "the whole B=8 H=12 problem per step: the reference's core "
                                   "(model/custom_attention.py:183-227) restated with the same "
                                   "torch ops, fp32 fwd+bwd on all host threads", **host_info()},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ---- GPT training --------------------------------------------------------------------
TRAIN_WORKLOADS = {
    # name: (config factory, sequences per GPU, sequence length)
    "gpt2-small": ("small", 16, 1024),
    "gpt2-medium-8k": ("medium", 8, 8192),
}


def train_record(args, workload, world, rank, local, steps, warmup):
    """GPT training step (fwd + bwd + clip + fused AdamW, bf16 autocast) with the
    sqrt-block attention; data-parallel over NCCL (DDP) when world > 1.
    Returns the record (on every rank)."""
    from llm_training_b200.config import gpt2_medium, gpt2_small
    from llm_training_b200.train import Trainer, synthetic_batch

    kind, batch, seq = TRAIN_WORKLOADS[workload]
    batch = args.train_batch or batch
    cfg = gpt2_small(block_size=seq) if kind == "small" else gpt2_medium(block_size=seq,
                                                                        sqrt_block_b=96)
    dev = torch.device("cuda", local)
    tr = Trainer(cfg, dev, lr=6e-4, weight_decay=0.1, seed=1337, ddp=world > 1)
    gen = torch.Generator().manual_seed(args.seed * 1000 + rank)
    x, y = synthetic_batch(gen, batch, seq, cfg.vocab_size, dev)
    stream = torch.cuda.current_stream(dev)

    def timed(n, no_sync=False):
        ctx = tr.model.no_sync() if (no_sync and world > 1) else contextlib.nullcontext()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ctx:
            e0.record(stream)
            for _ in range(n):
                loss, _ = tr.step(x, y)
            e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1), world) / n, loss

    for _ in range(max(warmup, 3)):
        tr.step(x, y)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        ms, loss = timed(steps)
    tokens = batch * seq * world
    rec = {"metric": f"{workload} train tokens/sec (sqrt-block attention)",
           "value": round(tokens / (ms * 1e-3), 1), "unit": "tokens/s",
           "tokens_per_s": round(tokens / (ms * 1e-3), 1), "n_gpus": world, "steps": steps,
           "warmup": max(warmup, 3), "ms_per_step": round(ms, 3), "scaling": "weak",
           "config": {"workload": workload, "model": kind,
                      "params": sum(p.numel() for p in tr.raw_model.parameters()),
                      "batch_per_gpu": batch, "global_batch": batch * world, "seq_len": seq,
                      "block": cfg.sqrt_block_b or "default", "parallelism": f"dp{world}",
                      "optimizer": "fused AdamW lr 6e-4 wd 0.1, clip 1.0", "dtype": "bf16 autocast",
                      "data": "synthetic uniform token ids, seeded per rank"},
           "clocks": clocks.summary()}
    if world > 1:
        # what the collective costs: the same steps without the gradient
        # all-reduce (DDP no_sync), and one all-reduce of the gradients' total
        # size as a single flat fp32 buffer, timed alone
        import torch.distributed as dist

        ms_ns, _ = timed(max(steps // 2, 5), no_sync=True)
        nparam = sum(p.numel() for p in tr.raw_model.parameters() if p.requires_grad)
        flat = torch.zeros(nparam, dtype=torch.float32, device=dev)
        for _ in range(3):
            dist.all_reduce(flat)
        torch.cuda.synchronize()
        barrier(world)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(10):
            dist.all_reduce(flat)
        a1.record(stream)
        torch.cuda.synchronize()
        ar_ms = max_over_ranks(a0.elapsed_time(a1), world) / 10
        del flat
        exposed = max(ms - ms_ns, 0.0)
        rec["allreduce"] = {
            "collective": "DDP bucketed all-reduce of the fp32 gradients (NCCL, NVLink)",
            "bucket_cap_mb": round(getattr(tr.model, "bucket_bytes_cap", 0) / 2**20, 1),
            "grad_bytes": nparam * 4,
            "step_ms_without_allreduce": round(ms_ns, 3),
            "flat_allreduce_ms": round(ar_ms, 3),
            "flat_busbw_GBps": round(2 * (world - 1) / world * nparam * 4 / (ar_ms * 1e-3) / 1e9,
                                     1),
            "exposed_ms": round(exposed, 3),
            "hidden_frac": round(1.0 - min(exposed / ar_ms, 1.0), 3) if ar_ms > 0 else None}
    # end to end: a fresh host batch copied in and the loss read back every step
    host = [torch.randint(0, cfg.vocab_size, (batch, seq + 1), generator=gen).pin_memory()
            for _ in range(2)]
    torch.cuda.synchronize()
    barrier(world)
    e_steps = max(steps, 10)
    e0 = time.perf_counter()
    for i in range(e_steps):
        tok = host[i % 2].to(dev, non_blocking=True)
        loss, _ = tr.step(tok[:, :-1], tok[:, 1:])
        lv = loss.item()
    torch.cuda.synchronize()
    e_ms = max_over_ranks((time.perf_counter() - e0) * 1e3, world) / e_steps
    rec["e2e"] = {"value": round(tokens / (e_ms * 1e-3), 1), "unit": "tokens/s",
                  "ms_per_step": round(e_ms, 3), "h2d_bytes_per_step": batch * (seq + 1) * 8,
                  "d2h_bytes_per_step": 4, "steps": e_steps,
                  "timing": "host clock, loss.item() every step, max over ranks"}
    rec["last_loss"] = round(float(lv), 4)
    if getattr(args, "metrics_out", None):
        rec["metrics_json"] = write_report(args, tr, cfg, host, batch, seq, world, rank, dev)
    del tr
    torch.cuda.empty_cache()
    return rec


def write_report(args, tr, cfg, host, batch, seq, world, rank, dev):
    """A run in the reference trainer's metrics.json schema (written by rank 0):
    the host batch copied in ("data"), forward, backward and optimizer phases,
    attention layers hooked, the first 5 steps excluded from the means."""
    from llm_training_b200.metrics import MetricsReport
    from llm_training_b200.model.attention_registry import BaseAttention

    steps = max(args.report_steps, 6)
    info = tr.run_info(cfg, batch, seq, max_steps=steps, lr=6e-4, seed=1337)
    info["data_parallel_ranks"] = world
    rep = MetricsReport(args.metrics_out if rank == 0 else None, info,
                        tokens_per_step=batch * seq * world, warmup_steps_skipped=5,
                        log_interval=1, device_type="cuda")
    rep.attach_attention(tr.raw_model, BaseAttention)
    for step in range(steps):
        rep.begin_step(step)
        with rep.phase("data"):
            tok = host[step % 2].to(dev, non_blocking=True)
        loss, norm = tr.step(tok[:, :-1], tok[:, 1:], report=rep)
        rep.end_step(step, float(loss), 6e-4, float(norm))
    doc = rep.write("finished")
    return {"path": args.metrics_out, "measured_steps": doc["aggregates"]["measured_steps"],
            "avg_tokens_per_sec": doc["aggregates"]["avg_tokens_per_sec"],
            "attention_fraction_of_step_time":
                doc["aggregates"].get("attention", {}).get("fraction_of_step_time"),
            "note": "per-step synchronize and hooks: slower than the timed tokens_per_s"}


def run_train(args, world, rank, local):
    rec = train_record(args, args.workload, world, rank, local, args.steps, args.warmup)
    if rank == 0:
        line = {"metric": rec.pop("metric"), "value": rec.pop("value"), "unit": rec.pop("unit"),
                "higher_is_better": True, "vs_baseline": None, "dtype": "bf16",
                "data": rec["config"]["data"], **rec}
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernels", choices=["auto", "tcgen05", "simt"], default="auto")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--no-train", action="store_true", help="skip the train sub-record")
    ap.add_argument("--no-h64", action="store_true", help="skip the h64_split sub-record")
    ap.add_argument("--no-train-medium", action="store_true",
                    help="skip the GPT-2 medium T=8K training sub-record")
    ap.add_argument("--train-steps", type=int, default=30)
    ap.add_argument("--train-warmup", type=int, default=5)
    ap.add_argument("--h64-steps", type=int, default=30)
    ap.add_argument("--metrics-out", default=None,
                    help="gpt2-* workloads: also write a metrics.json report (the reference "
                         "trainer's schema) of --report-steps profiled steps to this path")
    ap.add_argument("--report-steps", type=int, default=20)
    ap.add_argument("--train-batch", type=int, default=0,
                    help="sequences per GPU of the training workloads (0 = the config's)")
    ap.add_argument("--warmup-seconds", type=float, default=0.5,
                    help="keep warming up at least this long (clock sampler needs samples)")
    ap.add_argument("--workload", choices=sorted(ATTN) + sorted(TRAIN_WORKLOADS) + sorted(REFSEM),
                    default="attn-t16k",
                    help="attn-*: the attention op (attn-t16k is the default and carries the "
                         "h64_split and train sub-records); gpt2-*: a training step; "
                         "refsem-cfg2: the reference-semantics mode")
    args = ap.parse_args()
    world, rank, local = init_dist()
    try:
        if args.workload in REFSEM:
            if args.impl == "reference":
                run_refsem_reference(args, world, rank)
            else:
                run_refsem(args, world, rank, local)
        elif args.workload in TRAIN_WORKLOADS:
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable":
                                      "the reference has no implementation of this "
                                      "attention operator to train with"}), flush=True)
            else:
                run_train(args, world, rank, local)
        elif args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
