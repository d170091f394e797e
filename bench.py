"""Benchmark: sqrt-block attention forward+backward at B=1, H=16, T=16384, D=128, bf16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload attn-t4k|attn-t8k|attn-t16k|attn-t32k|attn-t64k|gpt2-small|
                                gpt2-medium-8k|refsem-cfg2]

One step = one forward (sqb_fwd) and one backward (sqb_bwd) of the attention
operator over the whole workload.  ``value`` is whole-job algorithmic HBM
throughput in GB/s (compulsory bytes 12*B*H*T*D*2 + 8*B*H*T per step, summed
over ranks, divided by the max-over-ranks device time).  Inputs (Q, K, V, dO:
4 x 67 MB, plus O and the gradients) exceed the 126 MB L2, so no flush is
needed between steps.  Multi-GPU: one process per GPU under torchrun, every
rank runs its own 16 heads (weak scaling; the (batch, head) units are
independent, so there is no data-path collective).

``--workload refsem-cfg2`` times the reference-semantics mode (the reference's
own sqrt_block attention core, ``sqb_refsem_fwd`` / ``sqb_refsem_bwd``) at the
B=8, H=12, T=1024, D=64 bf16 shape, with its float64 CPU oracle timed beside it.

``--impl reference`` times the CPU restatement of the operator (the
reference repository has no implementation of it) on the host cores, on a
bounded sample of the same workload (a subset of heads), and prints the same
metric.
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

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "sqrt-block attn fwd+bwd ms & HBM GB/s at T=16K; GPT-2 small train tokens/sec"
B, H, T, D = 1, 16, 16384, 128
ELT = 2  # bf16
# the long-context sweep (B=1, H=16, D=128, default block length); attn-t16k is
# the headline point and the default
SWEEP = {"attn-t4k": 4096, "attn-t8k": 8192, "attn-t16k": 16384, "attn-t32k": 32768,
         "attn-t64k": 65536}


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


def make_inputs(seed, rank, device, dtype=torch.bfloat16, H_=H):
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    return [torch.randn(B, T, H_, D, generator=g).to(dtype) for _ in range(4)]


def cpu_samples(heads=1, reps=1, seconds=0.0):
    """Time the oracle port (fp32 torch, all host threads) on `heads` heads of
    the workload, forward+backward, `reps` times and then until the timed work
    adds up to `seconds`; returns (list of seconds per sample, threads)."""
    from oracle.torch_port import sqrt_block_attention_ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v, do = [torch.randn(1, heads, T, D, generator=g) for _ in range(4)]
    times = []
    while len(times) < reps or (sum(times) < seconds and len(times) < 5000):
        qs, ks, vs = [x.clone().requires_grad_(True) for x in (q, k, v)]
        t0 = time.perf_counter()
        o, _ = sqrt_block_attention_ref(qs, ks, vs)
        (o * do).sum().backward()
        times.append(time.perf_counter() - t0)
    return times, threads


def cpu_sample_time(heads=1, reps=1):
    """Best of `reps` timed samples (see cpu_samples); returns (seconds, threads)."""
    times, threads = cpu_samples(heads, reps)
    return min(times), threads


def run_reference(args, world, rank):
    """CPU restatement of the operator, timed on the host cores."""
    if rank != 0:
        return
    from oracle.sqrtblock_oracle import default_block

    heads = 1
    sample_bytes = algorithmic_bytes(B, heads, T, D)
    cpu_sample_time(heads, 1)  # warm-up allocations and thread pool
    times = []
    for _ in range(max(args.warmup, 0)):
        cpu_sample_time(heads, 1)
    for _ in range(args.steps):
        dt, threads = cpu_sample_time(heads, 1)
        times.append(dt)
    per = statistics.median(times)
    gbs = sample_bytes / per / 1e9
    full_ms = per * (H / heads) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(full_ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": f"sqrt-block attention fwd+bwd (sweep point T={T})", "B": B,
                   "H": H, "T": T, "D": D, "block": default_block(T),
                   "parallelism": f"heads x {world} ranks (rank 0 timed)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{heads} of {H} heads per step, fp32 torch, "
                                   "ms_per_step scaled to all heads"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    from llm_training_b200 import _lib
    from llm_training_b200.ops import (read_status, sqrt_block_attention, sqrt_block_backward,
                                       sqrt_block_forward)

    dev = torch.device("cuda", local)
    host = make_inputs(args.seed, rank, dev)
    q, k, v, do = [x.to(dev) for x in host]
    block = _lib.geometry(T)[0]  # the default block length of this T
    fwd_impl = bwd_impl = args.kernels
    if args.kernels == "auto":
        # the tcgen05 family where it has a kernel for this shape, else SIMT
        qs, ks, vs, dos = q[:, :256], k[:, :256], v[:, :256], do[:, :256]
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
    launches_per_step = {"tcgen05": 1, "simt": 2}[fwd_impl] + {"tcgen05": 1, "simt": 4}[bwd_impl]
    impl = f"fwd:{fwd_impl},bwd:{bwd_impl}"

    stream = torch.cuda.current_stream(dev)
    # Q, K, V, dO and O resident: above 2x the 126 MB L2 nothing survives from
    # one step to the next; below it (T <= 8192 here) L2 is flushed between
    # timed steps (a 512 MB write) and a step is timed from the forward's start
    # to the backward's end, so the flush is not counted.
    resident = 5 * B * H * T * D * ELT
    flush = resident < 2 * 126 * 2**20
    flush_buf = torch.empty(512 * 2**20, dtype=torch.uint8, device=dev) if flush else None
    f_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    b_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]

    def step(i=None):
        if i is not None:
            f_ev[2 * i].record(stream)
        o, lse, kbar, vbar = sqrt_block_forward(q, k, v, block, None, fwd_impl)
        if i is not None:
            f_ev[2 * i + 1].record(stream)
            b_ev[2 * i].record(stream)
        dq, dk, dv = sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do, block, None, bwd_impl)
        if i is not None:
            b_ev[2 * i + 1].record(stream)
        return o, dq

    with ClockSampler(torch.cuda.current_device()) as clocks:
        # warm up for at least W steps and ~0.5 s so the clock sampler (100 ms
        # period) has samples under load when the timed region starts
        t_end = time.perf_counter() + args.warmup_seconds
        i = 0
        while i < max(args.warmup, 3) or time.perf_counter() < t_end:
            step()
            i += 1
            if i % 16 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(args.steps):
            if flush:
                flush_buf.zero_()
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = max_over_ranks(start.elapsed_time(end), world)
    status = read_status(dev)
    fwd_ms = statistics.mean(f_ev[2 * i].elapsed_time(f_ev[2 * i + 1]) for i in range(args.steps))
    bwd_ms = statistics.mean(b_ev[2 * i].elapsed_time(b_ev[2 * i + 1]) for i in range(args.steps))

    if flush:
        step_ms = statistics.mean(f_ev[2 * i].elapsed_time(b_ev[2 * i + 1])
                                  for i in range(args.steps))
        ms_per_step = max_over_ranks(step_ms, world)
    else:
        ms_per_step = total_ms / args.steps
    step_bytes = algorithmic_bytes(B, H, T, D)
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9

    # end to end through the public autograd op: every step copies its inputs
    # (Q, K, V, dO) in from pinned host memory and its results (O, dQ, dK, dV)
    # back out to pinned host memory.  Steps are pipelined on three streams, as
    # a host application streaming batches would run them: the H2D copy of
    # step i+1 and the D2H copy of step i-1 overlap step i.  Every step's copies
    # lie inside the timed region (first H2D start to last D2H end).
    pinned = [x.pin_memory() for x in host]
    outs = [[torch.empty(B, T, H, D, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
            for _ in range(2)]
    dev_in = [[torch.empty_like(x, device=dev) for x in host] for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_run(nsteps, timed):
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
            o = sqrt_block_attention(qd, kd, vd, block, None, args.kernels)  # as timed above
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

    e2e_run(2, False)
    barrier(world)
    # 30 streamed steps (~0.2 s): the pipeline's fill and drain (the first
    # step's H2D and the last step's D2H, which overlap nothing) are ~3 % of
    # the timed region, as in a long-running stream of batches
    e_steps = 30
    e2e_ms = max_over_ranks(e2e_run(e_steps, True), world) / e_steps
    h2d = sum(x.numel() * x.element_size() for x in pinned)
    d2h = sum(x.numel() * x.element_size() for x in outs[0])

    peak, peak_kind = load_peaks()
    bwd_bytes = algorithmic_bytes(B, H, T, D, fwd=False)
    fwd_bytes = algorithmic_bytes(B, H, T, D, bwd=False)
    dom = ("backward", bwd_bytes, bwd_ms) if bwd_ms >= fwd_ms else ("forward", fwd_bytes, fwd_ms)
    achieved = dom[1] / (dom[2] * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": None, "kernel": dom[0],
                "peak_source": peak_kind,
                "fwd": {"ms": round(fwd_ms, 4),
                        "GBps": round(fwd_bytes / (fwd_ms * 1e-3) / 1e9, 1)},
                "bwd": {"ms": round(bwd_ms, 4),
                        "GBps": round(bwd_bytes / (bwd_ms * 1e-3) / 1e9, 1)}}
    traffic_path = os.path.join(REPO, "profiles", "dram_traffic.json")
    if T == 16384 and os.path.exists(traffic_path):  # captured at T=16384
        try:
            roofline["traffic"] = json.load(open(traffic_path)).get(dom[0])
        except Exception:
            pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        # one head of the workload per sample, repeated until the timed CPU work
        # adds up to 10 s (median sample; a first, untimed call warms the pool)
        heads = 1
        cpu_sample_time(heads, 1)
        samples, threads = cpu_samples(heads, 1, seconds=10.0)
        dt = statistics.median(samples)
        cpu = {"value": round(algorithmic_bytes(B, heads, T, D) / dt / 1e9, 3), "unit": "GB/s",
               "cores": threads, "kind": "port",
               "sample": f"{heads} of {H} heads, fp32 torch fwd+bwd, median of {len(samples)} "
                         f"samples ({sum(samples):.1f} s; {dt * 1e3:.0f} ms each)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded per rank",
            "config": {"workload": f"sqrt-block attention fwd+bwd (sweep point T={T})",
                       "B": B, "H_per_rank": H, "T": T, "D": D, "block": block,
                       "parallelism": f"heads x {world} ranks", "kernels": impl,
                       "l2": (f"L2 flushed between steps (512 MB write, not timed); resident "
                              f"Q/K/V/dO/O {resident / 2**20:.0f} MB" if flush else
                              f"resident Q/K/V/dO/O {resident / 2**20:.0f} MB > 2 x 126 MB L2; "
                              "no flush")},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(step_bytes * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e_steps,
                    "pipelined": "H2D of step i+1 and D2H of step i-1 overlap step i "
                                 "(three streams); all copies inside the timed region"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "device_status": status,
        }
        print(json.dumps(line), flush=True)


# reference-semantics mode: (B, H, T, D) of the cfg-2 shape (T a perfect square)
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
        import numpy as np

        from oracle import refsem_oracle as rso

        x = [h[:1, :, :1].float().numpy().transpose(0, 2, 1, 3).astype(np.float64) for h in host]
        t0 = time.perf_counter()
        rso.fwd(*x[:3])
        rso.bwd(*x)
        dt = time.perf_counter() - t0
        cpu = {"value": round(11 * Tq * Dq * 2 / dt / 1e9, 4), "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": f"1 of {Bq * Hq} (batch, head) units, float64 numpy "
                                         f"oracle fwd+bwd, {dt * 1e3:.1f} ms"}
    if rank == 0:
        print(json.dumps({
            "metric": "reference-semantics sqrt_block attn fwd+bwd GB/s (B=8 H=12 T=1024 D=64)",
            "value": round(step_bytes * world / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded per rank",
            "config": {"workload": args.workload, "B": Bq, "H": Hq, "T": Tq, "D": Dq,
                       "mode": "reference semantics (CUDA-core kernels)",
                       "parallelism": f"replicas x {world} ranks"},
            "cpu_baseline": cpu, "gpu_launches": 7 * args.steps, "clocks": clocks.summary(),
            "device_status": read_status(dev),
        }), flush=True)


TRAIN_WORKLOADS = {
    # name: (config factory kwargs, sequences per GPU, sequence length)
    "gpt2-small": ("small", 16, 1024),
    "gpt2-medium-8k": ("medium", 8, 8192),
}


def run_train(args, world, rank, local):
    """GPT training step (fwd + bwd + clip + fused AdamW, bf16 autocast) with the
    sqrt-block attention; data-parallel over NCCL when run under torchrun."""
    from llm_training_b200.config import gpt2_medium, gpt2_small
    from llm_training_b200.train import Trainer, synthetic_batch

    kind, batch, seq = TRAIN_WORKLOADS[args.workload]
    cfg = gpt2_small(block_size=seq) if kind == "small" else gpt2_medium(block_size=seq,
                                                                        sqrt_block_b=96)
    dev = torch.device("cuda", local)
    tr = Trainer(cfg, dev, lr=6e-4, weight_decay=0.1, seed=1337, ddp=world > 1)
    gen = torch.Generator().manual_seed(args.seed * 1000 + rank)
    x, y = synthetic_batch(gen, batch, seq, cfg.vocab_size, dev)
    for _ in range(max(args.warmup, 3)):
        tr.step(x, y)
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            loss, _ = tr.step(x, y)
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world) / args.steps
    tokens = batch * seq * world
    # end to end: a fresh host batch copied in and the loss read back every step
    host = [torch.randint(0, cfg.vocab_size, (batch, seq + 1), generator=gen).pin_memory()
            for _ in range(2)]
    torch.cuda.synchronize()
    barrier(world)
    e0 = time.perf_counter()
    for i in range(max(1, min(args.steps, 5))):
        tok = host[i % 2].to(dev, non_blocking=True)
        loss, _ = tr.step(tok[:, :-1], tok[:, 1:])
        loss.item()
    torch.cuda.synchronize()
    e_ms = max_over_ranks((time.perf_counter() - e0) * 1e3, world) / max(1, min(args.steps, 5))
    if rank == 0:
        nparams = sum(p.numel() for p in tr.raw_model.parameters())
        print(json.dumps({
            "metric": f"{args.workload} train tokens/sec (sqrt-block attention)",
            "value": round(tokens / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform token ids, seeded per rank",
            "config": {"workload": args.workload, "model": kind, "params": nparams,
                       "global_batch": batch * world, "seq_len": seq,
                       "block": cfg.sqrt_block_b or "default", "parallelism": f"dp{world}",
                       "optimizer": "fused AdamW lr 6e-4 wd 0.1, clip 1.0"},
            "e2e": {"value": round(tokens / (e_ms * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e_ms, 3), "h2d_bytes_per_step": batch * (seq + 1) * 8,
                    "d2h_bytes_per_step": 4},
            "last_loss": round(float(loss), 4),
            "clocks": clocks.summary(),
        }), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernels", choices=["auto", "tcgen05", "simt"], default="auto")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--warmup-seconds", type=float, default=0.5,
                    help="keep warming up at least this long (clock sampler needs samples)")
    ap.add_argument("--workload", choices=sorted(SWEEP) + sorted(TRAIN_WORKLOADS) + sorted(REFSEM),
                    default="attn-t16k",
                    help="attn-t*: the attention op at that sweep length (attn-t16k is the "
                         "default); gpt2-*: a training step")
    args = ap.parse_args()
    global T
    T = SWEEP.get(args.workload, T)
    world, rank, local = init_dist()
    try:
        if args.workload in REFSEM:
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable":
                                      "the reference checkout is not present where the "
                                      "benchmark runs; the workload's cpu_baseline times its "
                                      "CPU oracle"}),
                          flush=True)
            else:
                run_refsem(args, world, rank, local)
        elif args.workload not in SWEEP:
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
