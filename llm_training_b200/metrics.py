"""Training-run report in the reference trainer's ``metrics.json`` schema.

The reference writes one JSON file per run (metrics.py:516-537) with five
sections, and this module writes the same keys so the same tooling reads
either run:

* ``run`` - the run description given by the caller, plus ``started_at``,
  ``tokens_per_step``, ``warmup_steps_skipped``, ``log_interval``, ``status``,
  ``elapsed_wall_clock_sec`` and ``updated_at``;
* ``aggregates`` - means over the measured steps (every step after the first
  ``warmup_steps_skipped``, metrics.py:382): step time, tokens/s, model
  (forward + backward) time, peak memory, and the attention layers' time, share
  of the step and peak memory;
* ``train`` / ``val`` - curve points (every ``log_interval`` steps for train);
* ``_stats`` - the running count/sum pairs the means come from.

Timing: phases are bracketed by CUDA events on the current stream and read
after the one synchronize of ``end_step``; the step time is the host clock
from ``begin_step`` to that synchronize, as in the reference.  The attention
layers are timed by forward-pre/forward and full-backward-pre/full-backward
hooks on every ``BaseAttention`` instance, each bracket also opening a memory
segment (the allocator peak is rebased on entry and read on exit).  The file
is replaced atomically (temporary file + ``os.replace``).
"""

from __future__ import annotations

import json
import math
import os
import time
from contextlib import contextmanager
from datetime import datetime, timezone

import torch

_MIB = float(1 << 20)


def _now():
    return datetime.now(timezone.utc).isoformat(timespec="seconds")


class _Mean:
    """count / sum pair (persisted as such in ``_stats``)."""

    def __init__(self, d=None):
        self.count = int((d or {}).get("count", 0))
        self.sum = float((d or {}).get("sum", 0.0))

    def add(self, x):
        self.count += 1
        self.sum += float(x)

    def value(self):
        return self.sum / self.count if self.count else None

    def state(self):
        return {"count": self.count, "sum": self.sum}


class _Spans:
    """Named durations of the current step: CUDA event pairs (host clock on
    CPU), summed per label, resolved after the step's synchronize."""

    def __init__(self, cuda: bool):
        self.cuda = cuda
        self.open: dict[str, object] = {}
        self.done: list[tuple[str, object, object]] = []

    def start(self, label):
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.open[label] = ev
        else:
            self.open[label] = time.perf_counter()

    def stop(self, label):
        begin = self.open.pop(label, None)
        if begin is None:
            return
        if self.cuda:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
        else:
            end = time.perf_counter()
        self.done.append((label, begin, end))

    def resolve(self):
        out: dict[str, float] = {}
        for label, a, b in self.done:
            ms = a.elapsed_time(b) if self.cuda else (b - a) * 1e3
            out[label] = out.get(label, 0.0) + ms
        self.done.clear()
        self.open.clear()
        return out


class MetricsReport:
    """Collects one run's curves and running means and writes ``metrics.json``."""

    def __init__(self, path, run_info, tokens_per_step, warmup_steps_skipped=10,
                 log_interval=1, device_type="cuda"):
        self.path = path
        self.tokens_per_step = int(tokens_per_step)
        self.skip = int(warmup_steps_skipped)
        self.log_interval = max(int(log_interval), 1)
        self.cuda = device_type == "cuda" and torch.cuda.is_available()
        self.spans = _Spans(self.cuda)
        self.run = dict(run_info, started_at=_now(), tokens_per_step=self.tokens_per_step,
                        warmup_steps_skipped=self.skip, log_interval=self.log_interval)
        self.train, self.val = [], []
        self.means = {k: _Mean() for k in ("step_time", "tokens_per_sec", "attn_forward",
                                           "attn_backward", "peak_alloc_avg",
                                           "peak_reserved_avg")}
        self.phase_means: dict[str, _Mean] = {}
        self.attn_layers = 0
        self.attn_peak_abs = 0
        self.attn_peak_delta = 0
        self._step_peak = [0, 0]        # allocated, reserved high-water marks of the step
        self._attn_step_peak = [0, 0]   # absolute, delta-over-entry inside attention
        self._entry_alloc = 0
        self._measuring = False
        self._profiling = False
        self._t0 = 0.0
        self._wall0 = time.time()

    # ---- phases and attention hooks ------------------------------------------------
    @contextmanager
    def phase(self, label):
        """Time a labelled part of the step (e.g. "forward", "backward")."""
        self.spans.start(label)
        try:
            yield
        finally:
            self.spans.stop(label)

    def _fold_peak(self):
        if self.cuda:
            self._step_peak[0] = max(self._step_peak[0], torch.cuda.max_memory_allocated())
            self._step_peak[1] = max(self._step_peak[1], torch.cuda.max_memory_reserved())

    def _enter_attention(self, label):
        if not self._profiling:
            return
        if self.cuda:
            self._fold_peak()
            torch.cuda.reset_peak_memory_stats()
            self._entry_alloc = torch.cuda.memory_allocated()
        self.spans.start(label)

    def _leave_attention(self, label):
        if not self._profiling:
            return
        self.spans.stop(label)
        if self.cuda:
            peak = torch.cuda.max_memory_allocated()
            self._attn_step_peak[0] = max(self._attn_step_peak[0], peak)
            self._attn_step_peak[1] = max(self._attn_step_peak[1], peak - self._entry_alloc)
            self._fold_peak()
            torch.cuda.reset_peak_memory_stats()

    def attach_attention(self, model, base_cls):
        """Hook every ``base_cls`` instance of ``model`` (the attention layers)."""
        for m in model.modules():
            if isinstance(m, base_cls):
                self.attn_layers += 1
                m.register_forward_pre_hook(lambda *a: self._enter_attention("attention_forward"))
                m.register_forward_hook(lambda *a: self._leave_attention("attention_forward"))
                m.register_full_backward_pre_hook(
                    lambda *a: self._enter_attention("attention_backward"))
                m.register_full_backward_hook(
                    lambda *a: self._leave_attention("attention_backward"))
        self.run["attention_layers_profiled"] = self.attn_layers
        return self.attn_layers

    # ---- step lifecycle --------------------------------------------------------------
    def begin_step(self, step):
        self._measuring = step >= self.skip
        self._step_peak = [0, 0]
        self._attn_step_peak = [0, 0]
        if self.cuda:
            torch.cuda.reset_peak_memory_stats()
        self._profiling = self.attn_layers > 0
        self._t0 = time.perf_counter()

    def end_step(self, step, loss, lr, grad_norm):
        """Synchronize once, fold the step into the means, log a curve point."""
        if self.cuda:
            torch.cuda.synchronize()
        step_ms = (time.perf_counter() - self._t0) * 1e3
        tok_s = self.tokens_per_step * 1e3 / step_ms
        phases = self.spans.resolve()
        self._fold_peak()
        self._profiling = False
        if self._measuring:
            self.means["step_time"].add(step_ms)
            self.means["tokens_per_sec"].add(tok_s)
            for label, ms in phases.items():
                self.phase_means.setdefault(label, _Mean()).add(ms)
            if self.cuda:
                self.means["peak_alloc_avg"].add(self._step_peak[0])
                self.means["peak_reserved_avg"].add(self._step_peak[1])
            if self.attn_layers:
                self.means["attn_forward"].add(phases.get("attention_forward", 0.0))
                self.means["attn_backward"].add(phases.get("attention_backward", 0.0))
                self.attn_peak_abs = max(self.attn_peak_abs, self._attn_step_peak[0])
                self.attn_peak_delta = max(self.attn_peak_delta, self._attn_step_peak[1])
        last = self.run.get("max_steps", 0) - 1
        if step % self.log_interval == 0 or step == last:
            loss = float(loss)
            self.train.append({"step": step, "train_loss": loss,
                               "train_perplexity": _exp(loss), "lr": lr,
                               "grad_norm": float(grad_norm), "step_time_ms": step_ms,
                               "tokens_per_sec": tok_s,
                               "tokens_seen": (step + 1) * self.tokens_per_step})
            self.write()
        return step_ms, tok_s, phases

    def log_validation(self, step, val_loss):
        self.val.append({"step": step, "val_loss": float(val_loss),
                         "val_perplexity": _exp(float(val_loss)),
                         "tokens_seen": step * self.tokens_per_step})

    # ---- output ----------------------------------------------------------------------
    def aggregates(self):
        fwd, bwd = self.phase_means.get("forward"), self.phase_means.get("backward")
        model_ms = (fwd.value() + bwd.value()) if (fwd and bwd and fwd.count and bwd.count) \
            else None
        step_mean = self.means["step_time"].value()
        out = {"measured_steps": self.means["step_time"].count,
               "note": (f"means over the steps after the first {self.skip} (warm-up steps "
                        "are excluded); one optimizer step each"),
               "avg_step_time_ms": step_mean,
               "avg_tokens_per_sec": self.means["tokens_per_sec"].value(),
               "avg_model_time_ms": model_ms}
        if self.cuda:
            pa, pr = self.means["peak_alloc_avg"].value(), self.means["peak_reserved_avg"].value()
            out["avg_peak_memory_mib"] = {"allocated": pa / _MIB if pa is not None else None,
                                          "reserved": pr / _MIB if pr is not None else None}
        if self.attn_layers:
            af, ab = self.means["attn_forward"], self.means["attn_backward"]
            attn_ms = af.value() + ab.value() if af.count else None
            attn = {"layers": self.attn_layers, "avg_time_ms": attn_ms,
                    "fraction_of_step_time": (attn_ms / step_mean
                                              if attn_ms is not None and step_mean else None)}
            if self.cuda:
                attn["peak_memory_mib"] = {"absolute": self.attn_peak_abs / _MIB,
                                           "delta_over_entry": self.attn_peak_delta / _MIB}
            out["attention"] = attn
        return out

    def stats(self):
        s = {k: m.state() for k, m in self.means.items()}
        s["phase_time"] = {k: m.state() for k, m in self.phase_means.items()}
        s["attn_peak_absolute"] = self.attn_peak_abs
        s["attn_peak_delta"] = self.attn_peak_delta
        return s

    def snapshot(self):
        return {"run": dict(self.run), "aggregates": self.aggregates(), "train": list(self.train),
                "val": list(self.val), "_stats": self.stats()}

    def write(self, status="running"):
        """Replace the file with the current snapshot (no file when path is None,
        e.g. on data-parallel ranks other than the first)."""
        doc = self.snapshot()
        doc["run"].update(status=status, elapsed_wall_clock_sec=time.time() - self._wall0,
                          updated_at=_now())
        if self.path is None:
            return doc
        folder = os.path.dirname(os.path.abspath(self.path))
        os.makedirs(folder, exist_ok=True)
        tmp = f"{self.path}.tmp"
        with open(tmp, "w") as f:
            json.dump(doc, f, indent=2)
        os.replace(tmp, self.path)
        return doc


def _exp(x):
    try:
        return math.exp(x)
    except OverflowError:
        return float("inf")
