"""Synthetic-token GPT training step driving the sqrt-block attention.

This is the op's caller for the training configurations (GPT-2 small at T=1024 on one
GPU; GPT-2 medium at T=8192 data-parallel over several GPUs).  One step mirrors the
reference trainer's inner loop (train.py:482-509): bf16-autocast forward and
cross-entropy (training_utils.py:8-17), backward, clip_grad_norm_(1.0), and AdamW with
the reference's decay / no-decay parameter groups (training_utils.py:25-51; fused on
CUDA; weight_decay 0.1, betas (0.9, 0.95) as at train.py:305-306).  With WORLD_SIZE > 1
the model is wrapped in DistributedDataParallel, whose bucketed NCCL all-reduce of the
gradients overlaps the backward pass.  Tokens are uniform over the vocabulary from a
seeded generator: no dataset is involved.
"""

from __future__ import annotations

import inspect
from contextlib import nullcontext

import torch
import torch.nn.functional as F

from .model.gpt import GPT
from .ops import check_status, cross_entropy


def calculate_loss(logits, targets):
    """Next-token cross-entropy over (B*T, vocab) (or over the padded vocabulary
    of ``GPT.forward(pad_vocab=True)``, whose extra columns are -inf).  On CUDA
    the library's fused cross-entropy computes it (the same fp32 math as the
    autocast ``F.cross_entropy`` of the reference, without its fp32 copies of
    the logits); on CPU ``F.cross_entropy``."""
    if logits.is_cuda:
        return cross_entropy(logits, targets)
    return F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1))


def configure_optimizers(model, weight_decay, learning_rate, betas=(0.9, 0.95),
                         device_type="cuda"):
    """AdamW with decay on every >= 2-D parameter and none on the rest."""
    params = [p for p in model.parameters() if p.requires_grad]
    decay = [p for p in params if p.dim() >= 2]
    nodecay = [p for p in params if p.dim() < 2]
    groups = [{"params": decay, "weight_decay": weight_decay},
              {"params": nodecay, "weight_decay": 0.0}]
    fused = "fused" in inspect.signature(torch.optim.AdamW).parameters and device_type == "cuda"
    return torch.optim.AdamW(groups, lr=learning_rate, betas=betas,
                             **({"fused": True} if fused else {}))


def synthetic_batch(gen, batch, seq, vocab, device):
    """(x, y) token ids uniform over [0, vocab), y = x shifted by one."""
    tok = torch.randint(0, vocab, (batch, seq + 1), generator=gen)
    x, y = tok[:, :-1], tok[:, 1:]
    if device.type == "cuda":
        x, y = x.pin_memory(), y.pin_memory()
    return x.to(device, non_blocking=True), y.to(device, non_blocking=True)


class Trainer:
    """One model + optimizer; ``step(x, y)`` runs forward, backward, clip, AdamW."""

    def __init__(self, config, device, lr=6e-4, weight_decay=0.1, seed=1337, ddp=False,
                 autocast=True, ddp_kwargs=None):
        torch.manual_seed(seed)
        self.device = device
        self.model = GPT(config).to(device)
        self.raw_model = self.model
        if ddp:
            from torch.nn.parallel import DistributedDataParallel

            ids = [device.index] if device.type == "cuda" else None
            # gradients live in DDP's communication buckets (no copy of the
            # 4-byte gradients into and out of them around each all-reduce);
            # 100 MB buckets: fewer, larger all-reduces overlapped with the
            # backward (measured on two B200s for GPT-2 small: 0.8 ms of the
            # all-reduce left exposed per step, 1.3 ms with 25 MB buckets)
            kw = dict(gradient_as_bucket_view=True, bucket_cap_mb=100)
            kw.update(ddp_kwargs or {})
            self.model = DistributedDataParallel(self.model, device_ids=ids, **kw)
        self.optimizer = configure_optimizers(self.raw_model, weight_decay, lr,
                                              device_type=device.type)
        self.autocast = autocast and device.type == "cuda"

    def step(self, x, y, report=None):
        """One optimizer step.  First raises if an attention kernel of an earlier
        step posted a device-side failure (a non-blocking check of the
        library's page-locked mailboxes: that step's gradients were invalid).
        ``report`` (a ``metrics.MetricsReport``) times the forward, backward and
        optimizer phases as the reference trainer does (train.py:488-505)."""
        if self.device.type == "cuda":
            check_status(self.device)
        span = report.phase if report is not None else (lambda _label: nullcontext())
        self.optimizer.zero_grad(set_to_none=True)
        with span("forward"), torch.autocast(device_type=self.device.type,
                                             dtype=torch.bfloat16, enabled=self.autocast):
            logits = self.model(x, pad_vocab=True)
            loss = calculate_loss(logits, y)
        with span("backward"):
            loss.backward()
        with span("optimizer"):
            norm = torch.nn.utils.clip_grad_norm_(self.model.parameters(), 1.0)
            self.optimizer.step()
        return loss.detach(), norm

    def run_info(self, config, batch, seq, max_steps, lr, seed, compiled=False):
        """The ``run`` section of a metrics.json report (the reference's keys,
        train.py's run description): device, model and training settings."""
        raw = self.raw_model
        n = sum(p.numel() for p in raw.parameters())
        emb = raw.transformer.wpe.weight.numel()
        dev = self.device
        return {
            "device": dev.type,
            "gpu_name": torch.cuda.get_device_name(dev) if dev.type == "cuda" else None,
            "torch_version": torch.__version__,
            "autocast_dtype": "bfloat16" if self.autocast else None,
            "torch_compile": compiled, "attention_profiling": True,
            "attention": config.attention, "seed": seed, "num_parameters": n,
            "num_parameters_non_embedding": n - emb,
            "model_config": {k: getattr(config, k) for k in (
                "block_size", "vocab_size", "n_layer", "n_head", "n_embd", "dropout", "bias",
                "attention")},
            "batch_size": batch, "seq_len": seq, "grad_accumulation_steps": 1,
            "max_steps": max_steps, "max_lr": lr, "min_lr": lr, "warmup_steps": 0,
            "eval_interval": 0, "eval_iters": 0, "data_dir": "synthetic (uniform token ids)",
        }
