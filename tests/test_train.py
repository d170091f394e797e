"""Host-side training-step logic: optimizer groups, a CPU step, and data-parallel
gradient averaging across two gloo ranks (no GPU involved)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_training_b200.config import ModelConfig, gpt2_small
from llm_training_b200.model.gpt import GPT
from llm_training_b200.train import Trainer, configure_optimizers, synthetic_batch

CPU_ATTN = "tests.cpu_attention:CausalAttentionCPU"


def tiny(**kw):
    base = dict(block_size=64, vocab_size=97, n_layer=2, n_head=2, n_embd=32, bias=False,
                attention=CPU_ATTN)
    base.update(kw)
    return ModelConfig(**base)


def test_optimizer_groups_follow_reference_rule():
    m = GPT(tiny())
    opt = configure_optimizers(m, 0.1, 6e-4, device_type="cpu")
    decay, nodecay = opt.param_groups
    assert decay["weight_decay"] == 0.1 and nodecay["weight_decay"] == 0.0
    assert all(p.dim() >= 2 for p in decay["params"])
    assert all(p.dim() < 2 for p in nodecay["params"])
    n = sum(p.numel() for g in opt.param_groups for p in g["params"])
    assert n == sum(p.numel() for p in m.parameters())


def test_gpt2_small_config_shapes():
    cfg = gpt2_small()
    assert (cfg.n_layer, cfg.n_head, cfg.n_embd, cfg.vocab_size, cfg.bias) == (12, 12, 768,
                                                                                50257, False)


def test_cpu_training_step_reduces_loss():
    tr = Trainer(tiny(), torch.device("cpu"), lr=3e-3, seed=0)
    gen = torch.Generator().manual_seed(0)
    x, y = synthetic_batch(gen, 4, 32, 97, torch.device("cpu"))
    first = float(tr.step(x, y)[0])
    for _ in range(30):
        last = float(tr.step(x, y)[0])
    assert last < first - 0.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ddp_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = Trainer(tiny(), torch.device("cpu"), lr=1e-3, seed=0, ddp=True)
        gen = torch.Generator().manual_seed(100 + rank)  # different data per rank
        x, y = synthetic_batch(gen, 2, 32, 97, torch.device("cpu"))
        tr.step(x, y)
        flat = torch.cat([p.detach().flatten() for p in tr.raw_model.parameters()])
        gathered = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(gathered, flat)
        out[rank] = float(max((g - flat).abs().max() for g in gathered))
        # the trainer's DDP settings (gradient bucket views, 100 MB buckets) and
        # their override
        tr2 = Trainer(tiny(), torch.device("cpu"), lr=1e-3, seed=0, ddp=True,
                      ddp_kwargs={"bucket_cap_mb": 1})
        out[f"ddp{rank}"] = (tr.model.gradient_as_bucket_view, tr.model.bucket_bytes_cap,
                             tr2.model.bucket_bytes_cap)
    finally:
        dist.destroy_process_group()


def test_two_rank_data_parallel_step_keeps_replicas_identical():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_ddp_worker, args=(world, _free_port(), out), nprocs=world, join=True)
        assert max(out[r] for r in range(world)) == 0.0
        for r in range(world):
            assert out[f"ddp{r}"] == (True, 100 * 2**20, 2**20)


@pytest.mark.gpu
def test_gpu_training_step_with_sqrt_block_attention():
    cfg = tiny(attention="sqrt_block", block_size=1024, n_embd=128, n_head=2, vocab_size=512)
    dev = torch.device("cuda", 0)
    tr = Trainer(cfg, dev, lr=3e-3, seed=0)
    gen = torch.Generator().manual_seed(0)
    x, y = synthetic_batch(gen, 4, 1024, 512, dev)
    first = float(tr.step(x, y)[0])
    for _ in range(20):
        loss, norm = tr.step(x, y)
    assert torch.isfinite(loss) and torch.isfinite(norm)
    assert float(loss) < first - 0.5


def test_padded_vocab_logits_give_the_same_loss_and_gradients():
    """The lm_head GEMM over a vocabulary padded to a multiple of 64 (-inf in the
    padded columns) is the unpadded cross-entropy, value and gradients."""
    from llm_training_b200.train import calculate_loss

    torch.manual_seed(0)
    cfg = tiny(vocab_size=97)
    m = GPT(cfg).double()
    gen = torch.Generator().manual_seed(1)
    x, y = synthetic_batch(gen, 3, 16, 97, torch.device("cpu"))
    losses, grads = [], []
    for pad in (False, True):
        m.zero_grad(set_to_none=True)
        logits = m(x, pad_vocab=pad)
        assert logits.shape[-1] == (128 if pad else 97)
        loss = calculate_loss(logits, y)
        loss.backward()
        losses.append(loss.detach())
        grads.append({n: p.grad.clone() for n, p in m.named_parameters()})
    assert torch.allclose(losses[0], losses[1], rtol=1e-12, atol=1e-12)
    for n in grads[0]:
        assert torch.allclose(grads[0][n], grads[1][n], rtol=1e-10, atol=1e-12), n
    # the padding is compute-only: the parameters and state-dict keys are unchanged
    assert "_pad_bias" not in m.state_dict()
    assert m.lm_head.weight.shape[0] == 97


@pytest.mark.gpu
def test_gpu_fused_caller_ops_match_torch_ops_end_to_end(monkeypatch):
    """One autocast step of a small GPT: the fused LayerNorm (and residual add +
    LayerNorm), the fused cross-entropy and the padded-vocabulary logits give the
    loss and gradients of the same model on torch's add, nn.LayerNorm,
    F.cross_entropy and unpadded logits."""
    import torch.nn.functional as F

    import llm_training_b200.model.gpt as gpt_mod

    cfg = tiny(attention="sqrt_block", block_size=256, n_embd=256, n_head=4, vocab_size=1001)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    m = GPT(cfg).to(dev)
    gen = torch.Generator().manual_seed(3)
    x, y = synthetic_batch(gen, 4, 256, 1001, dev)

    def run(fused):
        m.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                from llm_training_b200.train import calculate_loss

                loss = calculate_loss(m(x, pad_vocab=True), y)
            else:
                logits = m(x)
                loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), y.reshape(-1))
        loss.backward()
        return loss.detach().float(), {n: p.grad.float().clone() for n, p in m.named_parameters()}

    l_fused, g_fused = run(True)
    with monkeypatch.context() as mp_:
        mp_.setattr(gpt_mod, "layer_norm_supported", lambda *a: False)
        mp_.setattr(gpt_mod, "add_layer_norm_supported", lambda *a: False)
        l_ref, g_ref = run(False)
    # the same values reach every bf16 GEMM; the LayerNorm statistics are summed
    # in a different order, which bf16 rounding can amplify by an ulp here and there
    torch.testing.assert_close(l_fused, l_ref, rtol=2e-3, atol=2e-3)
    for n in g_ref:
        a, b = g_fused[n].flatten(), g_ref[n].flatten()
        cos = float(torch.dot(a, b) / (a.norm() * b.norm() + 1e-30))
        assert cos > 0.999, (n, cos)
        assert float((a.norm() - b.norm()).abs() / (b.norm() + 1e-30)) < 1e-2, n


def test_metrics_report_has_the_reference_schema(tmp_path):
    """A CPU run written by MetricsReport has every key path of the reference's
    metrics.json (tests/golden/ref_metrics_schema.json, read from the run the
    reference ships), and the warm-up steps are excluded from the means."""
    import json

    from llm_training_b200.metrics import MetricsReport
    from llm_training_b200.model.attention_registry import BaseAttention

    cfg = tiny()
    tr = Trainer(cfg, torch.device("cpu"), lr=3e-3, seed=0)
    gen = torch.Generator().manual_seed(0)
    x, y = synthetic_batch(gen, 2, 32, 97, torch.device("cpu"))
    path = str(tmp_path / "metrics.json")
    info = tr.run_info(cfg, 2, 32, max_steps=6, lr=3e-3, seed=0)
    rep = MetricsReport(path, info, tokens_per_step=64, warmup_steps_skipped=2, log_interval=2,
                        device_type="cpu")
    assert rep.attach_attention(tr.raw_model, BaseAttention) == cfg.n_layer
    for step in range(6):
        rep.begin_step(step)
        loss, norm = tr.step(x, y, report=rep)
        rep.end_step(step, float(loss), 3e-3, float(norm))
    rep.log_validation(6, 4.0)
    rep.write("finished")
    doc = json.load(open(path))

    def paths(d, prefix=""):
        if isinstance(d, dict):
            for k, v in d.items():
                yield f"{prefix}/{k}"
                yield from paths(v, f"{prefix}/{k}")
        elif isinstance(d, list) and d:
            yield from paths(d[0], f"{prefix}[]")

    ref = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                      "ref_metrics_schema.json")))["paths"]
    # the reference's CPU-less keys (peak memory) and the resume breadcrumb
    # appear only on CUDA runs / resumed runs; its phases include "data"
    optional = ("/run/resumed_at", "/aggregates/avg_peak_memory_mib",
                "/aggregates/attention/peak_memory_mib", "/_stats/phase_time/data")
    missing = [p for p in ref if p not in set(paths(doc)) and not p.startswith(optional)]
    assert missing == []
    agg = doc["aggregates"]
    assert agg["measured_steps"] == 4                      # steps 2..5
    assert doc["_stats"]["step_time"]["count"] == 4
    assert [r["step"] for r in doc["train"]] == [0, 2, 4, 5]
    assert agg["attention"]["layers"] == cfg.n_layer
    assert 0 < agg["attention"]["fraction_of_step_time"] < 1
    assert doc["run"]["status"] == "finished"
