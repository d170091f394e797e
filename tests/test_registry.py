"""The plugin boundary on CPU: registry semantics, state-dict compatibility with
the reference, profiler hooks, and the absence of any CPU compute path."""

import json
import os

import pytest
import torch
import torch.nn as nn

from llm_training_b200.config import ModelConfig
from llm_training_b200.model import attention_registry as reg
from llm_training_b200.model.gpt import GPT
from llm_training_b200.model.sqrt_block_attention import SqrtBlockAttention

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_names_registered_and_normalised():
    names = reg.available_attentions()
    assert "sqrt_block" in names and "custom" in names
    assert reg.get_attention("Sqrt-Block") is SqrtBlockAttention
    assert reg.get_attention("  SQRT_BLOCK ") is SqrtBlockAttention
    assert reg.discovery_errors() == {}


def test_unknown_name_lists_available():
    with pytest.raises(KeyError, match="sqrt_block"):
        reg.get_attention("nope")


def test_register_rejects_non_base_and_duplicates():
    with pytest.raises(TypeError):
        reg.register_attention("zz_bad")(nn.Linear)

    @reg.register_attention("zz_test_attn")
    class A(reg.BaseAttention):
        pass

    assert reg.get_attention("zz-test-attn") is A
    reg.register_attention("zz_test_attn")(A)  # same class again is fine
    with pytest.raises(ValueError, match="already registered"):
        @reg.register_attention("zz_test_attn")
        class B(reg.BaseAttention):
            pass
    reg.REGISTRY.remove("zz_test_attn")


def test_module_class_escape_hatch():
    cls = reg.get_attention("llm_training_b200.model.sqrt_block_attention:SqrtBlockAttention")
    assert cls is SqrtBlockAttention
    with pytest.raises(ValueError):
        reg.get_attention("llm_training_b200.model.sqrt_block_attention:Missing")
    with pytest.raises(TypeError):
        reg.get_attention("torch.nn:Linear")


def test_discovery_isolates_broken_modules(monkeypatch):
    monkeypatch.setattr(reg.REGISTRY, "extra_plugins", ["zz_missing_module"])
    report = reg.REGISTRY.scan(force=True)
    try:
        assert "zz_missing_module" in report.failed
        assert "ModuleNotFoundError" in report.failed["zz_missing_module"]
        assert any(m.endswith(".sqrt_block_attention") for m in report.imported)
        assert "sqrt_block" in reg.available_attentions()  # still found
        assert "zz_missing_module" in reg.discovery_errors()
    finally:
        monkeypatch.undo()
        reg.REGISTRY.scan(force=True)
    assert reg.discovery_errors() == {}


def test_build_attention_uses_config_name():
    cfg = ModelConfig(n_embd=64, n_head=4, block_size=64, attention="sqrt_block")
    m = reg.build_attention(cfg)
    assert isinstance(m, SqrtBlockAttention) and isinstance(m, reg.BaseAttention)


@pytest.mark.parametrize("bias", [False, True])
def test_state_dict_matches_reference(bias):
    d = json.load(open(os.path.join(GOLDEN, "ref_state_dict_keys.json")))
    c = d["config"]
    cfg = ModelConfig(block_size=c["block_size"], vocab_size=c["vocab_size"],
                      n_layer=c["n_layer"], n_head=c["n_head"], n_embd=c["n_embd"], bias=bias,
                      attention="sqrt_block")
    sd = GPT(cfg).state_dict()
    got = {k: list(v.shape) for k, v in sd.items()}
    assert got == d["keys"][f"bias={bias}"]


def test_no_persistent_buffers_and_loads_reference_style_weights():
    cfg = ModelConfig(n_embd=64, n_head=4, block_size=64, bias=False)
    m = SqrtBlockAttention(cfg)
    assert sorted(m.state_dict()) == ["Wk.weight", "Wq.weight", "Wv.weight", "c_proj.weight"]
    sd = {k: torch.randn_like(v) for k, v in m.state_dict().items()}
    m.load_state_dict(sd, strict=True)


def test_cpu_input_fails_loudly():
    cfg = ModelConfig(n_embd=64, n_head=4, block_size=64, bias=False)
    m = SqrtBlockAttention(cfg)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 32, 64))


def test_attention_dropout_rejected_in_training():
    cfg = ModelConfig(n_embd=64, n_head=4, block_size=64, bias=False, dropout=0.1)
    m = SqrtBlockAttention(cfg).train()
    with pytest.raises(NotImplementedError):
        m(torch.randn(1, 32, 64))


def test_profiler_hooks_register():
    """The reference profiler (metrics.py:156-162) registers these four hooks on
    every BaseAttention; they must be accepted by the module."""
    cfg = ModelConfig(n_embd=64, n_head=4, block_size=64, bias=False)
    m = SqrtBlockAttention(cfg)
    hs = [m.register_forward_pre_hook(lambda *a: None), m.register_forward_hook(lambda *a: None),
          m.register_full_backward_pre_hook(lambda *a: None),
          m.register_full_backward_hook(lambda *a: None)]
    for h in hs:
        h.remove()


@pytest.mark.parametrize("bias", [False, True])
def test_reference_semantics_plugin_is_a_drop_in(bias):
    """``sqrt_block_reference`` (the reference's own math) registers, has the
    reference module's parameters and no persistent buffers, and a GPT built with
    it has the reference GPT's state-dict keys, so reference checkpoints load."""
    from llm_training_b200.model.sqrt_block_reference_attention import (
        ReferenceSqrtBlockAttention)

    assert reg.get_attention("sqrt-block-reference") is ReferenceSqrtBlockAttention
    d = json.load(open(os.path.join(GOLDEN, "ref_state_dict_keys.json")))
    c = d["config"]
    cfg = ModelConfig(block_size=c["block_size"], vocab_size=c["vocab_size"],
                      n_layer=c["n_layer"], n_head=c["n_head"], n_embd=c["n_embd"], bias=bias,
                      attention="sqrt_block_reference")
    model = GPT(cfg)
    assert {k: list(v.shape) for k, v in model.state_dict().items()} == d["keys"][f"bias={bias}"]
    m = model.transformer.attn_blocks[0].attn
    assert isinstance(m, ReferenceSqrtBlockAttention)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 16, c["n_embd"]))
