"""CPU test of patch_model's wiring (no GPU): the fused-boundary decoder
layers, the norm handoff and the SwiGLU MLP module, with the four kernels
stood in for by the oracle's formulas (test-only monkeypatching; the product
has no CPU path). A patched tiny Qwen2 must produce the unpatched model's
logits (same rounding points), through prefill and a cached decode step, and
hand every layer's normalised output to the next norm instead of recomputing."""

from __future__ import annotations

import pytest
import torch

from tritonforge_b200 import kernels
from tritonforge_b200.integration import patch_model
from tritonforge_b200.integration import qwen as tq


def _rmsnorm_residual(x, residual, weight, eps=1e-6, config=None):
    s = (x + residual).to(x.dtype)
    v = s.float().pow(2).mean(-1, keepdim=True)
    return (weight * (s.float() * torch.rsqrt(v + eps)).to(x.dtype)).to(x.dtype), s


def _rmsnorm(x, weight, eps=1e-6, config=None):
    v = x.float().pow(2).mean(-1, keepdim=True)
    return (weight * (x.float() * torch.rsqrt(v + eps)).to(x.dtype)).to(x.dtype)


def _swiglu(gate, up, config=None):
    g = gate.float()
    return (g * torch.sigmoid(g) * up.float()).to(gate.dtype)


@pytest.fixture
def host_kernels(monkeypatch):
    calls = {"rmsnorm": 0, "rmsnorm_residual": 0, "swiglu": 0}

    def counted(name, fn):
        def wrap(*a, **k):
            calls[name] += 1
            return fn(*a, **k)
        return wrap

    monkeypatch.setattr(kernels, "rmsnorm", counted("rmsnorm", _rmsnorm))
    monkeypatch.setattr(kernels, "rmsnorm_residual", counted("rmsnorm_residual", _rmsnorm_residual))
    monkeypatch.setattr(kernels, "swiglu", counted("swiglu", _swiglu))
    return calls


def _tiny(layers=3):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
    return Qwen2ForCausalLM(cfg).float().eval(), cfg


def test_patched_layers_match_unpatched_and_hand_off(host_kernels):
    model, cfg = _tiny(3)
    ids = torch.randint(0, cfg.vocab_size, (2, 7), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(ids, use_cache=True)
        nxt = ref.logits[:, -1].argmax(-1, keepdim=True)
        ref_step = model(nxt, past_key_values=ref.past_key_values, use_cache=True).logits
    patch_model(model, quantize=False, fuse_norm=True, fuse_mlp=True)
    assert all(isinstance(l, tq._FusedBoundaryLayer) for l in model.model.layers)
    assert isinstance(model.model.norm, tq._BoundaryNorm)
    assert set(model.state_dict()) >= {"model.norm.weight", "model.layers.0.input_layernorm.weight",
                                       "model.layers.2.mlp.down_proj.weight"}
    with torch.no_grad():
        got = model(ids, use_cache=True)
        got_step = model(nxt, past_key_values=got.past_key_values, use_cache=True).logits
    torch.testing.assert_close(got.logits, ref.logits, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(got_step, ref_step, rtol=1e-5, atol=1e-5)
    # per forward: one plain rmsnorm (layer 0's input), two rmsnorm_residual per
    # layer (after attention, and after the MLP fused with the next norm)
    assert host_kernels["rmsnorm"] == 2 and host_kernels["rmsnorm_residual"] == 2 * 2 * 3
    assert host_kernels["swiglu"] == 2 * 3


def test_norm_recomputes_for_a_foreign_tensor(host_kernels):
    model, cfg = _tiny(1)
    patch_model(model, quantize=False)
    norm = model.model.norm
    h = torch.randn(1, 3, cfg.hidden_size)
    out = norm(h)  # nothing handed off for this tensor: computed here
    torch.testing.assert_close(out, _rmsnorm(h, norm.weight, norm.variance_epsilon))
    assert host_kernels["rmsnorm"] == 1


def test_patch_model_is_idempotent(host_kernels):
    model, _ = _tiny(2)
    patch_model(model, quantize=False)
    layers = list(model.model.layers)
    patch_model(model, quantize=False)
    assert list(model.model.layers) == layers
