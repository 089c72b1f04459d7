"""GPU model-level tests: the patched transformers model and the CUDA-graph
decoder against the reference's own CPU path (golden tokens recorded from the
reference, tests/golden/make_model_golden.py) and against transformers' own
unpatched model, mirroring the reference's tests/test_integration.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from oracle import ops as oops
from tests import golden_io as gio
from tests.parity import assert_rms_close, f32, oracle_linear
from tritonforge_b200 import kernels
from tritonforge_b200.decode import QwenDecoder, random_qwen2
from tritonforge_b200.integration import QuantLinear, patch_model

pytestmark = pytest.mark.gpu


def _golden():
    with np.load(gio.GOLDEN / "qwen05b_greedy.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="module")
def qwen05b():
    torch.manual_seed(0)
    model = random_qwen2("0.5b", seed=0)
    sd = model.state_dict()
    keys = ["model.embed_tokens.weight", "model.layers.0.self_attn.q_proj.weight",
            "model.layers.23.mlp.down_proj.weight", "model.norm.weight"]
    checksum = np.array([sd[k].double().sum().item() for k in keys])
    model = model.cuda()
    patch_model(model, group_size=128, dtype=torch.float16)
    return model, checksum


def test_random_init_matches_golden_weights(qwen05b):
    _, checksum = qwen05b
    assert np.allclose(checksum, _golden()["checksum"], rtol=0, atol=1e-6), "seeded weights differ"


def test_greedy_tokens_match_reference(qwen05b):
    """Greedy decode of 32 tokens (128-token random prompts, batch 2) through
    the CUDA-graph decoder must reproduce the reference's tokens."""
    model, _ = qwen05b
    gold = _golden()
    prompt = torch.from_numpy(gold["prompt"]).cuda()
    want = gold["tokens"]
    dec = QwenDecoder(model, batch=prompt.shape[0], max_len=prompt.shape[1] + want.shape[1] + 8)
    got = dec.generate(prompt, want.shape[1]).cpu().numpy()
    report = []
    for b in range(want.shape[0]):
        diff = np.nonzero(got[b] != want[b])[0]
        first = int(diff[0]) if diff.size else None
        gap = None if first is None else float(gold["top2_gap"][b, first])
        report.append((b, first, gap))
    assert all(r[1] is None for r in report), (
        "first divergent step per sequence (seq, step, reference top-2 logit gap at that step): "
        f"{report}")


def test_decoder_step_matches_eager_path(qwen05b):
    """The graph replay and the eager step produce the same tokens."""
    model, _ = qwen05b
    gold = _golden()
    prompt = torch.from_numpy(gold["prompt"][:1, :64]).cuda()
    a = QwenDecoder(model, batch=1, max_len=96).generate(prompt, 8, use_graph=True)
    b = QwenDecoder(model, batch=1, max_len=96).generate(prompt, 8, use_graph=False)
    assert torch.equal(a, b)


# ---- mirrors of the reference's tests/test_integration.py -------------------
def _tiny_model(dtype):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
    return Qwen2ForCausalLM(cfg).to(dtype=dtype).to("cuda").eval(), cfg


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quant_linear_matches_oracle(dtype):
    torch.manual_seed(0)
    lin = nn.Linear(128, 64, bias=True).to(device="cuda", dtype=dtype)
    qlin = QuantLinear.from_linear(lin, group_size=128, dtype=dtype, fuse_max_m=128)
    for m in (4, 32, 100):  # decode kernel and the larger-M kernel
        x = torch.randn(m, 128, device="cuda", dtype=dtype)
        got = qlin(x)
        ref = oracle_linear(x, qlin.packed, qlin.scales, qlin.zeros, qlin.bias, 128)
        assert_rms_close(got, ref, dtype, f"QuantLinear m={m}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_patch_model_logits_close(dtype):
    torch.manual_seed(0)
    model, cfg = _tiny_model(dtype)
    ids = torch.randint(0, cfg.vocab_size, (1, 8), device="cuda")
    with torch.no_grad():
        ref = model(ids).logits
    patch_model(model, group_size=128, dtype=dtype)
    with torch.no_grad():
        got = model(ids).logits
    rel = (got.float() - ref.float()).abs().mean() / ref.float().abs().mean()
    assert rel.item() < 0.2, rel.item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_norm_and_mlp_are_near_exact(dtype):
    torch.manual_seed(0)
    model, cfg = _tiny_model(dtype)
    ids = torch.randint(0, cfg.vocab_size, (1, 8), device="cuda")
    with torch.no_grad():
        ref = model(ids).logits
    patch_model(model, quantize=False, fuse_norm=True, fuse_mlp=True)
    with torch.no_grad():
        got = model(ids).logits
    rel = (got.float() - ref.float()).abs().mean() / ref.float().abs().mean()
    assert rel.item() < 1e-2, rel.item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_patch_model_cache_decode_close(dtype):
    torch.manual_seed(0)
    model, cfg = _tiny_model(dtype)
    prompt = torch.randint(0, cfg.vocab_size, (1, 6), device="cuda")
    with torch.no_grad():
        ref_pref = model(prompt, use_cache=True)
        nxt = ref_pref.logits[:, -1, :].argmax(-1, keepdim=True)
        ref_step = model(nxt, past_key_values=ref_pref.past_key_values, use_cache=True).logits
    patch_model(model, group_size=128, dtype=dtype)
    with torch.no_grad():
        got_pref = model(prompt, use_cache=True)
        got_step = model(nxt, past_key_values=got_pref.past_key_values, use_cache=True).logits
    rel = (got_step.float() - ref_step.float()).abs().mean() / ref_step.float().abs().mean()
    assert rel.item() < 0.2, rel.item()


def test_fused_rmsnorm_matches_reference_formula():
    torch.manual_seed(0)
    x = torch.randn(8, 128, device="cuda", dtype=torch.float16)
    weight = torch.randn(128, device="cuda", dtype=torch.float16)
    got = kernels.rmsnorm(x, weight)
    assert_rms_close(got, oops.rmsnorm(f32(x), f32(weight), 1e-6, "float16"), torch.float16, "rmsnorm")
