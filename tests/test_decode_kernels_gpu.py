"""GPU tests of the decode-loop kernels (tf_rope_kv_append, tf_decode_attention,
tf_swiglu_strided) against plain PyTorch references of the same math: the
rotary formula of transformers' Qwen2 (`apply_rotary_pos_emb`, model-dtype
rounding) and softmax(q k^T * scale) v computed in fp64."""

from __future__ import annotations

import pytest
import torch

from oracle import ops as oops
from tests.parity import assert_rms_close, f32
from tritonforge_b200 import _lib

pytestmark = pytest.mark.gpu


def _attn_ref(q, kc, vc, length, scale):
    # q [B, Hq, D], caches [B, Hkv, T, D] -> [B, Hq, D] in fp64
    b, hq, d = q.shape
    hkv = kc.shape[1]
    g = hq // hkv
    k = kc[:, :, :length].double().repeat_interleave(g, dim=1)
    v = vc[:, :, :length].double().repeat_interleave(g, dim=1)
    s = torch.einsum("bhd,bhtd->bht", q.double(), k) * scale
    return torch.einsum("bht,bhtd->bhd", torch.softmax(s, dim=-1), v)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b,hq,hkv,d,t_max,length", [
    (8, 14, 2, 64, 200, 137),      # 0.5B decode, batch 8
    (1, 14, 2, 64, 64, 1),         # first position
    (2, 28, 4, 128, 2304, 2049),   # 7B, 2048-token context
    (1, 64, 8, 128, 4352, 4097),   # 72B, 4096-token context
    (3, 8, 8, 64, 96, 96),         # MHA, full cache
])
def test_decode_attention(b, hq, hkv, d, t_max, length, dtype):
    g = torch.Generator(device="cuda").manual_seed(b * 100 + hq + length)
    q = torch.randn(b, hq, d, device="cuda", generator=g).to(dtype)
    kc = torch.randn(b, hkv, t_max, d, device="cuda", generator=g).to(dtype)
    vc = torch.randn(b, hkv, t_max, d, device="cuda", generator=g).to(dtype)
    out = torch.empty(b, hq * d, device="cuda", dtype=dtype)
    lens = torch.tensor([length - 1, length], dtype=torch.int32, device="cuda")
    scale = d ** -0.5
    lib = _lib.load()
    for _ in range(2):  # determinism
        rc = lib.tf_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), lens.data_ptr() + 4,
                                     b, hq, hkv, d, t_max, scale, _lib.dtype_code(dtype), _lib.stream_ptr(q.device))
        _lib.check(rc, "decode_attention")
        first = out.clone() if _ == 0 else first
    assert torch.equal(first, out)
    ref = _attn_ref(q, kc, vc, length, scale).reshape(b, hq * d)
    assert_rms_close(out, ref.float().cpu().numpy(), dtype, "decode attention")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128)])
def test_rope_kv_append(hq, hkv, d, dtype):
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding, apply_rotary_pos_emb

    from tritonforge_b200.decode import QWEN25, hf_config

    shape = QWEN25["0.5b" if d == 64 else "7b"]
    rot = Qwen2RotaryEmbedding(hf_config(shape)).cuda()
    b, t_max, pos = 3, 40, 17
    cos, sin = rot(torch.zeros(1, 1, 8, device="cuda", dtype=dtype), torch.arange(t_max, device="cuda")[None])
    cos, sin = cos[0].contiguous(), sin[0].contiguous()
    g = torch.Generator(device="cuda").manual_seed(hq)
    qkv = torch.randn(b, (hq + 2 * hkv) * d, device="cuda", generator=g).to(dtype)
    q_out = torch.empty(b, hq, d, device="cuda", dtype=dtype)
    kc = torch.zeros(b, hkv, t_max, d, device="cuda", dtype=dtype)
    vc = torch.zeros_like(kc)
    posb = torch.tensor([pos, pos + 1], dtype=torch.int32, device="cuda")
    rc = _lib.load().tf_rope_kv_append(qkv.data_ptr(), qkv.stride(0), q_out.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                       kc.data_ptr(), vc.data_ptr(), posb.data_ptr(), b, hq, hkv, d, t_max,
                                       _lib.dtype_code(dtype), _lib.stream_ptr(qkv.device))
    _lib.check(rc, "rope_kv_append")
    q = qkv[:, : hq * d].view(b, hq, 1, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(b, hkv, 1, d)
    v = qkv[:, (hq + hkv) * d:].view(b, hkv, d)
    q_ref, k_ref = apply_rotary_pos_emb(q, k, cos[pos][None, None], sin[pos][None, None], unsqueeze_dim=1)
    assert torch.equal(q_out, q_ref[:, :, 0]), "rotated q must equal transformers' formula bit for bit"
    assert torch.equal(kc[:, :, pos], k_ref[:, :, 0])
    assert torch.equal(vc[:, :, pos], v)
    assert kc[:, :, :pos].abs().sum() == 0 and kc[:, :, pos + 1:].abs().sum() == 0


def test_swiglu_strided_halves():
    g = torch.Generator(device="cuda").manual_seed(5)
    gu = (torch.randn(8, 2 * 4864, device="cuda", generator=g) * 3).half()
    out = torch.empty(8, 4864, device="cuda", dtype=torch.half)
    rc = _lib.load().tf_swiglu_strided(gu.data_ptr(), gu.data_ptr() + 4864 * 2, out.data_ptr(), 8, 4864,
                                       gu.stride(0), gu.stride(0), out.stride(0), _lib.F16, _lib.stream_ptr(gu.device))
    _lib.check(rc, "swiglu_strided")
    ref = oops.swiglu(f32(gu[:, :4864]), f32(gu[:, 4864:]), "float16")
    assert_rms_close(out, ref, torch.float16, "swiglu strided", max_mismatch=0.01)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b,hq,hkv,d,t_max,pos", [(8, 14, 2, 64, 200, 137), (2, 28, 4, 128, 2304, 2048),
                                                   (3, 64, 8, 128, 4352, 0), (1, 8, 1, 128, 600, 599),
                                                   (32, 16, 2, 128, 1100, 515)])
def test_fused_rope_attention_equals_separate(b, hq, hkv, d, t_max, pos, dtype):
    """tf_decode_attention_rope == tf_rope_kv_append then tf_decode_attention, bit for bit."""
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    from tritonforge_b200.decode import QwenShape, hf_config

    rot = Qwen2RotaryEmbedding(hf_config(QwenShape(hq * d, 128, 1, hq, hkv, d, 16))).cuda()
    cos, sin = rot(torch.zeros(1, 1, 8, device="cuda", dtype=dtype), torch.arange(t_max, device="cuda")[None])
    cos, sin = cos[0].contiguous(), sin[0].contiguous()
    g = torch.Generator(device="cuda").manual_seed(b * 7 + pos)
    qkv = torch.randn(b, (hq + 2 * hkv) * d, device="cuda", generator=g).to(dtype)
    kc = torch.randn(b, hkv, t_max, d, device="cuda", generator=g).to(dtype)
    vc = torch.randn(b, hkv, t_max, d, device="cuda", generator=g).to(dtype)
    kc2, vc2 = kc.clone(), vc.clone()
    posb = torch.tensor([pos, pos + 1], dtype=torch.int32, device="cuda")
    lib, st, dt = _lib.load(), _lib.stream_ptr(qkv.device), _lib.dtype_code(dtype)
    q = torch.empty(b, hq, d, device="cuda", dtype=dtype)
    out_ref = torch.empty(b, hq * d, device="cuda", dtype=dtype)
    _lib.check(lib.tf_rope_kv_append(qkv.data_ptr(), qkv.stride(0), q.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                     kc.data_ptr(), vc.data_ptr(), posb.data_ptr(), b, hq, hkv, d, t_max, dt, st),
               "rope_kv_append")
    _lib.check(lib.tf_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out_ref.data_ptr(),
                                       posb.data_ptr() + 4, b, hq, hkv, d, t_max, d ** -0.5, dt, st), "attention")
    out = torch.empty_like(out_ref)
    _lib.check(lib.tf_decode_attention_rope(qkv.data_ptr(), qkv.stride(0), cos.data_ptr(), sin.data_ptr(),
                                            kc2.data_ptr(), vc2.data_ptr(), posb.data_ptr(), out.data_ptr(), b, hq,
                                            hkv, d, t_max, d ** -0.5, dt, st), "attention_rope")
    torch.cuda.synchronize()
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc), "the same key and value appended"
    assert torch.equal(out, out_ref), "the same attention output"
