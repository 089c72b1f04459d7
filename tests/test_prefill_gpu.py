"""GPU tests of the engine's prompt prefill (QwenDecoder.prefill_tokens): the
prefill against the same prompt fed through the decode step one token at a
time (same weights, the same kernels but for the summation order and the
attention library), at a length that runs the chunked decode GEMV (40 rows)
and one that runs the tcgen05 GEMM (200 rows)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,length", [(2, 40), (1, 200)])
def test_prefill_matches_token_by_token_decode(batch, length):
    from tests.parity import assert_rms_close, f32
    from tests.tp_check import logits_close, near_tie
    from tritonforge_b200.decode import QwenDecoder, QwenWeights

    dev = torch.device("cuda", 0)
    w = QwenWeights.synthetic("7b", dtype=torch.bfloat16, device=dev, seed=3, layers=2)
    a = QwenDecoder(w, batch, length + 16, colmajor=False)
    b = QwenDecoder(w, batch, length + 16, colmajor=False)
    g = torch.Generator().manual_seed(length)
    prompt = torch.randint(0, w.embed.shape[0], (batch, length), generator=g)
    got = a.prefill_tokens(prompt)
    b.pos.copy_(torch.tensor([0, 1], dtype=torch.int32))
    for t in range(length):
        b.tokens.copy_(prompt[:, t].to(dev))
        b.step()
    torch.cuda.synchronize()
    assert a.pos.tolist() == b.pos.tolist() == [length, length + 1]
    ok, err, rms, mean = logits_close(a.buf["logits"], b.buf["logits"])
    assert ok, f"last-position logits: max beyond one ulp {err:.4g}, mean {mean:.4g}, RMS {rms:.4g}"
    tie_ok, gap = near_tie(b.buf["logits"], b.tokens, got.to(dev), rms)
    assert tie_ok, f"greedy tokens differ beyond a near tie (gap {gap:.4g})"
    # the caches hold the same keys and values: the first layer's within the
    # per-op contract (identical inputs; the projections' fp32 sums differ in
    # order only), later layers within the whole-decode bound (their inputs
    # already carry the earlier layers' one-ulp flips)
    for li in range(len(w.layers)):
        for name, ca, cb in (("k", a.k_cache, b.k_cache), ("v", a.v_cache, b.v_cache)):
            got, want = ca[li, :, :, :length], cb[li, :, :, :length]
            if li == 0:
                assert_rms_close(got, f32(want), torch.bfloat16, f"{name} cache layer 0", mean_frac=None)
            else:
                ok, err, rms, mean = logits_close(got, want)
                assert ok, f"{name} cache layer {li}: max beyond one ulp {err:.4g}, mean {mean:.4g}, RMS {rms:.4g}"
    # both continue decoding from the prefilled state
    b.tokens.copy_(a.tokens)
    for _ in range(2):
        a.step()
        b.step()
        ok, err, rms, mean = logits_close(a.buf["logits"], b.buf["logits"])
        assert ok, f"decode after prefill: max beyond one ulp {err:.4g}, mean {mean:.4g}"
        b.tokens.copy_(a.tokens)
    assert a.device_errors() == 0 and b.device_errors() == 0


def test_prefill_needs_k_major_projections():
    from tritonforge_b200.decode import QwenDecoder, QwenWeights

    w = QwenWeights.synthetic("7b", dtype=torch.bfloat16, device=torch.device("cuda", 0), seed=3, layers=1)
    d = QwenDecoder(w, 16, 64)  # batches 9..128: column-major projections
    with pytest.raises(RuntimeError, match="K-major"):
        d.prefill_tokens(torch.zeros(16, 8, dtype=torch.long))


def _rope_ref(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    # transformers' apply_rotary_pos_emb in the model dtype: each product and the sum rounded
    h = t.shape[-1] // 2
    return t * cos + torch.cat((-t[..., h:], t[..., :h]), dim=-1) * sin


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("t0,hq,hkv,d", [(37, 28, 4, 128), (200, 14, 2, 64), (1, 8, 8, 128)])
@pytest.mark.parametrize("in_place", [True, False])
def test_rope_kv_prefill_bit_exact(t0, hq, hkv, d, dtype, in_place):
    """tf_rope_kv_prefill against transformers' rounding in torch: q (in place
    over the projection, or into another buffer), k and v in the cache, bit
    for bit; cache positions past the prompt untouched."""
    from tritonforge_b200 import _lib

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(t0 + hq)
    width = (hq + 2 * hkv) * d
    ld = width + 16
    qkv = torch.randn(t0, ld, generator=g).to(dtype).to(dev)
    t_max = t0 + 5
    ang = torch.rand(t_max, d // 2, generator=g) * 6.0
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(dtype).to(dev)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(dtype).to(dev)
    kc = torch.full((hkv, t_max, d), float("nan"), dtype=dtype, device=dev)
    vc = torch.full_like(kc, float("nan"))
    c, s = cos[:t0, None, :], sin[:t0, None, :]
    want_q = _rope_ref(qkv[:, :hq * d].view(t0, hq, d), c, s)
    want_k = _rope_ref(qkv[:, hq * d:(hq + hkv) * d].view(t0, hkv, d), c, s).transpose(0, 1)
    want_v = qkv[:, (hq + hkv) * d:width].view(t0, hkv, d).transpose(0, 1).clone()
    before = qkv.clone()
    q_out = qkv if in_place else torch.zeros(t0, hq * d + 8, dtype=dtype, device=dev)
    _lib.check(_lib.load().tf_rope_kv_prefill(qkv.data_ptr(), ld, q_out.data_ptr(), q_out.stride(0), cos.data_ptr(),
                                              sin.data_ptr(), kc.data_ptr(), vc.data_ptr(), t0, hq, hkv, d, t_max,
                                              _lib.dtype_code(dtype), _lib.stream_ptr(dev)), "rope_kv_prefill")
    torch.cuda.synchronize()
    assert torch.equal(q_out[:, :hq * d].view(t0, hq, d), want_q)
    assert torch.equal(kc[:, :t0], want_k) and torch.equal(vc[:, :t0], want_v)
    assert torch.isnan(kc[:, t0:].float()).all() and torch.isnan(vc[:, t0:].float()).all()
    assert torch.equal(qkv[:, hq * d:], before[:, hq * d:]), "k, v columns and padding are read only"
    if not in_place:
        assert torch.equal(qkv, before)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m,inter", [(1, 64), (37, 4864), (2048, 18944)])
def test_swiglu_gu_matches_swiglu_on_the_halves(m, inter, dtype):
    """tf_swiglu_gu on the per-64 interleaved gate|up output equals tf_swiglu on
    the de-interleaved halves bit for bit (and so the oracle's rounding)."""
    from tritonforge_b200 import _lib, kernels

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(m + inter)
    gu = (torch.randn(m, 2 * inter + 32, generator=g) * 3).to(dtype).to(dev)
    v = gu[:, :2 * inter].view(m, inter // 64, 2, 64)
    want = kernels.swiglu(v[:, :, 0].contiguous(), v[:, :, 1].contiguous()).view(m, inter)
    act = torch.full((m, inter + 8), float("nan"), dtype=dtype, device=dev)
    _lib.check(_lib.load().tf_swiglu_gu(gu.data_ptr(), gu.stride(0), act.data_ptr(), act.stride(0), m, inter,
                                        _lib.dtype_code(dtype), _lib.stream_ptr(dev)), "swiglu_gu")
    torch.cuda.synchronize()
    assert torch.equal(act[:, :inter], want)
    assert torch.isnan(act[:, inter:].float()).all()
